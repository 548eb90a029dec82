// Gather-ceiling probe for the step kernel of libafb (a measurement utility built into its own library,
// libafb_probe.so; it has no counterpart in the reference and is not part of libafb.so's interface).
//
// The step kernel's cost is gathering, for every synapse of the light cone, one 512-byte row of state
// (256 float16 positions) from L2 into the SM.  afb_probe_gather runs that access pattern alone through
// the load path the step kernel uses -- 16-byte ld.global.nc per lane into registers -- with 8 rows in
// flight per lane, so bench.py can report the step kernel's gather rate as a fraction of what the device
// sustains on the same pattern.
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

#include "../../include/afb_probe.h"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxBlocksPerSm = 8;     // 64 warps per SM
constexpr int kInFlight = 8;           // rows in flight per lane
constexpr unsigned kAll = 0xffffffffu;

__device__ __forceinline__ uint32_t xor4(const uint4 &v) { return v.x ^ v.y ^ v.z ^ v.w; }

// Warp w reads rows w, w + W, ... (W = warps in the grid), kInFlight at a time; lane l takes bytes
// [16 l, 16 l + 16) of each row.  Every row is folded into one word per warp so that no load is dropped.
__global__ void __launch_bounds__(kThreads) gather_probe_ldg(const uint4 *__restrict__ slab, int64_t slab_rows,
                                                             const int *__restrict__ rows, int64_t n_rows,
                                                             uint32_t *__restrict__ sink) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
    const int64_t n_warps = ((int64_t)gridDim.x * kThreads) >> 5;
    uint32_t x = 0;
    int64_t r = warp;
    for (; r + (kInFlight - 1) * n_warps < n_rows; r += kInFlight * n_warps) {
        int idx[kInFlight];
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) idx[u] = __ldg(rows + r + u * n_warps);
        uint4 v[kInFlight];
#pragma unroll
        for (int u = 0; u < kInFlight; ++u)
            v[u] = (uint64_t)idx[u] < (uint64_t)slab_rows ? __ldg(slab + (int64_t)idx[u] * 32 + lane) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) x ^= xor4(v[u]);
    }
    for (; r < n_rows; r += n_warps) {
        const int i = __ldg(rows + r);
        if ((uint64_t)i < (uint64_t)slab_rows) x ^= xor4(__ldg(slab + (int64_t)i * 32 + lane));
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) x ^= __shfl_xor_sync(kAll, x, s);
    if (lane == 0) sink[warp] = x;
}

int sm_count() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return -1;
    return sms;
}

}  // namespace

extern "C" {

int64_t afb_probe_gather_sink_words(void) {
    const int sms = sm_count();
    return sms < 0 ? AFB_PROBE_ECUDA : (int64_t)sms * kMaxBlocksPerSm * kWarps;
}

int afb_probe_gather(int blocks_per_sm, const void *slab, int64_t slab_rows, const int32_t *rows, int64_t n_rows,
                     uint32_t *sink, int64_t sink_words, void *stream) {
    if (blocks_per_sm <= 0) blocks_per_sm = kMaxBlocksPerSm;
    if (blocks_per_sm > kMaxBlocksPerSm || !slab || !rows || !sink || ((uintptr_t)slab & 15) != 0 || slab_rows <= 0 ||
        slab_rows >= (1LL << 31) || n_rows < 0)
        return AFB_PROBE_EINVAL;
    const int sms = sm_count();
    if (sms < 0) return AFB_PROBE_ECUDA;
    if (sink_words < (int64_t)sms * kMaxBlocksPerSm * kWarps) return AFB_PROBE_EINVAL;
    if (n_rows == 0) return AFB_PROBE_OK;
    gather_probe_ldg<<<sms * blocks_per_sm, kThreads, 0, (cudaStream_t)stream>>>(static_cast<const uint4 *>(slab), slab_rows,
                                                                                  rows, n_rows, sink);
    return cudaGetLastError() == cudaSuccess ? AFB_PROBE_OK : AFB_PROBE_ECUDA;
}

}  // extern "C"
