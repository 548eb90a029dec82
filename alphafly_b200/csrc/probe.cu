// Ceiling probes for the step kernel's gather: 512-byte rows read from L2 in a caller-given order, by
// each of the three load paths a step kernel can use.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "../../include/afb_probe.h"

namespace afb {
namespace {

constexpr int kProbeThreads = 256;
constexpr int kProbeWarps = kProbeThreads / 32;
constexpr int kProbeBlocksPerSm = 8;     // register path: 64 warps per SM
constexpr int kRingBlocksPerSm = 3;      // shared-memory paths: 3 x 64 KB rings per SM
constexpr int kPStages = 4;              // ring paths: stages of 4 rows per warp
constexpr int kPStageBytes = 4 * 512;
constexpr int kPRingBytes = kProbeWarps * kPStages * kPStageBytes;
constexpr uint32_t kPWaitLimit = 1u << 22;
constexpr unsigned kAll = 0xffffffffu;

__device__ __forceinline__ uint32_t xor4(const uint4 &v) { return v.x ^ v.y ^ v.z ^ v.w; }

// Register path: warp w reads rows w, w + W, ... (W = warps in the grid), kProbeUnroll at a time (loads
// in flight per lane), lane l taking bytes [16 l, 16 l + 16) of each row.
template <int kProbeUnroll>
__global__ void __launch_bounds__(kProbeThreads) gather_probe_ldg(const uint4 *__restrict__ slab, int64_t slab_rows,
                                                                  const int *__restrict__ rows, int64_t n_rows,
                                                                  uint32_t *__restrict__ sink) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * kProbeThreads + threadIdx.x) >> 5;
    const int64_t n_warps = ((int64_t)gridDim.x * kProbeThreads) >> 5;
    uint32_t x = 0;
    int64_t r = warp;
    for (; r + (kProbeUnroll - 1) * n_warps < n_rows; r += kProbeUnroll * n_warps) {
        int idx[kProbeUnroll];
#pragma unroll
        for (int u = 0; u < kProbeUnroll; ++u) idx[u] = __ldg(rows + r + u * n_warps);
        uint4 v[kProbeUnroll];
#pragma unroll
        for (int u = 0; u < kProbeUnroll; ++u)
            v[u] = (uint64_t)idx[u] < (uint64_t)slab_rows ? __ldg(slab + (int64_t)idx[u] * 32 + lane) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < kProbeUnroll; ++u) x ^= xor4(v[u]);
    }
    for (; r < n_rows; r += n_warps) {
        const int i = __ldg(rows + r);
        if ((uint64_t)i < (uint64_t)slab_rows) x ^= xor4(__ldg(slab + (int64_t)i * 32 + lane));
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) x ^= __shfl_xor_sync(kAll, x, s);
    if (lane == 0) sink[warp] = x;
}

// Register path with 8-byte lanes: rows of 256 bytes (slab_rows x 2 of them), lane l taking bytes
// [8 l, 8 l + 8), kProbeUnroll loads in flight per lane.
template <int kProbeUnroll>
__global__ void __launch_bounds__(kProbeThreads) gather_probe_ldg_narrow(const uint2 *__restrict__ slab, int64_t slab_rows,
                                                                         const int *__restrict__ rows, int64_t n_rows,
                                                                         uint32_t *__restrict__ sink) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * kProbeThreads + threadIdx.x) >> 5;
    const int64_t n_warps = ((int64_t)gridDim.x * kProbeThreads) >> 5;
    const int64_t half_rows = 2 * slab_rows;
    uint32_t x = 0;
    int64_t r = warp;
    for (; r + (kProbeUnroll - 1) * n_warps < n_rows; r += kProbeUnroll * n_warps) {
        int idx[kProbeUnroll];
#pragma unroll
        for (int u = 0; u < kProbeUnroll; ++u) idx[u] = __ldg(rows + r + u * n_warps);
        uint2 v[kProbeUnroll];
#pragma unroll
        for (int u = 0; u < kProbeUnroll; ++u)
            v[u] = (uint64_t)idx[u] < (uint64_t)half_rows ? __ldg(slab + (int64_t)idx[u] * 32 + lane) : make_uint2(0, 0);
#pragma unroll
        for (int u = 0; u < kProbeUnroll; ++u) x ^= v[u].x ^ v[u].y;
    }
    for (; r < n_rows; r += n_warps) {
        const int i = __ldg(rows + r);
        if ((uint64_t)i < (uint64_t)half_rows) {
            const uint2 v = __ldg(slab + (int64_t)i * 32 + lane);
            x ^= v.x ^ v.y;
        }
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) x ^= __shfl_xor_sync(kAll, x, s);
    if (lane == 0) sink[warp] = x;
}

__device__ __forceinline__ uint4 lds16(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

// cp.async path: groups of 4 rows (entries 4g .. 4g+3 of `rows`), group g to warp g mod W; a warp's ring
// has kPStages stages and kPStages - 1 groups in flight.  READ: every lane also reads its 16 bytes of
// each row back from shared memory, as a step kernel's sums do.
template <bool READ>
__global__ void __launch_bounds__(kProbeThreads) gather_probe_cpasync(const uint4 *__restrict__ slab, int64_t slab_rows,
                                                                      const int *__restrict__ rows, int64_t n_groups,
                                                                      uint32_t *__restrict__ sink) {
    extern __shared__ __align__(128) unsigned char pring[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int64_t warp = ((int64_t)blockIdx.x * kProbeThreads + threadIdx.x) >> 5;
    const int64_t n_warps = ((int64_t)gridDim.x * kProbeThreads) >> 5;
    const uint32_t ring = (uint32_t)__cvta_generic_to_shared(pring) + wib * kPStages * kPStageBytes + lane * 16;
    const int64_t mine = warp < n_groups ? (n_groups - 1 - warp) / n_warps + 1 : 0;
    uint32_t x = 0;
    auto issue = [&](int64_t it) {
        if (it < mine) {
            const int64_t g = warp + it * n_warps;
            const uint32_t dst = ring + (uint32_t)(it % kPStages) * kPStageBytes;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = __ldg(rows + 4 * g + u);
                const int row = (uint64_t)i < (uint64_t)slab_rows ? i : 0;
                asm volatile("cp.async.ca.shared.global [%0], [%1], 16;\n" ::"r"(dst + u * 512), "l"(slab + (int64_t)row * 32 + lane)
                             : "memory");
            }
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    };
#pragma unroll
    for (int s = 0; s < kPStages - 1; ++s) issue(s);
    for (int64_t it = 0; it < mine; ++it) {
        issue(it + kPStages - 1);
        asm volatile("cp.async.wait_group %0;\n" ::"n"(kPStages - 1) : "memory");
        if (READ) {
            const uint32_t src = ring + (uint32_t)(it % kPStages) * kPStageBytes;
#pragma unroll
            for (int u = 0; u < 4; ++u) x ^= xor4(lds16(src + u * 512));
        }
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) x ^= __shfl_xor_sync(kAll, x, s);
    if (lane == 0) sink[warp] = x;
}

__device__ __forceinline__ void pbar_init(uint32_t bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool pbar_wait(uint32_t bar, uint32_t parity, uint32_t limit) {
    for (uint32_t it = 0; it < limit; ++it) {
        uint32_t ok;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
        if (ok) return true;
    }
    return false;
}

// TMA path: lane 0 of a warp copies each group's 4 rows with one tile::gather4 (box one row high, x = 0)
// into a ring stage and arms the stage's mbarrier with 2 KB; waits are bounded and a lost stage is
// reported as sink word 0xffffffff of that warp (never expected) after a bounded drain.
template <bool READ>
__global__ void __launch_bounds__(kProbeThreads) gather_probe_tma(const __grid_constant__ CUtensorMap map, int64_t slab_rows,
                                                                  const int *__restrict__ rows, int64_t n_groups,
                                                                  uint32_t *__restrict__ sink) {
    extern __shared__ __align__(128) unsigned char pring[];
    __shared__ __align__(8) uint64_t bars[kProbeWarps][kPStages];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int64_t warp = ((int64_t)blockIdx.x * kProbeThreads + threadIdx.x) >> 5;
    const int64_t n_warps = ((int64_t)gridDim.x * kProbeThreads) >> 5;
    const uint32_t ring = (uint32_t)__cvta_generic_to_shared(pring) + wib * kPStages * kPStageBytes;
    const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(&bars[wib][0]);
    if (lane < kPStages) pbar_init(bar0 + lane * 8);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    __syncwarp();
    const int64_t mine = warp < n_groups ? (n_groups - 1 - warp) / n_warps + 1 : 0;
    uint32_t x = 0;
    bool lost = false;
    auto issue = [&](int64_t it) {
        if (it < mine) {
            const int64_t g = warp + it * n_warps;
            const int st = (int)(it % kPStages);
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            if (lane == 0) {
                int c[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int i = __ldg(rows + 4 * g + u);
                    c[u] = (uint64_t)i < (uint64_t)slab_rows ? i : 0;
                }
                asm volatile("{\n .reg .b64 s;\n mbarrier.arrive.expect_tx.shared::cta.b64 s, [%0], %1;\n}\n"
                             ::"r"(bar0 + st * 8), "r"(kPStageBytes) : "memory");
                asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
                             " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];\n"
                             ::"r"(ring + st * kPStageBytes), "l"(reinterpret_cast<uint64_t>(&map)), "r"(0), "r"(c[0]), "r"(c[1]),
                             "r"(c[2]), "r"(c[3]), "r"(bar0 + st * 8) : "memory");
            }
        }
    };
#pragma unroll
    for (int s = 0; s < kPStages - 1; ++s) issue(s);
    for (int64_t it = 0; it < mine; ++it) {
        issue(it + kPStages - 1);
        const int st = (int)(it % kPStages);
        if (!pbar_wait(bar0 + st * 8, (uint32_t)((it / kPStages) & 1), lost ? 1024u : kPWaitLimit)) lost = true;
        if (READ) {
#pragma unroll
            for (int u = 0; u < 4; ++u) x ^= xor4(lds16(ring + st * kPStageBytes + u * 512 + lane * 16));
        }
        __syncwarp();
    }
    if (lost) {
        for (int st = 0; st < kPStages && st < mine; ++st) {
            const int64_t last = st + ((mine - 1 - st) / kPStages) * kPStages;
            pbar_wait(bar0 + st * 8, (uint32_t)((last / kPStages) & 1), 1u << 16);
        }
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) x ^= __shfl_xor_sync(kAll, x, s);
    if (lane == 0) sink[warp] = lost ? 0xffffffffu : x;
}

int sm_count() {
    int dev = 0, sms = 0;
    AFB_CUDA(cudaGetDevice(&dev));
    AFB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    return sms;
}

template <typename K>
void allow_ring(K kernel) {
    AFB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPRingBytes));
}

void encode_slab_map(CUtensorMap *map, const void *slab, int64_t slab_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        AFB_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        AFB_CHECK(q == cudaDriverEntryPointSuccess && fn, "cuTensorMapEncodeTiled is not available from the driver");
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const cuuint64_t dim[2] = {128, (cuuint64_t)slab_rows};
    const cuuint64_t stride[1] = {512};
    const cuuint32_t box[2] = {128, 1};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(slab), dim, stride, box, estride,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    AFB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
}

}  // namespace
}  // namespace afb

using namespace afb;

extern "C" {

int64_t afb_probe_gather_sink_words(void) {
    int64_t words = -1;
    const int rc = guarded([&] { words = (int64_t)sm_count() * kProbeBlocksPerSm * kProbeWarps; });
    return rc == AFB_OK ? words : rc;
}

int afb_probe_gather(int path, int blocks_per_sm, const void *slab, int64_t slab_rows, const int32_t *rows, int64_t n_rows,
                     uint32_t *sink, int64_t sink_words, void *stream) {
    return guarded([&] {
        AFB_CHECK(path >= AFB_PROBE_LDG && path <= AFB_PROBE_LDG_NARROW16, "afb_probe_gather: unknown path");
        const bool ldg = path == AFB_PROBE_LDG || path == AFB_PROBE_LDG4 || path == AFB_PROBE_LDG16 ||
                         path == AFB_PROBE_LDG_NARROW8 || path == AFB_PROBE_LDG_NARROW16;
        if (blocks_per_sm <= 0) blocks_per_sm = ldg ? kProbeBlocksPerSm : kRingBlocksPerSm;
        AFB_CHECK(blocks_per_sm <= (ldg ? kProbeBlocksPerSm : kRingBlocksPerSm), "afb_probe_gather: too many blocks per SM");
        AFB_CHECK(slab && rows && sink, "afb_probe_gather: null pointer");
        AFB_CHECK(((uintptr_t)slab & 15) == 0, "afb_probe_gather: slab must be 16-byte aligned");
        AFB_CHECK(slab_rows > 0 && slab_rows < (1LL << 31) && n_rows >= 0, "afb_probe_gather: bad sizes");
        AFB_CHECK(ldg || n_rows % 4 == 0, "afb_probe_gather: ring paths take rows in groups of 4");
        const int sms = sm_count();
        AFB_CHECK(sink_words >= (int64_t)sms * kProbeBlocksPerSm * kProbeWarps, "afb_probe_gather: sink too small");
        if (n_rows == 0) return;
        const cudaStream_t s = (cudaStream_t)stream;
        const uint4 *sl = static_cast<const uint4 *>(slab);
        const int grid = sms * blocks_per_sm, ring_grid = grid;
        switch (path) {
        case AFB_PROBE_LDG:
            gather_probe_ldg<8><<<grid, kProbeThreads, 0, s>>>(sl, slab_rows, rows, n_rows, sink);
            break;
        case AFB_PROBE_LDG4:
            gather_probe_ldg<4><<<grid, kProbeThreads, 0, s>>>(sl, slab_rows, rows, n_rows, sink);
            break;
        case AFB_PROBE_LDG16:
            gather_probe_ldg<16><<<grid, kProbeThreads, 0, s>>>(sl, slab_rows, rows, n_rows, sink);
            break;
        case AFB_PROBE_LDG_NARROW8:
            gather_probe_ldg_narrow<8><<<grid, kProbeThreads, 0, s>>>(static_cast<const uint2 *>(slab), slab_rows, rows,
                                                                      n_rows, sink);
            break;
        case AFB_PROBE_LDG_NARROW16:
            gather_probe_ldg_narrow<16><<<grid, kProbeThreads, 0, s>>>(static_cast<const uint2 *>(slab), slab_rows, rows,
                                                                       n_rows, sink);
            break;
        case AFB_PROBE_CPASYNC:
            allow_ring(gather_probe_cpasync<false>);
            gather_probe_cpasync<false><<<ring_grid, kProbeThreads, kPRingBytes, s>>>(sl, slab_rows, rows, n_rows / 4, sink);
            break;
        case AFB_PROBE_CPASYNC_READ:
            allow_ring(gather_probe_cpasync<true>);
            gather_probe_cpasync<true><<<ring_grid, kProbeThreads, kPRingBytes, s>>>(sl, slab_rows, rows, n_rows / 4, sink);
            break;
        default: {
            CUtensorMap map;
            encode_slab_map(&map, slab, slab_rows);
            if (path == AFB_PROBE_TMA) {
                allow_ring(gather_probe_tma<false>);
                gather_probe_tma<false><<<ring_grid, kProbeThreads, kPRingBytes, s>>>(map, slab_rows, rows, n_rows / 4, sink);
            } else {
                allow_ring(gather_probe_tma<true>);
                gather_probe_tma<true><<<ring_grid, kProbeThreads, kPRingBytes, s>>>(map, slab_rows, rows, n_rows / 4, sink);
            }
        }
        }
        AFB_LAUNCHED();
    });
}

}  // extern "C"
