// The float16 input map of the deviation path (chessfly/model.py:101-102, FlyChessNet.forward's drive):
//
//     u[i, p] = fp16( g * (sum_k W[i, k] x[p, k] + b[i]) )        i < n_in (input neurons), p < batch
//
// on the 5th-generation tensor cores.  W (n_in x k_dim) and x (batch x k_dim) are float16 and K-major
// (rows of k_dim elements, row strides multiples of 8 elements); u is written neuron-major (n_in x ldu),
// the layout the light-cone forward reads its drive in.
//
// A pair of CTAs (a cluster of two, on two SMs) computes 256 x 256 tiles of u with the two-SM MMA
// (tcgen05.mma.cta_group::2, M 256, N 256, K 16): CTA r of the pair holds W rows 128 r .. 128 r + 127 and
// x rows (positions) 128 r .. 128 r + 127 of every k-block, and its TMEM holds its 128 rows of the tile
// for all 256 positions.  Per k-block each SM loads 32 KB for a 128 x 256 x 64 product, the same bytes per
// FLOP as one SM computing 256 x 256, while an accumulator takes only 256 of the 512 TMEM columns: two
// accumulators alternate, so the epilogue of one tile overlaps the MMAs of the next.  The kernel is
// persistent: cluster c takes tiles c, c + (clusters), ..., neurons fastest, so concurrent pairs share x.
//   - warp 0, one lane, both CTAs: TMA producer into a ring of kStages stages.  Each CTA waits for its own
//     stage to be free (its `empty` barrier), and both CTAs' copies count their bytes on the leader's
//     (rank 0) `full` barrier, which the leader's producer arms with the bytes of both.
//   - warp 1, one lane, leader only: MMA issuer.  It waits for `full`, issues the four two-SM MMAs of the
//     k-block, and commits the stage's `empty` barrier in both CTAs; after a tile's last k-block it commits
//     the accumulator's `tfull` barrier in both CTAs, and before reusing an accumulator it waits for the
//     leader's `tempty` barrier, which the eight epilogue warps of the pair arrive on.
//   - warps 2-5, both CTAs: epilogue.  Warp w drains TMEM lanes 32 (w % 4) .. + 31 of its CTA's
//     accumulator 32 columns at a time, applies the gain and the bias in float32, rounds once to float16,
//     stages a 32 x 32 chunk (SWIZZLE_64B) and writes it with a TMA store; a u whose rows do not start on
//     16 bytes takes scalar stores.
// Every mbarrier wait is bounded and also gives up once the device status word is set: the failure is
// reported through *status and the kernel still reaches its exit, where TMEM is released.  Each CTA's
// TMA copies fill only its own shared memory.
#include <cstring>

#include "tc.cuh"

namespace afb {
namespace {

using tc::bar_init;
using tc::fail;
using tc::kBK;
using tc::kMmaK;
using tc::smem_desc;

constexpr int kHalf = 128;                       // W rows and x rows (positions) per CTA of the pair
constexpr int kTileRows = 2 * kHalf;             // neurons per pair tile (MMA M)
constexpr int kTileCols = 256;                   // positions per pair tile (MMA N)
constexpr int kStages = 5;
constexpr int kOperandBytes = kHalf * kBK * 2;   // 16 KB: one 128 x 64 float16 operand half
constexpr int kStageBytes = 2 * kOperandBytes;   // this CTA's W half and x half of a k-block
constexpr int kEpiWarps = 4;
constexpr int kThreads = 64 + 32 * kEpiWarps;    // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kChunkCols = 32;                   // one tcgen05.ld of 32 columns
constexpr int kStoreBytes = 32 * kChunkCols * 2; // one warp's 32 rows x 32 positions, float16
constexpr int kStagingBytes = kEpiWarps * 2 * kStoreBytes;
constexpr int kSmemBytes = kStages * kStageBytes + kStagingBytes + 1024 /* barriers */ + 1024 /* alignment */;
constexpr uint32_t kAccCols = kTileCols;         // one accumulator: 256 float32 columns
constexpr uint32_t kTmemCols = 2 * kAccCols;
constexpr uint32_t kIdesc = tc::idesc_f16(kTileRows, kTileCols);
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;\n" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;\n" : "=r"(r));
    return r;
}
// The shared::cluster address of the variable at `addr` (this CTA's shared window) in CTA `rank`.
__device__ __forceinline__ uint32_t map_to(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

// Bounded wait that also gives up as soon as another thread has reported a failure.
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, const int *status) {
    for (uint32_t it = 0; it < kWaitLimit; ++it) {
        uint32_t ok;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
        if (ok) return true;
        if ((it & 1023u) == 1023u && status && *reinterpret_cast<const volatile int *>(status) != 0) return false;
    }
    return false;
}

// A 2-D TMA load into this CTA's shared memory whose bytes count on an mbarrier of either CTA of the pair.
__device__ __forceinline__ void tma_load_pair(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar_cluster) {
    asm volatile("cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n"
                 ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster) : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n"
                 ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(accumulate) : "memory");
}
// Arrive on an mbarrier (shared::cluster address, either CTA) once every two-SM MMA issued so far is done.
__device__ __forceinline__ void commit_pair(uint32_t bar_cluster) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar_cluster) : "memory");
}
__device__ __forceinline__ void arrive_remote(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];\n" ::"r"(bar_cluster) : "memory");
}
__device__ __forceinline__ void tma_store(const CUtensorMap *map, int x, int y, uint32_t src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];\n"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(src) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1) input_map_kernel(const __grid_constant__ CUtensorMap map_w,
                                                                const __grid_constant__ CUtensorMap map_x,
                                                                const __grid_constant__ CUtensorMap map_u, int n_in,
                                                                int batch, int k_dim, const __half *__restrict__ bias,
                                                                float gain, __half *__restrict__ u, int64_t ldu, int tma_out,
                                                                int *__restrict__ status) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = (uint32_t)__cvta_generic_to_shared(smem_raw);
    const uint32_t ring = (raw + 1023u) & ~1023u;                        // stage s: W half, then x half
    const uint32_t staging = ring + kStages * kStageBytes;               // epilogue warp e, slot q: 2 KB
    const uint32_t bars = staging + kStagingBytes;
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (kStages + s); };
    auto tfull = [&](int b) { return bars + 8u * (2 * kStages + b); };
    auto tempty = [&](int b) { return bars + 8u * (2 * kStages + 2 + b); };
    const uint32_t tmem_slot = bars + 8u * (2 * kStages + 4);
    unsigned char *const slot_ptr = smem_raw + (tmem_slot - raw);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int n_kb = (k_dim + kBK - 1) / kBK;
    const int m_tiles = (n_in + kTileRows - 1) / kTileRows;
    const int total = m_tiles * ((batch + kTileCols - 1) / kTileCols);
    const int first = (int)cluster_id(), step = (int)cluster_count();

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            bar_init(full(s), 1);
            bar_init(empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            bar_init(tfull(b), 1);
            bar_init(tempty(b), 2 * kEpiWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&map_w)) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&map_x)) : "memory");
    }
    if (warp == 0) {                                                     // warp 0 of both CTAs allocates
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(tmem_slot), "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    cluster_sync();                                                      // both CTAs' barriers are initialised
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(slot_ptr);

    if (warp == 0 && lane == 0) {                                        // TMA producer (both CTAs)
        int it = 0;
        for (int t = first; t < total; t += step) {
            const int m0 = (t % m_tiles) * kTileRows, n0 = (t / m_tiles) * kTileCols;
            bool ok = true;
            for (int kb = 0; kb < n_kb; ++kb, ++it) {
                const int s = it % kStages, use = it / kStages;
                if (use > 0 && !wait_bar(empty(s), (use - 1) & 1, status)) {
                    fail(status, 1);
                    ok = false;
                    break;
                }
                const uint32_t leader_full = map_to(full(s), 0);
                if (rank == 0) tc::bar_expect_tx(full(s), 2 * kStageBytes);
                const uint32_t a_dst = ring + s * kStageBytes, b_dst = a_dst + kOperandBytes;
                tma_load_pair(a_dst, &map_w, kb * kBK, m0 + (int)rank * kHalf, leader_full);
                tma_load_pair(b_dst, &map_x, kb * kBK, n0 + (int)rank * kHalf, leader_full);
            }
            if (!ok) break;
        }
    } else if (warp == 1 && lane == 0 && rank == 0) {                    // MMA issuer (leader)
        int it = 0, ti = 0;
        for (int t = first; t < total; t += step, ++ti) {
            const int b = ti & 1, use_b = ti >> 1;
            if (use_b > 0 && !wait_bar(tempty(b), (use_b - 1) & 1, status)) {
                fail(status, 2);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            const uint32_t d = tmem + (uint32_t)b * kAccCols;
            bool ok = true;
            for (int kb = 0; kb < n_kb; ++kb, ++it) {
                const int s = it % kStages, use = it / kStages;
                if (!wait_bar(full(s), use & 1, status)) {
                    fail(status, 4);
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
                const uint32_t a_src = ring + s * kStageBytes, b_src = a_src + kOperandBytes;
                // the last k block takes only the 16-wide steps that hold features (K = 838: 1 of 4); the
                // skipped steps would multiply TMA's zero fill, so the sums are the same
                const int nj = min(kBK / kMmaK, (k_dim - kb * kBK + kMmaK - 1) / kMmaK);
#pragma unroll
                for (int j = 0; j < kBK / kMmaK; ++j)
                    if (j < nj)
                        mma_pair(d, smem_desc(a_src + j * kMmaK * 2), smem_desc(b_src + j * kMmaK * 2), (kb > 0 || j > 0) ? 1u : 0u);
                commit_pair(empty(s));                                   // the stage is free in both CTAs once
                commit_pair(map_to(empty(s), 1));                        // these MMAs have read it
            }
            if (!ok) break;
            commit_pair(tfull(b));                                       // the accumulator is complete
            commit_pair(map_to(tfull(b), 1));
        }
    } else if (warp >= 2) {                                              // epilogue (both CTAs)
        const int e = warp - 2, quarter = warp & 3;
        const int row = quarter * 32 + lane;                             // TMEM lane of this thread
        const uint32_t leader_tempty0 = map_to(tempty(0), 0), leader_tempty1 = map_to(tempty(1), 0);
        int ti = 0, stores = 0;
        for (int t = first; t < total; t += step, ++ti) {
            const int b = ti & 1, use_b = ti >> 1;
            const int m0 = (t % m_tiles) * kTileRows + (int)rank * kHalf, n0 = (t / m_tiles) * kTileCols;
            const bool ready = __all_sync(0xffffffffu, wait_bar(tfull(b), use_b & 1, status));
            if (!ready) {
                if (lane == 0) fail(status, 8);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            const int m = m0 + row;
            const float gb = m < n_in ? gain * __half2float(bias[m]) : 0.f;
#pragma unroll 1
            for (int c = 0; c < kTileCols / kChunkCols; ++c) {
                const int n = n0 + c * kChunkCols;
                if (n >= batch) break;                                   // uniform over the warp
                uint32_t r[32];
                tc::tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)b * kAccCols + (uint32_t)(c * kChunkCols), r);
                tc::tmem_wait_ld();
                if (tma_out) {
                    const int q = stores & 1;
                    const uint32_t dst = staging + (uint32_t)(e * 2 + q) * kStoreBytes;
                    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;\n" ::: "memory");   // slot q is free
                    __syncwarp();
                    // row `lane` of the 32 x 32 chunk: 64 bytes, 16-byte pieces in SWIZZLE_64B order
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        uint32_t h[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const int j = 8 * p + 2 * k;
                            const __half2 v = __floats2half2_rn(fmaf(gain, __uint_as_float(r[j]), gb),
                                                                fmaf(gain, __uint_as_float(r[j + 1]), gb));
                            h[k] = *reinterpret_cast<const uint32_t *>(&v);
                        }
                        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(dst + lane * 64 + ((p ^ ((lane >> 1) & 3)) << 4)),
                                     "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3]) : "memory");
                    }
                    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                    __syncwarp();
                    if (lane == 0) {
                        tma_store(&map_u, n, m0 + quarter * 32, dst);    // rows and columns past u: clipped
                        asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
                    }
                    ++stores;
                } else if (m < n_in) {
                    __half *urow = u + (int64_t)m * ldu;
#pragma unroll
                    for (int j = 0; j < kChunkCols; ++j)
                        if (n + j < batch) urow[n + j] = __float2half_rn(fmaf(gain, __uint_as_float(r[j]), gb));
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
            __syncwarp();
            if (lane == 0) arrive_remote(b ? leader_tempty1 : leader_tempty0);   // this accumulator is drained
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
    }
    __syncwarp();
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    cluster_sync();                                                      // both CTAs are done with TMEM and barriers
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// The output u: n_in rows x batch float16 columns, row stride ldu elements, boxes of 32 rows x 32 columns
// staged SWIZZLE_64B.
void encode_output(CUtensorMap *map, void *base, int64_t n_in, int64_t batch, int64_t ldu) {
    const cuuint64_t dim[2] = {(cuuint64_t)batch, (cuuint64_t)n_in};
    const cuuint64_t stride[1] = {(cuuint64_t)ldu * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kChunkCols, 32u};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult r = tc::tensor_map_encoder()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dim, stride, box, estride,
                                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                                                CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    AFB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (output) failed with code " + std::to_string((int)r));
}

}  // namespace

namespace tc {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        AFB_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        AFB_CHECK(q == cudaDriverEntryPointSuccess && fn, "cuTensorMapEncodeTiled is not available from the driver");
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    return encode;
}

void encode_operand(CUtensorMap *map, const void *base, int64_t rows, int64_t k_dim, int64_t ld, uint32_t box_rows) {
    const cuuint64_t dim[2] = {(cuuint64_t)k_dim, (cuuint64_t)rows};
    const cuuint64_t stride[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, box_rows};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dim, stride, box,
                                            estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    AFB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
}

}  // namespace tc
}  // namespace afb

using namespace afb;

extern "C" int afb_input_map_f16(int64_t n_in, int64_t batch, int64_t k_dim, const void *w, int64_t ldw, const void *x,
                                 int64_t ldx, const void *bias, float gain, void *u, int64_t ldu, int *status, void *stream) {
    return guarded([&] {
        AFB_CHECK(n_in >= 0 && batch >= 0 && k_dim >= 0, "negative size");
        AFB_CHECK(n_in < (1LL << 31) && batch < (1LL << 31) && k_dim < (1LL << 31), "size above 2^31");
        if (n_in == 0 || batch == 0) return;
        AFB_CHECK(w && x && bias && u, "NULL pointer");
        AFB_CHECK(k_dim >= 1, "k_dim must be positive");
        AFB_CHECK(ldw >= k_dim && ldx >= k_dim && ldu >= batch, "a leading dimension is below the row length");
        AFB_CHECK(ldw % 8 == 0 && ldx % 8 == 0, "W and x rows must start on 16-byte boundaries (leading dimension a multiple of 8)");
        AFB_CHECK((reinterpret_cast<uintptr_t>(w) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0,
                  "W and x must be 16-byte aligned");
        CUtensorMap map_w, map_x, map_u;
        tc::encode_operand(&map_w, w, n_in, k_dim, ldw, kHalf);
        tc::encode_operand(&map_x, x, batch, k_dim, ldx, kHalf);
        const int tma_out = (ldu % 8 == 0 && (reinterpret_cast<uintptr_t>(u) & 15) == 0) ? 1 : 0;
        if (tma_out) encode_output(&map_u, u, n_in, batch, ldu);
        else std::memset(&map_u, 0, sizeof(map_u));
        const int64_t m_tiles = (n_in + kTileRows - 1) / kTileRows, n_tiles = (batch + kTileCols - 1) / kTileCols;
        const int64_t total = m_tiles * n_tiles;
        AFB_CHECK(total < (1LL << 31), "batch too large for one launch");

        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = kSmemBytes;
        cfg.stream = (cudaStream_t)stream;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        // pairs that fit on the device at once, per device (the kernel is persistent)
        static int pairs[64] = {0};
        int dev = 0;
        AFB_CUDA(cudaGetDevice(&dev));
        AFB_CHECK(dev >= 0 && dev < 64, "device index out of range");
        if (!pairs[dev]) {
            AFB_CUDA(cudaFuncSetAttribute(input_map_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
            int sms = 0;
            AFB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
            cfg.gridDim = dim3((unsigned)sms, 1, 1);
            int n = 0;
            AFB_CUDA(cudaOccupancyMaxActiveClusters(&n, input_map_kernel, &cfg));
            AFB_CHECK(n >= 1, "no pair of CTAs of the input map fits on this device");
            pairs[dev] = n;
        }
        const int64_t clusters = total < pairs[dev] ? total : pairs[dev];
        cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
        const __half *bias_h = static_cast<const __half *>(bias);
        __half *u_h = static_cast<__half *>(u);
        AFB_CUDA(cudaLaunchKernelEx(&cfg, input_map_kernel, map_w, map_x, map_u, (int)n_in, (int)batch, (int)k_dim, bias_h,
                                    gain, u_h, ldu, tma_out, status));
    });
}
