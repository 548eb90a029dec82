// The float16 input map of the deviation path (chessfly/model.py:101-102, FlyChessNet.forward's drive):
//
//     u[i, p] = fp16( g * (sum_k W[i, k] x[p, k] + b[i]) )        i < n_in (input neurons), p < batch
//
// on the 5th-generation tensor cores.  W (n_in x k_dim) and x (batch x k_dim) are float16 and K-major
// (rows of k_dim elements, row strides multiples of 8 elements); u is written neuron-major (n_in x ldu),
// the layout the light-cone forward reads its drive in.
//
// One CTA computes a (kSub x 128) x 256 tile of u: kSub MMA tiles of 128 neurons (the 128 TMEM lanes) by
// 256 positions, their float32 accumulators side by side in TMEM (kSub x 256 columns).  Two sub-tiles
// share every x tile, which cuts the L2 -> SM bytes per FLOP by a third against one.
//   - warp 0, one lane: TMA producer.  Each k-block is a (kSub x 128) x 64 tile of W and a 256 x 64 tile
//     of x (128 bytes per row, SWIZZLE_128B), loaded by cp.async.bulk.tensor into a ring of kStages
//     stages; an mbarrier per stage counts the bytes in.  Columns past k_dim, and rows past n_in or
//     batch, are zero-filled by the TMA unit.
//   - warp 1, one lane: MMA issuer.  4 x kSub tcgen05.mma (M 128, N 256, K 16, float16 in, float32 out) per
//     k-block into TMEM; tcgen05.commit frees the stage when its MMAs have read it, and after the last
//     k-block signals the accumulator barrier.
//   - all warps: epilogue.  Warp w reads TMEM lanes 32(w%4)..32(w%4)+31 of sub-tile w/4 32 columns at a
//     time with tcgen05.ld, applies the gain and the bias in float32 and rounds once to float16.  The
//     128 x 32 chunks are staged in the (now idle) operand ring, SWIZZLE_64B, and written by TMA bulk
//     stores, so the global writes are whole lines; a u whose rows do not start on 16 bytes takes scalar
//     stores.
// Every mbarrier wait is bounded: a wait that gives up sets *status (the host reads it) and the CTA
// skips ahead instead of hanging; TMEM is always released.  No thread-block clusters: every TMA load fills
// this CTA's own shared memory.
#include <cstring>

#include "tc.cuh"

namespace afb {
namespace {

using tc::bar_init;
using tc::bar_wait;
using tc::fail;
using tc::kBK;
using tc::kMmaK;
using tc::smem_desc;
using tc::tma_load;

constexpr int kBM = 128;                        // neurons per MMA (TMEM lanes)
constexpr int kSub = 2;                         // MMA tiles per CTA along the neurons (one was measured 15% slower)
constexpr int kRows = kSub * kBM;               // neurons per CTA
constexpr int kBN = 256;                        // positions per CTA (TMEM columns per sub-tile)
// one CTA per SM with two sub-tiles (3 stages of 64 KB); with one, two CTAs per SM of 2 stages of 48 KB
constexpr int kStages = kSub == 2 ? 3 : 2;
constexpr int kThreads = 128 * kSub;            // one epilogue warp per (TMEM lane quarter, sub-tile)
constexpr int kABytes = kRows * kBK * 2;        // 16 KB per sub-tile
constexpr int kBBytes = kBN * kBK * 2;          // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /* barriers */ + 1024 /* alignment slack */;
constexpr uint32_t kTmemCols = kSub * kBN;      // float32 accumulators: one column per position and sub-tile
static_assert(kSub == 1 || kSub == 2, "one or two MMA tiles per CTA");
constexpr uint32_t kIdesc = tc::idesc_f16(kBM, kBN);

__device__ __forceinline__ void tma_store(const CUtensorMap *map, int x, int y, uint32_t src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];\n"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(src) : "memory");
}

constexpr int kChunkCols = 32;                         // one tcgen05.ld of 32 columns = one TMA store box
constexpr int kChunkBytes = kBM * kChunkCols * 2;      // 8 KB staged per chunk
static_assert(kSub * (kBN / kChunkCols) * kChunkBytes <= kStages * kStageBytes, "the staged tile must fit in the operand ring");

__global__ void __launch_bounds__(kThreads, 1) input_map_kernel(const __grid_constant__ CUtensorMap map_w,
                                                             const __grid_constant__ CUtensorMap map_x,
                                                             const __grid_constant__ CUtensorMap map_u, int n_in,
                                                             int batch, int k_dim, const __half *__restrict__ bias,
                                                             float gain, __half *__restrict__ u, int64_t ldu, int tma_out,
                                                             int *__restrict__ status) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = (uint32_t)__cvta_generic_to_shared(smem_raw);
    const uint32_t tiles = (raw + 1023u) & ~1023u;                       // stage s at +s*kStageBytes: W tile, then x tile
    const uint32_t bars = tiles + kStages * kStageBytes;                 // full[s], empty[s], acc, tmem slot
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (kStages + s); };
    const uint32_t acc_bar = bars + 16u * kStages;
    const uint32_t tmem_slot = acc_bar + 8u;
    unsigned char *const slot_ptr = smem_raw + (tmem_slot - raw);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kRows, n0 = blockIdx.y * kBN;
    const int n_kb = (k_dim + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            bar_init(full(s), 1);
            bar_init(empty(s), 1);
        }
        bar_init(acc_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&map_w)) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&map_x)) : "memory");
    }
    if (warp == 0) {                                                     // the whole warp allocates TMEM
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(tmem_slot), "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(slot_ptr);

    if (warp == 0 && lane == 0) {                                        // TMA producer
        for (int kb = 0; kb < n_kb; ++kb) {
            const int s = kb % kStages, use = kb / kStages;
            if (use > 0 && !bar_wait(empty(s), (use - 1) & 1)) {
                fail(status, 1);
                break;
            }
            const uint32_t a_dst = tiles + s * kStageBytes, b_dst = a_dst + kABytes;
            asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}\n" ::"r"(full(s)), "r"(kStageBytes)
                         : "memory");
            tma_load(a_dst, &map_w, kb * kBK, m0, full(s));
            tma_load(b_dst, &map_x, kb * kBK, n0, full(s));
        }
    } else if (warp == 1 && lane == 0) {                                 // MMA issuer
        int kb = 0;
        for (; kb < n_kb; ++kb) {
            const int s = kb % kStages;
            if (!bar_wait(full(s), (kb / kStages) & 1)) {
                fail(status, 2);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            const uint32_t a_src = tiles + s * kStageBytes, b_src = a_src + kABytes;
#pragma unroll
            for (int j = 0; j < kBK / kMmaK; ++j) {
                const uint64_t db = smem_desc(b_src + j * kMmaK * 2);
                const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
#pragma unroll
                for (int t = 0; t < kSub; ++t) {              // sub-tile t: W rows 128t.., TMEM columns 256t..
                    const uint64_t da = smem_desc(a_src + t * kBM * 128 + j * kMmaK * 2);
                    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                                 " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
                                 ::"r"(tmem + (uint32_t)(t * kBN)), "l"(da), "l"(db), "r"(kIdesc), "r"(acc) : "memory");
                }
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(empty(s)) : "memory");
        }
        // the accumulator barrier fires once every MMA issued above has completed
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(acc_bar) : "memory");
    }
    __syncwarp();

    // epilogue: every thread owns one row (neuron) of the tile
    const bool acc_ok = __syncthreads_and(bar_wait(acc_bar, 0)) != 0;   // the same answer in every thread
    if (!acc_ok && threadIdx.x == 0) fail(status, 4);
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const int quarter = warp & 3, sub = warp >> 2;
    const int row = quarter * 32 + lane, m = m0 + sub * kBM + row;   // row: TMEM lane, and row of a staged chunk
    const float gb = m < n_in ? gain * __half2float(bias[m]) : 0.f;
    __half *const urow = u + (int64_t)(m < n_in ? m : 0) * ldu;
    const bool staged = tma_out && acc_ok;                               // every MMA is done: the ring is free
#pragma unroll 1
    for (int c = 0; c < kBN / kChunkCols; ++c) {
        const int n = n0 + c * kChunkCols;
        if (n >= batch) break;                                           // uniform over the CTA
        uint32_t r[32];
        const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(sub * kBN + c * kChunkCols);
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
                     " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                       "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                       "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                       "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                     : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
        if (staged) {
            // row `row` of chunk c: 64 bytes at c*8K + row*64, its 16-byte pieces in SWIZZLE_64B order
            // (piece q at q ^ ((row >> 1) & 3), the pattern the TMA store un-swizzles)
            const uint32_t dst = tiles + (sub * (kBN / kChunkCols) + c) * kChunkBytes + row * 64;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint32_t h[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int j = 8 * q + 2 * e;
                    const __half2 v = __floats2half2_rn(fmaf(gain, __uint_as_float(r[j]), gb), fmaf(gain, __uint_as_float(r[j + 1]), gb));
                    h[e] = *reinterpret_cast<const uint32_t *>(&v);
                }
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(dst + ((q ^ ((row >> 1) & 3)) << 4)), "r"(h[0]),
                             "r"(h[1]), "r"(h[2]), "r"(h[3]) : "memory");
            }
        } else if (m < n_in && acc_ok) {
#pragma unroll
            for (int j = 0; j < kChunkCols; ++j)
                if (n + j < batch) urow[n + j] = __float2half_rn(fmaf(gain, __uint_as_float(r[j]), gb));
        }
    }
    if (staged) {
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // the staged chunks, visible to TMA
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int t = 0; t < kSub && m0 + t * kBM < n_in; ++t)
                for (int c = 0; c < kBN / kChunkCols && n0 + c * kChunkCols < batch; ++c)   // past u: clipped
                    tma_store(&map_u, n0 + c * kChunkCols, m0 + t * kBM, tiles + (t * (kBN / kChunkCols) + c) * kChunkBytes);
            asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
            asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");         // smem read before the CTA exits
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// The output u: n_in rows x batch float16 columns, row stride ldu elements, boxes of 128 rows x 32 columns
// staged SWIZZLE_64B.
void encode_output(CUtensorMap *map, void *base, int64_t n_in, int64_t batch, int64_t ldu) {
    const cuuint64_t dim[2] = {(cuuint64_t)batch, (cuuint64_t)n_in};
    const cuuint64_t stride[1] = {(cuuint64_t)ldu * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kChunkCols, (cuuint32_t)kBM};
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
        tc::encode_operand(&map_w, w, n_in, k_dim, ldw, kRows);
        tc::encode_operand(&map_x, x, batch, k_dim, ldx, kBN);
        const int tma_out = (ldu % 8 == 0 && (reinterpret_cast<uintptr_t>(u) & 15) == 0) ? 1 : 0;
        if (tma_out) encode_output(&map_u, u, n_in, batch, ldu);
        else std::memset(&map_u, 0, sizeof(map_u));
        static bool configured[64] = {false};
        int dev = 0;
        AFB_CUDA(cudaGetDevice(&dev));
        if (dev < 64 && !configured[dev]) {
            AFB_CUDA(cudaFuncSetAttribute(input_map_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
            configured[dev] = true;
        }
        const dim3 grid((unsigned)((n_in + kRows - 1) / kRows), (unsigned)((batch + kBN - 1) / kBN));
        AFB_CHECK(grid.y < 65536, "batch too large for one launch");
        input_map_kernel<<<grid, kThreads, kSmemBytes, (cudaStream_t)stream>>>(map_w, map_x, map_u, (int)n_in, (int)batch,
                                                                               (int)k_dim, static_cast<const __half *>(bias), gain,
                                                                               static_cast<__half *>(u), ldu, tma_out, status);
        AFB_LAUNCHED();
    });
}
