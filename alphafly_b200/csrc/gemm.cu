// Float32 GEMMs of the training path on the 5th-generation tensor cores.
//
// FlyChessNet trains its encoder and heads as float32 layers (chessfly/model.py:95-105, nn.Linear in the
// reference's train_step, chessfly/train.py:126-138); cuBLAS runs those products as float32 SIMT GEMMs.
// afb_gemm_f32 computes
//
//     R (P x Q, row-major) = alpha X Y^T + beta bias          X (P x K), Y (Q x K), bias per row or column
//
// at float32 accuracy from float16 tensor-core products, the readout kernel's scheme (readout.cu) made
// general: each operand is scaled by a power of two s chosen from its largest magnitude (so that
// max |x s| lies in [2^14, 2^15), inside float16's range) and split into hi = fp16(x s) and
// lo = fp16((x s - hi) 2^11); two float32 TMEM accumulators take D_hi = Y_hi X_hi^T and
// D_lo = Y_hi X_lo^T + Y_lo X_hi^T, and R = alpha (D_hi + D_lo / 2^11) / (s_X s_Y) + beta bias.  The dropped
// lo lo term and the roundings of the lo parts are ~2^-22 of the largest products.
//
// Kernels (all on the caller's stream):
//   amax_kernel      max |S| of each operand (atomicMax on the float's bits, which order like the values)
//   split_kernel     the scaled hi / lo float16 operand, K-major with rows padded to 16 bytes; an operand
//                    given transposed (element (p, k) at S[k ld + p]) goes through a 64 x 64 shared tile
//   gemm_kernel      one CTA per 128 (Q) x 128 (P) tile of R: warp 0 lane 0 streams the four operand tiles
//                    of each 64-wide k block by TMA into a 3-stage mbarrier ring, warp 1 lane 0 issues 3
//                    tcgen05.mma (M 128, N 128, K 16) per 16-wide k step, then the four warps read their
//                    32 TMEM lanes (Q) 32 columns (P) at a time: for one p the 32 lanes of a warp write 32
//                    consecutive q of R, one coalesced line.
// Every mbarrier wait is bounded and reports through a device status word; TMEM is always released.
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

constexpr float kLoScale = 2048.f;              // lo parts are stored times 2^11
constexpr int kBM = 128;                        // Q per CTA (TMEM lanes)
constexpr int kBN = 128;                        // P per CTA (TMEM columns per accumulator)
constexpr int kStages = 3;
constexpr int kThreads = 128;
constexpr int kTileBytes = kBM * kBK * 2;       // 16 KB: one 128 x 64 float16 operand tile
static_assert(kBN == kBM, "the four operand tiles of a stage share one size");
constexpr int kStageBytes = 4 * kTileBytes;     // Y_hi, Y_lo, X_hi, X_lo
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /* barriers */ + 1024 /* alignment slack */;
constexpr uint32_t kTmemCols = 2 * kBN;         // D_hi at column 0, D_lo at column kBN
constexpr uint32_t kIdesc = tc::idesc_f16(kBM, kBN);
constexpr int kT = 64;                          // transpose tile of split_kernel
constexpr int kScaleTop = 14;                   // max |x s| in [2^14, 2^15)
constexpr int kScaleLimit = 100;                // |log2 s| at most this: s and 1 / s are normal floats

// Largest |S| over a rows x cols operand (row stride ld) into *amax (the float's bits).
__global__ void amax_kernel(const float *__restrict__ src, int64_t rows, int64_t cols, int64_t ld, unsigned *__restrict__ amax) {
    const int lane = threadIdx.x & 31;
    float m = 0.f;
    for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += ((int64_t)gridDim.x * blockDim.x) >> 5)
        for (int64_t c = lane; c < cols; c += 32) m = fmaxf(m, fabsf(src[r * ld + c]));
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0 && m > 0.f) atomicMax(amax, __float_as_uint(m));
}

// 2^n as a float, n in [-126, 127].
__device__ __forceinline__ float pow2(int n) { return __int_as_float((n + 127) << 23); }

// log2 of the operand scale for a largest magnitude with bits `a` (0 when it is 0 or not finite).
__device__ __forceinline__ int scale_log2(unsigned a) {
    const int biased = (int)((a >> 23) & 0xFF);
    if (a == 0u || biased == 0xFF) return 0;
    const int e = biased == 0 ? -127 : biased - 127;          // floor(log2 |x|) for normal |x|
    const int n = kScaleTop - e;
    return n > kScaleLimit ? kScaleLimit : (n < -kScaleLimit ? -kScaleLimit : n);
}

__device__ __forceinline__ void split_store(float x, float s, __half *hi, __half *lo) {
    const float xs = x * s;                                   // exact: s is a power of two
    const __half h = __float2half_rn(xs);
    *hi = h;
    *lo = __float2half_rn((xs - __half2float(h)) * kLoScale);
}

// dst (rows x ldd, K-major, zero past k_dim) = split(S s).  TRANS = 0: element (p, k) at src[p ld + k];
// TRANS = 1: at src[k ld + p].  Block (x, y) covers rows [64 x, 64 x + 64) and k [64 y, 64 y + 64).
template <int TRANS>
__global__ void __launch_bounds__(256) split_kernel(const float *__restrict__ src, int64_t rows, int64_t k_dim, int64_t ld,
                                                    const unsigned *__restrict__ amax, __half *__restrict__ hi,
                                                    __half *__restrict__ lo, int64_t ldd, float *__restrict__ inv_scale) {
    __shared__ float tile[kT][kT + 1];
    const int n = scale_log2(*amax);
    const float s = pow2(n);
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *inv_scale = pow2(-n);
    const int64_t p0 = (int64_t)blockIdx.x * kT, k0 = (int64_t)blockIdx.y * kT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (TRANS) {
        // load along p (contiguous in the source), store along k
        for (int kk = warp; kk < kT; kk += 8) {
            const int64_t k = k0 + kk;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int64_t p = p0 + lane + 32 * h;
                tile[lane + 32 * h][kk] = (k < k_dim && p < rows) ? src[k * ld + p] : 0.f;
            }
        }
        __syncthreads();
    }
    for (int pp = warp; pp < kT; pp += 8) {
        const int64_t p = p0 + pp;
        if (p >= rows) break;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int64_t k = k0 + lane + 32 * h;
            if (k >= ldd) continue;
            const float x = TRANS ? tile[pp][lane + 32 * h] : (k < k_dim ? src[p * ld + k] : 0.f);
            split_store(x, s, hi + p * ldd + k, lo + p * ldd + k);
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap map_y_hi,
                                                           const __grid_constant__ CUtensorMap map_y_lo,
                                                           const __grid_constant__ CUtensorMap map_x_hi,
                                                           const __grid_constant__ CUtensorMap map_x_lo, int p_dim, int q_dim,
                                                           int k_dim, float alpha, const float *__restrict__ inv_scales,
                                                           const float *__restrict__ bias, int bias_dim, float beta,
                                                           float *__restrict__ r, int64_t ld_r, int *__restrict__ status) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = (uint32_t)__cvta_generic_to_shared(smem_raw);
    const uint32_t tiles = (raw + 1023u) & ~1023u;                       // stage s: Y_hi, Y_lo, X_hi, X_lo tiles
    const uint32_t bars = tiles + kStages * kStageBytes;                 // full[s], empty[s], acc, tmem slot
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (kStages + s); };
    const uint32_t acc_bar = bars + 16u * kStages;
    const uint32_t tmem_slot = acc_bar + 8u;
    unsigned char *const slot_ptr = smem_raw + (tmem_slot - raw);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * kBM, p0 = blockIdx.y * kBN;
    const int n_kb = (k_dim + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            bar_init(full(s), 1);
            bar_init(empty(s), 1);
        }
        bar_init(acc_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&map_y_hi)) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&map_y_lo)) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&map_x_hi)) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&map_x_lo)) : "memory");
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
            const uint32_t dst = tiles + s * kStageBytes;
            tc::bar_expect_tx(full(s), kStageBytes);
            tma_load(dst, &map_y_hi, kb * kBK, q0, full(s));
            tma_load(dst + kTileBytes, &map_y_lo, kb * kBK, q0, full(s));
            tma_load(dst + 2 * kTileBytes, &map_x_hi, kb * kBK, p0, full(s));
            tma_load(dst + 3 * kTileBytes, &map_x_lo, kb * kBK, p0, full(s));
        }
    } else if (warp == 1 && lane == 0) {                                 // MMA issuer
        for (int kb = 0; kb < n_kb; ++kb) {
            const int s = kb % kStages;
            if (!bar_wait(full(s), (kb / kStages) & 1)) {
                fail(status, 2);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            const uint32_t y_hi = tiles + s * kStageBytes, y_lo = y_hi + kTileBytes, x_hi = y_hi + 2 * kTileBytes,
                           x_lo = y_hi + 3 * kTileBytes;
            // the last k block takes only the 16-wide steps that hold data; the others would multiply zero fill
            const int nj = min(kBK / kMmaK, (k_dim - kb * kBK + kMmaK - 1) / kMmaK);
#pragma unroll
            for (int j = 0; j < kBK / kMmaK; ++j) {
                if (j >= nj) break;
                const uint32_t off = j * kMmaK * 2;
                const uint32_t first = (kb > 0 || j > 0) ? 1u : 0u;
                tc::mma_f16(tmem, smem_desc(y_hi + off), smem_desc(x_hi + off), kIdesc, first);
                tc::mma_f16(tmem + kBN, smem_desc(y_hi + off), smem_desc(x_lo + off), kIdesc, first);
                tc::mma_f16(tmem + kBN, smem_desc(y_lo + off), smem_desc(x_hi + off), kIdesc, 1u);
            }
            tc::mma_commit(empty(s));                                    // the stage is free once these MMAs read it
        }
        tc::mma_commit(acc_bar);                                         // every MMA issued above has completed
    }
    __syncwarp();

    // epilogue: thread t owns q = q0 + t (TMEM lane t)
    const bool acc_ok = __syncthreads_and(bar_wait(acc_bar, 0)) != 0;   // the same answer in every thread
    if (!acc_ok && threadIdx.x == 0) fail(status, 4);
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const int q = q0 + warp * 32 + lane;
    const float f_x = inv_scales[0], f_y = alpha * inv_scales[1];   // alpha / (s_X s_Y), applied in two steps
    const float bq = (bias_dim == 2 && q < q_dim) ? beta * bias[q] : 0.f;
#pragma unroll 1
    for (int c = 0; c < kBN / 32 && acc_ok; ++c) {
        const int pc = p0 + c * 32;
        if (pc >= p_dim) break;                                          // uniform over the CTA
        uint32_t hi[32], lo[32];
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 32);
        tc::tmem_ld32(taddr, hi);
        tc::tmem_ld32(taddr + kBN, lo);
        tc::tmem_wait_ld();
        if (q >= q_dim) continue;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int p = pc + j;
            if (p >= p_dim) break;
            const float d = __uint_as_float(hi[j]) + __uint_as_float(lo[j]) * (1.f / kLoScale);
            const float b = bias_dim == 1 ? beta * __ldg(bias + p) : bq;
            r[(int64_t)p * ld_r + q] = (d * f_x) * f_y + b;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

int64_t round8(int64_t x) { return (x + 7) / 8 * 8; }
size_t align256(size_t b) { return (b + 255) / 256 * 256; }

// Split one operand into its scaled float16 hi / lo pair (rows x ldd, K-major).
void split_operand(const float *src, int64_t rows, int64_t k_dim, int64_t ld, int trans, unsigned *amax, __half *hi,
                   __half *lo, int64_t ldd, float *inv_scale, cudaStream_t s) {
    const int64_t src_rows = trans ? k_dim : rows, src_cols = trans ? rows : k_dim;
    amax_kernel<<<grid_for(src_rows * 32, 256, 148 * 16), 256, 0, s>>>(src, src_rows, src_cols, ld, amax);
    const dim3 grid((unsigned)((rows + kT - 1) / kT), (unsigned)((ldd + kT - 1) / kT));
    if (trans) split_kernel<1><<<grid, 256, 0, s>>>(src, rows, k_dim, ld, amax, hi, lo, ldd, inv_scale);
    else split_kernel<0><<<grid, 256, 0, s>>>(src, rows, k_dim, ld, amax, hi, lo, ldd, inv_scale);
    AFB_LAUNCHED();
}

}  // namespace
}  // namespace afb

using namespace afb;

extern "C" {

size_t afb_gemm_workspace(int64_t p, int64_t q, int64_t k) {
    if (p <= 0 || q <= 0 || k <= 0) return 0;
    const int64_t ldk = round8(k);
    return 4 * align256((size_t)std::max(p, q) * ldk * 2) + 256 + 256;
}

int afb_gemm_f32(int64_t p, int64_t q, int64_t k, float alpha, const float *x, int64_t ld_x, int x_trans, const float *y,
                 int64_t ld_y, int y_trans, const float *bias, int bias_dim, float beta, float *r, int64_t ld_r,
                 void *workspace, size_t workspace_bytes, int *status, void *stream) {
    return guarded([&] {
        AFB_CHECK(p >= 0 && q >= 0 && k >= 0, "negative size");
        AFB_CHECK(p < (1LL << 31) && q < (1LL << 31) && k < (1LL << 31), "size above 2^31");
        AFB_CHECK(bias_dim >= 0 && bias_dim <= 2, "bias_dim must be 0 (none), 1 (per row of R) or 2 (per column)");
        if (p == 0 || q == 0) return;
        AFB_CHECK(r && (bias_dim == 0 || bias), "NULL pointer");
        AFB_CHECK(ld_r >= q, "ld_r is below the row length");
        const cudaStream_t s = as_stream(stream);
        if (k == 0) {                                                // R = beta bias (or 0)
            AFB_CHECK(bias_dim == 0, "k = 0 with a bias: add the bias on the caller's side");
            AFB_CUDA(cudaMemset2DAsync(r, (size_t)ld_r * 4, 0, (size_t)q * 4, (size_t)p, s));
            return;
        }
        AFB_CHECK(x && y && workspace, "NULL pointer");
        AFB_CHECK(ld_x >= (x_trans ? p : k) && ld_y >= (y_trans ? q : k), "a leading dimension is below the row length");
        AFB_CHECK(workspace_bytes >= afb_gemm_workspace(p, q, k), "workspace too small (afb_gemm_workspace)");
        const int64_t ldk = round8(k);
        AFB_CHECK((ldk + kT - 1) / kT < 65536, "k too large for one launch");
        const size_t part = align256((size_t)std::max(p, q) * ldk * 2);
        char *ws = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
        __half *x_hi = reinterpret_cast<__half *>(ws), *x_lo = reinterpret_cast<__half *>(ws + part);
        __half *y_hi = reinterpret_cast<__half *>(ws + 2 * part), *y_lo = reinterpret_cast<__half *>(ws + 3 * part);
        unsigned *amax = reinterpret_cast<unsigned *>(ws + 4 * part);          // [x, y]
        float *inv_scales = reinterpret_cast<float *>(ws + 4 * part + 8);      // [x, y]
        AFB_CUDA(cudaMemsetAsync(amax, 0, 8, s));
        split_operand(x, p, k, ld_x, x_trans, amax, x_hi, x_lo, ldk, inv_scales, s);
        split_operand(y, q, k, ld_y, y_trans, amax + 1, y_hi, y_lo, ldk, inv_scales + 1, s);
        CUtensorMap my_hi, my_lo, mx_hi, mx_lo;
        tc::encode_operand(&my_hi, y_hi, q, k, ldk, kBM);
        tc::encode_operand(&my_lo, y_lo, q, k, ldk, kBM);
        tc::encode_operand(&mx_hi, x_hi, p, k, ldk, kBN);
        tc::encode_operand(&mx_lo, x_lo, p, k, ldk, kBN);
        static bool configured[64] = {false};
        int dev = 0;
        AFB_CUDA(cudaGetDevice(&dev));
        if (dev < 64 && !configured[dev]) {
            AFB_CUDA(cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
            configured[dev] = true;
        }
        const dim3 grid((unsigned)((q + kBM - 1) / kBM), (unsigned)((p + kBN - 1) / kBN));
        AFB_CHECK(grid.y < 65536, "p too large for one launch");
        gemm_kernel<<<grid, kThreads, kSmemBytes, s>>>(my_hi, my_lo, mx_hi, mx_lo, (int)p, (int)q, (int)k, alpha, inv_scales,
                                                        bias, bias_dim, beta, r, ld_r, status);
        AFB_LAUNCHED();
    });
}

}  // extern "C"
