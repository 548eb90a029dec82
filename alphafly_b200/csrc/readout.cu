// The readout of FlyChessNet on the 5th-generation tensor cores (chessfly/model.py:103-105):
//
//     r      = clamp((out^T - mean) / sqrt(var + eps), -clip, clip)        RunningNorm, eval mode
//     logits = r Wp^T + bp + (r Wf^T + bf)[:, from] + (r Wt^T + bt)[:, to]  policy with factorised terms
//     wdl    = r Wv^T + bv                                                 value head
//
// The factorised from/to terms are linear in r, so the caller folds them into the policy rows once per
// weight version (W[m] = Wp[m] + Wf[from[m]] + Wt[to[m]], b[m] likewise) and stacks the value rows
// under them: the whole readout is then one GEMM D = W r^T + b over n_rows = n_policy + n_value rows,
// with no gather in it.
//
// float32 accuracy from float16 operands.  Both operands are split, x = hi + lo / 2^11 with hi = fp16(x)
// and lo = fp16((x - hi) 2^11) (the scaling keeps lo in float16's normal range), and two float32 TMEM
// accumulators take  D_hi = W_hi r_hi^T  and  D_lo = W_hi r_lo^T + W_lo r_hi^T;  D = D_hi + D_lo / 2^11.
// The dropped W_lo r_lo term and the roundings of the lo parts are ~2^-22 relative, so D matches a
// float32 product to ~1e-6 (the reference computes the heads in float32).
//
// Kernels.
//   readout_normalize_kernel: out (n_out, batch) float32, the light-cone forward's layout, is transposed
//     through shared memory, normalised and split into r_hi, r_lo (batch, ldn) float16, K-major.
//   readout_heads_kernel: one CTA per 128 rows x kBN positions of D.  Warp 0 lane 0 issues TMA loads of
//     the four 128-byte-swizzled operand tiles of a k-block (W_hi, W_lo, r_hi, r_lo) into a 3-stage
//     mbarrier ring; warp 1 lane 0 issues 3 tcgen05.mma (M 128, N kBN, K 16) per 16-wide k step; then all
//     four warps read their 32 TMEM lanes (rows) 32 columns (positions) at a time, add the bias and
//     write logits[p, m] (float32 or float16) or wdl[p, m - n_policy]: for a fixed position the 32 lanes
//     of a warp write 32 consecutive outputs, one coalesced line.
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
constexpr int kBM = 128;                        // rows of D per CTA (TMEM lanes)
constexpr int kBN = 128;                        // positions per CTA (TMEM columns per accumulator)
constexpr int kStages = 3;
constexpr int kThreads = 128;
constexpr int kTileBytes = kBM * kBK * 2;       // 16 KB: one 128 x 64 float16 operand tile
static_assert(kBN == kBM, "the four operand tiles of a stage share one size");
constexpr int kStageBytes = 4 * kTileBytes;     // W_hi, W_lo, r_hi, r_lo
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /* barriers */ + 1024 /* alignment slack */;
constexpr uint32_t kTmemCols = 2 * kBN;         // D_hi at column 0, D_lo at column kBN
constexpr uint32_t kIdesc = tc::idesc_f16(kBM, kBN);

constexpr int kNormTile = 64;                   // the transpose tile of the normaliser: 64 neurons x 64 positions

__global__ void __launch_bounds__(256) readout_normalize_kernel(int n_out, int batch, const float *__restrict__ r, int64_t ldr,
                                                                const float *__restrict__ mean, const float *__restrict__ var,
                                                                float eps, float clip, __half *__restrict__ r_hi,
                                                                __half *__restrict__ r_lo, int64_t ldn) {
    __shared__ float tile[kNormTile][kNormTile + 1];
    const int k0 = blockIdx.x * kNormTile, p0 = blockIdx.y * kNormTile;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // load: warp w takes neuron rows w, w + 8, ...; each lane two positions (coalesced along the batch)
    for (int kk = warp; kk < kNormTile; kk += 8) {
        const int k = k0 + kk;
        float s = 0.f, m = 0.f;
        if (k < n_out) {
            m = mean[k];
            s = sqrtf(var[k] + eps);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int pp = lane + 32 * h, p = p0 + pp;
            float x = 0.f;
            if (k < n_out && p < batch) x = fminf(fmaxf((r[(int64_t)k * ldr + p] - m) / s, -clip), clip);
            tile[kk][pp] = x;
        }
    }
    __syncthreads();
    // store: warp w takes position rows w, w + 8, ...; each lane a pair of neurons (coalesced along K)
    for (int pp = warp; pp < kNormTile; pp += 8) {
        const int p = p0 + pp;
        const int k = k0 + 2 * lane;
        if (p >= batch || k >= ldn) continue;
        const float x0 = tile[2 * lane][pp], x1 = tile[2 * lane + 1][pp];
        const __half2 hi = __floats2half2_rn(x0, x1);
        const float2 hf = __half22float2(hi);
        const __half2 lo = __floats2half2_rn((x0 - hf.x) * kLoScale, (x1 - hf.y) * kLoScale);
        *reinterpret_cast<__half2 *>(r_hi + (int64_t)p * ldn + k) = hi;
        *reinterpret_cast<__half2 *>(r_lo + (int64_t)p * ldn + k) = lo;
    }
}

__global__ void split_kernel(int64_t rows, int64_t cols, const float *__restrict__ src, int64_t ld_src, __half *__restrict__ hi,
                             __half *__restrict__ lo, int64_t ld_dst) {
    const int64_t total = rows * ld_dst;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / ld_dst, col = i % ld_dst;
        const float x = col < cols ? src[row * ld_src + col] : 0.f;
        const __half h = __float2half_rn(x);
        hi[i] = h;
        lo[i] = __float2half_rn((x - __half2float(h)) * kLoScale);
    }
}

__global__ void __launch_bounds__(kThreads, 1) readout_heads_kernel(const __grid_constant__ CUtensorMap map_w_hi,
                                                                    const __grid_constant__ CUtensorMap map_w_lo,
                                                                    const __grid_constant__ CUtensorMap map_r_hi,
                                                                    const __grid_constant__ CUtensorMap map_r_lo, int n_rows,
                                                                    int n_policy, int batch, int k_dim,
                                                                    const float *__restrict__ bias, void *__restrict__ logits,
                                                                    int64_t ld_logits, int logits_f16, float *__restrict__ values,
                                                                    int64_t ld_values, int *__restrict__ status) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = (uint32_t)__cvta_generic_to_shared(smem_raw);
    const uint32_t tiles = (raw + 1023u) & ~1023u;                       // stage s: W_hi, W_lo, r_hi, r_lo tiles
    const uint32_t bars = tiles + kStages * kStageBytes;                 // full[s], empty[s], acc, tmem slot
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (kStages + s); };
    const uint32_t acc_bar = bars + 16u * kStages;
    const uint32_t tmem_slot = acc_bar + 8u;
    unsigned char *const slot_ptr = smem_raw + (tmem_slot - raw);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * kBN;
    const int n_kb = (k_dim + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            bar_init(full(s), 1);
            bar_init(empty(s), 1);
        }
        bar_init(acc_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&map_w_hi)) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&map_w_lo)) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&map_r_hi)) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&map_r_lo)) : "memory");
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
            tma_load(dst, &map_w_hi, kb * kBK, m0, full(s));
            tma_load(dst + kTileBytes, &map_w_lo, kb * kBK, m0, full(s));
            tma_load(dst + 2 * kTileBytes, &map_r_hi, kb * kBK, n0, full(s));
            tma_load(dst + 3 * kTileBytes, &map_r_lo, kb * kBK, n0, full(s));
        }
    } else if (warp == 1 && lane == 0) {                                 // MMA issuer
        for (int kb = 0; kb < n_kb; ++kb) {
            const int s = kb % kStages;
            if (!bar_wait(full(s), (kb / kStages) & 1)) {
                fail(status, 2);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            const uint32_t w_hi = tiles + s * kStageBytes, w_lo = w_hi + kTileBytes, r_hi = w_hi + 2 * kTileBytes,
                           r_lo = w_hi + 3 * kTileBytes;
            // the last k block takes only the 16-wide steps that hold data; the others would multiply zero fill
            const int nj = min(kBK / kMmaK, (k_dim - kb * kBK + kMmaK - 1) / kMmaK);
#pragma unroll
            for (int j = 0; j < kBK / kMmaK; ++j) {
                if (j >= nj) break;
                const uint32_t off = j * kMmaK * 2;
                const uint32_t first = (kb > 0 || j > 0) ? 1u : 0u;
                tc::mma_f16(tmem, smem_desc(w_hi + off), smem_desc(r_hi + off), kIdesc, first);
                tc::mma_f16(tmem + kBN, smem_desc(w_hi + off), smem_desc(r_lo + off), kIdesc, first);
                tc::mma_f16(tmem + kBN, smem_desc(w_lo + off), smem_desc(r_hi + off), kIdesc, 1u);
            }
            tc::mma_commit(empty(s));                                    // the stage is free once these MMAs read it
        }
        tc::mma_commit(acc_bar);                                         // every MMA issued above has completed
    }
    __syncwarp();

    // epilogue: thread t owns row m0 + t of D (TMEM lane t)
    const bool acc_ok = __syncthreads_and(bar_wait(acc_bar, 0)) != 0;   // the same answer in every thread
    if (!acc_ok && threadIdx.x == 0) fail(status, 4);
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const int m = m0 + warp * 32 + lane;
    const float b = m < n_rows ? bias[m] : 0.f;
#pragma unroll 1
    for (int c = 0; c < kBN / 32 && acc_ok; ++c) {
        const int p0 = n0 + c * 32;
        if (p0 >= batch) break;                                          // uniform over the CTA
        uint32_t hi[32], lo[32];
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 32);
        tc::tmem_ld32(taddr, hi);
        tc::tmem_ld32(taddr + kBN, lo);
        tc::tmem_wait_ld();
        if (m >= n_rows) continue;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int p = p0 + j;
            if (p >= batch) break;
            const float v = __uint_as_float(hi[j]) + __uint_as_float(lo[j]) * (1.f / kLoScale) + b;
            if (m < n_policy) {
                if (logits_f16) static_cast<__half *>(logits)[(int64_t)p * ld_logits + m] = __float2half_rn(v);
                else static_cast<float *>(logits)[(int64_t)p * ld_logits + m] = v;
            } else {
                values[(int64_t)p * ld_values + (m - n_policy)] = v;
            }
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

}  // namespace
}  // namespace afb

using namespace afb;

extern "C" {

int afb_heads_split(int64_t rows, int64_t cols, const float *src, int64_t ld_src, void *hi, void *lo, int64_t ld_dst,
                    void *stream) {
    return guarded([&] {
        AFB_CHECK(rows >= 0 && cols >= 0, "negative size");
        if (rows == 0) return;
        AFB_CHECK(src && hi && lo, "NULL pointer");
        AFB_CHECK(ld_src >= cols && ld_dst >= cols, "a leading dimension is below the row length");
        split_kernel<<<grid_for(rows * ld_dst, 256), 256, 0, as_stream(stream)>>>(rows, cols, src, ld_src, static_cast<__half *>(hi),
                                                                                  static_cast<__half *>(lo), ld_dst);
        AFB_LAUNCHED();
    });
}

size_t afb_readout_workspace(int64_t batch, int64_t n_out) {
    if (batch <= 0 || n_out <= 0) return 0;
    return (size_t)(2 * batch * round8(n_out) * 2 + 256);
}

int afb_readout_heads(int64_t n_out, int64_t batch, const float *r, int64_t ld_r, const float *mean, const float *var,
                      float eps, float clip, int64_t n_rows, int64_t n_policy, const void *w_hi, const void *w_lo, int64_t ldw,
                      const float *bias, void *logits, int64_t ld_logits, int logits_f16, float *values, int64_t ld_values,
                      void *workspace, size_t workspace_bytes, int *status, void *stream) {
    return guarded([&] {
        AFB_CHECK(n_out >= 1 && batch >= 0 && n_rows >= 1 && n_policy >= 0 && n_policy <= n_rows, "bad sizes");
        AFB_CHECK(n_out < (1LL << 31) && batch < (1LL << 31) && n_rows < (1LL << 31), "size above 2^31");
        if (batch == 0) return;
        AFB_CHECK(r && mean && var && w_hi && w_lo && bias && workspace, "NULL pointer");
        AFB_CHECK(n_policy == 0 || logits, "logits is NULL");
        AFB_CHECK(n_policy == n_rows || values, "values is NULL");
        AFB_CHECK(ld_r >= batch && (n_policy == 0 || ld_logits >= n_policy) && (n_policy == n_rows || ld_values >= n_rows - n_policy),
                  "a leading dimension is below the row length");
        AFB_CHECK(ldw >= n_out && ldw % 8 == 0, "ldw must be >= n_out and a multiple of 8 (16-byte rows for TMA)");
        AFB_CHECK((reinterpret_cast<uintptr_t>(w_hi) & 15) == 0 && (reinterpret_cast<uintptr_t>(w_lo) & 15) == 0,
                  "w_hi and w_lo must be 16-byte aligned");
        AFB_CHECK(workspace_bytes >= afb_readout_workspace(batch, n_out), "workspace too small (afb_readout_workspace)");
        const cudaStream_t s = as_stream(stream);
        const int64_t ldn = round8(n_out);
        auto base = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255);
        __half *r_hi = reinterpret_cast<__half *>(base);
        __half *r_lo = r_hi + batch * ldn;
        const dim3 ngrid((unsigned)((ldn + kNormTile - 1) / kNormTile), (unsigned)((batch + kNormTile - 1) / kNormTile));
        AFB_CHECK(ngrid.y < 65536, "batch too large for one launch");
        readout_normalize_kernel<<<ngrid, 256, 0, s>>>((int)n_out, (int)batch, r, ld_r, mean, var, eps, clip, r_hi, r_lo, ldn);
        AFB_LAUNCHED();
        CUtensorMap mw_hi, mw_lo, mr_hi, mr_lo;
        tc::encode_operand(&mw_hi, w_hi, n_rows, n_out, ldw, kBM);
        tc::encode_operand(&mw_lo, w_lo, n_rows, n_out, ldw, kBM);
        tc::encode_operand(&mr_hi, r_hi, batch, n_out, ldn, kBN);
        tc::encode_operand(&mr_lo, r_lo, batch, n_out, ldn, kBN);
        static bool configured[64] = {false};
        int dev = 0;
        AFB_CUDA(cudaGetDevice(&dev));
        if (dev < 64 && !configured[dev]) {
            AFB_CUDA(cudaFuncSetAttribute(readout_heads_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
            configured[dev] = true;
        }
        const dim3 grid((unsigned)((n_rows + kBM - 1) / kBM), (unsigned)((batch + kBN - 1) / kBN));
        AFB_CHECK(grid.y < 65536, "batch too large for one launch");
        readout_heads_kernel<<<grid, kThreads, kSmemBytes, s>>>(mw_hi, mw_lo, mr_hi, mr_lo, (int)n_rows, (int)n_policy,
                                                                 (int)batch, (int)n_out, bias, logits, ld_logits, logits_f16,
                                                                 values, ld_values, status);
        AFB_LAUNCHED();
    });
}

}  // extern "C"
