// Light-cone steps with short rows, float16 deviation forward, on the tensor cores.
//
// Step 2 of configuration 3 has 7.3 synapses per row (median 5).  The CUDA-core kernels spend most of
// their time there on per-row and per-synapse bookkeeping (index shuffles, row ends, the epilogue): the
// ring kernel measures 62 warp-instructions per gathered row with the issue slots 72% busy.  Here the
// sums of a unit of 128 consecutive rows over one 256-column batch tile are one tcgen05 MMA chain:
//
//     D (128 rows x 256 columns, float32 in TMEM) += A (128 rows x 64 synapses) x B (64 synapses x 256)
//
// A holds each synapse's float16 weight in its own row and zeros elsewhere (1/128 dense: the tensor
// cores do ~128x the useful multiply-adds, still well under their peak at this gather rate); B holds the
// gathered float16 state rows of the 64 synapses.  The products are exact in float32; the sums follow
// the MMA's order, so results equal the CUDA-core kernels' within float32 summation order.
//   - warps 0-3 (128 threads) produce each 64-synapse k-block of a 2-stage ring: the gathered rows by
//     cp.async into B (MN-major, SWIZZLE_128B layout written by address), the weights into A (K-major,
//     SWIZZLE_128B; a thread first clears the entry it wrote into the stage one round before).  A thread
//     waits for its copies, fences them to the async proxy and arrives on the stage's mbarrier.
//   - warp 4, one lane, issues 4 MMAs (M 128, N 256, K 16) per k-block; tcgen05.commit frees the stage,
//     and after the last k-block signals the accumulator barrier.
//   - warps 0-3 then run the epilogue: thread = row = TMEM lane; 32 columns per tcgen05.ld, the step
//     update of the CUDA-core kernels' epilogue (same float32 arithmetic, one float16 rounding), float16
//     chunks staged in the idle ring (SWIZZLE_64B) and written by TMA stores into the tile-major state.
// Every mbarrier wait is bounded and reports through the device status word; TMEM is always released.
// No cluster, no multicast.
#include <cudaTypedefs.h>

#include "internal.cuh"

namespace afb {
namespace {

constexpr int kRows = 128;                          // rows per unit = MMA M = TMEM lanes
constexpr int kCols = 256;                          // one float16 batch tile = MMA N = TMEM columns
constexpr int kKb = 64;                             // synapses per k-block
constexpr int kMmaK = 16;
#ifndef AFB_TC_STAGES
#define AFB_TC_STAGES 2
#endif
constexpr int kStg = AFB_TC_STAGES;                 // ring stages (2: two CTAs per SM; 3-4: one)
constexpr int kProd = 128;                          // producer / epilogue threads (warps 0-3)
constexpr int kThreadsTc = kProd + 32;              // + the MMA warp
constexpr int kABytesTc = kRows * kKb * 2;          // 16 KB: weights, K-major
constexpr int kBBytesTc = kKb * kCols * 2;          // 32 KB: gathered rows, MN-major
constexpr int kStageTc = kABytesTc + kBBytesTc;
constexpr int kSmemTc = kStg * kStageTc + 1024 /* barriers */ + 1024 /* alignment slack */;
constexpr uint32_t kTmemTc = kCols;
constexpr uint32_t kWaitLimitTc = 1u << 22;
constexpr int kChunkColsTc = 32;                    // one tcgen05.ld and one TMA store box of columns
constexpr int kChunkBytesTc = kRows * kChunkColsTc * 2;
static_assert(kCols / kChunkColsTc * kChunkBytesTc <= kStg * kStageTc, "the staged tile must fit in the ring");

// tcgen05.mma kind::f16 instruction descriptor: D float32 (bits 4-5 = 1), A and B float16, A K-major
// (bit 15 = 0), B MN-major (bit 16 = 1), N >> 3 in bits 17-22, M >> 4 in bits 24-28.
constexpr uint32_t kIdescTc = (1u << 4) | (1u << 16) | ((uint32_t)(kCols >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);

// Shared-memory descriptors (start >> 4 in bits 0-13, leading byte offset >> 4 in 16-29, stride byte
// offset >> 4 in 32-45, version 1 in 46-47, layout 2 = SWIZZLE_128B in 61-63).
//   A, K-major: rows of 128 bytes (64 synapses), 8-row groups 1024 bytes apart (stride offset); the
//   leading offset is unused by this layout.
//   B, MN-major: 1024-byte atoms of 8 synapses x 64 columns; the 4 column blocks are 8 KB apart (leading
//   offset), the 8 synapse groups 1 KB apart (stride offset).
__device__ __forceinline__ uint64_t desc_a(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}
__device__ __forceinline__ uint64_t desc_b(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(8192 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// byte offset of A[row][k] (K-major, SWIZZLE_128B) and of B[k][16-byte unit q] (MN-major, SWIZZLE_128B)
__device__ __forceinline__ uint32_t a_off(int row, int k) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((k >> 3) ^ (row & 7)) & 7) << 4) + (k & 7) * 2);
}
__device__ __forceinline__ uint32_t b_off(int k, int q) {
    return (uint32_t)((q >> 3) * 8192 + (k >> 3) * 1024 + (k & 7) * 128 + ((((q & 7) ^ (k & 7)) & 7) << 4));
}

__device__ __forceinline__ void tc_bar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ bool tc_bar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t it = 0; it < kWaitLimitTc; ++it) {
        uint32_t ok;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
        if (ok) return true;
    }
    return false;
}
__device__ __forceinline__ void tc_arrive(uint32_t bar) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fail(int *err, int code) {
    if (err) atomicOr(err, code);
}

__global__ void __launch_bounds__(kThreadsTc, kStg == 2 ? 2 : 1) step_kernel_tc(const __grid_constant__ CUtensorMap map_out, const StepArgs a,
                                                                int n_groups) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = (uint32_t)__cvta_generic_to_shared(smem_raw);
    const uint32_t ring = (raw + 1023u) & ~1023u;                        // stage s at +s*kStageTc: A, then B
    const uint32_t bars = ring + kStg * kStageTc;                        // full[s], empty[s], acc, tmem slot
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (kStg + s); };
    const uint32_t acc_bar = bars + 16u * kStg;
    const uint32_t tmem_slot = acc_bar + 8u;
    unsigned char *const slot_ptr = smem_raw + (tmem_slot - raw);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x / n_groups, group = blockIdx.x % n_groups;
    const int r0 = group * kRows, r1 = min(r0 + kRows, a.n_rows);
    const int e_lo = __ldg(a.crow + r0), e_hi = __ldg(a.crow + r1);
    const int n_kb = (e_hi - e_lo + kKb - 1) / kKb;
    const __half *x_tile = static_cast<const __half *>(a.x_in) + (int64_t)tile * a.ts_in;
    const __half *val = static_cast<const __half *>(a.val);

    if (tid == 0) {
        for (int s = 0; s < kStg; ++s) {
            tc_bar_init(full(s), kProd);
            tc_bar_init(empty(s), 1);
        }
        tc_bar_init(acc_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&map_out)) : "memory");
    }
    if (tid < kProd) {                                                   // the weight tiles start all zero
        for (int k = tid; k < kStg * kABytesTc / 16; k += kProd) {
            const uint32_t at = ring + (k / (kABytesTc / 16)) * kStageTc + (k % (kABytesTc / 16)) * 16;
            asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};\n" ::"r"(at), "r"(0) : "memory");
        }
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(tmem_slot), "r"(kTmemTc) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(slot_ptr);

    if (tid < kProd) {
        // ---- producers ----
        bool ok = true;
        for (int kb = 0; kb < n_kb && ok; ++kb) {
            const int s = kb % kStg, use = kb / kStg;
            if (use > 0 && !tc_bar_wait(empty(s), (use - 1) & 1)) {
                tc_fail(a.err, 1);
                ok = false;
                break;
            }
            const uint32_t a_s = ring + s * kStageTc, b_s = a_s + kABytesTc;
            const int kbase = e_lo + kb * kKb;
            if (tid < kKb) {                                             // synapse tid of the k-block
                const int e_old = kbase - kStg * kKb + tid;              // its entry of the stage's previous use
                if (use > 0 && e_old < e_hi)
                    asm volatile("st.shared.b16 [%0], %1;\n" ::"r"(a_s + a_off(__ldg(a.post + e_old) - r0, tid)),
                                 "h"((unsigned short)0) : "memory");
                const int e = kbase + tid;
                if (e < e_hi)
                    asm volatile("st.shared.b16 [%0], %1;\n" ::"r"(a_s + a_off(__ldg(a.post + e) - r0, tid)),
                                 "h"(__half_as_ushort(val[e])) : "memory");
            }
            // gathered rows: warp w copies synapses w, w + 4, ..., lane l the 16 bytes of columns 8l..8l+7
            int my_col = -1;
            if (lane < kKb / 4) {
                const int e = kbase + warp + 4 * lane;
                if (e < e_hi) my_col = __ldg(a.col + e);
            }
#pragma unroll 4
            for (int i = 0; i < kKb / 4; ++i) {
                const int c = __shfl_sync(0xffffffffu, my_col, i);
                const uint32_t dst = b_s + b_off(warp + 4 * i, lane);
                const __half *src = x_tile + (int64_t)(c >= 0 ? c : 0) * kCols + lane * 8;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(c >= 0 ? 16 : 0)
                             : "memory");                                // past the unit's synapses: zero-filled
            }
            asm volatile("cp.async.commit_group;\n" ::: "memory");
            if (kb >= kStg - 1) {                                        // the oldest k-block in flight is complete
                asm volatile("cp.async.wait_group %0;\n" ::"n"(kStg - 1) : "memory");
                asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                tc_arrive(full((kb - (kStg - 1)) % kStg));
            }
        }
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        if (ok)
            for (int kb = n_kb - (kStg - 1) > 0 ? n_kb - (kStg - 1) : 0; kb < n_kb; ++kb) tc_arrive(full(kb % kStg));
    } else if (lane == 0) {
        // ---- MMA issuer ----
        for (int kb = 0; kb < n_kb; ++kb) {
            const int s = kb % kStg;
            if (!tc_bar_wait(full(s), (kb / kStg) & 1)) {
                tc_fail(a.err, 2);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            const uint32_t a_s = ring + s * kStageTc, b_s = a_s + kABytesTc;
#pragma unroll
            for (int j = 0; j < kKb / kMmaK; ++j) {
                const uint64_t da = desc_a(a_s + j * kMmaK * 2), db = desc_b(b_s + j * (kMmaK / 8) * 1024);
                const uint32_t accumulate = (kb > 0 || j > 0) ? 1u : 0u;
                asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                             " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
                             ::"r"(tmem), "l"(da), "l"(db), "r"(kIdescTc), "r"(accumulate) : "memory");
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(empty(s)) : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(acc_bar) : "memory");
    }
    __syncwarp();

    // ---- epilogue (warps 0-3): thread = row ----
    const bool acc_ok = __syncthreads_and(tc_bar_wait(acc_bar, 0)) != 0;
    if (!acc_ok && tid == 0) tc_fail(a.err, 4);
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    if (tid < kProd) {
        const int row = tid, grow = r0 + row;
        RowConst q{};
        q.prev = -1;
        q.usrc = -1;
        if (grow < r1) q = a.rc[grow];
        const __half *u = static_cast<const __half *>(a.u) + (int64_t)(q.usrc >= 0 ? q.usrc : 0) * a.ld_u;
        const __half *pv = x_tile + (int64_t)(q.prev >= 0 ? q.prev : 0) * kCols;
#pragma unroll 1
        for (int c = 0; c < kCols / kChunkColsTc; ++c) {
            uint32_t r[32];
            const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * kChunkColsTc);
            asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
                         " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
                         : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                           "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                           "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                           "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                         : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
            const uint32_t stage_row = ring + c * kChunkBytesTc + row * 64;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const int cc = c * kChunkColsTc + g * 8;                 // column within the tile
                const int64_t col0 = (int64_t)tile * kCols + cc;
                uint4 up = make_uint4(0, 0, 0, 0), pp = make_uint4(0, 0, 0, 0);
                const bool u_vec = q.usrc >= 0 && a.u_vec_ok && col0 + 8 <= a.batch;
                if (u_vec) up = __ldg(reinterpret_cast<const uint4 *>(u + col0));
                if (q.prev >= 0) pp = __ldg(reinterpret_cast<const uint4 *>(pv + cc));
                const uint32_t ur[4] = {up.x, up.y, up.z, up.w}, pr[4] = {pp.x, pp.y, pp.z, pp.w};
                uint32_t h[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 u2 = __half22float2(*reinterpret_cast<const __half2 *>(&ur[k]));
                    const float2 p2 = __half22float2(*reinterpret_cast<const __half2 *>(&pr[k]));
                    const float uv[2] = {u2.x, u2.y}, pvv[2] = {p2.x, p2.y};
                    float o[2];
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int cj = 2 * k + j;
                        float uu = 0.f;
                        if (q.usrc >= 0) uu = u_vec ? uv[j] : (col0 + cj < a.batch ? __half2float(u[col0 + cj]) : 0.f);
                        const float acc = acc_ok && n_kb > 0 ? __uint_as_float(r[g * 8 + cj]) : 0.f;
                        const float y = acc + q.kk + uu;
                        const float x = fminf(fmaxf(y, q.lo), q.hi) + q.e;
                        const float pk = q.prev >= 0 ? pvv[j] : q.pc;
                        o[j] = pk + q.a * (x - pk);
                    }
                    const __half2 hv = __floats2half2_rn(o[0], o[1]);
                    h[k] = *reinterpret_cast<const uint32_t *>(&hv);
                }
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(stage_row + ((g ^ ((row >> 1) & 3)) << 4)),
                             "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3]) : "memory");
            }
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        asm volatile("bar.sync 1, %0;\n" ::"n"(kProd) : "memory");        // the 128 epilogue threads
        if (tid == 0 && acc_ok) {
            for (int c = 0; c < kCols / kChunkColsTc; ++c)
                asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];\n"
                             ::"l"(reinterpret_cast<uint64_t>(&map_out)), "r"(c * kChunkColsTc), "r"(r0), "r"(tile),
                             "r"(ring + c * kChunkBytesTc) : "memory");
            asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
            asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemTc) : "memory");
    }
}

PFN_cuTensorMapEncodeTiled_v12000 tc_encoder() {
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

}  // namespace

bool step_tc_eligible(const StepArgs &a) {
#ifdef AFB_NO_TC_STEP
    return false;
#else
    return a.post && a.nnz > 0 && a.n_rows > 0 && (reinterpret_cast<uintptr_t>(a.x_out) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(a.x_in) & 15) == 0;
#endif
}

void launch_step_tc(const StepArgs &a, cudaStream_t s) {
    if (a.n_rows == 0 || a.batch == 0) return;
    const int64_t tiles = (a.batch + kCols - 1) / kCols;
    const int n_groups = (a.n_rows + kRows - 1) / kRows;
    AFB_CHECK(tiles * n_groups < (1LL << 31), "grid too large: reduce the batch");
    AFB_CHECK(a.ts_out == (int64_t)a.n_rows * kCols, "the tensor-core step expects a dense tile-major state");
    // the tile-major output state as a 3-d tensor: 256 columns x n_rows rows x tiles
    CUtensorMap map;
    const cuuint64_t dim[3] = {(cuuint64_t)kCols, (cuuint64_t)a.n_rows, (cuuint64_t)tiles};
    const cuuint64_t stride[2] = {(cuuint64_t)kCols * 2, (cuuint64_t)a.ts_out * 2};
    const cuuint32_t box[3] = {(cuuint32_t)kChunkColsTc, (cuuint32_t)kRows, 1};
    const cuuint32_t estride[3] = {1, 1, 1};
    const CUresult r = tc_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, a.x_out, dim, stride, box, estride,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    AFB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (step state) failed with code " + std::to_string((int)r));
    static unsigned long long configured = 0;
    int dev = 0;
    AFB_CUDA(cudaGetDevice(&dev));
    if (dev < 64 && !(configured >> dev & 1ull)) {
        AFB_CUDA(cudaFuncSetAttribute(step_kernel_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTc));
        configured |= 1ull << dev;
    }
    step_kernel_tc<<<(unsigned)(tiles * n_groups), kThreadsTc, kSmemTc, s>>>(map, a, n_groups);
    AFB_LAUNCHED();
}

}  // namespace afb
