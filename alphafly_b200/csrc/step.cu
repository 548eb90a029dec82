// The fused light-cone step: one CSR SpMM over a batch tile with the whole state update in its
// epilogue (chessfly/brain.py:273-277 float16 deviation, brain.py:310-314 float32).
//
// Layout.  State and drive are (rows, batch) row-major; a CTA owns one batch tile of kLanesPerEdge
// lanes x 16 bytes (with 16 lanes: 128 half or 64 float columns) and one "item" -- a contiguous run of
// rows whose cost (edges + 4 per row) is about kItemCost.  blockIdx.x = tile * n_items + k, so all items of a
// tile run before the next tile starts: the gathered slab R_{t-1} x tile stays resident in L2.
//
// Load balance.  Inside a CTA the item's rows and edges are split evenly over the 8 warps by the
// merge-path partition of Merrill & Garland ("Merge-based parallel sparse matrix-vector
// multiplication", SC'16): the merge of row ends with edge indices is cut into equal diagonals, so a
// 5,000-synapse row and 60 short rows cost the same.  A row cut by warp boundaries leaves one partial
// per warp in shared memory; after a barrier one warp sums them in warp order and finishes the row,
// so results are bitwise reproducible and independent of the batch width.
//
// Gather.  kLanesPerEdge lanes cover the tile with one 16-byte load each per edge; the 32 / kLanesPerEdge
// lane groups of a warp take interleaved edges of the same row and are summed with xor-shuffles at the
// row end.  Column indices and values are loaded 32 edges at a time, coalesced, and broadcast with
// shuffles.
// Accumulation is float32 in every mode.
#include <cudaTypedefs.h>

#include "internal.cuh"

namespace afb {
namespace {

#ifndef AFB_WARPS
#define AFB_WARPS 8
#endif
#ifndef AFB_UNROLL
#define AFB_UNROLL 4
#endif
#ifndef AFB_MINBLOCKS
#define AFB_MINBLOCKS 1
#endif
constexpr int kWarps = AFB_WARPS;              // warps per CTA
constexpr int kLanesPerEdge = AFB_LPE;         // lanes that cover one gathered row tile (16 bytes each)
constexpr int kGroups = 32 / kLanesPerEdge;    // edges a warp gathers side by side
constexpr int kUnroll = AFB_UNROLL;            // gathers in flight per lane
constexpr unsigned kFull = 0xffffffffu;
static_assert(kLanesPerEdge == 8 || kLanesPerEdge == 16 || kLanesPerEdge == 32, "lanes per edge");

template <typename T>
struct Lane;  // 16 bytes of state per lane

template <>
struct Lane<float> {
    static constexpr int V = 4;
    __device__ static void load(const float *p, float (&x)[V]) {
        float4 v = __ldg(reinterpret_cast<const float4 *>(p));
        x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
    }
    __device__ static void store(float *p, const float (&x)[V]) {
        *reinterpret_cast<float4 *>(p) = make_float4(x[0], x[1], x[2], x[3]);
    }
    __device__ static float scalar(const float *p) { return __ldg(p); }
};

template <>
struct Lane<__half> {
    static constexpr int V = 8;
    __device__ static void load(const __half *p, float (&x)[V]) {
        uint4 v = __ldg(reinterpret_cast<const uint4 *>(p));
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float2 f = __half22float2(h[k]);
            x[2 * k] = f.x;
            x[2 * k + 1] = f.y;
        }
    }
    __device__ static void store(__half *p, const float (&x)[V]) {
        uint4 v;
        __half2 *h = reinterpret_cast<__half2 *>(&v);
#pragma unroll
        for (int k = 0; k < 4; ++k) h[k] = __floats2half2_rn(x[2 * k], x[2 * k + 1]);
        *reinterpret_cast<uint4 *>(p) = v;
    }
    __device__ static float scalar(const __half *p) { return __half2float(p[0]); }
};

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

// Finish one row: epilogue of the state update, writes V columns of this lane.
// State buffers are tile-major: element (row, column c) of a step's state lives at
// tile * ts + row * BT + (c % BT) with tile = c / BT, so one tile's slab is contiguous.
template <typename T, int BT>
__device__ __forceinline__ void finish_row(const StepArgs &a, int row, int64_t tile, int off, float (&acc)[Lane<T>::V]) {
    constexpr int V = Lane<T>::V;
    const int64_t col0 = tile * BT + off;          // batch column of this lane's first element
    const int4 w0 = __ldg(reinterpret_cast<const int4 *>(a.rc + row));
    const int4 w1 = __ldg(reinterpret_cast<const int4 *>(a.rc + row) + 1);
    const float kk = __int_as_float(w0.x), lo = __int_as_float(w0.y), hi = __int_as_float(w0.z), e = __int_as_float(w0.w);
    const float pc = __int_as_float(w1.x), al = __int_as_float(w1.y);
    const int prev = w1.z, usrc = w1.w;
    float y[V];
#pragma unroll
    for (int k = 0; k < V; ++k) y[k] = acc[k] + kk;
    if (usrc >= 0) {
        const T *u = static_cast<const T *>(a.u) + (int64_t)usrc * a.ld_u + col0;
        if (a.u_vec_ok && col0 + V <= a.batch) {
            float x[V];
            Lane<T>::load(u, x);
#pragma unroll
            for (int k = 0; k < V; ++k) y[k] += x[k];
        } else {
#pragma unroll
            for (int k = 0; k < V; ++k)
                if (col0 + k < a.batch) y[k] += Lane<T>::scalar(u + k);
        }
    }
    float p[V];
    if (prev >= 0) {
        Lane<T>::load(static_cast<const T *>(a.x_in) + tile * a.ts_in + (int64_t)prev * BT + off, p);
    } else {
#pragma unroll
        for (int k = 0; k < V; ++k) p[k] = pc;
    }
    float o[V];
#pragma unroll
    for (int k = 0; k < V; ++k) {
        const float x = fminf(fmaxf(y[k], lo), hi) + e;
        o[k] = p[k] + al * (x - p[k]);
    }
    Lane<T>::store(static_cast<T *>(a.x_out) + tile * a.ts_out + (int64_t)row * BT + off, o);
    if constexpr (sizeof(T) == 4)
        if (a.y_out) Lane<float>::store(a.y_out + tile * a.ts_out + (int64_t)row * BT + off, y);
}

template <typename T, typename TV>
__global__ void __launch_bounds__(kWarps * 32, AFB_MINBLOCKS) step_kernel(const StepArgs a) {
    using L = Lane<T>;
    constexpr int V = L::V;
    constexpr int BT = kLanesPerEdge * V;
    __shared__ float s_first[kWarps][BT], s_last[kWarps][BT];   // partials of rows cut by warp boundaries
    __shared__ int s_bi[kWarps + 1], s_bj[kWarps + 1];

    const int item = __ldg(a.item_order + (blockIdx.x % a.n_items));
    const int64_t tile = blockIdx.x / a.n_items;
    const int r0 = __ldg(a.item_rows + item), r1 = __ldg(a.item_rows + item + 1);
    const int e0 = __ldg(a.crow + r0);
    const int nrows = r1 - r0, nnz = __ldg(a.crow + r1) - e0;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = lane / kLanesPerEdge, sub = lane % kLanesPerEdge;
    const int off = sub * V;
    const T *x_tile = static_cast<const T *>(a.x_in) + tile * a.ts_in + off;

    if (tid <= kWarps) {  // merge-path coordinates of the warp boundaries (precomputed per item)
        const int2 bd = __ldg(a.bounds + item * (kWarps + 1) + tid);
        s_bi[tid] = bd.x;
        s_bj[tid] = bd.y;
    }
    for (int k = tid; k < kWarps * BT; k += kWarps * 32) (&s_first[0][0])[k] = (&s_last[0][0])[k] = 0.f;
    __syncthreads();

    // a boundary b (1..W-1) cuts a row if that row started before it
    auto cut = [&](int b) -> bool {
        return b >= 1 && b < kWarps && s_bj[b] > __ldg(a.crow + r0 + s_bi[b]) - e0;
    };
    auto first_cut = [&](int b) -> int {  // the first boundary cutting the row cut by b
        while (b > 1 && s_bi[b - 1] == s_bi[b] && cut(b - 1)) --b;
        return b;
    };

    const TV *val = static_cast<const TV *>(a.val);
    const int is = s_bi[warp], js = s_bj[warp], ie = s_bi[warp + 1], je = s_bj[warp + 1];
    const bool cut_lo = cut(warp), cut_hi = cut(warp + 1);
    for (int i = is; i <= ie && i < nrows; ++i) {
        const int rs = __ldg(a.crow + r0 + i) - e0, re = __ldg(a.crow + r0 + i + 1) - e0;
        const int eb = rs > js ? rs : js;
        const int ee = re < je ? re : je;
        if (i == ie && ee <= eb) break;  // the next warp's row, no edges of it here
        float acc[V];
#pragma unroll
        for (int k = 0; k < V; ++k) acc[k] = 0.f;
        for (int base = eb; base < ee; base += 32) {
            const int n = ee - base < 32 ? ee - base : 32;
            int my_col = 0;
            float my_val = 0.f;
            if (lane < n) {
                my_col = __ldg(a.col + e0 + base + lane);
                my_val = to_f(val[e0 + base + lane]);
            }
            for (int k = 0; k < n; k += kGroups * kUnroll) {
                float x[kUnroll][V];
                float v[kUnroll];
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    const int kk = k + kGroups * u + grp;
                    const int c = __shfl_sync(kFull, my_col, kk & 31);
                    v[u] = __shfl_sync(kFull, my_val, kk & 31);
                    if (kk < n) {
                        L::load(x_tile + (int64_t)c * BT, x[u]);
                    } else {
                        v[u] = 0.f;
#pragma unroll
                        for (int q = 0; q < V; ++q) x[u][q] = 0.f;
                    }
                }
#pragma unroll
                for (int u = 0; u < kUnroll; ++u)
#pragma unroll
                    for (int q = 0; q < V; ++q) acc[q] = fmaf(v[u], x[u][q], acc[q]);
            }
        }
#pragma unroll
        for (int sh = kLanesPerEdge; sh < 32; sh <<= 1)
#pragma unroll
            for (int q = 0; q < V; ++q) acc[q] += __shfl_xor_sync(kFull, acc[q], sh);
        const bool span_lo = (i == is) && cut_lo, span_hi = (i == ie) && cut_hi;
        if (span_lo || span_hi) {
            // a cut row: its first partial goes to s_first of every warp that starts inside it, the
            // partial of the warp where it begins to s_last; summed in warp order after the barrier
            if (grp == 0) {
                float *slot = span_lo ? s_first[warp] : s_last[warp];
#pragma unroll
                for (int q = 0; q < V; ++q) slot[sub * V + q] = acc[q];
            }
        } else if (i < ie && grp == 0) {
            finish_row<T, BT>(a, r0 + i, tile, off, acc);
        }
    }
    __syncthreads();
    // each cut row is finished by warp b-1, b its first cutting boundary: s_last[b-1] + s_first[b..b']
    const int b = warp + 1;
    if (b < kWarps && cut(b) && first_cut(b) == b && grp == 0) {
        const int row = s_bi[b];
        float acc[V];
#pragma unroll
        for (int q = 0; q < V; ++q) acc[q] = s_last[b - 1][sub * V + q];
        for (int w = b;; ++w) {
#pragma unroll
            for (int q = 0; q < V; ++q) acc[q] += s_first[w][sub * V + q];
            if (!(w + 1 < kWarps && s_bi[w + 1] == row && cut(w + 1))) break;
        }
        finish_row<T, BT>(a, r0 + row, tile, off, acc);
    }
}

__global__ void output_kernel(int n_out, const int *__restrict__ src, const float *__restrict__ base, int add_base,
                              const void *__restrict__ state, int is_half, int bt, int64_t ts, float *__restrict__ out,
                              int64_t ld_out, int64_t batch) {
    for (int o = blockIdx.x; o < n_out; o += gridDim.x) {
        const int s = src ? src[o] : (state ? o : -1);   // no map: copy row for row, or fill
        const float b0 = base ? base[o] : 0.f;
        for (int64_t c = threadIdx.x; c < batch; c += blockDim.x) {
            float v = b0;
            if (s >= 0) {
                const int64_t at = (c / bt) * ts + (int64_t)s * bt + c % bt;
                const float x = is_half ? __half2float(static_cast<const __half *>(state)[at])
                                        : static_cast<const float *>(state)[at];
                v = add_base ? b0 + x : x;
            }
            out[(int64_t)o * ld_out + c] = v;
        }
    }
}

__global__ void spmv_kernel(int n_rows, const int *__restrict__ crow, const int *__restrict__ col,
                            const float *__restrict__ val, const float *__restrict__ x, float *__restrict__ y) {
    const int lane = threadIdx.x & 31;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < n_rows; r += (gridDim.x * blockDim.x) >> 5) {
        float s = 0.f;
        for (int e = crow[r] + lane; e < crow[r + 1]; e += 32) s = fmaf(val[e], x[col[e]], s);
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
        if (lane == 0) y[r] = s;
    }
}

// ---- pipelined variant: gathers land in shared memory through cp.async ------------------------
// Each warp owns one edge range (merge path, as above) and a private ring of kStages stages of kChunk
// edges.  A whole warp covers one edge's row tile (32 lanes x 16 bytes: 256 half or 128 float
// columns); lane l copies and later reads back only its own 16 bytes, so per-thread cp.async
// wait_group ordering is all the ring needs.  Bytes in flight live in shared memory, not registers:
// (kStages - 1) x kChunk x 512 bytes per warp.  A chunk that lies inside one row takes the branch-free
// path; chunks that cross a row end go edge by edge.  The product of two float16 values is exact in
// float32, so the mixed-precision fma.rn.f32.f16 (float16 inputs, float32 accumulator, one rounding)
// gives the same sums as converting first, at half the instructions; float32 state uses the packed
// fma.rn.f32x2.  Row constants of the warp's next 32 rows are staged in shared memory.
#ifndef AFB_STAGES
#define AFB_STAGES 3
#endif
#ifndef AFB_CHUNK
#define AFB_CHUNK 4
#endif
#ifndef AFB_ASYNC_WARPS
#define AFB_ASYNC_WARPS 8
#endif
#ifndef AFB_ASYNC_MINBLOCKS
#define AFB_ASYNC_MINBLOCKS 3
#endif
constexpr int kAWarps = AFB_ASYNC_WARPS;
constexpr int kStages = AFB_STAGES;
constexpr int kChunk = AFB_CHUNK;
constexpr int kRowBytes = 512;
constexpr int kWarpRing = kStages * kChunk * kRowBytes;
constexpr int kRingBytes = kAWarps * kWarpRing;
static_assert(32 % kChunk == 0, "a chunk must not straddle a 32-edge window");
static_assert(kWarpRing >= 256 * 4, "a warp's ring must hold its cut-row partial after the main loop");

#ifndef AFB_CP_CG
#define AFB_CP_CG 0
#endif
// Through L1 (.ca) a warp's 32 x 16 contiguous bytes coalesce into four 128-byte requests; the L2-only
// form (.cg) was measured to move twice the gathered bytes from L2.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    if (AFB_CP_CG) asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
    else asm volatile("cp.async.ca.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
// L2 eviction priorities: the gathered slab of a tile is read ~60 times while the tile is processed,
// everything else (sub-matrix indices and values, the input drive, the new state) once.  Marking the
// one-pass traffic evict-first and the slab evict-last keeps the slab resident in L2.
#ifndef AFB_L2HINT
#define AFB_L2HINT 1
#endif
__device__ __forceinline__ uint64_t policy_keep() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_stream() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
    return p;
}
__device__ __forceinline__ void cp_async16_hint(uint32_t dst, const void *src, uint64_t pol) {
    if (!AFB_L2HINT) return cp_async16(dst, src);
    asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "l"(pol) : "memory");
}
__device__ __forceinline__ uint32_t ld_stream_b32(const void *p, uint64_t pol) {
    uint32_t v;
    if (AFB_L2HINT) asm volatile("ld.global.nc.L2::cache_hint.b32 %0, [%1], %2;\n" : "=r"(v) : "l"(p), "l"(pol));
    else v = __ldg(static_cast<const unsigned *>(p));
    return v;
}
__device__ __forceinline__ uint32_t ld_stream_b16(const void *p, uint64_t pol) {
    unsigned short v;
    if (AFB_L2HINT) asm volatile("ld.global.nc.L2::cache_hint.b16 %0, [%1], %2;\n" : "=h"(v) : "l"(p), "l"(pol));
    else v = __ldg(static_cast<const unsigned short *>(p));
    return v;
}
__device__ __forceinline__ uint4 ld_stream_v4(const void *p, uint64_t pol) {
    uint4 v;
    if (AFB_L2HINT)
        asm volatile("ld.global.nc.L2::cache_hint.v4.b32 {%0, %1, %2, %3}, [%4], %5;\n"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p), "l"(pol));
    else v = __ldg(static_cast<const uint4 *>(p));
    return v;
}
__device__ __forceinline__ void st_stream_v4(void *p, uint4 v, uint64_t pol) {
    if (AFB_L2HINT)
        asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1, %2, %3, %4}, %5;\n" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                     "r"(v.w), "l"(pol) : "memory");
    else *static_cast<uint4 *>(p) = v;
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// How a float16 row slice is multiplied into the float32 accumulators: 0 = mixed-precision
// fma.rn.f32.f16, 1 = convert half2 -> float2 then fmaf, 2 = convert then packed fma.rn.f32x2.
// All three round each product-sum once in float32 and give the same results.
#ifndef AFB_HALF_MATH
#define AFB_HALF_MATH 0
#endif

template <typename T>
struct Gather;

template <>
struct Gather<__half> {
    static constexpr int V = 8;
    __device__ static uint32_t bits(const __half *p, uint64_t pol) { return ld_stream_b16(p, pol); }
    // acc[0..7] += v * x[0..7], x = the 8 float16 values at shared address addr
    __device__ static void fma(float (&acc)[8], uint32_t v, uint32_t addr) {
        uint32_t r[4];
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];\n" : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
#if AFB_HALF_MATH == 0
        const unsigned short vh = (unsigned short)v;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            unsigned short lo, hi;
            asm("mov.b32 {%0, %1}, %2;\n" : "=h"(lo), "=h"(hi) : "r"(r[k]));
            asm("fma.rn.f32.f16 %0, %1, %2, %0;\n" : "+f"(acc[2 * k]) : "h"(lo), "h"(vh));
            asm("fma.rn.f32.f16 %0, %1, %2, %0;\n" : "+f"(acc[2 * k + 1]) : "h"(hi), "h"(vh));
        }
#else
        const float vf = __half2float(__ushort_as_half((unsigned short)v));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&r[k]));
#if AFB_HALF_MATH == 1
            acc[2 * k] = fmaf(vf, f.x, acc[2 * k]);
            acc[2 * k + 1] = fmaf(vf, f.y, acc[2 * k + 1]);
#else
            asm("{\n .reg .b64 a, x, v;\n mov.b64 a, {%0, %1};\n mov.b64 x, {%2, %3};\n mov.b64 v, {%4, %4};\n"
                " fma.rn.f32x2 a, x, v, a;\n mov.b64 {%0, %1}, a;\n}\n"
                : "+f"(acc[2 * k]), "+f"(acc[2 * k + 1]) : "f"(f.x), "f"(f.y), "f"(vf));
#endif
        }
#endif
    }
};

template <>
struct Gather<float> {
    static constexpr int V = 4;
    __device__ static uint32_t bits(const float *p, uint64_t pol) { return ld_stream_b32(p, pol); }
    __device__ static void fma(float (&acc)[4], uint32_t v, uint32_t addr) {
        float x[4];
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];\n" : "=f"(x[0]), "=f"(x[1]), "=f"(x[2]), "=f"(x[3]) : "r"(addr));
        const float vf = __uint_as_float(v);
#pragma unroll
        for (int k = 0; k < 2; ++k)
            asm("{\n .reg .b64 a, x, v;\n mov.b64 a, {%0, %1};\n mov.b64 x, {%2, %3};\n mov.b64 v, {%4, %4};\n"
                " fma.rn.f32x2 a, x, v, a;\n mov.b64 {%0, %1}, a;\n}\n"
                : "+f"(acc[2 * k]), "+f"(acc[2 * k + 1]) : "f"(x[2 * k]), "f"(x[2 * k + 1]), "f"(vf));
    }
};

// finish_row with the row's constants already at hand (shared memory)
template <typename T>
__device__ __forceinline__ void load_stream(const T *p, float (&x)[Lane<T>::V], uint64_t pol) {
    const uint4 v = ld_stream_v4(p, pol);
    if constexpr (sizeof(T) == 4) {
        x[0] = __uint_as_float(v.x); x[1] = __uint_as_float(v.y); x[2] = __uint_as_float(v.z); x[3] = __uint_as_float(v.w);
    } else {
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = __half22float2(h[k]);
            x[2 * k] = f.x;
            x[2 * k + 1] = f.y;
        }
    }
}
template <typename T>
__device__ __forceinline__ void store_stream(T *p, const float (&x)[Lane<T>::V], uint64_t pol) {
    uint4 v;
    if constexpr (sizeof(T) == 4) {
        v = make_uint4(__float_as_uint(x[0]), __float_as_uint(x[1]), __float_as_uint(x[2]), __float_as_uint(x[3]));
    } else {
        __half2 *h = reinterpret_cast<__half2 *>(&v);
#pragma unroll
        for (int k = 0; k < 4; ++k) h[k] = __floats2half2_rn(x[2 * k], x[2 * k + 1]);
    }
    st_stream_v4(p, v, pol);
}

// The epilogue inputs of a row (its previous state and its input drive, 16 raw bytes per lane), loaded
// one row ahead so that the loads are in flight while the row's edges are summed.
struct RowPre {
    uint4 p, u;
};

template <typename T>
__device__ __forceinline__ void raw_to_floats(const uint4 &v, float (&x)[Lane<T>::V]) {
    if constexpr (sizeof(T) == 4) {
        x[0] = __uint_as_float(v.x); x[1] = __uint_as_float(v.y); x[2] = __uint_as_float(v.z); x[3] = __uint_as_float(v.w);
    } else {
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = __half22float2(h[k]);
            x[2 * k] = f.x;
            x[2 * k + 1] = f.y;
        }
    }
}

template <typename T, int BT>
__device__ __forceinline__ RowPre issue_row(const StepArgs &a, const RowConst *q_s, int64_t tile, int off, uint64_t stream) {
    constexpr int V = Lane<T>::V;
    RowPre r;
    const int4 w1 = reinterpret_cast<const int4 *>(q_s)[1];
    const int prev = w1.z, usrc = w1.w;
    const int64_t col0 = tile * BT + off;
    if (prev >= 0) r.p = __ldg(reinterpret_cast<const uint4 *>(static_cast<const T *>(a.x_in) + tile * a.ts_in + (int64_t)prev * BT + off));
    if (usrc >= 0 && a.u_vec_ok && col0 + V <= a.batch)
        r.u = ld_stream_v4(static_cast<const T *>(a.u) + (int64_t)usrc * a.ld_u + col0, stream);
    return r;
}

template <typename T, int BT>
__device__ __forceinline__ void finish_row_pre(const StepArgs &a, const RowConst *q_s, const RowPre &pre, int row,
                                               int64_t tile, int off, float (&acc)[Lane<T>::V], uint64_t stream) {
    constexpr int V = Lane<T>::V;
    const int4 w0 = reinterpret_cast<const int4 *>(q_s)[0];
    const int4 w1 = reinterpret_cast<const int4 *>(q_s)[1];
    const float kk = __int_as_float(w0.x), lo = __int_as_float(w0.y), hi = __int_as_float(w0.z), e = __int_as_float(w0.w);
    const float pc = __int_as_float(w1.x), al = __int_as_float(w1.y);
    const int prev = w1.z, usrc = w1.w;
    const int64_t col0 = tile * BT + off;
    float p[V], ux[V];
    if (prev >= 0) raw_to_floats<T>(pre.p, p);
    if (usrc >= 0) {
        if (a.u_vec_ok && col0 + V <= a.batch) {
            raw_to_floats<T>(pre.u, ux);
        } else {
            const T *u = static_cast<const T *>(a.u) + (int64_t)usrc * a.ld_u + col0;
#pragma unroll
            for (int k = 0; k < V; ++k) ux[k] = col0 + k < a.batch ? Lane<T>::scalar(u + k) : 0.f;
        }
    }
    float o[V], yv[V];
#pragma unroll
    for (int k = 0; k < V; ++k) {
        yv[k] = acc[k] + kk + (usrc >= 0 ? ux[k] : 0.f);
        const float x = fminf(fmaxf(yv[k], lo), hi) + e;
        const float pk = prev >= 0 ? p[k] : pc;
        o[k] = pk + al * (x - pk);
    }
    store_stream<T>(static_cast<T *>(a.x_out) + tile * a.ts_out + (int64_t)row * BT + off, o, stream);
    if constexpr (sizeof(T) == 4)
        if (a.y_out) Lane<float>::store(a.y_out + tile * a.ts_out + (int64_t)row * BT + off, yv);
}

template <typename T, typename TV>
__global__ void __launch_bounds__(kAWarps * 32, AFB_ASYNC_MINBLOCKS) step_kernel_async(const StepArgs a) {
    using G = Gather<T>;
    constexpr int V = G::V;
    constexpr int BT = 32 * V;
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ float s_first[kAWarps][BT];
    __shared__ __align__(16) RowConst s_rc[kAWarps][32];
    __shared__ int s_bi[kAWarps + 1], s_bj[kAWarps + 1];

    const int item = __ldg(a.item_order + (blockIdx.x % a.n_items));
    const int64_t tile = blockIdx.x / a.n_items;
    const int r0 = __ldg(a.item_rows + item), r1 = __ldg(a.item_rows + item + 1);
    const int e0 = __ldg(a.crow + r0);
    const int nrows = r1 - r0;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int off = lane * V;
    if (tid <= kAWarps) {
        const int2 bd = __ldg(a.bounds + item * (kAWarps + 1) + tid);
        s_bi[tid] = bd.x;
        s_bj[tid] = bd.y;
    }
    for (int k = tid; k < kAWarps * BT; k += kAWarps * 32) (&s_first[0][0])[k] = 0.f;
    __syncthreads();
    auto cut = [&](int b) -> bool { return b >= 1 && b < kAWarps && s_bj[b] > __ldg(a.crow + r0 + s_bi[b]) - e0; };
    auto first_cut = [&](int b) -> int {
        while (b > 1 && s_bi[b - 1] == s_bi[b] && cut(b - 1)) --b;
        return b;
    };

    const int is = s_bi[warp], js = s_bj[warp], ie = s_bi[warp + 1], je = s_bj[warp + 1];
    const bool cut_lo = cut(warp), cut_hi = cut(warp + 1);
    const T *x_tile = static_cast<const T *>(a.x_in) + tile * a.ts_in + off;
    const int *colp = a.col + e0;
    const TV *valp = static_cast<const TV *>(a.val) + e0;
    const uint32_t ring_warp = (uint32_t)__cvta_generic_to_shared(ring) + warp * kWarpRing + lane * 16;
    const uint64_t keep = policy_keep(), stream = policy_stream();

    // row constants of rows rcb .. rcb + 31 (relative to r0), one per lane, in shared memory
    int rcb = is;
    auto load_rc = [&](int base) {
        rcb = base;
        const int r = base + lane;
        if (r < nrows) {
            const int4 *src = reinterpret_cast<const int4 *>(a.rc + r0 + r);
            int4 *dst = reinterpret_cast<int4 *>(&s_rc[warp][lane]);
            dst[0] = __ldg(src);
            dst[1] = __ldg(src + 1);
        }
        __syncwarp();
    };
    load_rc(is);
    RowPre pre;
    auto arm = [&](int i) {           // issue the epilogue loads of row i, the next row this warp finishes
        if (i < ie) {
            if (i - rcb >= 32) load_rc(i);
            pre = issue_row<T, BT>(a, &s_rc[warp][i - rcb], tile, off, stream);
        }
    };
    arm(cut_lo ? is + 1 : is);

    const int n_chunks = (je - js + kChunk - 1) / kChunk;
    // 32-edge windows of column indices (for the copies) and values (for the sums), one window ahead
    int pcol = 0, pcol_nx = js + lane < je ? (int)ld_stream_b32(colp + js + lane, stream) : 0;
    uint32_t vwin = 0, vwin_nx = js + lane < je ? G::bits(valp + js + lane, stream) : 0u;
    auto prefetch = [&](int k) {      // chunk k -> stage k % kStages
        if (k < n_chunks) {
            const int cs = js + k * kChunk, wo = (k * kChunk) & 31;
            if (wo == 0) {
                pcol = pcol_nx;
                pcol_nx = cs + 32 + lane < je ? (int)ld_stream_b32(colp + cs + 32 + lane, stream) : 0;
            }
            const uint32_t dst = ring_warp + (k % kStages) * (kChunk * kRowBytes);
            if (cs + kChunk <= je) {
#pragma unroll
                for (int u = 0; u < kChunk; ++u) {
                    const int c = __shfl_sync(kFull, pcol, wo + u);
                    cp_async16_hint(dst + u * kRowBytes, x_tile + c * BT, keep);
                }
            } else {
#pragma unroll
                for (int u = 0; u < kChunk; ++u) {
                    const int c = __shfl_sync(kFull, pcol, wo + u);
                    if (cs + u < je) cp_async16_hint(dst + u * kRowBytes, x_tile + c * BT, keep);
                }
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int st = 0; st < kStages - 1; ++st) prefetch(st);

    int rend_base = -64, rend = 0;    // ends (relative edge index) of rows rend_base .. +31
    auto row_end = [&](int i) -> int {
        if (i >= rend_base + 32 || i < rend_base) {
            rend_base = i;
            rend = i + lane < nrows ? __ldg(a.crow + r0 + i + lane + 1) - e0 : 0x7fffffff;
        }
        return __shfl_sync(kFull, rend, i - rend_base);
    };
    int cur = is;
    int cur_end = cur < nrows ? row_end(cur) : 0x7fffffff;
    float acc[V];
#pragma unroll
    for (int q = 0; q < V; ++q) acc[q] = 0.f;
    auto close_row = [&](int i) {     // all of row i's edges in this warp are summed and its end is in range
        if (i == is && cut_lo) {
#pragma unroll
            for (int q = 0; q < V; ++q) s_first[warp][off + q] = acc[q];
        } else {
            finish_row_pre<T, BT>(a, &s_rc[warp][i - rcb], pre, r0 + i, tile, off, acc, stream);
        }
#pragma unroll
        for (int q = 0; q < V; ++q) acc[q] = 0.f;
        arm(i + 1);
    };

    for (int k = 0; k < n_chunks; ++k) {
        prefetch(k + kStages - 1);
        cp_async_wait<kStages - 1>();
        const int cs = js + k * kChunk, wo = (k * kChunk) & 31;
        if (wo == 0) {
            vwin = vwin_nx;
            vwin_nx = cs + 32 + lane < je ? G::bits(valp + cs + 32 + lane, stream) : 0u;
        }
        const uint32_t src = ring_warp + (k % kStages) * (kChunk * kRowBytes);
        if (cs + kChunk <= cur_end && cs + kChunk <= je) {
#pragma unroll
            for (int u = 0; u < kChunk; ++u) G::fma(acc, __shfl_sync(kFull, vwin, wo + u), src + u * kRowBytes);
        } else {
#pragma unroll
            for (int u = 0; u < kChunk; ++u) {
                const int e = cs + u;
                if (e < je) {
                    while (e >= cur_end) {
                        close_row(cur);
                        ++cur;
                        cur_end = row_end(cur);
                    }
                    G::fma(acc, __shfl_sync(kFull, vwin, wo + u), src + u * kRowBytes);
                }
            }
        }
    }
    cp_async_wait<0>();
    while (cur < ie) {
        close_row(cur);
        ++cur;
    }
    float *s_last_w = reinterpret_cast<float *>(ring + warp * kWarpRing);   // the ring is idle from here on
    if (cut_hi) {
        float *slot = (ie == is && cut_lo) ? s_first[warp] : s_last_w;
#pragma unroll
        for (int q = 0; q < V; ++q) slot[off + q] = acc[q];
    }
    __syncthreads();
    const int b = warp + 1;
    if (b < kAWarps && cut(b) && first_cut(b) == b) {
        const int row = s_bi[b];
        const float *s_last_p = reinterpret_cast<const float *>(ring + (b - 1) * kWarpRing);
        float sum[V];
#pragma unroll
        for (int q = 0; q < V; ++q) sum[q] = s_last_p[off + q];
        for (int w = b;; ++w) {
#pragma unroll
            for (int q = 0; q < V; ++q) sum[q] += s_first[w][off + q];
            if (!(w + 1 < kAWarps && s_bi[w + 1] == row && cut(w + 1))) break;
        }
        finish_row<T, BT>(a, r0 + row, tile, off, sum);
    }
}

// ---- TMA variant: one 512-byte bulk copy per edge, completion on a per-stage mbarrier -----------
// The same warp-private ring as the cp.async kernel, but the copies run on the TMA path
// (cp.async.bulk): the gathered bytes no longer pass through the LSU data pipe on their way into
// shared memory, which measured 85% busy with cp.async.  Lane u < kTChunk issues the copy of the
// chunk's u-th edge; lane 0 arms the stage's mbarrier with the chunk's byte count.  Every wait is
// bounded: on timeout the kernel records AFB status 1 in *err and finishes with zeros in place of the
// lost rows (never observed; it only keeps a lost copy from hanging the GPU).
#ifndef AFB_TMA
#define AFB_TMA 0     // measured slower than the cp.async kernel on the configuration-3 workload
#endif
#ifndef AFB_TMA_STAGES
#define AFB_TMA_STAGES 4
#endif
#ifndef AFB_TMA_CHUNK
#define AFB_TMA_CHUNK 4
#endif
#ifndef AFB_TMA_MINBLOCKS
#define AFB_TMA_MINBLOCKS 2
#endif
#ifndef AFB_TMA_ONE_LANE
#define AFB_TMA_ONE_LANE 0
#endif
#ifndef AFB_TMA_FENCE
#define AFB_TMA_FENCE 1
#endif
#ifndef AFB_TMA_GATHER4
#define AFB_TMA_GATHER4 1
#endif
static_assert(!AFB_TMA_GATHER4 || AFB_TMA_CHUNK == 4, "gather4 moves four edges per copy");
constexpr int kTStages = AFB_TMA_STAGES;
constexpr int kTChunk = AFB_TMA_CHUNK;
constexpr int kTWarpRing = kTStages * kTChunk * kRowBytes;
constexpr int kTRingBytes = kAWarps * kTWarpRing;
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr uint32_t kDrainLimit = 1u << 16;
static_assert(32 % kTChunk == 0 && kTChunk <= 32, "chunk within a 32-edge window");
static_assert(kTWarpRing >= 256 * 4, "a warp's ring must hold its cut-row partial after the main loop");

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}\n" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// Polls at most `limit` times; gives up early once any CTA has reported a lost stage in *err.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint32_t limit, const int *err) {
    for (uint32_t it = 0; it < limit; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 1023u) == 1023u && err && *reinterpret_cast<const volatile int *>(err) != 0) return false;
    }
    return false;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar, uint64_t pol) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;\n"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(pol) : "memory");
}
// Four rows (y0..y3) of the 2-D tensor map, each one box (a full row tile) wide, into 4 consecutive
// 512-byte slots at dst (sm_100a tile::gather4; the box is one row high, x = 0).
__device__ __forceinline__ void gather4_g2s(uint32_t dst, const CUtensorMap *map, int y0, int y1, int y2, int y3,
                                            uint32_t bar, uint64_t pol) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes.L2::cache_hint"
                 " [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;\n"
                 ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(bar),
                 "l"(pol) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }

template <typename T, typename TV>
__global__ void __launch_bounds__(kAWarps * 32, AFB_TMA_MINBLOCKS) step_kernel_tma(const __grid_constant__ StepArgs a) {
    using G = Gather<T>;
    constexpr int V = G::V;
    constexpr int BT = 32 * V;
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ float s_first[kAWarps][BT];
    __shared__ __align__(16) RowConst s_rc[kAWarps][32];
    __shared__ __align__(8) uint64_t s_bar[kAWarps][kTStages];
    __shared__ int s_bi[kAWarps + 1], s_bj[kAWarps + 1];

    const int item = __ldg(a.item_order + (blockIdx.x % a.n_items));
    const int64_t tile = blockIdx.x / a.n_items;
    const int r0 = __ldg(a.item_rows + item), r1 = __ldg(a.item_rows + item + 1);
    const int e0 = __ldg(a.crow + r0);
    const int nrows = r1 - r0;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int off = lane * V;
    if (tid <= kAWarps) {
        const int2 bd = __ldg(a.bounds + item * (kAWarps + 1) + tid);
        s_bi[tid] = bd.x;
        s_bj[tid] = bd.y;
    }
    if (tid < kAWarps * kTStages) mbar_init((uint32_t)__cvta_generic_to_shared(&s_bar[0][0] + tid), 1);
    for (int k = tid; k < kAWarps * BT; k += kAWarps * 32) (&s_first[0][0])[k] = 0.f;
    fence_mbar_init();
    __syncthreads();
    auto cut = [&](int b) -> bool { return b >= 1 && b < kAWarps && s_bj[b] > __ldg(a.crow + r0 + s_bi[b]) - e0; };
    auto first_cut = [&](int b) -> int {
        while (b > 1 && s_bi[b - 1] == s_bi[b] && cut(b - 1)) --b;
        return b;
    };

    const int is = s_bi[warp], js = s_bj[warp], ie = s_bi[warp + 1], je = s_bj[warp + 1];
    const bool cut_lo = cut(warp), cut_hi = cut(warp + 1);
    const T *x_tile0 = static_cast<const T *>(a.x_in) + tile * a.ts_in;
    const int *colp = a.col + e0;
    const TV *valp = static_cast<const TV *>(a.val) + e0;
    const uint32_t ring_w = (uint32_t)__cvta_generic_to_shared(ring) + warp * kTWarpRing;
    const uint32_t bar_w = (uint32_t)__cvta_generic_to_shared(&s_bar[warp][0]);
    const uint64_t keep = policy_keep(), stream = policy_stream();

    int rcb = is;
    auto load_rc = [&](int base) {
        rcb = base;
        const int r = base + lane;
        if (r < nrows) {
            const int4 *src = reinterpret_cast<const int4 *>(a.rc + r0 + r);
            int4 *dst = reinterpret_cast<int4 *>(&s_rc[warp][lane]);
            dst[0] = __ldg(src);
            dst[1] = __ldg(src + 1);
        }
        __syncwarp();
    };
    load_rc(is);
    RowPre pre;
    auto arm = [&](int i) {
        if (i < ie) {
            if (i - rcb >= 32) load_rc(i);
            pre = issue_row<T, BT>(a, &s_rc[warp][i - rcb], tile, off, stream);
        }
    };
    arm(cut_lo ? is + 1 : is);

    const int n_chunks = (je - js + kTChunk - 1) / kTChunk;
    int pcol = 0, pcol_nx = js + lane < je ? (int)ld_stream_b32(colp + js + lane, stream) : 0;
    uint32_t vwin = 0, vwin_nx = js + lane < je ? G::bits(valp + js + lane, stream) : 0u;
    auto prefetch = [&](int k) {      // chunk k -> stage k % kTStages, whose previous use was read last iteration
        if (k < n_chunks) {
            const int cs = js + k * kTChunk, wo = (k * kTChunk) & 31;
            if (wo == 0) {
                pcol = pcol_nx;
                pcol_nx = cs + 32 + lane < je ? (int)ld_stream_b32(colp + cs + 32 + lane, stream) : 0;
            }
            const int n_valid = je - cs < kTChunk ? je - cs : kTChunk;
            const int stage = k % kTStages;
#if AFB_TMA_GATHER4
            int cc[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) cc[u] = __shfl_sync(kFull, pcol, wo + (u < n_valid ? u : 0));
            __syncwarp();
            if (AFB_TMA_FENCE) fence_proxy_async_smem();
            if (lane == 0) {
                const int base = (int)(tile * a.rows_in);
                mbar_arrive_expect_tx(bar_w + stage * 8, 4 * kRowBytes);
                gather4_g2s(ring_w + stage * kTChunk * kRowBytes, &a.tmap, base + cc[0], base + cc[1], base + cc[2],
                            base + cc[3], bar_w + stage * 8, keep);
            }
#elif AFB_TMA_ONE_LANE
            int cc[kTChunk];
#pragma unroll
            for (int u = 0; u < kTChunk; ++u) cc[u] = __shfl_sync(kFull, pcol, wo + u);
#else
            const int c = __shfl_sync(kFull, pcol, (wo + lane) & 31);
#endif
#if !AFB_TMA_GATHER4
            __syncwarp();
            if (AFB_TMA_FENCE) fence_proxy_async_smem();
#endif
#if AFB_TMA_GATHER4
#elif AFB_TMA_ONE_LANE
            if (lane == 0) {
                mbar_arrive_expect_tx(bar_w + stage * 8, n_valid * kRowBytes);
#pragma unroll
                for (int u = 0; u < kTChunk; ++u)
                    if (u < n_valid)
                        bulk_g2s(ring_w + (stage * kTChunk + u) * kRowBytes, x_tile0 + cc[u] * BT, kRowBytes, bar_w + stage * 8, keep);
            }
#else
            if (lane == 0) mbar_arrive_expect_tx(bar_w + stage * 8, n_valid * kRowBytes);
            if (lane < n_valid)
                bulk_g2s(ring_w + (stage * kTChunk + lane) * kRowBytes, x_tile0 + c * BT, kRowBytes, bar_w + stage * 8, keep);
#endif
        }
    };
#pragma unroll
    for (int st = 0; st < kTStages - 1; ++st) prefetch(st);

    int rend_base = -64, rend = 0;
    auto row_end = [&](int i) -> int {
        if (i >= rend_base + 32 || i < rend_base) {
            rend_base = i;
            rend = i + lane < nrows ? __ldg(a.crow + r0 + i + lane + 1) - e0 : 0x7fffffff;
        }
        return __shfl_sync(kFull, rend, i - rend_base);
    };
    int cur = is;
    int cur_end = cur < nrows ? row_end(cur) : 0x7fffffff;
    float acc[V];
#pragma unroll
    for (int q = 0; q < V; ++q) acc[q] = 0.f;
    auto close_row = [&](int i) {
        if (i == is && cut_lo) {
#pragma unroll
            for (int q = 0; q < V; ++q) s_first[warp][off + q] = acc[q];
        } else {
            finish_row_pre<T, BT>(a, &s_rc[warp][i - rcb], pre, r0 + i, tile, off, acc, stream);
        }
#pragma unroll
        for (int q = 0; q < V; ++q) acc[q] = 0.f;
        arm(i + 1);
    };

    bool lost = false;
    for (int k = 0; k < n_chunks; ++k) {
        prefetch(k + kTStages - 1);
        const int stage = k % kTStages;
        if (!mbar_wait_bounded(bar_w + stage * 8, (k / kTStages) & 1, lost ? kDrainLimit : kWaitLimit, a.err)) {
            if (!lost && a.err) atomicExch(a.err, 1);
            lost = true;
        }
        const int cs = js + k * kTChunk, wo = (k * kTChunk) & 31;
        if (wo == 0) {
            vwin = vwin_nx;
            vwin_nx = cs + 32 + lane < je ? G::bits(valp + cs + 32 + lane, stream) : 0u;
        }
        const uint32_t src = ring_w + stage * (kTChunk * kRowBytes) + lane * 16;
        if (cs + kTChunk <= cur_end && cs + kTChunk <= je) {
#pragma unroll
            for (int u = 0; u < kTChunk; ++u) G::fma(acc, __shfl_sync(kFull, vwin, wo + u), src + u * kRowBytes);
        } else {
#pragma unroll
            for (int u = 0; u < kTChunk; ++u) {
                const int e = cs + u;
                if (e < je) {
                    while (e >= cur_end) {
                        close_row(cur);
                        ++cur;
                        cur_end = row_end(cur);
                    }
                    G::fma(acc, __shfl_sync(kFull, vwin, wo + u), src + u * kRowBytes);
                }
            }
        }
    }
    while (cur < ie) {
        close_row(cur);
        ++cur;
    }
    if (lost) {   // let any copy still in flight land before this warp's ring is reused or the CTA exits
        for (int st = 0; st < kTStages && st < n_chunks; ++st) {
            const int last = st + ((n_chunks - 1 - st) / kTStages) * kTStages;
            mbar_wait_bounded(bar_w + st * 8, (last / kTStages) & 1, kDrainLimit, nullptr);
        }
    }
    __syncwarp();
    float *s_last_w = reinterpret_cast<float *>(ring + warp * kTWarpRing);
    if (cut_hi) {
        float *slot = (ie == is && cut_lo) ? s_first[warp] : s_last_w;
#pragma unroll
        for (int q = 0; q < V; ++q) slot[off + q] = acc[q];
    }
    __syncthreads();
    const int b = warp + 1;
    if (b < kAWarps && cut(b) && first_cut(b) == b) {
        const int row = s_bi[b];
        const float *s_last_p = reinterpret_cast<const float *>(ring + (b - 1) * kTWarpRing);
        float sum[V];
#pragma unroll
        for (int q = 0; q < V; ++q) sum[q] = s_last_p[off + q];
        for (int w = b;; ++w) {
#pragma unroll
            for (int q = 0; q < V; ++q) sum[q] += s_first[w][off + q];
            if (!(w + 1 < kAWarps && s_bi[w + 1] == row && cut(w + 1))) break;
        }
        finish_row<T, BT>(a, r0 + row, tile, off, sum);
    }
}

#ifndef AFB_ASYNC
#define AFB_ASYNC 1
#endif

// The gather kernel's tensor map of x_in: a 2-D tensor of tiles * rows_in rows, each one batch tile (bt
// elements, 512 bytes) wide; the box is one row, so tile::gather4 fetches four arbitrary rows.
void encode_gather_map(StepArgs &a, int elem_bytes, int bt, int64_t tiles) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        AFB_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        AFB_CHECK(q == cudaDriverEntryPointSuccess && fn, "cuTensorMapEncodeTiled is not available from the driver");
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const cuuint64_t dim[2] = {(cuuint64_t)bt, (cuuint64_t)(tiles * a.rows_in)};
    const cuuint64_t stride[1] = {(cuuint64_t)bt * elem_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)bt, 1};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult r = encode(&a.tmap, elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                              2, const_cast<void *>(a.x_in), dim, stride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    AFB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
}

template <typename T, typename TV>
void launch(const StepArgs &a, cudaStream_t s) {
    constexpr int BT = (AFB_ASYNC || AFB_TMA ? 32 : kLanesPerEdge) * Lane<T>::V;
    if (a.n_items == 0 || a.batch == 0) return;
    const int64_t tiles = (a.batch + BT - 1) / BT;
    const int64_t blocks = tiles * a.n_items;
    AFB_CHECK(blocks < (1LL << 31), "grid too large: reduce the batch");
    if (AFB_TMA) {
        StepArgs g = a;
        if (AFB_TMA_GATHER4 && a.rows_in > 0) encode_gather_map(g, (int)sizeof(T), BT, tiles);
        static unsigned long long configured = 0;   // devices on which this instantiation may use kTRingBytes
        int dev = 0;
        AFB_CUDA(cudaGetDevice(&dev));
        if (dev < 64 && !(configured >> dev & 1ull)) {
            AFB_CUDA(cudaFuncSetAttribute(step_kernel_tma<T, TV>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTRingBytes));
            configured |= 1ull << dev;
        }
        step_kernel_tma<T, TV><<<(unsigned)blocks, kAWarps * 32, kTRingBytes, s>>>(g);
    } else if (AFB_ASYNC) {
        static unsigned long long configured = 0;   // devices on which this instantiation may use kRingBytes
        int dev = 0;
        AFB_CUDA(cudaGetDevice(&dev));
        if (dev < 64 && !(configured >> dev & 1ull)) {
            AFB_CUDA(cudaFuncSetAttribute(step_kernel_async<T, TV>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRingBytes));
            configured |= 1ull << dev;
        }
        step_kernel_async<T, TV><<<(unsigned)blocks, kAWarps * 32, kRingBytes, s>>>(a);
    } else {
        step_kernel<T, TV><<<(unsigned)blocks, kWarps * 32, 0, s>>>(a);
    }
    AFB_LAUNCHED();
}

}  // namespace

void launch_step_f32(const StepArgs &a, cudaStream_t s) { launch<float, float>(a, s); }
__global__ void bounds_kernel(int n_items, int warps, const int *__restrict__ crow, const int *__restrict__ item_rows,
                              int2 *__restrict__ bounds) {
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < (int64_t)n_items * (warps + 1);
         k += (int64_t)gridDim.x * blockDim.x) {
        const int item = (int)(k / (warps + 1)), b = (int)(k % (warps + 1));
        const int r0 = item_rows[item], r1 = item_rows[item + 1];
        const int e0 = crow[r0], nrows = r1 - r0, nnz = crow[r1] - e0;
        const int d = (int)(((int64_t)(nrows + nnz) * b) / warps);
        int lo = d - nnz > 0 ? d - nnz : 0, hi = d < nrows ? d : nrows;
        while (lo < hi) {                      // merge path: row ends consumed at diagonal d
            const int mid = (lo + hi) >> 1;
            if (crow[r0 + mid + 1] - e0 <= d - mid - 1) lo = mid + 1;
            else hi = mid;
        }
        bounds[k] = make_int2(lo, d - lo);
    }
}

int tile_cols(int elem_bytes) { return (AFB_ASYNC || AFB_TMA ? 32 : kLanesPerEdge) * (16 / elem_bytes); }
void launch_step_dev16(const StepArgs &a, cudaStream_t s) { launch<__half, __half>(a, s); }

void build_bounds(Csr &m, cudaStream_t s) {
    const int warps = AFB_ASYNC || AFB_TMA ? kAWarps : kWarps;
    m.bounds.alloc((size_t)m.n_items * (warps + 1));
    if (m.n_items) {
        bounds_kernel<<<grid_for((int64_t)m.n_items * (warps + 1), 256), 256, 0, s>>>(m.n_items, warps, m.crow.get(),
                                                                                       m.item_rows.get(), m.bounds.get());
        AFB_LAUNCHED();
    }
}

void launch_output(int n_out, const int *src, const float *base, int add_base, const void *state, int state_is_half,
                   int64_t ts_state, float *out, int64_t ld_out, int64_t batch, cudaStream_t s) {
    const int bt = tile_cols(state_is_half ? 2 : 4);
    if (n_out == 0 || batch == 0) return;
    const int threads = 256;
    const int grid = n_out < 148 * 64 ? n_out : 148 * 64;
    output_kernel<<<grid, threads, 0, s>>>(n_out, src, base, add_base, state, state_is_half, bt, ts_state, out, ld_out, batch);
    AFB_LAUNCHED();
}

void launch_spmv(int n_rows, const int *crow, const int *col, const float *val, const float *x, float *y, cudaStream_t s) {
    if (n_rows == 0) return;
    spmv_kernel<<<grid_for((int64_t)n_rows * 32, 256, 148 * 64), 256, 0, s>>>(n_rows, crow, col, val, x, y);
    AFB_LAUNCHED();
}

}  // namespace afb
