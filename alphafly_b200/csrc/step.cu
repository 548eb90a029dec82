// The fused light-cone step: one CSR SpMM over a batch tile with the whole state update in its
// epilogue (chessfly/brain.py:273-277 float16 deviation, brain.py:310-314 float32).
//
// Layout.  State and drive are (rows, batch); the state is tile-major: a batch tile is 32 lanes x 16
// bytes (256 float16 or 128 float32 columns), element (row, c) lives at (c / BT) * ts + row * BT + c % BT,
// so one tile's rows are contiguous 512-byte lines and a gathered row is one fully coalesced warp load.
// A CTA owns one batch tile and one "item" -- a contiguous run of rows whose cost (edges + 4 per row) is
// about kItemCost.  blockIdx.x = tile * n_items + k, items heaviest first, so all items of a tile run
// before the next tile starts: the gathered slab R_{t-1} x tile stays resident in L2.
//
// Load balance.  Inside a CTA the item's rows and edges are split evenly over the 8 warps by the
// merge-path partition of Merrill & Garland ("Merge-based parallel sparse matrix-vector
// multiplication", SC'16): the merge of row ends with edge indices is cut into equal diagonals, so a
// 5,000-synapse row and 60 short rows cost the same.  A row cut by warp boundaries leaves one partial
// per warp in shared memory; after a barrier one warp sums them in warp order and finishes the row,
// so results are bitwise reproducible, and independent of the batch width among widths that select the same
// item schedule (see launch: narrow launches take a finer one).
//
// The cost is the gather: every synapse pulls one 512-byte row of the previous state from L2.  Two
// kernels implement it.  The default (step_kernel) loads kChunk gathered rows per lane straight into
// registers; its throughput is set by the loads in flight per SM, so it is written to fit 48 registers
// (5 CTAs, 40 warps per SM).  The other (step_kernel_ring) stages the rows in a shared-memory ring with
// cp.async, which keeps gathers in flight across row ends but moves every row through the L1 data pipe
// three times; on B200 it reaches 10 TB/s (its own ceiling), the register kernel 12 TB/s.  The ring
// kernel runs the sub-matrices whose rows are short (see launch).
// Accumulation is float32 in every mode.
#include "internal.cuh"

namespace afb {
namespace {

constexpr int kWarps = 8;                      // warps per CTA (both kernels)
constexpr int kRowBytes = 512;                 // a gathered row tile: 32 lanes x 16 bytes
constexpr unsigned kFull = 0xffffffffu;

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


// Epilogue of one row, this lane's V columns: y = acc + kk (+ drive), x = clamp(y, lo, hi) + e,
// p = previous state (or the constant pc), out = p + a (x - p); written to the tile-major x_out (and
// y to y_out in the training forward).  The previous state and the drive are kept packed and converted
// a pair at a time, to keep few registers live.
template <typename T, int BT>
__device__ __forceinline__ void finish_row(const StepArgs &a, int row, int64_t tile, int off, const float (&acc)[Lane<T>::V]) {
    constexpr int V = Lane<T>::V;
    const int64_t col0 = tile * BT + off;
    const int4 w0 = __ldg(reinterpret_cast<const int4 *>(a.rc + row));
    const int4 w1 = __ldg(reinterpret_cast<const int4 *>(a.rc + row) + 1);
    const int prev = w1.z, usrc = w1.w;
    uint4 up = make_uint4(0, 0, 0, 0), pp = make_uint4(0, 0, 0, 0);
    const T *u = static_cast<const T *>(a.u) + (int64_t)(usrc >= 0 ? usrc : 0) * a.ld_u + col0;
    const bool u_vec = usrc >= 0 && a.u_vec_ok && col0 + V <= a.batch;
    if (u_vec) up = __ldg(reinterpret_cast<const uint4 *>(u));
    if (prev >= 0) pp = __ldg(reinterpret_cast<const uint4 *>(static_cast<const T *>(a.x_in) + tile * a.ts_in + (int64_t)prev * BT + off));
    const float kk = __int_as_float(w0.x), lo = __int_as_float(w0.y), hi = __int_as_float(w0.z), e = __int_as_float(w0.w);
    const float pc = __int_as_float(w1.x), al = __int_as_float(w1.y);
    const uint32_t ur[4] = {up.x, up.y, up.z, up.w}, pr[4] = {pp.x, pp.y, pp.z, pp.w};
    uint32_t outr[4], yr[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float y[2], pv[2], uv[2];
        if constexpr (sizeof(T) == 2) {
            const float2 u2 = __half22float2(*reinterpret_cast<const __half2 *>(&ur[k]));
            const float2 p2 = __half22float2(*reinterpret_cast<const __half2 *>(&pr[k]));
            uv[0] = u2.x; uv[1] = u2.y; pv[0] = p2.x; pv[1] = p2.y;
        } else {
            uv[0] = __uint_as_float(ur[k]); pv[0] = __uint_as_float(pr[k]);
        }
        constexpr int P = sizeof(T) == 2 ? 2 : 1;   // state elements in this 32-bit word
        float o[2];
#pragma unroll
        for (int j = 0; j < P; ++j) {
            const int c = P * k + j;
            float uu = 0.f;
            if (usrc >= 0) uu = u_vec ? uv[j] : (col0 + c < a.batch ? Lane<T>::scalar(u + c) : 0.f);
            y[j] = acc[c] + kk + uu;
            const float x = fminf(fmaxf(y[j], lo), hi) + e;
            const float pk = prev >= 0 ? pv[j] : pc;
            o[j] = pk + al * (x - pk);
        }
        if constexpr (sizeof(T) == 2) {
            const __half2 h = __floats2half2_rn(o[0], o[1]);
            outr[k] = *reinterpret_cast<const uint32_t *>(&h);
        } else {
            outr[k] = __float_as_uint(o[0]);
            yr[k] = __float_as_uint(y[0]);
        }
    }
    *reinterpret_cast<uint4 *>(static_cast<T *>(a.x_out) + tile * a.ts_out + (int64_t)row * BT + off) =
        make_uint4(outr[0], outr[1], outr[2], outr[3]);
    if constexpr (sizeof(T) == 4)
        if (a.y_out)
            *reinterpret_cast<uint4 *>(a.y_out + tile * a.ts_out + (int64_t)row * BT + off) = make_uint4(yr[0], yr[1], yr[2], yr[3]);
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

// ---- ring kernel: gathers land in shared memory through cp.async -------------------------------
// Each warp owns one edge range (merge path) and a private ring of kStages stages of kChunk
// edges.  A whole warp covers one edge's row tile (32 lanes x 16 bytes: 256 half or 128 float
// columns); lane l copies and later reads back only its own 16 bytes, so per-thread cp.async
// wait_group ordering is all the ring needs.  Bytes in flight live in shared memory, not registers:
// (kStages - 1) x kChunk x 512 bytes per warp.  A chunk that lies inside one row takes the branch-free
// path; chunks that cross a row end go edge by edge.  The product of two float16 values is exact in
// float32, so the mixed-precision fma.rn.f32.f16 (float16 inputs, float32 accumulator, one rounding)
// gives the same sums as converting first, at half the instructions; float32 state uses the packed
// fma.rn.f32x2.  Row constants of the warp's next 32 rows are staged in shared memory.
constexpr int kStages = 3;      // tuned on configuration 3's step 2: 3 stages of 4 synapses, 3 CTAs per SM
constexpr int kChunk = 4;
constexpr int kRingMinBlocks = 3;
constexpr int kWarpRing = kStages * kChunk * kRowBytes;
constexpr int kRingBytes = kWarps * kWarpRing;
static_assert(32 % kChunk == 0, "a chunk must not straddle a 32-edge window");
static_assert(kWarpRing >= 256 * 4, "a warp's ring must hold its cut-row partial after the main loop");

// L2 eviction priorities of the ring kernel: the gathered slab of a tile is read ~60 times while the tile
// is processed, everything else (sub-matrix indices and values, the input drive, the new state) once.
// Marking the one-pass traffic evict-first and the slab evict-last keeps the slab resident in L2.
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
// Through L1 (.ca) a warp's 32 x 16 contiguous bytes coalesce into four 128-byte requests; the L2-only
// form (.cg) was measured to move twice the gathered bytes from L2.
__device__ __forceinline__ void cp_async16_hint(uint32_t dst, const void *src, uint64_t pol) {
    asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "l"(pol) : "memory");
}
__device__ __forceinline__ uint32_t ld_stream_b32(const void *p, uint64_t pol) {
    uint32_t v;
    asm volatile("ld.global.nc.L2::cache_hint.b32 %0, [%1], %2;\n" : "=r"(v) : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ uint32_t ld_stream_b16(const void *p, uint64_t pol) {
    unsigned short v;
    asm volatile("ld.global.nc.L2::cache_hint.b16 %0, [%1], %2;\n" : "=h"(v) : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ uint4 ld_stream_v4(const void *p, uint64_t pol) {
    uint4 v;
    asm volatile("ld.global.nc.L2::cache_hint.v4.b32 {%0, %1, %2, %3}, [%4], %5;\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ void st_stream_v4(void *p, uint4 v, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1, %2, %3, %4}, %5;\n" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w), "l"(pol) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

template <typename T>
struct Gather;

template <>
struct Gather<__half> {
    static constexpr int V = 8;
    __device__ static uint32_t bits(const __half *p, uint64_t pol) { return ld_stream_b16(p, pol); }
    __device__ static uint32_t bits_plain(const __half *p) { return __ldg(reinterpret_cast<const unsigned short *>(p)); }
    // acc[0..7] += v * x[0..7], x = the 8 float16 values at shared address addr
    __device__ static void fma(float (&acc)[8], uint32_t v, uint32_t addr) {
        uint4 x;
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];\n" : "=r"(x.x), "=r"(x.y), "=r"(x.z), "=r"(x.w) : "r"(addr));
        fma(acc, v, x);
    }
    // acc[0..7] += v * x[0..7], x = 8 float16 values in registers.  The mixed-precision fma.rn.f32.f16
    // multiplies two float16 values exactly in float32 and rounds the sum once, so it equals converting
    // first, at half the instructions.
    __device__ static void fma(float (&acc)[8], uint32_t v, const uint4 &x) {
        const uint32_t r[4] = {x.x, x.y, x.z, x.w};
        const unsigned short vh = (unsigned short)v;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            unsigned short lo, hi;
            asm("mov.b32 {%0, %1}, %2;\n" : "=h"(lo), "=h"(hi) : "r"(r[k]));
            asm("fma.rn.f32.f16 %0, %1, %2, %0;\n" : "+f"(acc[2 * k]) : "h"(lo), "h"(vh));
            asm("fma.rn.f32.f16 %0, %1, %2, %0;\n" : "+f"(acc[2 * k + 1]) : "h"(hi), "h"(vh));
        }
    }
};

template <>
struct Gather<float> {
    static constexpr int V = 4;
    __device__ static uint32_t bits(const float *p, uint64_t pol) { return ld_stream_b32(p, pol); }
    __device__ static uint32_t bits_plain(const float *p) { return __ldg(reinterpret_cast<const unsigned *>(p)); }
    __device__ static void fma(float (&acc)[4], uint32_t v, uint32_t addr) {
        uint4 x;
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];\n" : "=r"(x.x), "=r"(x.y), "=r"(x.z), "=r"(x.w) : "r"(addr));
        fma(acc, v, x);
    }
    __device__ static void fma(float (&acc)[4], uint32_t v, const uint4 &xr) {
        const float x[4] = {__uint_as_float(xr.x), __uint_as_float(xr.y), __uint_as_float(xr.z), __uint_as_float(xr.w)};
        const float vf = __uint_as_float(v);
#pragma unroll
        for (int k = 0; k < 2; ++k)
            asm("{\n .reg .b64 a, x, v;\n mov.b64 a, {%0, %1};\n mov.b64 x, {%2, %3};\n mov.b64 v, {%4, %4};\n"
                " fma.rn.f32x2 a, x, v, a;\n mov.b64 {%0, %1}, a;\n}\n"
                : "+f"(acc[2 * k]), "+f"(acc[2 * k + 1]) : "f"(x[2 * k]), "f"(x[2 * k + 1]), "f"(vf));
    }
};

// V state values of this lane stored as one 16-byte word with an L2 eviction policy
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
__global__ void __launch_bounds__(kWarps * 32, kRingMinBlocks) step_kernel_ring(const StepArgs a) {
    using G = Gather<T>;
    constexpr int V = G::V;
    constexpr int BT = 32 * V;
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ float s_first[kWarps][BT];
    __shared__ __align__(16) RowConst s_rc[kWarps][32];
    __shared__ int s_bi[kWarps + 1], s_bj[kWarps + 1];

    const int item = __ldg(a.item_order + (blockIdx.x % a.n_items));
    const int64_t tile = blockIdx.x / a.n_items;
    const int r0 = __ldg(a.item_rows + item), r1 = __ldg(a.item_rows + item + 1);
    const int e0 = __ldg(a.crow + r0);
    const int nrows = r1 - r0;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int off = lane * V;
    if (tid <= kWarps) {
        const int2 bd = __ldg(a.bounds + item * (kWarps + 1) + tid);
        s_bi[tid] = bd.x;
        s_bj[tid] = bd.y;
    }
    for (int k = tid; k < kWarps * BT; k += kWarps * 32) (&s_first[0][0])[k] = 0.f;
    __syncthreads();
    auto cut = [&](int b) -> bool { return b >= 1 && b < kWarps && s_bj[b] > __ldg(a.crow + r0 + s_bi[b]) - e0; };
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
    if (b < kWarps && cut(b) && first_cut(b) == b) {
        const int row = s_bi[b];
        const float *s_last_p = reinterpret_cast<const float *>(ring + (b - 1) * kWarpRing);
        float sum[V];
#pragma unroll
        for (int q = 0; q < V; ++q) sum[q] = s_last_p[off + q];
        for (int w = b;; ++w) {
#pragma unroll
            for (int q = 0; q < V; ++q) sum[q] += s_first[w][off + q];
            if (!(w + 1 < kWarps && s_bi[w + 1] == row && cut(w + 1))) break;
        }
        finish_row<T, BT>(a, r0 + row, tile, off, sum);
    }
}


// ---- register kernel (default) --------------------------------------------------------------------
// Row by row, one warp per 512-byte row tile, kChunk gathered rows in flight per lane in registers; a
// chunk never straddles a row, so the gathered registers are dead when a row's epilogue runs.  The
// column indices and values of 32 edges are loaded coalesced and broadcast with shuffles.  A gather's
// address is the tile's slab base (the same for the whole CTA) plus a 32-bit byte offset, which keeps
// the per-lane address state to one register (measured 150 vs 154 ms per configuration-3 forward
// against 64-bit per-lane pointers).  Measured on
// the configuration-3 workload: the gather's throughput grows with the warps per SM, and a spill in the
// loop costs more than any occupancy gains, so the tuned point is kChunk = 4 at 5 CTAs per SM (48
// registers, no spills).
constexpr int kChunkR = 4;      // gathered rows in flight per lane
constexpr int kMinBlocks = 5;   // CTAs per SM: 40 warps at 48 registers per thread

// Per-warp loop bounds live in shared memory and are re-read where they are needed (volatile), so
// that they do not hold registers through the gather loop.
struct LeanWarp {
    int is, ie, js, je, ilast, flags;   // flags: 1 = first row cut (partial to s_first), 2 = last row cut
};
__device__ __forceinline__ int vld(const int &x) { return *reinterpret_cast<const volatile int *>(&x); }

template <typename T, typename TV>
__global__ void __launch_bounds__(kWarps * 32, kMinBlocks) step_kernel(const StepArgs a) {
    using G = Gather<T>;
    constexpr int V = G::V;
    constexpr int BT = 32 * V;
    __shared__ float s_first[kWarps][BT], s_last[kWarps][BT];
    __shared__ int s_bi[kWarps + 1], s_bj[kWarps + 1];
    __shared__ LeanWarp s_w[kWarps];
    __shared__ int s_r0, s_e0, s_nrows;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    {
        const int item = __ldg(a.item_order + (blockIdx.x % a.n_items));
        if (tid <= kWarps) {
            const int2 bd = __ldg(a.bounds + item * (kWarps + 1) + tid);
            s_bi[tid] = bd.x;
            s_bj[tid] = bd.y;
        }
        if (tid == 0) {
            const int r0 = __ldg(a.item_rows + item);
            s_r0 = r0;
            s_e0 = __ldg(a.crow + r0);
            s_nrows = __ldg(a.item_rows + item + 1) - r0;
        }
    }
    __syncthreads();
    auto cut = [&](int b) -> bool { return b >= 1 && b < kWarps && s_bj[b] > __ldg(a.crow + s_r0 + s_bi[b]) - s_e0; };
    if (lane == 0) {
        LeanWarp w;
        w.is = s_bi[warp];
        w.ie = s_bi[warp + 1];
        w.js = s_bj[warp];
        w.je = s_bj[warp + 1];
        w.ilast = w.ie < s_nrows - 1 ? w.ie : s_nrows - 1;
        w.flags = (cut(warp) ? 1 : 0) | (cut(warp + 1) ? 2 : 0);
        s_w[warp] = w;
    }
    __syncwarp();

    const int tile = blockIdx.x / a.n_items;
    const int off = lane * V;
    // uniform base of this tile's slab + a 32-bit per-lane byte offset (a slab is far below 4 GB)
    const char *x_base = reinterpret_cast<const char *>(static_cast<const T *>(a.x_in) + (int64_t)tile * a.ts_in);
    const uint32_t lane_b = (uint32_t)lane * 16u;
    const LeanWarp &me = s_w[warp];
    for (int i = vld(me.is); i <= vld(me.ilast); ++i) {
        int eb, ee;
        {
            const int r0 = vld(s_r0), e0 = vld(s_e0);
            const int rs = __ldg(a.crow + r0 + i) - e0, re = __ldg(a.crow + r0 + i + 1) - e0;
            const int js = vld(me.js), je = vld(me.je);
            eb = rs > js ? rs : js;
            ee = re < je ? re : je;
        }
        if (i == vld(me.ie) && ee <= eb) break;
        float acc[V];
#pragma unroll
        for (int q = 0; q < V; ++q) acc[q] = 0.f;
        for (int base = eb; base < ee; base += 32) {
            const int n = ee - base < 32 ? ee - base : 32;
            const int eoff = vld(s_e0) + base + lane;
            int my_col = 0;
            uint32_t my_val = 0u;
            if (lane < n) {
                my_col = __ldg(a.col + eoff);
                my_val = G::bits_plain(static_cast<const TV *>(a.val) + eoff);
            }
            // full chunks: nothing predicated (chunks kept in sequence: one chunk's rows in registers at a time)
            const int n_full = n / kChunkR * kChunkR;
#pragma unroll 1
            for (int k = 0; k < n_full; k += kChunkR) {
                uint4 x[kChunkR];
#pragma unroll
                for (int u = 0; u < kChunkR; ++u)
                    x[u] = __ldg(reinterpret_cast<const uint4 *>(x_base + ((uint32_t)__shfl_sync(kFull, my_col, k + u) * 512u + lane_b)));
#pragma unroll
                for (int u = 0; u < kChunkR; ++u) G::fma(acc, __shfl_sync(kFull, my_val, k + u), x[u]);
            }
            // the window's last, partial chunk
            for (int k = n_full; k < n; k += kChunkR) {
                uint4 x[kChunkR];
#pragma unroll
                for (int u = 0; u < kChunkR; ++u) {
                    const int c = __shfl_sync(kFull, my_col, (k + u) & 31);
                    x[u] = k + u >= n ? make_uint4(0, 0, 0, 0) : __ldg(reinterpret_cast<const uint4 *>(x_base + ((uint32_t)c * 512u + lane_b)));
                }
#pragma unroll
                for (int u = 0; u < kChunkR; ++u) G::fma(acc, __shfl_sync(kFull, my_val, (k + u) & 31), x[u]);
            }
        }
        const int flags = vld(me.flags);
        const bool span_lo = (i == vld(me.is)) && (flags & 1), span_hi = (i == vld(me.ie)) && (flags & 2);
        if (span_lo || span_hi) {
            float *slot = span_lo ? s_first[warp] : s_last[warp];
#pragma unroll
            for (int q = 0; q < V; ++q) slot[off + q] = acc[q];
        } else if (i < vld(me.ie)) {
            finish_row<T, BT>(a, vld(s_r0) + i, tile, off, acc);
        }
    }
    __syncthreads();
    const int b = warp + 1;
    if (b < kWarps && cut(b)) {
        int fb = b;                               // the first boundary cutting the row cut by b
        while (fb > 1 && s_bi[fb - 1] == s_bi[fb] && cut(fb - 1)) --fb;
        if (fb == b) {
            const int row = s_bi[b];
            float sum[V];
#pragma unroll
            for (int q = 0; q < V; ++q) sum[q] = s_last[b - 1][off + q];
            for (int w = b;; ++w) {
#pragma unroll
                for (int q = 0; q < V; ++q) sum[q] += s_first[w][off + q];
                if (!(w + 1 < kWarps && s_bi[w + 1] == row && cut(w + 1))) break;
            }
            finish_row<T, BT>(a, s_r0 + row, tile, off, sum);
        }
    }
}

// Sub-matrices whose mean row is shorter than this take the ring kernel.
constexpr int64_t kRingMaxDegree = 16;

// CTAs below which a step takes the fine schedule: two waves of the register kernel's 5 CTAs per SM.
int64_t fine_grid_limit() {
    static int sms[64] = {0};
    int dev = 0;
    AFB_CUDA(cudaGetDevice(&dev));
    if (dev >= 64) return 0;
    if (!sms[dev]) AFB_CUDA(cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev));
    return 2LL * kMinBlocks * sms[dev];
}

template <typename T, typename TV>
void launch(const StepArgs &args, cudaStream_t s) {
    constexpr int BT = 32 * Lane<T>::V;
    if (args.n_items == 0 || args.batch == 0) return;
    const int64_t tiles = (args.batch + BT - 1) / BT;
    StepArgs a = args;
    // Too few CTAs for two waves: the fine schedule (one batch tile of a small graph 2.8x faster).  The
    // schedule fixes where rows are cut between warps, hence the summation order of those rows: results are
    // bitwise the same for batch widths that pick the same schedules, and may differ in the last place of
    // cut rows otherwise.
    if (a.n_items_fine > a.n_items && tiles * a.n_items < fine_grid_limit()) {
        a.n_items = a.n_items_fine;
        a.item_rows = a.item_rows_fine;
        a.item_order = a.item_order_fine;
        a.bounds = a.bounds_fine;
    }
    const int64_t blocks = tiles * a.n_items;
    AFB_CHECK(blocks < (1LL << 31), "grid too large: reduce the batch");
    // The ring kernel keeps gathers in flight across row ends, which pays on sub-matrices whose rows are
    // shorter than half a 32-synapse window (configuration 3's steps 1 and 2: 0.85 vs 1.04 ms on step 1,
    // which has no synapses, equal on step 2); the register kernel wins on the others.  Both give bitwise
    // the same results.
    const bool ring = a.nnz < kRingMaxDegree * (int64_t)a.n_rows;
    if (ring) {
        static unsigned long long configured = 0;   // devices on which this instantiation may use kRingBytes
        int dev = 0;
        AFB_CUDA(cudaGetDevice(&dev));
        if (dev < 64 && !(configured >> dev & 1ull)) {
            AFB_CUDA(cudaFuncSetAttribute(step_kernel_ring<T, TV>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRingBytes));
            configured |= 1ull << dev;
        }
        step_kernel_ring<T, TV><<<(unsigned)blocks, kWarps * 32, kRingBytes, s>>>(a);
    } else {
        // the register kernel addresses a tile's slab with 32-bit byte offsets
        AFB_CHECK(a.ts_in * (int64_t)sizeof(T) <= (int64_t)UINT32_MAX, "a step's state tile exceeds 4 GB");
        step_kernel<T, TV><<<(unsigned)blocks, kWarps * 32, 0, s>>>(a);
    }
    AFB_LAUNCHED();
}

}  // namespace

void launch_step_f32(const StepArgs &a, cudaStream_t s) { launch<float, float>(a, s); }
void launch_step_dev16(const StepArgs &a, cudaStream_t s) { launch<__half, __half>(a, s); }

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

int tile_cols(int elem_bytes) { return 32 * (16 / elem_bytes); }

void build_bounds(const Csr &m, int n_items, const int *item_rows, DevBuf<int2> &bounds, cudaStream_t s) {
    const int warps = kWarps;
    bounds.alloc((size_t)n_items * (warps + 1));
    if (n_items) {
        bounds_kernel<<<grid_for((int64_t)n_items * (warps + 1), 256), 256, 0, s>>>(n_items, warps, m.crow.get(), item_rows,
                                                                                     bounds.get());
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
