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
// The cost is the gather: every synapse pulls one 512-byte row of the previous state from L2.  The
// kernels load the gathered rows straight into registers; the throughput is set by the loads in flight
// per SM, so step_kernel is written to fit 48 registers (5 CTAs, 40 warps per SM).  Sub-matrices whose
// rows are short take step_kernel_pair, which covers the same row for two batch tiles, so the index
// window, the shuffles and the row bookkeeping serve two row tiles; a step without synapses takes
// step_kernel_nosyn, the epilogue alone (see launch).
// Accumulation is float32 in every mode.
#include "internal.cuh"

namespace afb {
namespace {

constexpr int kWarps = 8;                      // warps per CTA (both kernels)
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

template <typename T>
struct Gather;

template <>
struct Gather<__half> {
    static constexpr int V = 8;
    __device__ static uint32_t bits_plain(const __half *p) { return __ldg(reinterpret_cast<const unsigned short *>(p)); }
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
    __device__ static uint32_t bits_plain(const float *p) { return __ldg(reinterpret_cast<const unsigned *>(p)); }
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
    __shared__ int s_r0, s_e0, s_nrows, s_tile;

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
            s_tile = blockIdx.x / a.n_items;
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

    // uniform base of this tile's slab + a 32-bit per-lane byte offset (a slab is far below 4 GB); the tile
    // and the lane's column offset are re-derived at a row's end (from shared memory and the lane), so that
    // they hold no registers through the gather loop (which otherwise spills 12 bytes: 147.4 vs 144.5 ms)
    const char *x_base = reinterpret_cast<const char *>(static_cast<const T *>(a.x_in) + (int64_t)vld(s_tile) * a.ts_in);
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
            for (int q = 0; q < V; ++q) slot[lane * V + q] = acc[q];
        } else if (i < vld(me.ie)) {
            finish_row<T, BT>(a, vld(s_r0) + i, vld(s_tile), lane * V, acc);
        }
    }
    __syncthreads();
    const int b = warp + 1;
    if (b < kWarps && cut(b)) {
        int fb = b;                               // the first boundary cutting the row cut by b
        while (fb > 1 && s_bi[fb - 1] == s_bi[fb] && cut(fb - 1)) --fb;
        if (fb == b) {
            const int row = s_bi[b];
            const int off = lane * V;
            float sum[V];
#pragma unroll
            for (int q = 0; q < V; ++q) sum[q] = s_last[b - 1][off + q];
            for (int w = b;; ++w) {
#pragma unroll
                for (int q = 0; q < V; ++q) sum[q] += s_first[w][off + q];
                if (!(w + 1 < kWarps && s_bi[w + 1] == row && cut(w + 1))) break;
            }
            finish_row<T, BT>(a, s_r0 + row, s_tile, off, sum);
        }
    }
}

// ---- short-row kernel --------------------------------------------------------------------------------
// The register kernel's structure with one warp on the same row for two batch tiles (a CTA covers tiles
// 2p and 2p + 1): the index window, the shuffles, the row bookkeeping and the row constants serve two row
// tiles, and each round trip to L2 brings 2 synapses x 2 tiles per lane.  On short rows the register
// kernel is a chain of dependent round trips per row (row end, index window, gathers, epilogue); here each
// chain does twice the work.  Configuration 3's step 2 (7.3 synapses per row): 11.5 ms against 14.0 for
// the shared-memory ring kernel this replaced and 14.3 for the register kernel.  64 registers, 4 CTAs per
// SM (48 registers spill 108 bytes: 14.2 ms).  Per tile the arithmetic and its order are the register
// kernel's, so the results are bitwise the same.
constexpr int kChunkP = 2;          // synapses per round trip (x 2 tiles)
constexpr int kPairMinBlocks = 4;
template <typename T, typename TV>
__global__ void __launch_bounds__(kWarps * 32, kPairMinBlocks) step_kernel_pair(const StepArgs a) {
    using G = Gather<T>;
    constexpr int V = G::V;
    constexpr int BT = 32 * V;
    __shared__ float s_first[2][kWarps][BT], s_last[2][kWarps][BT];
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

    const int tiles = (int)((a.batch + BT - 1) / BT);
    const int tile_a = 2 * (blockIdx.x / a.n_items), tile_b = tile_a + 1;
    const bool has_b = tile_b < tiles;
    const int off = lane * V;
    const char *base_a = reinterpret_cast<const char *>(static_cast<const T *>(a.x_in) + (int64_t)tile_a * a.ts_in);
    const char *base_b = has_b ? reinterpret_cast<const char *>(static_cast<const T *>(a.x_in) + (int64_t)tile_b * a.ts_in) : base_a;
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
        float acc_a[V], acc_b[V];
#pragma unroll
        for (int q = 0; q < V; ++q) acc_a[q] = acc_b[q] = 0.f;
        for (int base = eb; base < ee; base += 32) {
            const int n = ee - base < 32 ? ee - base : 32;
            const int eoff = vld(s_e0) + base + lane;
            int my_col = 0;
            uint32_t my_val = 0u;
            if (lane < n) {
                my_col = __ldg(a.col + eoff);
                my_val = G::bits_plain(static_cast<const TV *>(a.val) + eoff);
            }
            const int n_full = n / kChunkP * kChunkP;
#pragma unroll 1
            for (int k = 0; k < n_full; k += kChunkP) {
                uint4 xa[kChunkP], xb[kChunkP];
#pragma unroll
                for (int u = 0; u < kChunkP; ++u) {
                    const uint32_t o = (uint32_t)__shfl_sync(kFull, my_col, k + u) * 512u + lane_b;
                    xa[u] = __ldg(reinterpret_cast<const uint4 *>(base_a + o));
                    xb[u] = __ldg(reinterpret_cast<const uint4 *>(base_b + o));
                }
#pragma unroll
                for (int u = 0; u < kChunkP; ++u) {
                    const uint32_t v = __shfl_sync(kFull, my_val, k + u);
                    G::fma(acc_a, v, xa[u]);
                    G::fma(acc_b, v, xb[u]);
                }
            }
            for (int k = n_full; k < n; ++k) {               // the window's last synapses, one at a time
                const uint32_t o = (uint32_t)__shfl_sync(kFull, my_col, k) * 512u + lane_b;
                const uint32_t v = __shfl_sync(kFull, my_val, k);
                const uint4 xa = __ldg(reinterpret_cast<const uint4 *>(base_a + o));
                const uint4 xb = __ldg(reinterpret_cast<const uint4 *>(base_b + o));
                G::fma(acc_a, v, xa);
                G::fma(acc_b, v, xb);
            }
        }
        const int flags = vld(me.flags);
        const bool span_lo = (i == vld(me.is)) && (flags & 1), span_hi = (i == vld(me.ie)) && (flags & 2);
        if (span_lo || span_hi) {
#pragma unroll
            for (int q = 0; q < V; ++q) {
                (span_lo ? s_first[0][warp] : s_last[0][warp])[off + q] = acc_a[q];
                (span_lo ? s_first[1][warp] : s_last[1][warp])[off + q] = acc_b[q];
            }
        } else if (i < vld(me.ie)) {
            finish_row<T, BT>(a, vld(s_r0) + i, tile_a, off, acc_a);
            if (has_b) finish_row<T, BT>(a, vld(s_r0) + i, tile_b, off, acc_b);
        }
    }
    __syncthreads();
    const int b = warp + 1;
    if (b < kWarps && cut(b)) {
        int fb = b;
        while (fb > 1 && s_bi[fb - 1] == s_bi[fb] && cut(fb - 1)) --fb;
        if (fb == b) {
            const int row = s_bi[b];
            for (int h = 0; h < (has_b ? 2 : 1); ++h) {
                float sum[V];
#pragma unroll
                for (int q = 0; q < V; ++q) sum[q] = s_last[h][b - 1][off + q];
                for (int w = b;; ++w) {
#pragma unroll
                    for (int q = 0; q < V; ++q) sum[q] += s_first[h][w][off + q];
                    if (!(w + 1 < kWarps && s_bi[w + 1] == row && cut(w + 1))) break;
                }
                finish_row<T, BT>(a, s_r0 + row, h ? tile_b : tile_a, off, sum);
            }
        }
    }
}

// ---- narrow batches ----------------------------------------------------------------------------------
// A batch of at most 16 V columns (128 float16 or 64 float32 positions: one partly used tile) needs only
// the first G x 16 bytes of each gathered 512-byte row line, G = the smallest power of two with G V >= batch.
// The register kernel would still move whole lines; here the warp splits into S = 32 / G groups of G lanes
// and each group gathers its own synapse, so one warp load brings S synapses (at B = 1, 32 synapses x 16
// bytes).  A row's group sums are joined with log2 S shuffle steps and group 0 runs the row's epilogue for
// its G V columns; columns past them are neither read nor written.  Inference only (the training backward
// reads whole tiles of the saved state).  The sums are the same as the register kernel's up to their order.
template <typename T, typename TV, int G>
__global__ void __launch_bounds__(kWarps * 32, kMinBlocks) step_kernel_narrow(const StepArgs a) {
    using Gt = Gather<T>;
    constexpr int V = Gt::V;
    constexpr int BT = 32 * V;
    constexpr int S = 32 / G;                 // synapses per warp load
    __shared__ float s_first[kWarps][G * V], s_last[kWarps][G * V];
    __shared__ int s_bi[kWarps + 1], s_bj[kWarps + 1];
    __shared__ LeanWarp s_w[kWarps];
    __shared__ int s_r0, s_e0, s_nrows;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    {
        const int item = __ldg(a.item_order + blockIdx.x);
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

    const char *x_base = static_cast<const char *>(a.x_in);            // the one tile
    const int grp = lane / G;
    const uint32_t lane_b = (uint32_t)(lane % G) * 16u;
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
                my_val = Gt::bits_plain(static_cast<const TV *>(a.val) + eoff);
            }
            // uniform trip count: group g takes synapses k + u S + g of the window
            for (int k = 0; k < n; k += S * kChunkR) {
                uint4 x[kChunkR];
#pragma unroll
                for (int u = 0; u < kChunkR; ++u) {
                    const int e = k + u * S + grp;
                    const uint32_t c = (uint32_t)__shfl_sync(kFull, my_col, e & 31);
                    x[u] = e < n ? __ldg(reinterpret_cast<const uint4 *>(x_base + (c * (uint32_t)(BT * sizeof(T)) + lane_b)))
                                 : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int u = 0; u < kChunkR; ++u) Gt::fma(acc, __shfl_sync(kFull, my_val, (k + u * S + grp) & 31), x[u]);
            }
        }
#pragma unroll
        for (int o = 16; o >= G; o >>= 1)
#pragma unroll
            for (int q = 0; q < V; ++q) acc[q] += __shfl_xor_sync(kFull, acc[q], o);
        if (lane < G) {
            const int flags = vld(me.flags);
            const bool span_lo = (i == vld(me.is)) && (flags & 1), span_hi = (i == vld(me.ie)) && (flags & 2);
            if (span_lo || span_hi) {
                float *slot = span_lo ? s_first[warp] : s_last[warp];
#pragma unroll
                for (int q = 0; q < V; ++q) slot[lane * V + q] = acc[q];
            } else if (i < vld(me.ie)) {
                finish_row<T, BT>(a, vld(s_r0) + i, 0, lane * V, acc);
            }
        }
    }
    __syncthreads();
    const int b = warp + 1;
    if (lane < G && b < kWarps && cut(b)) {
        int fb = b;
        while (fb > 1 && s_bi[fb - 1] == s_bi[fb] && cut(fb - 1)) --fb;
        if (fb == b) {
            const int row = s_bi[b], off = lane * V;
            float sum[V];
#pragma unroll
            for (int q = 0; q < V; ++q) sum[q] = s_last[b - 1][off + q];
            for (int w = b;; ++w) {
#pragma unroll
                for (int q = 0; q < V; ++q) sum[q] += s_first[w][off + q];
                if (!(w + 1 < kWarps && s_bi[w + 1] == row && cut(w + 1))) break;
            }
            finish_row<T, BT>(a, s_r0 + row, 0, off, sum);
        }
    }
}

// ---- a step without synapses ---------------------------------------------------------------------
// R_{t-1} is empty (the first step): every row is the epilogue alone, y = k (+ drive).  One warp per
// (row, tile), rows fastest, so consecutive warps write consecutive 512-byte lines of the tile.
template <typename T>
__global__ void __launch_bounds__(256) step_kernel_nosyn(const StepArgs a, int64_t tiles) {
    constexpr int V = Lane<T>::V;
    constexpr int BT = 32 * V;
    const int lane = threadIdx.x & 31;
    const int64_t total = (int64_t)a.n_rows * tiles;
    const float zero[V] = {};
    for (int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < total;
         w += ((int64_t)gridDim.x * blockDim.x) >> 5)
        finish_row<T, BT>(a, (int)(w % a.n_rows), w / a.n_rows, lane * V, zero);
}

// Sub-matrices whose mean row is shorter than this take the short-row kernel.
constexpr int64_t kShortRowDegree = 16;

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
    // Short rows (configuration 3's step 2: 7.3 synapses per row) take the two-tile kernel; a step without
    // synapses the epilogue alone (all three give bitwise the same results); a narrow inference batch the
    // narrow kernel (the same sums in another order).
    if (a.nnz == 0) {
        step_kernel_nosyn<T><<<grid_for((int64_t)a.n_rows * tiles * 32, 256, 148 * 64), 256, 0, s>>>(a, tiles);
    } else {
        // the gathers address a tile's slab with 32-bit byte offsets
        AFB_CHECK(a.ts_in * (int64_t)sizeof(T) <= (int64_t)UINT32_MAX, "a step's state tile exceeds 4 GB");
        constexpr int V = Lane<T>::V;
        if (!a.y_out && a.batch <= 16 * V) {          // a narrow inference batch: G lanes per synapse
            const int g = a.batch <= V ? 1 : a.batch <= 2 * V ? 2 : a.batch <= 4 * V ? 4 : a.batch <= 8 * V ? 8 : 16;
            const unsigned grid = (unsigned)a.n_items;
            switch (g) {
                case 1: step_kernel_narrow<T, TV, 1><<<grid, kWarps * 32, 0, s>>>(a); break;
                case 2: step_kernel_narrow<T, TV, 2><<<grid, kWarps * 32, 0, s>>>(a); break;
                case 4: step_kernel_narrow<T, TV, 4><<<grid, kWarps * 32, 0, s>>>(a); break;
                case 8: step_kernel_narrow<T, TV, 8><<<grid, kWarps * 32, 0, s>>>(a); break;
                default: step_kernel_narrow<T, TV, 16><<<grid, kWarps * 32, 0, s>>>(a); break;
            }
        } else if (a.nnz < kShortRowDegree * (int64_t)a.n_rows) {
            const int64_t pairs = (tiles + 1) / 2;
            step_kernel_pair<T, TV><<<(unsigned)(pairs * a.n_items), kWarps * 32, 0, s>>>(a);
        } else {
            step_kernel<T, TV><<<(unsigned)blocks, kWarps * 32, 0, s>>>(a);
        }
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
