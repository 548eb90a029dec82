// The fused light-cone step: one CSR SpMM over a batch tile with the whole state update in its
// epilogue (chessfly/brain.py:273-277 float16 deviation, brain.py:310-314 float32).
//
// Layout.  State and drive are (rows, batch) row-major; a CTA owns one batch tile of kTile = 16
// lanes x 16 bytes (128 half or 64 float columns) and one "item" -- a contiguous run of rows whose
// cost (edges + 4 per row) is about kItemCost.  blockIdx.x = tile * n_items + k, so all items of a
// tile run before the next tile starts: the gathered slab R_{t-1} x tile stays resident in L2.
//
// Load balance.  Inside a CTA the item's rows and edges are split evenly over the 8 warps by the
// merge-path partition of Merrill & Garland ("Merge-based parallel sparse matrix-vector
// multiplication", SC'16): the merge of row ends with edge indices is cut into equal diagonals, so a
// 5,000-synapse row and 60 short rows cost the same.  A row cut by warp boundaries leaves one partial
// per warp in shared memory; after a barrier one warp sums them in warp order and finishes the row,
// so results are bitwise reproducible and independent of the batch width.
//
// Gather.  A half-warp covers the tile with one 16-byte load per lane per edge; the two half-warps
// take alternate edges of the same row and are summed with one xor-shuffle at the row end.  Column
// indices and values are loaded 32 edges at a time, coalesced, and broadcast with shuffles.
// Accumulation is float32 in every mode.
#include "internal.cuh"

namespace afb {
namespace {

constexpr int kWarps = 8;
constexpr int kLanesPerEdge = 16;
constexpr int kUnroll = 4;
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

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

// Finish one row: epilogue of the state update, writes V columns of this lane.
template <typename T>
__device__ __forceinline__ void finish_row(const StepArgs &a, int row, int64_t col0, float (&acc)[Lane<T>::V]) {
    constexpr int V = Lane<T>::V;
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
        Lane<T>::load(static_cast<const T *>(a.x_in) + (int64_t)prev * a.ld_in + col0, p);
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
    Lane<T>::store(static_cast<T *>(a.x_out) + (int64_t)row * a.ld_out + col0, o);
}

template <typename T, typename TV>
__global__ void __launch_bounds__(kWarps * 32) step_kernel(const StepArgs a) {
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
    const int L_ = nrows + nnz;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = lane >> 4, sub = lane & 15;
    const int64_t col0 = tile * BT + sub * V;

    if (tid <= kWarps) {  // merge-path coordinates of the warp boundaries
        const int d = (int)(((int64_t)L_ * tid) / kWarps);
        int lo = d - nnz > 0 ? d - nnz : 0, hi = d < nrows ? d : nrows;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (__ldg(a.crow + r0 + mid + 1) - e0 <= d - mid - 1) lo = mid + 1;
            else hi = mid;
        }
        s_bi[tid] = lo;
        s_bj[tid] = d - lo;
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
    const T *x_in = static_cast<const T *>(a.x_in);
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
            for (int k = 0; k < n; k += 2 * kUnroll) {
                float x[kUnroll][V];
                float v[kUnroll];
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    const int kk = k + 2 * u + grp;
                    const int c = __shfl_sync(kFull, my_col, kk & 31);
                    v[u] = __shfl_sync(kFull, my_val, kk & 31);
                    if (kk < n) {
                        L::load(x_in + (int64_t)c * a.ld_in + col0, x[u]);
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
        for (int q = 0; q < V; ++q) acc[q] += __shfl_xor_sync(kFull, acc[q], 16);
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
            finish_row<T>(a, r0 + i, col0, acc);
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
        finish_row<T>(a, r0 + row, col0, acc);
    }
}

__global__ void output_kernel(int n_out, const int *__restrict__ src, const float *__restrict__ base, int add_base,
                              const void *__restrict__ state, int is_half, int64_t ld_state, float *__restrict__ out,
                              int64_t ld_out, int64_t batch) {
    for (int o = blockIdx.x; o < n_out; o += gridDim.x) {
        const int s = src ? src[o] : (state ? o : -1);   // no map: copy row for row, or fill
        const float b0 = base ? base[o] : 0.f;
        for (int64_t c = threadIdx.x; c < batch; c += blockDim.x) {
            float v = b0;
            if (s >= 0) {
                const float x = is_half ? __half2float(static_cast<const __half *>(state)[(int64_t)s * ld_state + c])
                                        : static_cast<const float *>(state)[(int64_t)s * ld_state + c];
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

template <typename T, typename TV>
void launch(const StepArgs &a, cudaStream_t s) {
    constexpr int BT = kLanesPerEdge * Lane<T>::V;
    if (a.n_items == 0 || a.batch == 0) return;
    const int64_t tiles = (a.batch + BT - 1) / BT;
    const int64_t blocks = tiles * a.n_items;
    AFB_CHECK(blocks < (1LL << 31), "grid too large: reduce the batch");
    step_kernel<T, TV><<<(unsigned)blocks, kWarps * 32, 0, s>>>(a);
    AFB_LAUNCHED();
}

}  // namespace

void launch_step_f32(const StepArgs &a, cudaStream_t s) { launch<float, float>(a, s); }
void launch_step_dev16(const StepArgs &a, cudaStream_t s) { launch<__half, __half>(a, s); }

void launch_output(int n_out, const int *src, const float *base, int add_base, const void *state, int state_is_half,
                   int64_t ld_state, float *out, int64_t ld_out, int64_t batch, cudaStream_t s) {
    if (n_out == 0 || batch == 0) return;
    const int threads = 256;
    const int grid = n_out < 148 * 64 ? n_out : 148 * 64;
    output_kernel<<<grid, threads, 0, s>>>(n_out, src, base, add_base, state, state_is_half, ld_state, out, ld_out, batch);
    AFB_LAUNCHED();
}

void launch_spmv(int n_rows, const int *crow, const int *col, const float *val, const float *x, float *y, cudaStream_t s) {
    if (n_rows == 0) return;
    spmv_kernel<<<grid_for((int64_t)n_rows * 32, 256, 148 * 64), 256, 0, s>>>(n_rows, crow, col, val, x, y);
    AFB_LAUNCHED();
}

}  // namespace afb
