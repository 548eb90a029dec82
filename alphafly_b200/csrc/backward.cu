// Training path: the float32 light-cone forward that keeps what the backward needs, and the backward.
//
// Forward (chessfly/brain.py:289-294, 315-329 with grad enabled): the fused step kernel in float32,
// writing per step the new state h_t and the pre-clamp drive y_t = A_t h_{t-1} + k_t + u (both
// tile-major, kept in the caller's `saved` buffer).
//
// Backward, per step t = T..1 (the autograd graph of forward_io and _constants, brain.py:238-252,
// 315-329, with torch's rules: lerp(s, e, a) passes (1 - a) g, a g and (e - s) g; clamp passes the
// gradient where lo <= y <= hi):
//   bwd_rows     g_y = a g_h [lo <= y <= hi]; per row sum_b g_h (x - p) -> dL/dalpha,
//                sum_b g_y -> dL/dk_t, sum_b (1 - a) g_h -> dL/dc_{t-1} for rows not carried;
//                g_y of fed rows -> dL/du_in
//   bwd_spmm_t   over the transposed sub-matrix (rows of R_{t-1}): dL/dh_{t-1} = A_t^T g_y + (1 - a) g_h of
//                the row carried from it, and, from the same gathered g_y rows, the per-synapse products
//                sum_b g_y[post, b] h_{t-1}[pre, b] of this batch tile (SDDMM)
//   bwd_edge_sum the SDDMM partials summed over tiles in a fixed order -> dL/dw
//   constants    the batch-1 recurrence of the resting trajectory c_t and the constant drive k_t:
//                k_t = (W c_{t-1} + b)[R_t] - A_t c_{t-1}[R_{t-1}],  c_t = lerp(c_{t-1}, clamp(W c_{t-1} + b), alpha)
// The outputs are dL/du_in, dL/dw (w = sign * w0 * exp(log_gain)), dL/db and dL/dalpha; the chain rule
// to log_gain and alpha_logit is the caller's (two elementwise products).
#include <algorithm>

#include "internal.cuh"

namespace afb {
namespace {

constexpr int kBlock = 256;
constexpr unsigned kFull = 0xffffffffu;

inline size_t align256(size_t b) { return (b + 255) / 256 * 256; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

__global__ void zero_kernel(float *__restrict__ p, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = 0.f;
}

// Output gradient into the last step: rows inside R_T go to g_h_T; outputs outside the cone are the
// constant c_T[out_idx] and send their batch sum to dL/dc_T.
__global__ void bwd_out(int n_out, const int *__restrict__ out_row, const int *__restrict__ out_idx,
                        const float *__restrict__ g_out, int64_t ld_g, int64_t batch, float *__restrict__ gh, int64_t ts,
                        int bt, float *__restrict__ gc_T) {
    __shared__ float red[kBlock / 32];
    for (int o = blockIdx.x; o < n_out; o += gridDim.x) {
        const int r = out_row[o];
        if (r >= 0) {
            for (int64_t c = threadIdx.x; c < batch; c += blockDim.x)
                atomicAdd(&gh[(c / bt) * ts + (int64_t)r * bt + c % bt], g_out[(int64_t)o * ld_g + c]);
        } else {
            float sum = 0.f;
            for (int64_t c = threadIdx.x; c < batch; c += blockDim.x) sum += g_out[(int64_t)o * ld_g + c];
            sum = warp_sum(sum);
            if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
            __syncthreads();
            if (threadIdx.x == 0) {
                float t = 0.f;
                for (int k = 0; k < kBlock / 32; ++k) t += red[k];
                atomicAdd(&gc_T[out_idx[o]], t);
            }
            __syncthreads();
        }
    }
}

// One warp per row of R_t (see the file comment).
__global__ void bwd_rows(int n_rows, const RowConst *__restrict__ rc, const int *__restrict__ rows, int64_t batch,
                         int64_t cols, const float *__restrict__ gh, const float *__restrict__ y, int64_t ts,
                         const float *__restrict__ h_prev, int64_t ts_prev, float *__restrict__ gy,
                         float *__restrict__ g_alpha, float *__restrict__ gc_prev, float *__restrict__ g_k,
                         float *__restrict__ g_u, int64_t ld_gu, int gu_vec) {
    constexpr int bt = 128;                      // float32 batch tile: one float4 per lane
    const int lane = threadIdx.x & 31;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < n_rows; r += (gridDim.x * blockDim.x) >> 5) {
        const RowConst q = rc[r];
        float s_alpha = 0.f, s_k = 0.f, s_pc = 0.f;
        for (int64_t c0 = lane * 4; c0 < cols; c0 += bt) {
            const int64_t tile = c0 / bt, at = tile * ts + (int64_t)r * bt + lane * 4;
            const float4 g4 = *reinterpret_cast<const float4 *>(gh + at), y4 = *reinterpret_cast<const float4 *>(y + at);
            const float4 p4 = q.prev >= 0 ? *reinterpret_cast<const float4 *>(h_prev + tile * ts_prev + (int64_t)q.prev * bt + lane * 4)
                                          : make_float4(q.pc, q.pc, q.pc, q.pc);
            const float g[4] = {g4.x, g4.y, g4.z, g4.w}, yv[4] = {y4.x, y4.y, y4.z, y4.w}, p[4] = {p4.x, p4.y, p4.z, p4.w};
            float g_y[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                g_y[k] = 0.f;
                if (c0 + k < batch) {
                    const float x = fminf(fmaxf(yv[k], q.lo), q.hi) + q.e;
                    g_y[k] = (yv[k] >= q.lo && yv[k] <= q.hi) ? q.a * g[k] : 0.f;
                    s_alpha += g[k] * (x - p[k]);
                    s_k += g_y[k];
                    s_pc += (1.f - q.a) * g[k];
                }
            }
            *reinterpret_cast<float4 *>(gy + at) = make_float4(g_y[0], g_y[1], g_y[2], g_y[3]);
            if (q.usrc >= 0) {
                float *gu = g_u + (int64_t)q.usrc * ld_gu + c0;
                if (gu_vec && c0 + 4 <= batch) {
                    float4 v = *reinterpret_cast<float4 *>(gu);
                    v.x += g_y[0]; v.y += g_y[1]; v.z += g_y[2]; v.w += g_y[3];
                    *reinterpret_cast<float4 *>(gu) = v;
                } else {
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        if (c0 + k < batch) gu[k] += g_y[k];
                }
            }
        }
        s_alpha = warp_sum(s_alpha);
        s_k = warp_sum(s_k);
        s_pc = warp_sum(s_pc);
        if (lane == 0) {
            g_alpha[rows[r]] += s_alpha;
            g_k[r] = s_k;
            if (q.prev < 0 && gc_prev) gc_prev[rows[r]] += s_pc;
        }
    }
}

// One warp per (row j of R_{t-1}, float32 batch tile of 128 columns; lane = 4 columns).
// Sums of four values over the warp, reduce-scatter style: 6 shuffles instead of 4 x 5.  Lane 8 q ends
// with the sum of v_q (q = 0..3); the addition order is fixed, so results are reproducible.
__device__ __forceinline__ float warp_sum4(float v0, float v1, float v2, float v3, int lane) {
    const bool h16 = lane & 16, h8 = lane & 8;
    float k0 = h16 ? v2 : v0, k1 = h16 ? v3 : v1;
    const float s0 = h16 ? v0 : v2, s1 = h16 ? v1 : v3;
    k0 += __shfl_xor_sync(0xffffffffu, s0, 16);
    k1 += __shfl_xor_sync(0xffffffffu, s1, 16);
    float k = h8 ? k1 : k0;
    k += __shfl_xor_sync(0xffffffffu, h8 ? k0 : k1, 8);
    k += __shfl_xor_sync(0xffffffffu, k, 4);
    k += __shfl_xor_sync(0xffffffffu, k, 2);
    k += __shfl_xor_sync(0xffffffffu, k, 1);
    return k;
}

// Transposed step of the backward, one warp per row j of R_{t-1} (taken longest first from `order`, so
// that the longest rows do not finish last) and one 128-column float32 tile:
//   g_prev[j] = sum_e w_e gy[post_e] + (1 - a_i) gh[i]      (i = the row of R_t carrying j, if any)
//   part[tile][e] = sum over the tile's columns of h_prev[j] * gy[post_e]      (the SDDMM of dL/dw)
// Column indices and values come 32 edges at a time (coalesced, broadcast with shuffles); the rows of gy
// are gathered 4 edges at a time (4 loads in flight per lane), and the 4 edges' dot products are reduced
// together (warp_sum4).
__global__ void __launch_bounds__(256, 5) bwd_spmm_t(int n_cols, const int *__restrict__ order, const int *__restrict__ t_crow,
                                                   const int *__restrict__ t_col,
                                                   const float *__restrict__ val_t, const float *__restrict__ gy,
                                                   const float *__restrict__ gh, int64_t ts, const RowConst *__restrict__ rc,
                                                   const int *__restrict__ inv, const float *__restrict__ h_prev,
                                                   int64_t ts_prev, float *__restrict__ gh_prev, float *__restrict__ part,
                                                   int64_t nnz) {
    constexpr int bt = 128;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int jj = blockIdx.x * (blockDim.x >> 5) + warp;
    if (jj >= n_cols) return;
    const int j = __ldg(order + jj);
    const int64_t tile = blockIdx.y;
    const int off = lane * 4;
    const float4 hj = *reinterpret_cast<const float4 *>(h_prev + tile * ts_prev + (int64_t)j * bt + off);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const float *gy_tile = gy + tile * ts + off;
    float *part_tile = part + tile * nnz;
    const int e0 = t_crow[j], e1 = t_crow[j + 1];
    for (int base = e0; base < e1; base += 32) {
        const int n = e1 - base < 32 ? e1 - base : 32;
        const int my_r = lane < n ? __ldg(t_col + base + lane) : 0;
        const float my_v = lane < n ? __ldg(val_t + base + lane) : 0.f;
        for (int k = 0; k < n; k += 4) {
            float4 g[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int r = __shfl_sync(0xffffffffu, my_r, (k + u) & 31);
                g[u] = k + u < n ? *reinterpret_cast<const float4 *>(gy_tile + (int64_t)r * bt) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            float d[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float v = __shfl_sync(0xffffffffu, my_v, (k + u) & 31);
                acc.x = fmaf(v, g[u].x, acc.x);
                acc.y = fmaf(v, g[u].y, acc.y);
                acc.z = fmaf(v, g[u].z, acc.z);
                acc.w = fmaf(v, g[u].w, acc.w);
                d[u] = g[u].x * hj.x + g[u].y * hj.y + g[u].z * hj.z + g[u].w * hj.w;
            }
            const float s = warp_sum4(d[0], d[1], d[2], d[3], lane);
            const int q = lane >> 3;
            if ((lane & 7) == 0 && k + q < n) part_tile[base + k + q] = s;
        }
    }
    const int i = inv[j];
    if (i >= 0) {
        const float keep = 1.f - rc[i].a;
        const float4 g = *reinterpret_cast<const float4 *>(gh + tile * ts + (int64_t)i * bt + off);
        acc.x = fmaf(keep, g.x, acc.x);
        acc.y = fmaf(keep, g.y, acc.y);
        acc.z = fmaf(keep, g.z, acc.z);
        acc.w = fmaf(keep, g.w, acc.w);
    }
    *reinterpret_cast<float4 *>(gh_prev + tile * ts_prev + (int64_t)j * bt + off) = acc;
}

// dL/dw of the step: the per-tile partials of each transpose position summed in tile order (deterministic),
// added at that synapse's edge of W (t_edges = edges[t_order], one gather instead of two dependent ones).
__global__ void bwd_edge_sum(int64_t nnz, int64_t tiles, const float *__restrict__ part, const int *__restrict__ t_edges,
                             float *__restrict__ g_w) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < nnz; e += (int64_t)gridDim.x * blockDim.x) {
        float s = 0.f;
        for (int64_t t = 0; t < tiles; ++t) s += part[t * nnz + e];
        g_w[t_edges[e]] += s;
    }
}

// ---- the batch-1 constants ----------------------------------------------------------------------
__global__ void scatter_set(int m, const int *__restrict__ rows, const float *__restrict__ v, float *__restrict__ dst) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < m; i += gridDim.x * blockDim.x) dst[rows[i]] = v[i];
}

// gc[rows_prev[j]] += scale * sum_e val_t[e] x[t_col[e]]  (one warp per row of a transposed CSR)
__global__ void spmv_t_acc(int n_rows, const int *__restrict__ t_crow, const int *__restrict__ t_col,
                           const float *__restrict__ val_t, const float *__restrict__ x, const int *__restrict__ map,
                           float scale, float *__restrict__ dst) {
    const int lane = threadIdx.x & 31;
    for (int j = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; j < n_rows; j += (gridDim.x * blockDim.x) >> 5) {
        float s = 0.f;
        for (int e = t_crow[j] + lane; e < t_crow[j + 1]; e += 32) s = fmaf(val_t[e], x[t_col[e]], s);
        s = warp_sum(s);
        if (lane == 0) dst[map ? map[j] : j] += scale * s;
    }
}

// g_w[edge(e)] += scale * g[row(e)] * c[col(e)] over the entries e of a CSR
__global__ void sddmm1_acc(int64_t nnz, const int *__restrict__ post, const int *__restrict__ col,
                           const int *__restrict__ edges, const float *__restrict__ g, const float *__restrict__ c,
                           const int *__restrict__ col_map, float scale, float *__restrict__ g_w) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < nnz; e += (int64_t)gridDim.x * blockDim.x) {
        const int j = col[e];
        g_w[edges ? edges[e] : e] += scale * g[post[e]] * c[col_map ? col_map[j] : j];
    }
}

// c_t = lerp(c_{t-1}, clamp(z_t, 0, h_max), alpha), z_t = W c_{t-1} + b  (kfull), per neuron
__global__ void bwd_resting(int64_t n, const float *__restrict__ z, const float *__restrict__ c_prev,
                            const float *__restrict__ alpha, float h_max, const float *__restrict__ gc,
                            float *__restrict__ gc_prev, float *__restrict__ g_sb, float *__restrict__ g_alpha,
                            float *__restrict__ g_bias) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float g = gc[i], a = alpha[i], zi = z[i];
        const float gz = (zi >= 0.f && zi <= h_max) ? a * g : 0.f;
        const float sb = g_sb[i] + gz;
        g_sb[i] = sb;
        gc_prev[i] += (1.f - a) * g;
        g_alpha[i] += g * (fminf(fmaxf(zi, 0.f), h_max) - c_prev[i]);
        g_bias[i] += sb;
    }
}

size_t train_saved_bytes(const afb_cone *c, int64_t batch) {
    const int64_t ld = padded_ld(batch, 4);
    size_t b = 0;
    for (int t = 1; t <= c->steps; ++t) b += 2 * align256((size_t)c->st[t].n_rows * ld * 4);
    return b + 256;
}

int64_t max_nnz(const afb_cone *c) {
    int64_t m = 0;
    for (int t = 1; t <= c->steps; ++t) m = std::max<int64_t>(m, c->st[t].op.nnz);
    return m;
}

}  // namespace
}  // namespace afb

using namespace afb;

extern "C" {

size_t afb_cone_train_workspace(const afb_cone *c, int64_t batch) {
    if (!c || batch < 0) return 0;
    return train_saved_bytes(c, batch);
}

int afb_cone_forward_train(const afb_cone *c, const float *u_in, int64_t ld_u, int64_t batch, float *out, int64_t ld_out,
                           void *saved, size_t saved_bytes, void *stream) {
    return guarded([&] {
        AFB_CHECK(c, "cone is NULL");
        if (!c->ready[AFB_MODE_F32])
            throw Error(AFB_ESTATE, "afb_cone_set_weights(AFB_MODE_F32) has not been called since the cone was built");
        AFB_CHECK(batch >= 0 && ld_u >= batch && ld_out >= batch, "bad batch or leading dimension");
        AFB_CHECK(out && (c->n_in == 0 || batch == 0 || u_in), "NULL pointer");
        AFB_CHECK(saved_bytes >= train_saved_bytes(c, batch), "saved-state buffer too small");
        if (batch == 0) return;
        check_aligned(saved, 256, "saved");
        cudaStream_t s = as_stream(stream);
        const int64_t ld = padded_ld(batch, 4), bt = tile_cols(4);
        char *p = static_cast<char *>(saved);
        const int u_vec_ok = (ld_u % 4 == 0) && (reinterpret_cast<uintptr_t>(u_in) % 16 == 0);
        const void *x_in = p;   // never read at step 1
        int64_t ts_in = 0;
        for (int t = 1; t <= c->steps; ++t) {
            const Step &sp = c->st[t];
            const size_t slab = align256((size_t)sp.n_rows * ld * 4);
            float *h = reinterpret_cast<float *>(p);
            float *y = reinterpret_cast<float *>(p + slab);
            StepArgs a{};
            a.crow = sp.op.crow.get();
            a.col = sp.op.col.get();
            a.val = sp.val32.get();
            a.item_rows = sp.op.item_rows.get();
            a.item_order = sp.op.item_order.get();
            a.bounds = sp.op.bounds.get();
            a.n_items = sp.op.n_items;
            a.item_rows_fine = sp.op.fine.item_rows.get();
            a.item_order_fine = sp.op.fine.item_order.get();
            a.bounds_fine = sp.op.fine.bounds.get();
            a.n_items_fine = sp.op.fine.n_items;
            a.n_rows = sp.op.n_rows;
            a.nnz = sp.op.nnz;
            a.rc = sp.rc[AFB_MODE_F32].get();
            a.x_in = x_in;
            a.ts_in = ts_in;
            a.u = u_in;
            a.ld_u = ld_u;
            a.u_vec_ok = u_vec_ok;
            a.x_out = h;
            a.ts_out = (int64_t)sp.n_rows * bt;
            a.batch = batch;
            a.err = c->err.get();
            a.y_out = y;
            launch_step_f32(a, s);
            x_in = h;
            ts_in = a.ts_out;
            p += 2 * slab;
        }
        launch_output((int)c->n_out, c->out_row.get(), c->out_base[AFB_MODE_F32].get(), 0, x_in, 0, ts_in, out, ld_out,
                      batch, s);
    });
}

size_t afb_cone_backward_workspace(const afb_cone *c, int64_t batch) {
    if (!c || batch < 0) return 0;
    const int64_t ld = padded_ld(batch, 4), tiles = ld / tile_cols(4);
    return 3 * align256((size_t)c->max_rows * ld * 4) + align256((size_t)tiles * max_nnz(c) * 4) +
           align256((size_t)c->max_rows * 4) + align256((size_t)(c->steps + 1) * c->n * 4) + align256((size_t)c->n * 4) + 256;
}

int afb_cone_backward(const afb_cone *c, const float *g_out, int64_t ld_g, int64_t batch, const void *saved,
                      size_t saved_bytes, float *g_u_in, int64_t ld_gu, float *g_w, float *g_bias, float *g_alpha,
                      void *workspace, size_t workspace_bytes, void *stream) {
    return guarded([&] {
        AFB_CHECK(c, "cone is NULL");
        if (!c->ready[AFB_MODE_F32])
            throw Error(AFB_ESTATE, "afb_cone_set_weights(AFB_MODE_F32) has not been called since the cone was built");
        AFB_CHECK(batch >= 0 && ld_g >= batch && ld_gu >= batch, "bad batch or leading dimension");
        AFB_CHECK(g_out && g_w && g_bias && g_alpha && (c->n_in == 0 || g_u_in), "NULL pointer");
        AFB_CHECK(saved_bytes >= train_saved_bytes(c, batch), "saved-state buffer too small");
        AFB_CHECK(workspace_bytes >= afb_cone_backward_workspace(c, batch), "workspace too small");
        check_aligned(workspace, 256, "workspace");
        cudaStream_t s = as_stream(stream);
        const int64_t n = c->n, e = c->e, T = c->steps;
        const int64_t ld = padded_ld(batch, 4), bt = tile_cols(4), tiles = ld / bt;
        AFB_CHECK(bt == 128, "the backward kernels assume 128-column float32 tiles");
        const int gu_vec = ld_gu % 4 == 0 && reinterpret_cast<uintptr_t>(g_u_in) % 16 == 0;
        AFB_CHECK(bt == 128, "the backward kernels assume 128-column float32 tiles");
        char *ws = static_cast<char *>(workspace);
        const size_t state_b = align256((size_t)c->max_rows * ld * 4);
        float *gh[2] = {reinterpret_cast<float *>(ws), reinterpret_cast<float *>(ws + state_b)};
        float *gy = reinterpret_cast<float *>(ws + 2 * state_b);
        float *part = reinterpret_cast<float *>(ws + 3 * state_b);
        char *q = ws + 3 * state_b + align256((size_t)tiles * max_nnz(c) * 4);
        float *g_k = reinterpret_cast<float *>(q);
        q += align256((size_t)c->max_rows * 4);
        float *gc = reinterpret_cast<float *>(q);   // (T + 1) x n: dL/dc_t
        q += align256((size_t)(T + 1) * n * 4);
        float *g_sb = reinterpret_cast<float *>(q);

        auto zero = [&](float *p, int64_t m) {
            if (m > 0) zero_kernel<<<grid_for(m, kBlock), kBlock, 0, s>>>(p, m);
        };
        zero(g_w, e);
        zero(g_bias, n);
        zero(g_alpha, n);
        zero(gc, (T + 1) * n);
        if (c->n_in) AFB_CUDA(cudaMemset2DAsync(g_u_in, ld_gu * 4, 0, batch * 4, c->n_in, s));
        AFB_LAUNCHED();
        if (batch == 0) return;

        // per-step slabs of the saved forward
        std::vector<const float *> h(T + 1, nullptr), y(T + 1, nullptr);
        const char *p = static_cast<const char *>(saved);
        for (int t = 1; t <= T; ++t) {
            const size_t slab = align256((size_t)c->st[t].n_rows * ld * 4);
            h[t] = reinterpret_cast<const float *>(p);
            y[t] = reinterpret_cast<const float *>(p + slab);
            p += 2 * slab;
        }
        // output gradient
        {
            const int64_t ts = (int64_t)c->st[T].n_rows * bt;
            zero(gh[T & 1], c->st[T].n_rows * ld);
            bwd_out<<<std::min<int64_t>(c->n_out, 148 * 16), kBlock, 0, s>>>((int)c->n_out, c->out_row.get(), c->out_idx.get(),
                                                                           g_out, ld_g, batch, gh[T & 1], ts, (int)bt,
                                                                           gc + T * n);
            AFB_LAUNCHED();
        }
        for (int t = (int)T; t >= 1; --t) {
            const Step &sp = c->st[t], &pv = c->st[t - 1];
            const Csr &m = sp.op;
            const int64_t ts = (int64_t)sp.n_rows * bt, ts_prev = (int64_t)pv.n_rows * bt;
            float *g_here = gh[t & 1], *g_prev = gh[(t + 1) & 1];
            const float *c_prev = c->resting.get() + (t - 1) * n;
            if (sp.n_rows) {
                bwd_rows<<<grid_for((int64_t)sp.n_rows * 32, kBlock, 148 * 64), kBlock, 0, s>>>(
                    sp.n_rows, sp.rc[AFB_MODE_F32].get(), sp.rows.get(), batch, ld, g_here, y[t], ts,
                    t > 1 ? h[t - 1] : nullptr, ts_prev, gy, g_alpha, gc + (t - 1) * n, g_k, g_u_in, ld_gu, gu_vec);
                AFB_LAUNCHED();
            }
            if (m.present && pv.n_rows) {
                dim3 grid((unsigned)((pv.n_rows + 7) / 8), (unsigned)tiles);
                bwd_spmm_t<<<grid, kBlock, 0, s>>>(pv.n_rows, m.t_heavy.get(), m.t_crow.get(), m.t_col.get(), sp.val32_t.get(), gy, g_here, ts,
                                                  sp.rc[AFB_MODE_F32].get(), sp.inv_prev.get(), h[t - 1], ts_prev, g_prev,
                                                  part, m.nnz);
                AFB_LAUNCHED();
                if (m.nnz) {
                    bwd_edge_sum<<<grid_for(m.nnz, kBlock), kBlock, 0, s>>>(m.nnz, tiles, part, m.t_edges.get(), g_w);
                    AFB_LAUNCHED();
                }
            }
            // the constants of step t (batch 1)
            zero(g_sb, n);
            if (sp.n_rows) {
                scatter_set<<<grid_for(sp.n_rows, kBlock), kBlock, 0, s>>>(sp.n_rows, sp.rows.get(), g_k, g_sb);
                AFB_LAUNCHED();
            }
            if (m.present && m.nnz) {   // k_t -= A_t c_{t-1}[R_{t-1}]
                spmv_t_acc<<<grid_for((int64_t)pv.n_rows * 32, kBlock, 148 * 64), kBlock, 0, s>>>(
                    pv.n_rows, m.t_crow.get(), m.t_col.get(), sp.val32_t.get(), g_k, pv.rows.get(), -1.f, gc + (t - 1) * n);
                sddmm1_acc<<<grid_for(m.nnz, kBlock), kBlock, 0, s>>>(m.nnz, m.post.get(), m.col.get(), m.edges.get(), g_k,
                                                                     c_prev, pv.rows.get(), -1.f, g_w);
                AFB_LAUNCHED();
            }
            bwd_resting<<<grid_for(n, kBlock), kBlock, 0, s>>>(n, c->kfull.get() + t * n, c_prev, c->alpha.get(),
                                                              c->h_max, gc + t * n, gc + (t - 1) * n, g_sb, g_alpha, g_bias);
            AFB_LAUNCHED();
            if (t > 1 && e) {   // z_t = W c_{t-1} + b
                spmv_t_acc<<<grid_for(n * 32, kBlock, 148 * 64), kBlock, 0, s>>>((int)n, c->full_tcrow.get(), c->full_tcol.get(),
                                                                              c->w_t.get(), g_sb, nullptr, 1.f,
                                                                              gc + (t - 1) * n);
                sddmm1_acc<<<grid_for(e, kBlock), kBlock, 0, s>>>(e, c->full_post.get(), c->full_col.get(), nullptr, g_sb,
                                                                 c_prev, nullptr, 1.f, g_w);
                AFB_LAUNCHED();
            }
        }
    });
}

}  // extern "C"
