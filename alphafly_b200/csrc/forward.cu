// Weight-version precompute and the inference drivers.
//
// afb_cone_set_weights restates the cached part of forward_io (chessfly/brain.py:257-270, 296-306)
// and _constants (brain.py:238-252) as a short kernel sequence: sigmoid(alpha_logit); the resting
// trajectory c_t by T full batch-1 SpMVs; per step the row constants of the chosen mode (for float32,
// k_t = (W c_{t-1} + b)[R_t] - A_t c_{t-1}[R_{t-1}] with one warp per row); the sub-matrix values
// w[edges].  afb_cone_forward then runs one fused step kernel per step and one output kernel.
#include <mutex>

#include "internal.cuh"

namespace afb {
namespace {

constexpr int kBlock = 256;

__global__ void edge_weights_kernel(int64_t e, const float *__restrict__ sign, const float *__restrict__ w0,
                                    const float *__restrict__ lg, float *__restrict__ w) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < e; i += (int64_t)gridDim.x * blockDim.x)
        w[i] = sign[i] * w0[i] * expf(lg[i]);
}

__global__ void sigmoid_kernel(int64_t n, const float *__restrict__ x, float *__restrict__ y) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = 1.f / (1.f + expf(-x[i]));
}

__device__ __forceinline__ float lerp_t(float s, float e, float w) {  // torch.lerp's two-branch form
    return w < 0.5f ? s + w * (e - s) : e - (e - s) * (1.f - w);
}

// k_full = (t > 1 ? W c_prev : 0) + b ;  c_next = lerp(c_prev, clamp(k_full, 0, h_max), alpha)
__global__ void resting_kernel(int64_t n, const float *__restrict__ wc, const float *__restrict__ bias,
                               const float *__restrict__ alpha, const float *__restrict__ c_prev, float h_max,
                               float *__restrict__ kfull, float *__restrict__ c_next) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float k = (wc ? wc[i] : 0.f) + bias[i];
        kfull[i] = k;
        c_next[i] = lerp_t(c_prev[i], fminf(fmaxf(k, 0.f), h_max), alpha[i]);
    }
}

__global__ void gather_values(int64_t m, const int *__restrict__ edges, const float *__restrict__ w,
                              float *__restrict__ v32, __half *__restrict__ v16) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x) {
        const float x = w[edges[i]];
        if (v32) v32[i] = x;
        if (v16) v16[i] = __float2half_rn(x);
    }
}

// One warp per row of R_t: the row constants of the step (see RowConst).
__global__ void row_constants(int n_rows, int mode, const int *__restrict__ rows, const int *__restrict__ prev,
                              const int *__restrict__ usrc, const int *__restrict__ crow, const int *__restrict__ col,
                              const float *__restrict__ val, const int *__restrict__ rows_prev,
                              const float *__restrict__ kfull, const float *__restrict__ c_prev,
                              const float *__restrict__ alpha, float h_max, RowConst *__restrict__ rc) {
    const int lane = threadIdx.x & 31;
    for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < n_rows; i += (gridDim.x * blockDim.x) >> 5) {
        const int r = rows[i];
        float sub = 0.f;
        if (mode == AFB_MODE_F32 && crow) {
            for (int e = crow[i] + lane; e < crow[i + 1]; e += 32) sub = fmaf(val[e], c_prev[rows_prev[col[e]]], sub);
#pragma unroll
            for (int o = 16; o; o >>= 1) sub += __shfl_xor_sync(0xffffffffu, sub, o);
        }
        if (lane == 0) {
            const float k = kfull[r];
            RowConst q;
            if (mode == AFB_MODE_F32) {
                q.kk = k - sub;
                q.lo = 0.f;
                q.hi = h_max;
                q.e = 0.f;
                q.pc = c_prev[r];
            } else {
                q.kk = 0.f;
                q.lo = -k;
                q.hi = h_max - k;
                q.e = k - fminf(fmaxf(k, 0.f), h_max);
                q.pc = 0.f;
            }
            q.a = alpha[r];
            q.prev = prev[i];
            q.usrc = usrc[i];
            rc[i] = q;
        }
    }
}

// Literal recurrence constants: kk = b, clamp to [0, h_max], prev = row (or -1 on the first step), usrc = row.
__global__ void graph_constants(int64_t n, const float *__restrict__ bias, const float *__restrict__ alpha_logit,
                                float h_max, RowConst *__restrict__ first, RowConst *__restrict__ rest) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        RowConst q;
        q.kk = bias[i];
        q.lo = 0.f;
        q.hi = h_max;
        q.e = 0.f;
        q.pc = 0.f;
        q.a = 1.f / (1.f + expf(-alpha_logit[i]));
        q.usrc = (int)i;
        q.prev = -1;
        first[i] = q;
        q.prev = (int)i;
        rest[i] = q;
    }
}

__global__ void gather_float(const float *__restrict__ table, const int *__restrict__ ids, float *__restrict__ out, int64_t m);
}  // namespace

void gather_floats(const float *table, const int *ids, float *out, int64_t m, cudaStream_t s) {
    if (m <= 0) return;
    gather_float<<<grid_for(m, kBlock), kBlock, 0, s>>>(table, ids, out, m);
    AFB_LAUNCHED();
}

namespace {
__global__ void gather_float(const float *__restrict__ table, const int *__restrict__ ids, float *__restrict__ out, int64_t m) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = table[ids[i]];
}

inline size_t align256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace
}  // namespace afb

using namespace afb;

extern "C" {

int afb_edge_weights(int64_t e, const float *sign, const float *w0, const float *log_gain, float *w, void *stream) {
    return guarded([&] {
        AFB_CHECK(e >= 0, "e must be >= 0");
        AFB_CHECK(e == 0 || (sign && w0 && log_gain && w), "NULL pointer");
        if (!e) return;
        edge_weights_kernel<<<grid_for(e, kBlock), kBlock, 0, as_stream(stream)>>>(e, sign, w0, log_gain, w);
        AFB_LAUNCHED();
    });
}

int afb_cone_set_weights(afb_cone *c, int mode, const float *w, const float *bias, const float *alpha_logit,
                         float h_max, void *stream) {
    return guarded([&] {
        AFB_CHECK(c, "cone is NULL");
        AFB_CHECK(mode == AFB_MODE_F32 || mode == AFB_MODE_DEV16, "unknown mode");
        AFB_CHECK((c->e == 0 || w) && bias && alpha_logit, "NULL pointer");
        cudaStream_t s = as_stream(stream);
        const int64_t n = c->n;
        const int T = c->steps;
        if (!c->alpha.p) {
            c->alpha.alloc(n);
            c->resting.alloc((size_t)(T + 1) * n);
            c->kfull.alloc((size_t)(T + 1) * n);
            c->wc.alloc(n);
        }
        if (!c->out_base[mode].p) c->out_base[mode].alloc(c->n_out);
        c->ready[mode] = false;
        c->h_max = h_max;
        sigmoid_kernel<<<grid_for(n, kBlock), kBlock, 0, s>>>(n, alpha_logit, c->alpha.get());
        AFB_CUDA(cudaMemsetAsync(c->resting.get(), 0, n * sizeof(float), s));
        float *wc = c->wc.get();
        for (int t = 1; t <= T; ++t) {
            const float *cp = c->resting.get() + (size_t)(t - 1) * n;
            if (t > 1) launch_spmv((int)n, c->full_crow.get(), c->full_col.get(), w, cp, wc, s);
            resting_kernel<<<grid_for(n, kBlock), kBlock, 0, s>>>(n, t > 1 ? wc : nullptr, bias, c->alpha.get(), cp,
                                                                 h_max, c->kfull.get() + (size_t)t * n,
                                                                 c->resting.get() + (size_t)t * n);
            AFB_LAUNCHED();
        }
        for (int t = 1; t <= T; ++t) {
            Step &sp = c->st[t];
            Csr &m = sp.op;
            if (mode == AFB_MODE_F32) {
                if (sp.val32.n < (size_t)m.nnz) sp.val32.alloc(m.nnz);
            } else if (sp.val16.n < (size_t)m.nnz) {
                sp.val16.alloc(m.nnz);
            }
            if (m.nnz) {
                gather_values<<<grid_for(m.nnz, kBlock), kBlock, 0, s>>>(m.nnz, m.edges.get(), w,
                                                                        mode == AFB_MODE_F32 ? sp.val32.get() : nullptr,
                                                                        mode == AFB_MODE_DEV16 ? sp.val16.get() : nullptr);
                AFB_LAUNCHED();
            }
            if (mode == AFB_MODE_F32 && m.nnz) {   // values of the transpose, for the training backward
                if (sp.val32_t.n < (size_t)m.nnz) sp.val32_t.alloc(m.nnz);
                gather_floats(sp.val32.get(), m.t_order.get(), sp.val32_t.get(), m.nnz, s);
            }
            if (sp.rc[mode].n < (size_t)sp.n_rows) sp.rc[mode].alloc(sp.n_rows);
            if (sp.n_rows) {
                row_constants<<<grid_for((int64_t)sp.n_rows * 32, kBlock, 148 * 64), kBlock, 0, s>>>(
                    sp.n_rows, mode, sp.rows.get(), sp.prev.get(), sp.usrc.get(), m.nnz ? m.crow.get() : nullptr,
                    m.col.get(), sp.val32.get(), c->st[t - 1].rows.get(), c->kfull.get() + (size_t)t * n,
                    c->resting.get() + (size_t)(t - 1) * n, c->alpha.get(), h_max, sp.rc[mode].get());
                AFB_LAUNCHED();
            }
        }
        if (mode == AFB_MODE_F32 && c->e) {
            if (!c->w_t.p) c->w_t.alloc(c->e);
            gather_floats(w, c->full_torder.get(), c->w_t.get(), c->e, s);
        }
        gather_float<<<grid_for(c->n_out, kBlock), kBlock, 0, s>>>(c->resting.get() + (size_t)T * n, c->out_idx.get(),
                                                                 c->out_base[mode].get(), c->n_out);
        AFB_LAUNCHED();
        c->ready[mode] = true;
    });
}

int afb_cone_resting(const afb_cone *c, int t, float *dst, void *stream) {
    return guarded([&] {
        AFB_CHECK(c && dst, "NULL pointer");
        AFB_CHECK(c->resting.p, "afb_cone_set_weights has not been called");
        AFB_CHECK(t >= 0 && t <= c->steps, "step out of range");
        AFB_CUDA(cudaMemcpyAsync(dst, c->resting.get() + (size_t)t * c->n, c->n * sizeof(float), cudaMemcpyDeviceToDevice,
                                 as_stream(stream)));
    });
}

size_t afb_cone_forward_workspace(const afb_cone *c, int mode, int64_t batch) {
    if (!c || batch < 0 || (mode != AFB_MODE_F32 && mode != AFB_MODE_DEV16)) return 0;
    const size_t es = mode == AFB_MODE_F32 ? 4 : 2;
    return 2 * align256((size_t)c->max_rows * padded_ld(batch, (int)es) * es) + 256;
}

int afb_cone_forward_timed(const afb_cone *c, int mode, const void *u_in, int64_t ld_u, int64_t batch, float *out,
                           int64_t ld_out, void *workspace, size_t workspace_bytes, void *const *events, void *stream) {
    return guarded([&] {
        AFB_CHECK(c, "cone is NULL");
        AFB_CHECK(mode == AFB_MODE_F32 || mode == AFB_MODE_DEV16, "unknown mode");
        if (!c->ready[mode])
            throw Error(AFB_ESTATE, "afb_cone_set_weights has not been called for this mode since the last weight change");
        AFB_CHECK(batch >= 0, "batch must be >= 0");
        AFB_CHECK(ld_u >= batch && ld_out >= batch, "leading dimensions must be >= batch");
        AFB_CHECK(out, "out is NULL");
        AFB_CHECK(c->n_in == 0 || batch == 0 || u_in, "u_in is NULL");
        AFB_CHECK(workspace_bytes >= afb_cone_forward_workspace(c, mode, batch), "workspace too small");
        if (batch == 0) return;
        check_aligned(workspace, 256, "workspace");
        cudaStream_t s = as_stream(stream);
        const size_t es = mode == AFB_MODE_F32 ? 4 : 2;
        const int64_t ld = padded_ld(batch, (int)es);
        char *ws = static_cast<char *>(workspace);
        void *buf[2] = {ws, ws + align256((size_t)c->max_rows * ld * es)};
        const int vec = mode == AFB_MODE_F32 ? 4 : 8;
        const int u_vec_ok = (ld_u % vec == 0) && (reinterpret_cast<uintptr_t>(u_in) % 16 == 0);
        const void *x_in = nullptr;
        const int64_t bt = tile_cols((int)es);
        int64_t ts_in = 0;
        for (int t = 1; t <= c->steps; ++t) {
            const Step &sp = c->st[t];
            StepArgs a{};
            a.crow = sp.op.crow.get();
            a.col = sp.op.col.get();
            a.val = mode == AFB_MODE_F32 ? (const void *)sp.val32.get() : (const void *)sp.val16.get();
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
            a.rc = sp.rc[mode].get();
            a.x_in = x_in ? x_in : buf[(t + 1) & 1];   // step 1 reads no state (R_0 is empty)
            a.ts_in = ts_in;
            a.u = u_in;
            a.ld_u = ld_u;
            a.u_vec_ok = u_vec_ok;
            a.x_out = buf[t & 1];
            a.ts_out = (int64_t)sp.n_rows * bt;
            a.batch = batch;
            a.err = c->err.get();
            if (events) AFB_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(events[t - 1]), s));
            if (mode == AFB_MODE_F32) launch_step_f32(a, s);
            else launch_step_dev16(a, s);
            x_in = buf[t & 1];
            ts_in = a.ts_out;
        }
        if (events) AFB_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(events[c->steps]), s));
        launch_output((int)c->n_out, c->out_row.get(), c->out_base[mode].get(), mode == AFB_MODE_DEV16, x_in,
                      mode == AFB_MODE_DEV16, ts_in, out, ld_out, batch, s);
        if (events) AFB_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(events[c->steps + 1]), s));
    });
}

int afb_cone_forward(const afb_cone *c, int mode, const void *u_in, int64_t ld_u, int64_t batch, float *out,
                     int64_t ld_out, void *workspace, size_t workspace_bytes, void *stream) {
    return afb_cone_forward_timed(c, mode, u_in, ld_u, batch, out, ld_out, workspace, workspace_bytes, nullptr, stream);
}

size_t afb_graph_forward_workspace(const afb_graph *g, int64_t batch) {
    if (!g || batch < 0) return 0;
    return 2 * align256((size_t)g->n * padded_ld(batch, 4) * 4) + 2 * align256((size_t)g->n * sizeof(RowConst)) + 256;
}

int afb_graph_forward(const afb_graph *g, const float *w, const float *bias, const float *alpha_logit, float h_max,
                      const float *u, int64_t ld_u, int64_t batch, int steps, float *h, int64_t ld_h, void *workspace,
                      size_t workspace_bytes, void *stream) {
    return guarded([&] {
        AFB_CHECK(g, "graph is NULL");
        AFB_CHECK((g->e == 0 || w) && bias && alpha_logit && h, "NULL pointer");
        AFB_CHECK(batch >= 0 && steps >= 0, "batch and steps must be >= 0");
        AFB_CHECK(ld_u >= batch && ld_h >= batch, "leading dimensions must be >= batch");
        AFB_CHECK(workspace_bytes >= afb_graph_forward_workspace(g, batch), "workspace too small");
        if (batch == 0) return;
        AFB_CHECK(u, "u is NULL");
        check_aligned(workspace, 256, "workspace");
        cudaStream_t s = as_stream(stream);
        const int64_t n = g->n, ld = padded_ld(batch, 4);
        char *ws = static_cast<char *>(workspace);
        const size_t sb = align256((size_t)n * ld * 4);
        void *buf[2] = {ws, ws + sb};
        RowConst *rc_first = reinterpret_cast<RowConst *>(ws + 2 * sb);
        RowConst *rc_rest = reinterpret_cast<RowConst *>(ws + 2 * sb + align256((size_t)n * sizeof(RowConst)));
        graph_constants<<<grid_for(n, kBlock), kBlock, 0, s>>>(n, bias, alpha_logit, h_max, rc_first, rc_rest);
        AFB_LAUNCHED();
        if (steps == 0) {  // h stays zero
            launch_output((int)n, nullptr, nullptr, 0, nullptr, 0, 0, h, ld_h, batch, s);
            return;
        }
        const int u_vec_ok = (ld_u % 4 == 0) && (reinterpret_cast<uintptr_t>(u) % 16 == 0);
        const void *x_in = buf[1];
        const int64_t ts = n * tile_cols(4);
        for (int t = 1; t <= steps; ++t) {
            const Csr &m = t == 1 ? g->empty : g->full;
            StepArgs a{};
            a.crow = m.crow.get();
            a.col = m.col.get();
            a.val = w;
            a.item_rows = m.item_rows.get();
            a.item_order = m.item_order.get();
            a.bounds = m.bounds.get();
            a.n_items = m.n_items;
            a.item_rows_fine = m.fine.item_rows.get();
            a.item_order_fine = m.fine.item_order.get();
            a.bounds_fine = m.fine.bounds.get();
            a.n_items_fine = m.fine.n_items;
            a.n_rows = m.n_rows;
            a.nnz = m.nnz;
            a.rc = t == 1 ? rc_first : rc_rest;
            a.x_in = x_in;
            a.ts_in = ts;
            a.u = u;
            a.ld_u = ld_u;
            a.u_vec_ok = u_vec_ok;
            a.x_out = buf[t & 1];
            a.ts_out = ts;
            a.batch = batch;
            a.err = g->err.get();
            launch_step_f32(a, s);
            x_in = buf[t & 1];
        }
        launch_output((int)n, nullptr, nullptr, 0, x_in, 0, ts, h, ld_h, batch, s);   // row-for-row copy
    });
}

// ---- forward without any allocation -----------------------------------------------------------
// Some callers cannot allocate device memory when they evaluate: a host process whose device memory
// is owned by another framework's pooling allocator (a cudaMalloc behind its back fragments the pool
// or fails against its reservation), or a latency-bound serving loop that cannot afford the implicit
// device synchronisation of cudaMalloc / cudaFree.  For them the forward's two ping-pong state
// buffers live in this file-scope device array instead of a caller workspace.  Its size is fixed:
// every GPU that loads the library holds these 32 MiB until the process exits.
#define AFB_NOALLOC_SCRATCH_BYTES (32u << 20)
static __device__ __align__(256) unsigned char g_noalloc_scratch[AFB_NOALLOC_SCRATCH_BYTES];

namespace {
// Device address of g_noalloc_scratch on device `dev`, which must be current.  In host code the symbol's
// name is a host-side stand-in, not a device address, so it is resolved once per device with
// cudaGetSymbolAddress (with that device current) and cached for the life of the process.
void *noalloc_scratch(int dev) {
    static std::mutex lock;
    static void *addr[64] = {};
    AFB_CHECK(dev >= 0 && dev < 64, "device index out of range for the built-in scratch");
    std::lock_guard<std::mutex> g(lock);
    if (!addr[dev]) {
        void *p = nullptr;
        AFB_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        addr[dev] = p;
    }
    return addr[dev];
}
}  // namespace

int afb_cone_forward_noalloc(const afb_cone *c, int mode, const void *u_in, int64_t ld_u, int64_t batch, float *out,
                             int64_t ld_out, void *stream) {
    void *ws = nullptr;
    const int rc = guarded([&] {
        AFB_CHECK(c, "cone is NULL");
        AFB_CHECK(mode == AFB_MODE_F32 || mode == AFB_MODE_DEV16, "unknown mode");
        AFB_CHECK(batch >= 0, "batch must be >= 0");
        const size_t need = afb_cone_forward_workspace(c, mode, batch);
        AFB_CHECK(need <= AFB_NOALLOC_SCRATCH_BYTES,
                  "afb_cone_forward_noalloc: this cone and batch need " + std::to_string(need) +
                      " bytes of state, more than the built-in scratch of " + std::to_string(AFB_NOALLOC_SCRATCH_BYTES) +
                      " bytes; use afb_cone_forward with a caller-provided workspace or a smaller batch");
        // The scratch is picked by device, so the device must be the cone's, and the stream's: a mismatch
        // would run this cone's kernels against another GPU's array.
        int dev = -1;
        AFB_CUDA(cudaGetDevice(&dev));
        AFB_CHECK(dev == c->device, "afb_cone_forward_noalloc: the current device (" + std::to_string(dev) +
                                        ") is not the cone's device (" + std::to_string(c->device) + ")");
        if (stream) {
            int sdev = -1;
            AFB_CUDA(cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev));
            AFB_CHECK(sdev == c->device, "afb_cone_forward_noalloc: the stream belongs to device " + std::to_string(sdev) +
                                             ", not the cone's device (" + std::to_string(c->device) + ")");
        }
        ws = noalloc_scratch(dev);
    });
    if (rc != AFB_OK) return rc;
    return afb_cone_forward_timed(c, mode, u_in, ld_u, batch, out, ld_out, ws, AFB_NOALLOC_SCRATCH_BYTES, nullptr, stream);
}

}  // extern "C"
