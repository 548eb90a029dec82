// Light-cone construction on the GPU: the per-step row sets R_t, the sub-matrices W[R_t, R_{t-1}]
// with their transposes, the carried / fed row maps and the output map, plus the work schedule of
// the fused step kernel.  Restates chessfly/brain.py:102-173 (LightCone, _SubMatrix) with int32
// indices; every compaction keeps ascending order, so the index arrays equal the reference's
// torch.nonzero results element for element.
#include <cub/cub.cuh>
#include <thrust/iterator/counting_iterator.h>

#include <algorithm>
#include <numeric>

#include "internal.cuh"

namespace afb {

thread_local std::string g_last_error;
void set_last_error(const std::string &msg) { g_last_error = msg; }

namespace {

constexpr int kBlock = 256;

__global__ void narrow_indices(const int64_t *__restrict__ src, int *__restrict__ dst, int64_t m, int64_t n,
                               int *__restrict__ bad) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t v = src[i];
        if (v < 0 || v >= n) {
            atomicExch(bad, 1);
            v = 0;
        }
        dst[i] = (int)v;
    }
}

// post must be non-decreasing (edges in CSR order of W[post, pre]) and (post, pre) non-decreasing.
__global__ void check_sorted(const int *__restrict__ post, const int *__restrict__ pre, int64_t e, int *__restrict__ bad) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x + 1; i < e; i += (int64_t)gridDim.x * blockDim.x) {
        if (post[i] < post[i - 1] || (post[i] == post[i - 1] && pre[i] < pre[i - 1])) atomicExch(bad, 1);
    }
}

__global__ void count_rows(const int *__restrict__ rows_of_edge, int64_t e, int *__restrict__ counts) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < e; i += (int64_t)gridDim.x * blockDim.x)
        atomicAdd(&counts[rows_of_edge[i]], 1);
}

__global__ void fill_mask(uint8_t *__restrict__ mask, const int *__restrict__ idx, int64_t m) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x)
        mask[idx[i]] = 1;
}

// next |= (cur[from[e]] ? to[e] : -)   -- one hop of the light-cone BFS (brain.py:143,148)
__global__ void hop(const uint8_t *__restrict__ cur, uint8_t *__restrict__ next, const int *__restrict__ from,
                    const int *__restrict__ to, int64_t e) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < e; i += (int64_t)gridDim.x * blockDim.x)
        if (cur[from[i]]) next[to[i]] = 1;
}

__global__ void and_flags(const uint8_t *__restrict__ a, const uint8_t *__restrict__ b, uint8_t *__restrict__ f, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        f[i] = a[i] & b[i];
}

__global__ void fill_int(int *__restrict__ p, int v, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = v;
}

__global__ void scatter_iota(int *__restrict__ where, const int *__restrict__ ids, int m) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < m; i += gridDim.x * blockDim.x) where[ids[i]] = i;
}

// in_pos[in_idx[j]] = j; on duplicates the last j wins (atomicMax), like a sequential index_put.
__global__ void scatter_last(int *__restrict__ where, const int *__restrict__ ids, int64_t m) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x)
        atomicMax(&where[ids[i]], (int)i);
}

__global__ void gather_int(const int *__restrict__ table, const int *__restrict__ ids, int *__restrict__ out, int m) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < m; i += gridDim.x * blockDim.x) out[i] = table[ids[i]];
}

__global__ void nonneg_flags(const int *__restrict__ v, uint8_t *__restrict__ f, int m) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < m; i += gridDim.x * blockDim.x) f[i] = v[i] >= 0;
}

__global__ void edge_flags(const int *__restrict__ post, const int *__restrict__ pre, const int *__restrict__ row_of,
                           const int *__restrict__ col_of, uint8_t *__restrict__ f, int64_t e) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < e; i += (int64_t)gridDim.x * blockDim.x)
        f[i] = (row_of[post[i]] >= 0) & (col_of[pre[i]] >= 0);
}

__global__ void local_edges(const int *__restrict__ edges, const int *__restrict__ post, const int *__restrict__ pre,
                            const int *__restrict__ row_of, const int *__restrict__ col_of, int *__restrict__ lpost,
                            int *__restrict__ lcol, long long *__restrict__ key, int *__restrict__ iota, int n_rows,
                            int64_t m) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x) {
        int ed = edges[i];
        int r = row_of[post[ed]], c = col_of[pre[ed]];
        lpost[i] = r;
        lcol[i] = c;
        key[i] = (long long)c * n_rows + r;   // CSR order of the transpose (brain.py:116)
        iota[i] = (int)i;
    }
}

__global__ void full_keys(const int *__restrict__ post, const int *__restrict__ pre, long long *__restrict__ key,
                          int *__restrict__ iota, int64_t n, int64_t e) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < e; i += (int64_t)gridDim.x * blockDim.x) {
        key[i] = (long long)pre[i] * n + post[i];
        iota[i] = (int)i;
    }
}

// inv[prev[i]] = i for the carried rows i of R_t (prev is one-to-one onto its image)
__global__ void row_lengths(const int *__restrict__ crow, int n, int *__restrict__ len, int *__restrict__ iota) {
    for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x) {
        len[r] = crow[r + 1] - crow[r];
        iota[r] = (int)r;
    }
}

__global__ void invert_prev(const int *__restrict__ prev, int n_rows, int *__restrict__ inv) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_rows; i += gridDim.x * blockDim.x)
        if (prev[i] >= 0) inv[prev[i]] = i;
}

__global__ void widen(const int *__restrict__ src, int64_t *__restrict__ dst, int64_t m, int mode) {
    // mode 0: copy; mode 1: (v >= 0) as 0/1; mode 2: max(v, 0)
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x) {
        int v = src[i];
        dst[i] = mode == 0 ? (int64_t)v : (mode == 1 ? (int64_t)(v >= 0) : (int64_t)(v > 0 ? v : 0));
    }
}

struct Temp {
    DevBuf<uint8_t> buf;
    void *need(size_t bytes) {
        if (buf.n < bytes) buf.alloc(bytes);
        return buf.get();
    }
};

// Ascending positions i < m with flags[i] != 0, into an exact-size buffer; synchronous.
int select_flagged(const uint8_t *flags, int64_t m, DevBuf<int> &out, Temp &tmp, cudaStream_t s) {
    DevBuf<int> all(m > 0 ? m : 1);
    DevBuf<int> count(1);
    thrust::counting_iterator<int> iota(0);
    size_t bytes = 0;
    AFB_CUDA(cub::DeviceSelect::Flagged(nullptr, bytes, iota, flags, all.get(), count.get(), (int)m, s));
    AFB_CUDA(cub::DeviceSelect::Flagged(tmp.need(bytes), bytes, iota, flags, all.get(), count.get(), (int)m, s));
    int c = to_host(count.get(), 1, s)[0];
    out.alloc(c);
    if (c) AFB_CUDA(cudaMemcpyAsync(out.get(), all.get(), c * sizeof(int), cudaMemcpyDeviceToDevice, s));
    return c;
}

// crow (n_rows + 1) from per-row counts: exclusive prefix sum; counts must have n_rows + 1 entries.
void counts_to_crow(DevBuf<int> &counts, int n_rows, DevBuf<int> &crow, Temp &tmp, cudaStream_t s) {
    crow.alloc(n_rows + 1);
    size_t bytes = 0;
    AFB_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, bytes, counts.get(), crow.get(), n_rows + 1, s));
    AFB_CUDA(cub::DeviceScan::ExclusiveSum(tmp.need(bytes), bytes, counts.get(), crow.get(), n_rows + 1, s));
}

void crow_from_rows(const int *rows_of_edge, int64_t m, int n_rows, DevBuf<int> &crow, Temp &tmp, cudaStream_t s) {
    DevBuf<int> counts(n_rows + 1);
    AFB_CUDA(cudaMemsetAsync(counts.get(), 0, (n_rows + 1) * sizeof(int), s));
    if (m) {
        count_rows<<<grid_for(m, kBlock), kBlock, 0, s>>>(rows_of_edge, m, counts.get());
        AFB_LAUNCHED();
    }
    counts_to_crow(counts, n_rows, crow, tmp, s);
}

int bits_for(long long v) {
    int b = 1;
    while (b < 63 && (1LL << b) <= v) ++b;
    return b;
}

}  // namespace

// Items of about `target` cost units (a unit is a synapse, a row is kRowCost), heaviest first.
static void make_items(const std::vector<int> &crow, int n_rows, int64_t target, std::vector<int> &starts,
                       std::vector<int> &order) {
    std::vector<int64_t> cost;
    starts.assign(1, 0);
    int64_t acc = 0;
    for (int r = 0; r < n_rows; ++r) {
        acc += (int64_t)(crow[r + 1] - crow[r]) + kRowCost;
        if (acc >= target || r + 1 == n_rows) {
            starts.push_back(r + 1);
            cost.push_back(acc);
            acc = 0;
        }
    }
    if (n_rows == 0) cost.clear(), starts.assign(1, 0);
    order.resize(cost.size());
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return cost[a] > cost[b]; });
}

void build_schedule(Csr &m, cudaStream_t s) {
    std::vector<int> crow = to_host(m.crow.get(), (size_t)m.n_rows + 1, s);
    std::vector<int> starts, order;
    make_items(crow, m.n_rows, kItemCost, starts, order);
    m.n_items = (int)order.size();
    m.item_rows.alloc(starts.size());
    to_device(m.item_rows.get(), starts, s);
    m.item_order.alloc(order.size());
    to_device(m.item_order.get(), order, s);
    build_bounds(m, m.n_items, m.item_rows.get(), m.bounds, s);
    make_items(crow, m.n_rows, kFineItemCost, starts, order);
    m.fine.n_items = (int)order.size();
    m.fine.item_rows.alloc(starts.size());
    to_device(m.fine.item_rows.get(), starts, s);
    m.fine.item_order.alloc(order.size());
    to_device(m.fine.item_order.get(), order, s);
    build_bounds(m, m.fine.n_items, m.fine.item_rows.get(), m.fine.bounds, s);
}

}  // namespace afb

using namespace afb;

extern "C" {

const char *afb_last_error(void) { return g_last_error.c_str(); }
int afb_version(void) { return 1; }
int afb_compiled_arch(void) { return AFB_ARCH; }

int afb_cone_create(afb_cone **out, int64_t n, int64_t e, const int64_t *pre, const int64_t *post,
                    const int64_t *in_idx, int64_t n_in, const int64_t *out_idx, int64_t n_out, int steps,
                    void *stream) {
    return guarded([&] {
        AFB_CHECK(out != nullptr, "cone output pointer is NULL");
        AFB_CHECK(n > 0 && n < (1LL << 31), "n must be in [1, 2^31)");
        AFB_CHECK(e >= 0 && e < (1LL << 31), "e must be in [0, 2^31)");
        AFB_CHECK(steps >= 1 && steps <= 64, "steps must be in [1, 64]");
        AFB_CHECK(n_in >= 0 && n_out >= 1, "need n_in >= 0 and n_out >= 1");
        AFB_CHECK(e == 0 || (pre && post), "pre / post are NULL");
        AFB_CHECK(n_in == 0 || in_idx, "in_idx is NULL");
        AFB_CHECK(out_idx, "out_idx is NULL");
        cudaStream_t s = as_stream(stream);
        auto c = std::make_unique<afb_cone>();
        c->n = n;
        c->e = e;
        c->steps = steps;
        AFB_CUDA(cudaGetDevice(&c->device));
        c->n_in = n_in;
        c->n_out = n_out;
        Temp tmp;
        DevBuf<int> bad(1);
        AFB_CUDA(cudaMemsetAsync(bad.get(), 0, sizeof(int), s));
        DevBuf<int> pre32(e ? e : 1), post32(e ? e : 1), in32(n_in ? n_in : 1);
        c->out_idx.alloc(n_out);
        if (e) {
            narrow_indices<<<grid_for(e, kBlock), kBlock, 0, s>>>(pre, pre32.get(), e, n, bad.get());
            narrow_indices<<<grid_for(e, kBlock), kBlock, 0, s>>>(post, post32.get(), e, n, bad.get());
        }
        if (n_in) narrow_indices<<<grid_for(n_in, kBlock), kBlock, 0, s>>>(in_idx, in32.get(), n_in, n, bad.get());
        narrow_indices<<<grid_for(n_out, kBlock), kBlock, 0, s>>>(out_idx, c->out_idx.get(), n_out, n, bad.get());
        AFB_LAUNCHED();
        AFB_CHECK(to_host(bad.get(), 1, s)[0] == 0, "an edge, input or output index is outside [0, n)");
        if (e > 1) {
            check_sorted<<<grid_for(e, kBlock), kBlock, 0, s>>>(post32.get(), pre32.get(), e, bad.get());
            AFB_LAUNCHED();
            AFB_CHECK(to_host(bad.get(), 1, s)[0] == 0, "edges must be sorted by (post, pre), the CSR order of W[post, pre]");
        }
        crow_from_rows(post32.get(), e, (int)n, c->full_crow, tmp, s);
        // W^T: edges sorted by (pre, post), stable (the reference's t_order, brain.py:192-195)
        c->full_torder.alloc(e ? e : 1);
        c->full_tcol.alloc(e ? e : 1);
        if (e) {
            DevBuf<long long> key(e), key_sorted(e);
            DevBuf<int> iota(e);
            full_keys<<<grid_for(e, kBlock), kBlock, 0, s>>>(post32.get(), pre32.get(), key.get(), iota.get(), n, e);
            AFB_LAUNCHED();
            size_t bytes = 0;
            const int end_bit = bits_for((long long)n * n);
            AFB_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, bytes, key.get(), key_sorted.get(), iota.get(),
                                                     c->full_torder.get(), (int)e, 0, end_bit, s));
            AFB_CUDA(cub::DeviceRadixSort::SortPairs(tmp.need(bytes), bytes, key.get(), key_sorted.get(), iota.get(),
                                                     c->full_torder.get(), (int)e, 0, end_bit, s));
            gather_int<<<grid_for(e, kBlock), kBlock, 0, s>>>(post32.get(), c->full_torder.get(), c->full_tcol.get(), (int)e);
            AFB_LAUNCHED();
        }
        crow_from_rows(pre32.get(), e, (int)n, c->full_tcrow, tmp, s);
        c->full_col = std::move(pre32);
        c->full_post = std::move(post32);
        const int *post32_p = c->full_post.get();

        // V_t (forward reachability from the inputs) and D_t (backward reachability of the outputs)
        const int T = steps;
        DevBuf<uint8_t> V((size_t)(T + 1) * n), D((size_t)(T + 1) * n), F(n);
        AFB_CUDA(cudaMemsetAsync(V.get(), 0, V.n, s));
        AFB_CUDA(cudaMemsetAsync(D.get(), 0, D.n, s));
        if (n_in) fill_mask<<<grid_for(n_in, kBlock), kBlock, 0, s>>>(V.get() + n, in32.get(), n_in);
        for (int t = 2; t <= T; ++t) {
            AFB_CUDA(cudaMemcpyAsync(V.get() + t * n, V.get() + (t - 1) * n, n, cudaMemcpyDeviceToDevice, s));
            if (e) hop<<<grid_for(e, kBlock), kBlock, 0, s>>>(V.get() + (t - 1) * n, V.get() + t * n, c->full_col.get(), post32_p, e);
        }
        fill_mask<<<grid_for(n_out, kBlock), kBlock, 0, s>>>(D.get() + (size_t)T * n, c->out_idx.get(), n_out);
        for (int t = T - 1; t >= 0; --t) {
            AFB_CUDA(cudaMemcpyAsync(D.get() + t * n, D.get() + (t + 1) * n, n, cudaMemcpyDeviceToDevice, s));
            if (e) hop<<<grid_for(e, kBlock), kBlock, 0, s>>>(D.get() + (t + 1) * n, D.get() + t * n, post32_p, c->full_col.get(), e);
        }
        AFB_LAUNCHED();
        c->st.resize(T + 1);
        for (int t = 0; t <= T; ++t) {
            and_flags<<<grid_for(n, kBlock), kBlock, 0, s>>>(V.get() + t * n, D.get() + t * n, F.get(), n);
            AFB_LAUNCHED();
            c->st[t].n_rows = select_flagged(F.get(), n, c->st[t].rows, tmp, s);
            c->max_rows = std::max(c->max_rows, c->st[t].n_rows);
        }

        DevBuf<int> in_pos(n), where_prev(n), where_next(n);
        fill_int<<<grid_for(n, kBlock), kBlock, 0, s>>>(in_pos.get(), -1, n);
        if (n_in) scatter_last<<<grid_for(n_in, kBlock), kBlock, 0, s>>>(in_pos.get(), in32.get(), n_in);
        DevBuf<uint8_t> rflags(c->max_rows ? c->max_rows : 1);
        DevBuf<uint8_t> eflags(e ? e : 1);
        for (int t = 1; t <= T; ++t) {
            Step &sp = c->st[t], &pv = c->st[t - 1];
            const int nr = sp.n_rows, nc = pv.n_rows;
            fill_int<<<grid_for(n, kBlock), kBlock, 0, s>>>(where_prev.get(), -1, n);
            fill_int<<<grid_for(n, kBlock), kBlock, 0, s>>>(where_next.get(), -1, n);
            if (nc) scatter_iota<<<grid_for(nc, kBlock), kBlock, 0, s>>>(where_prev.get(), pv.rows.get(), nc);
            if (nr) scatter_iota<<<grid_for(nr, kBlock), kBlock, 0, s>>>(where_next.get(), sp.rows.get(), nr);
            sp.prev.alloc(nr ? nr : 1);
            sp.usrc.alloc(nr ? nr : 1);
            if (nr) {
                gather_int<<<grid_for(nr, kBlock), kBlock, 0, s>>>(where_prev.get(), sp.rows.get(), sp.prev.get(), nr);
                gather_int<<<grid_for(nr, kBlock), kBlock, 0, s>>>(in_pos.get(), sp.rows.get(), sp.usrc.get(), nr);
            }
            AFB_LAUNCHED();
            sp.inv_prev.alloc(nc ? nc : 1);
            if (nc) fill_int<<<grid_for(nc, kBlock), kBlock, 0, s>>>(sp.inv_prev.get(), -1, nc);
            if (nr) invert_prev<<<grid_for(nr, kBlock), kBlock, 0, s>>>(sp.prev.get(), nr, sp.inv_prev.get());
            // carried rows (brain.py:161-165) and fed rows (brain.py:166-168)
            if (nr) nonneg_flags<<<grid_for(nr, kBlock), kBlock, 0, s>>>(sp.prev.get(), rflags.get(), nr);
            sp.n_keep = select_flagged(rflags.get(), nr, sp.keep_next, tmp, s);
            sp.keep_prev.alloc(sp.n_keep ? sp.n_keep : 1);
            if (sp.n_keep) gather_int<<<grid_for(sp.n_keep, kBlock), kBlock, 0, s>>>(sp.prev.get(), sp.keep_next.get(), sp.keep_prev.get(), sp.n_keep);
            if (nr) nonneg_flags<<<grid_for(nr, kBlock), kBlock, 0, s>>>(sp.usrc.get(), rflags.get(), nr);
            sp.n_fed = select_flagged(rflags.get(), nr, sp.u_pos, tmp, s);
            sp.u_src.alloc(sp.n_fed ? sp.n_fed : 1);
            if (sp.n_fed) gather_int<<<grid_for(sp.n_fed, kBlock), kBlock, 0, s>>>(sp.usrc.get(), sp.u_pos.get(), sp.u_src.get(), sp.n_fed);
            AFB_LAUNCHED();

            // the sub-matrix W[R_t, R_{t-1}] in W's edge order (brain.py:106-117)
            Csr &m = sp.op;
            m.n_rows = nr;
            m.n_cols = nc;
            m.present = nc > 0;
            if (m.present && e) {
                edge_flags<<<grid_for(e, kBlock), kBlock, 0, s>>>(post32_p, c->full_col.get(), where_next.get(), where_prev.get(), eflags.get(), e);
                AFB_LAUNCHED();
                m.nnz = select_flagged(eflags.get(), e, m.edges, tmp, s);
            } else {
                m.nnz = 0;
                m.edges.alloc(0);
            }
            const int64_t nnz = m.nnz;
            m.post.alloc(nnz);
            m.col.alloc(nnz);
            m.t_col.alloc(nnz);
            m.t_order.alloc(nnz);
            m.t_edges.alloc(nnz);
            if (nnz) {
                DevBuf<long long> key(nnz), key_sorted(nnz);
                DevBuf<int> iota(nnz);
                local_edges<<<grid_for(nnz, kBlock), kBlock, 0, s>>>(m.edges.get(), post32_p, c->full_col.get(), where_next.get(),
                                                                     where_prev.get(), m.post.get(), m.col.get(), key.get(), iota.get(), nr, nnz);
                AFB_LAUNCHED();
                // stable radix sort: equal keys (duplicate synapses) keep edge order
                size_t bytes = 0;
                int end_bit = bits_for((long long)nc * nr);
                AFB_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, bytes, key.get(), key_sorted.get(), iota.get(), m.t_order.get(),
                                                         (int)nnz, 0, end_bit, s));
                AFB_CUDA(cub::DeviceRadixSort::SortPairs(tmp.need(bytes), bytes, key.get(), key_sorted.get(), iota.get(),
                                                         m.t_order.get(), (int)nnz, 0, end_bit, s));
                gather_int<<<grid_for(nnz, kBlock), kBlock, 0, s>>>(m.post.get(), m.t_order.get(), m.t_col.get(), (int)nnz);
                gather_int<<<grid_for(nnz, kBlock), kBlock, 0, s>>>(m.edges.get(), m.t_order.get(), m.t_edges.get(), (int)nnz);
                AFB_LAUNCHED();
            }
            crow_from_rows(m.post.get(), nnz, nr, m.crow, tmp, s);
            crow_from_rows(m.col.get(), nnz, nc, m.t_crow, tmp, s);
            m.t_heavy.alloc(nc);
            if (nc) {                          // rows of the transpose by decreasing length
                DevBuf<int> len(nc), len_sorted(nc), iota(nc);
                row_lengths<<<grid_for(nc, kBlock), kBlock, 0, s>>>(m.t_crow.get(), nc, len.get(), iota.get());
                AFB_LAUNCHED();
                size_t bytes = 0;
                const int end_bit = bits_for((long long)nnz + 1);
                AFB_CUDA(cub::DeviceRadixSort::SortPairsDescending(nullptr, bytes, len.get(), len_sorted.get(), iota.get(),
                                                                   m.t_heavy.get(), nc, 0, end_bit, s));
                AFB_CUDA(cub::DeviceRadixSort::SortPairsDescending(tmp.need(bytes), bytes, len.get(), len_sorted.get(), iota.get(),
                                                                   m.t_heavy.get(), nc, 0, end_bit, s));
            }
            build_schedule(m, s);
            c->edge_visits += m.present ? nnz : 0;
        }
        // outputs inside R_T (brain.py:169-172)
        {
            Step &last = c->st[T];
            fill_int<<<grid_for(n, kBlock), kBlock, 0, s>>>(where_next.get(), -1, n);
            if (last.n_rows) scatter_iota<<<grid_for(last.n_rows, kBlock), kBlock, 0, s>>>(where_next.get(), last.rows.get(), last.n_rows);
            c->out_row.alloc(n_out);
            gather_int<<<grid_for(n_out, kBlock), kBlock, 0, s>>>(where_next.get(), c->out_idx.get(), c->out_row.get(), (int)n_out);
            DevBuf<uint8_t> of(n_out);
            nonneg_flags<<<grid_for(n_out, kBlock), kBlock, 0, s>>>(c->out_row.get(), of.get(), (int)n_out);
            AFB_LAUNCHED();
            c->n_hit = select_flagged(of.get(), n_out, c->out_pos, tmp, s);
            c->out_src.alloc(c->n_hit ? c->n_hit : 1);
            if (c->n_hit) gather_int<<<grid_for(c->n_hit, kBlock), kBlock, 0, s>>>(c->out_row.get(), c->out_pos.get(), c->out_src.get(), c->n_hit);
            AFB_LAUNCHED();
        }
        c->err.alloc(1);
        AFB_CUDA(cudaMemsetAsync(c->err.get(), 0, sizeof(int), s));
        AFB_CUDA(cudaStreamSynchronize(s));
        *out = c.release();
    });
}

void afb_cone_destroy(afb_cone *cone) { delete cone; }

static int read_status(int *word, int *status, int reset, void *stream) {
    return guarded([&] {
        AFB_CHECK(word && status, "NULL pointer");
        cudaStream_t s = as_stream(stream);
        AFB_CUDA(cudaMemcpyAsync(status, word, sizeof(int), cudaMemcpyDeviceToHost, s));
        if (reset) AFB_CUDA(cudaMemsetAsync(word, 0, sizeof(int), s));
        AFB_CUDA(cudaStreamSynchronize(s));
    });
}

int afb_cone_status(const afb_cone *c, int *status, int reset, void *stream) {
    if (!c) { set_last_error("cone is NULL"); return AFB_EINVAL; }
    return read_status(c->err.get(), status, reset, stream);
}

int afb_graph_status(const afb_graph *g, int *status, int reset, void *stream) {
    if (!g) { set_last_error("graph is NULL"); return AFB_EINVAL; }
    return read_status(g->err.get(), status, reset, stream);
}

int afb_cone_sizes(const afb_cone *c, int64_t *rows_len, int64_t *nnz, int64_t *n_keep, int64_t *n_fed,
                   int64_t *n_hit, int64_t *edge_visits) {
    return guarded([&] {
        AFB_CHECK(c, "cone is NULL");
        for (int t = 0; t <= c->steps; ++t) {
            if (rows_len) rows_len[t] = c->st[t].n_rows;
            if (nnz) nnz[t] = (t == 0 || !c->st[t].op.present) ? -1 : c->st[t].op.nnz;
            if (n_keep) n_keep[t] = t ? c->st[t].n_keep : 0;
            if (n_fed) n_fed[t] = t ? c->st[t].n_fed : 0;
        }
        if (n_hit) *n_hit = c->n_hit;
        if (edge_visits) *edge_visits = c->edge_visits;
    });
}

int afb_cone_export(const afb_cone *c, int field, int t, int64_t *dst, void *stream) {
    return guarded([&] {
        AFB_CHECK(c, "cone is NULL");
        AFB_CHECK(dst, "dst is NULL");
        const bool per_step = field != AFB_F_OUT_POS && field != AFB_F_OUT_SRC;
        AFB_CHECK(!per_step || (t >= 0 && t <= c->steps), "step out of range");
        AFB_CHECK(field == AFB_F_ROWS || !per_step || t >= 1, "step 0 has rows only");
        const Step *sp = per_step ? &c->st[t] : nullptr;
        const int *src = nullptr;
        int64_t m = 0;
        int mode = 0;
        auto need_op = [&] { AFB_CHECK(sp->op.present, "this step has no sub-matrix (R_{t-1} is empty)"); };
        switch (field) {
            case AFB_F_ROWS: src = sp->rows.get(); m = sp->n_rows; break;
            case AFB_F_CARRIED: src = sp->prev.get(); m = sp->n_rows; mode = 1; break;
            case AFB_F_KEEP_NEXT: src = sp->keep_next.get(); m = sp->n_keep; break;
            case AFB_F_KEEP_PREV: src = sp->keep_prev.get(); m = sp->n_keep; break;
            case AFB_F_PREV_ROW: src = sp->prev.get(); m = sp->n_rows; mode = 2; break;
            case AFB_F_U_POS: src = sp->u_pos.get(); m = sp->n_fed; break;
            case AFB_F_U_SRC: src = sp->u_src.get(); m = sp->n_fed; break;
            case AFB_F_OP_EDGES: need_op(); src = sp->op.edges.get(); m = sp->op.nnz; break;
            case AFB_F_OP_POST: need_op(); src = sp->op.post.get(); m = sp->op.nnz; break;
            case AFB_F_OP_PRE: need_op(); src = sp->op.col.get(); m = sp->op.nnz; break;
            case AFB_F_OP_CROW: need_op(); src = sp->op.crow.get(); m = sp->op.n_rows + 1; break;
            case AFB_F_OP_T_ORDER: need_op(); src = sp->op.t_order.get(); m = sp->op.nnz; break;
            case AFB_F_OP_T_CROW: need_op(); src = sp->op.t_crow.get(); m = sp->op.n_cols + 1; break;
            case AFB_F_OP_T_COL: need_op(); src = sp->op.t_col.get(); m = sp->op.nnz; break;
            case AFB_F_OUT_POS: src = c->out_pos.get(); m = c->n_hit; break;
            case AFB_F_OUT_SRC: src = c->out_src.get(); m = c->n_hit; break;
            default: AFB_CHECK(false, "unknown field id");
        }
        if (m) {
            widen<<<grid_for(m, kBlock), kBlock, 0, as_stream(stream)>>>(src, dst, m, mode);
            AFB_LAUNCHED();
        }
    });
}

int afb_graph_create(afb_graph **out, int64_t n, int64_t e, const int64_t *pre, const int64_t *post, void *stream) {
    return guarded([&] {
        AFB_CHECK(out, "graph output pointer is NULL");
        AFB_CHECK(n > 0 && n < (1LL << 31), "n must be in [1, 2^31)");
        AFB_CHECK(e >= 0 && e < (1LL << 31), "e must be in [0, 2^31)");
        AFB_CHECK(e == 0 || (pre && post), "pre / post are NULL");
        cudaStream_t s = as_stream(stream);
        auto g = std::make_unique<afb_graph>();
        g->n = n;
        g->e = e;
        Temp tmp;
        DevBuf<int> bad(1), post32(e ? e : 1);
        AFB_CUDA(cudaMemsetAsync(bad.get(), 0, sizeof(int), s));
        g->full.col.alloc(e ? e : 1);
        if (e) {
            narrow_indices<<<grid_for(e, kBlock), kBlock, 0, s>>>(pre, g->full.col.get(), e, n, bad.get());
            narrow_indices<<<grid_for(e, kBlock), kBlock, 0, s>>>(post, post32.get(), e, n, bad.get());
            AFB_LAUNCHED();
        }
        AFB_CHECK(to_host(bad.get(), 1, s)[0] == 0, "an edge index is outside [0, n)");
        if (e > 1) {
            check_sorted<<<grid_for(e, kBlock), kBlock, 0, s>>>(post32.get(), g->full.col.get(), e, bad.get());
            AFB_LAUNCHED();
            AFB_CHECK(to_host(bad.get(), 1, s)[0] == 0, "edges must be sorted by (post, pre), the CSR order of W[post, pre]");
        }
        g->full.n_rows = g->full.n_cols = (int)n;
        g->full.nnz = e;
        g->full.present = true;
        crow_from_rows(post32.get(), e, (int)n, g->full.crow, tmp, s);
        build_schedule(g->full, s);
        g->empty.n_rows = (int)n;
        g->empty.n_cols = 0;
        g->empty.crow.alloc(n + 1);
        AFB_CUDA(cudaMemsetAsync(g->empty.crow.get(), 0, (n + 1) * sizeof(int), s));
        g->empty.col.alloc(1);
        build_schedule(g->empty, s);
        g->err.alloc(1);
        AFB_CUDA(cudaMemsetAsync(g->err.get(), 0, sizeof(int), s));
        AFB_CUDA(cudaStreamSynchronize(s));
        *out = g.release();
    });
}

void afb_graph_destroy(afb_graph *g) { delete g; }

}  // extern "C"
