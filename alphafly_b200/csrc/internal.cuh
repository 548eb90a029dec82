// Internal data structures shared by the library's translation units.
#pragma once

#include "common.cuh"

namespace afb {

// Per-row constants of one step, read once per row by the fused step kernel's epilogue:
//   y = acc + kk (+ u[usrc]) ; x = clamp(y, lo, hi) + e ; p = prev >= 0 ? x_in[prev] : pc ;
//   out = p + a (x - p)
// float32 state:  kk = k_t, lo = 0, hi = h_max, e = 0, pc = c_{t-1}            (brain.py:40-46)
// float16 deviation: kk = 0, lo = -k, hi = h_max - k, e = k - clamp(k, 0, h_max), pc = 0
//                    with k = (W c_{t-1} + b)[row]                              (brain.py:53-58, 264-267)
struct __align__(16) RowConst {
    float kk, lo, hi, e;
    float pc, a;
    int prev, usrc;
};
static_assert(sizeof(RowConst) == 32, "RowConst is two 16-byte words");

// A work schedule of the fused step kernel: contiguous row ranges ("items") of similar cost, launched
// heaviest first, each with its merge-path cut over the CTA's warps.
struct Schedule {
    int n_items = 0;
    DevBuf<int> item_rows;         // (n_items + 1) row boundaries
    DevBuf<int> item_order;        // (n_items) launch order
    DevBuf<int2> bounds;           // (n_items x (warps + 1)) merge-path cut of each item over the CTA's warps
};

// A CSR matrix (int32 indices) with the work schedules of the fused step kernel.
struct Csr {
    int n_rows = 0, n_cols = 0;
    int64_t nnz = 0;
    bool present = false;          // false: the reference has no matrix for this step (R_{t-1} empty)
    DevBuf<int> crow, col;         // crow (n_rows + 1), col (nnz): local column index
    DevBuf<int> edges, post;       // edges (nnz): index into W's edge list; post (nnz): local row
    DevBuf<int> t_crow, t_col, t_order;  // CSR of the transpose, and the edge permutation into it
    DevBuf<int> t_edges;           // (nnz) edges[t_order]: W's edge index at each position of the transpose
    DevBuf<int> t_heavy;           // (n_cols) rows of the transpose, longest first (backward launch order)
    // schedule of items of ~kItemCost, and of ~kFineItemCost for launches whose kItemCost items would be
    // too few CTAs to fill the GPU (narrow batches on small graphs or small light-cone steps)
    int n_items = 0;
    DevBuf<int> item_rows;         // (n_items + 1) row boundaries
    DevBuf<int> item_order;        // (n_items) launch order
    DevBuf<int2> bounds;           // (n_items x (warps + 1)) merge-path cut of each item over the CTA's warps
    Schedule fine;
};

struct Step {
    int n_rows = 0;
    DevBuf<int> rows;              // global neuron ids of R_t, ascending
    Csr op;                        // W[R_t, R_{t-1}]
    DevBuf<int> prev;              // (n_rows) local index in R_{t-1}, or -1 (not carried)
    DevBuf<int> usrc;              // (n_rows) position in in_idx, or -1 (not fed)
    DevBuf<int> keep_next, keep_prev, u_pos, u_src;
    int n_keep = 0, n_fed = 0;
    DevBuf<RowConst> rc[2];        // per mode
    DevBuf<int> inv_prev;          // (|R_{t-1}|) the row of R_t carried from each row of R_{t-1}, or -1
    DevBuf<float> val32;           // w[edges], AFB_MODE_F32
    DevBuf<float> val32_t;         // w[edges[t_order]], the transpose's values (training)
    DevBuf<__half> val16;          // half(w[edges]), AFB_MODE_DEV16
};

// Schedule target: cost units (edges + kRowCost per row) per CTA work item, and the finer target of
// launches whose kItemCost items would be too few CTAs to fill the GPU.
constexpr int kRowCost = 4;
constexpr int kItemCost = 4096;
constexpr int kFineItemCost = 512;

// Builds the item schedule of `m` from its crow (device), then its merge-path table; synchronous.
void build_schedule(Csr &m, cudaStream_t s);
void build_bounds(const Csr &m, int n_items, const int *item_rows, DevBuf<int2> &bounds, cudaStream_t s);

// Launch helpers of the fused step kernel (step.cu).
struct StepArgs {
    const int *crow;
    const int *col;
    const void *val;
    const int *item_rows;
    const int *item_order;
    const int2 *bounds;
    int n_items;
    const int *item_rows_fine;     // the fine schedule (Csr::fine); the launcher picks one of the two
    const int *item_order_fine;
    const int2 *bounds_fine;
    int n_items_fine;
    int n_rows;                    // rows of this step's sub-matrix
    int64_t nnz;                   // its synapses (chooses the kernel: see launch in step.cu)
    const RowConst *rc;
    const void *x_in;              // state of R_{t-1}, tile-major (see tile_cols)
    int64_t ts_in;                 // elements between consecutive batch tiles of x_in
    const void *u;                 // drive (n_in, batch), row-major with ld_u
    int64_t ld_u;
    int u_vec_ok;
    void *x_out;                   // state of R_t, tile-major
    int64_t ts_out;
    int64_t batch;
    int *err;                      // device status word (afb_cone_status); no current step kernel waits, so none sets it
    float *y_out;                  // training forward: pre-clamp drive of R_t, tile-major (float32 state only)
};

// Batch columns one CTA covers for a state element of `elem_bytes`; the state's leading dimension is
// padded to a multiple of it.
int tile_cols(int elem_bytes);
inline int64_t padded_ld(int64_t batch, int elem_bytes) {
    const int64_t t = tile_cols(elem_bytes);
    return (batch + t - 1) / t * t;
}

void launch_step_f32(const StepArgs &a, cudaStream_t s);
void launch_step_dev16(const StepArgs &a, cudaStream_t s);

// out[o, b] = src[o] >= 0 ? (add_base ? base[o] : 0) + state[src[o], b] : base[o]   (float32 out, row-major);
// src NULL: row o of the state (or, with state NULL too, base[o] / zero); base NULL: zero.  The state is
// tile-major with tile stride ts_state.
void launch_output(int n_out, const int *src, const float *base, int add_base, const void *state, int state_is_half,
                   int64_t ts_state, float *out, int64_t ld_out, int64_t batch, cudaStream_t s);

// out[i] = table[ids[i]], i < m
void gather_floats(const float *table, const int *ids, float *out, int64_t m, cudaStream_t s);

// Warp-per-row y = A x for one column vector (float32), A given by (crow, col, val).
void launch_spmv(int n_rows, const int *crow, const int *col, const float *val, const float *x, float *y,
                 cudaStream_t s);

}  // namespace afb

struct afb_cone {
    int64_t n = 0, e = 0;
    int steps = 0;
    int device = -1;                  // the CUDA device that was current at creation: the cone's buffers live there
    std::vector<afb::Step> st;        // st[0..steps]; st[0] holds R_0 only
    afb::DevBuf<int> full_crow, full_col, full_post;   // W in CSR (edge order) with each edge's row
    afb::DevBuf<int> full_tcrow, full_tcol, full_torder; // W^T in CSR and the edge permutation into it
    int64_t n_in = 0, n_out = 0;
    afb::DevBuf<int> out_idx, out_row, out_pos, out_src;
    int n_hit = 0;
    int max_rows = 0;
    int64_t edge_visits = 0;
    // weight version state
    afb::DevBuf<float> alpha;          // sigmoid(alpha_logit)
    afb::DevBuf<float> resting;        // (steps + 1) x n
    afb::DevBuf<float> kfull;          // (steps + 1) x n: W c_{t-1} + b
    afb::DevBuf<float> wc;             // (n) scratch of the resting-trajectory SpMV
    afb::DevBuf<float> w_t;            // (e) w[full_torder]: values of W^T (training)
    afb::DevBuf<float> out_base[2];    // c_T[out_idx], per mode
    bool ready[2] = {false, false};    // per mode: constants set since the handle was built
    afb::DevBuf<int> err;              // device status word of the step kernels (0 = ok)
    float h_max = 10.f;                // clamp of the last afb_cone_set_weights
};

struct afb_graph {
    int64_t n = 0, e = 0;
    afb::Csr full;                     // W over all neurons (edge order = CSR order)
    afb::Csr empty;                    // no entries: the first step multiplies a zero state
    afb::DevBuf<int> err;              // device status word of the step kernels (0 = ok)
};
