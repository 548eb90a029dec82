/*
 * CPU oracle kernels for the connectome recurrence -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this file's
 * library, and only as the checker or as the timed CPU baseline; the product path never does.
 *
 * These are plain restatements of what the reference computes through torch's sparse CSR
 * tensors (chessfly/brain.py):
 *   ref_spmm_f64 / ref_spmm_f32   y = A x for A in CSR, x laid out (cols, B) row-major
 *                                 (torch.sparse_csr_tensor @ dense, chessfly/brain.py:76,83,221,275,311,320)
 *   ref_sddmm_f64                 g_e = sum_b G[row_e, b] * X[col_e, b]  (the per-synapse gradient,
 *                                 chessfly/brain.py:85-98)
 *   ref_step_f32                  one fused light-cone step in float32, the reference's FUSED_UPDATE
 *                                 path (chessfly/brain.py:40-46, 310-314); used as the timed CPU
 *                                 baseline with OpenMP over rows
 * Accumulation order: edges in CSR order, one accumulator per (row, column).
 */
#include <stdint.h>
#include <string.h>

void ref_spmm_f64(int64_t n_rows, const int64_t *crow, const int64_t *col, const double *val,
                  const double *x, int64_t batch, double *y) {
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t r = 0; r < n_rows; ++r) {
        double *yr = y + r * batch;
        memset(yr, 0, sizeof(double) * (size_t)batch);
        for (int64_t e = crow[r]; e < crow[r + 1]; ++e) {
            const double v = val[e];
            const double *xr = x + col[e] * batch;
            for (int64_t b = 0; b < batch; ++b) yr[b] += v * xr[b];
        }
    }
}

void ref_spmm_f32(int64_t n_rows, const int64_t *crow, const int64_t *col, const float *val,
                  const float *x, int64_t batch, float *y) {
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t r = 0; r < n_rows; ++r) {
        float *yr = y + r * batch;
        memset(yr, 0, sizeof(float) * (size_t)batch);
        for (int64_t e = crow[r]; e < crow[r + 1]; ++e) {
            const float v = val[e];
            const float *xr = x + col[e] * batch;
            for (int64_t b = 0; b < batch; ++b) yr[b] += v * xr[b];
        }
    }
}

void ref_sddmm_f64(int64_t n_rows, const int64_t *crow, const int64_t *col, const double *g,
                   const double *x, int64_t batch, double *out) {
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t r = 0; r < n_rows; ++r) {
        const double *gr = g + r * batch;
        for (int64_t e = crow[r]; e < crow[r + 1]; ++e) {
            const double *xr = x + col[e] * batch;
            double s = 0.0;
            for (int64_t b = 0; b < batch; ++b) s += gr[b] * xr[b];
            out[e] = s;
        }
    }
}

static inline float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* torch.lerp's two-branch form: start + w (end - start) for w < 0.5, else end - (end - start)(1 - w). */
static inline float lerpf(float s, float e, float w) {
    return w < 0.5f ? s + w * (e - s) : e - (e - s) * (1.0f - w);
}

/*
 * One light-cone step in float32 (chessfly/brain.py:310-314):
 *   y = A h_prev (+ u_in[u_src[r]] on fed rows);  x = clamp(y + k_r, 0, h_max)
 *   p = prev_row[r] >= 0 ? h_prev[prev_row[r]] : c_r;  h[r] = lerp(p, x, a_r)
 * h_prev may be NULL when the step has no matrix (its rows then see y = 0 + input).
 */
void ref_step_f32(int64_t n_rows, const int64_t *crow, const int64_t *col, const float *val,
                  const float *h_prev, const float *k, const float *c, const float *a,
                  const int64_t *prev_row, const int64_t *u_src, const float *u_in, float h_max,
                  int64_t batch, float *h) {
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t r = 0; r < n_rows; ++r) {
        float *hr = h + r * batch;
        memset(hr, 0, sizeof(float) * (size_t)batch);
        if (h_prev) {
            for (int64_t e = crow[r]; e < crow[r + 1]; ++e) {
                const float v = val[e];
                const float *xr = h_prev + col[e] * batch;
                for (int64_t b = 0; b < batch; ++b) hr[b] += v * xr[b];
            }
        }
        if (u_src[r] >= 0) {
            const float *ur = u_in + u_src[r] * batch;
            for (int64_t b = 0; b < batch; ++b) hr[b] += ur[b];
        }
        const float kr = k[r], ar = a[r];
        const float *pr = (prev_row[r] >= 0 && h_prev) ? h_prev + prev_row[r] * batch : 0;
        for (int64_t b = 0; b < batch; ++b) {
            const float x = clampf(hr[b] + kr, 0.0f, h_max);
            const float p = pr ? pr[b] : c[r];
            hr[b] = lerpf(p, x, ar);
        }
    }
}

int ref_num_threads(void) {
#ifdef _OPENMP
    extern int omp_get_max_threads(void);
    return omp_get_max_threads();
#else
    return 1;
#endif
}
