// The policy head's legal-move logits without the dense (batch, n_moves) product: the evaluator's
// gather of logits[rows, cols] (chessfly/model.py:124-126) fused into the head (model.py:104).
#include "internal.cuh"

namespace afb {
namespace {

constexpr int kHeadThreads = 256;

// One warp per requested entry: the dot product of a readout row with a policy-weight row (both read
// coalesced, 32 floats per step), plus the bias and the factorised from/to terms.
__global__ void __launch_bounds__(kHeadThreads) legal_logits_kernel(int64_t m, const int64_t *__restrict__ rows,
                                                                    const int64_t *__restrict__ cols, int64_t batch,
                                                                    int64_t n_out, const float *__restrict__ r,
                                                                    int64_t n_moves, const float *__restrict__ w,
                                                                    const float *__restrict__ b, int64_t n_sq,
                                                                    const float *__restrict__ f, const float *__restrict__ t,
                                                                    const int64_t *__restrict__ move_from,
                                                                    const int64_t *__restrict__ move_to,
                                                                    float *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = ((int64_t)gridDim.x * kHeadThreads) >> 5;
    for (int64_t i = ((int64_t)blockIdx.x * kHeadThreads + threadIdx.x) >> 5; i < m; i += warps) {
        const int64_t row = __ldg(rows + i), col = __ldg(cols + i);
        if (row < 0 || row >= batch || col < 0 || col >= n_moves) {
            if (lane == 0) out[i] = __int_as_float(0x7fc00000);   // NaN: the index was out of range
            continue;
        }
        const float *rr = r + row * n_out, *ww = w + col * n_out;
        float s = 0.f;
        for (int64_t k = lane; k < n_out; k += 32) s = fmaf(__ldg(rr + k), __ldg(ww + k), s);
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) {
            const int64_t sf = __ldg(move_from + col), st = __ldg(move_to + col);
            const bool ok = sf >= 0 && sf < n_sq && st >= 0 && st < n_sq;
            out[i] = ok ? s + __ldg(b + col) + __ldg(f + row * n_sq + sf) + __ldg(t + row * n_sq + st)
                        : __int_as_float(0x7fc00000);
        }
    }
}

}  // namespace
}  // namespace afb

using namespace afb;

extern "C" int afb_legal_logits(int64_t m, const int64_t *rows, const int64_t *cols, int64_t batch, int64_t n_out,
                                const float *r, int64_t n_moves, const float *w, const float *b, int64_t n_sq,
                                const float *f, const float *t, const int64_t *move_from, const int64_t *move_to,
                                float *out, void *stream) {
    return guarded([&] {
        AFB_CHECK(m >= 0 && batch >= 0 && n_out >= 0 && n_moves >= 0 && n_sq >= 0, "negative size");
        if (m == 0) return;
        AFB_CHECK(rows && cols && r && w && b && f && t && move_from && move_to && out, "NULL pointer");
        const int64_t grid64 = (m + kHeadThreads / 32 - 1) / (kHeadThreads / 32);
        const int grid = (int)(grid64 < 148 * 64 ? grid64 : 148 * 64);
        legal_logits_kernel<<<grid, kHeadThreads, 0, (cudaStream_t)stream>>>(m, rows, cols, batch, n_out, r, n_moves, w, b,
                                                                             n_sq, f, t, move_from, move_to, out);
        AFB_LAUNCHED();
    });
}
