"""The reference's CPU inference path restated on torch CPU sparse tensors -- TEST INFRASTRUCTURE ONLY.

Only bench.py's CPU-baseline legs (``cpu_baseline`` and ``--impl reference``) and tests/ use this module.
It times what the reference itself runs on a machine without CUDA: ``ConnectomeRNN.forward_io`` under
``torch.no_grad()`` with float32 input takes the generic light-cone path (chessfly/brain.py:307-329;
FUSED_UPDATE needs CUDA, brain.py:310), whose per-step work is

    x = (A_t @ h).add_(k_t)                          torch CPU CSR x dense SpMM   (brain.py:320-321)
    x.index_add_(0, u_pos_t, u_in[u_src_t])           the position's input         (brain.py:322-323)
    x.clamp_(0, h_max)                                                             (brain.py:324)
    prev = c_{t-1}[R_t] with the carried rows of h    index_copy                   (brain.py:325-327)
    h = lerp(prev, x, alpha[R_t])                                                  (brain.py:328)

and the output c_T[out_idx] with the reached outputs taken from h (brain.py:328-329).  The same torch
calls run here, on the same library kernels, so the timing is the reference's: in this repository's build
container (8 threads) the reference's own forward_io on configuration 3's graph ran 317 / 342 / 277
positions/s at B = 16 / 64 / 256 and this restatement 375 / 371 / 236 (run-to-run spread of the host),
with outputs equal to 9e-8 relative L2.  The weight-dependent constants (resting trajectory c_t, constant drive k_t) are computed
once per weight version by the reference (brain.py:296-306) and here by the numpy oracle in float64 and
rounded to float32, outside any timed region.  The reference's Python source is not needed at run time.
"""

from __future__ import annotations

import warnings

import numpy as np
import torch

from . import oracle as orc


class TorchCpuForward:
    """forward_io of the reference on the host cores (float32, torch CPU sparse CSR), for one graph."""

    def __init__(self, n, pre, post, sign, w0, log_gain, bias, alpha_logit, in_idx, out_idx, steps,
                 h_max=orc.H_MAX, cone=None):
        pre = np.asarray(pre, np.int64)
        post = np.asarray(post, np.int64)
        self.cone = cone = cone or orc.light_cone(n, pre, post, in_idx, out_idx, steps)
        w = orc.edge_weights(sign, w0, log_gain, np.float64)
        alpha = orc.sigmoid(np.asarray(alpha_logit, np.float64))
        cs, ks = orc.constants(orc.full_csr(n, pre, post), cone, w, np.asarray(bias, np.float64), alpha, h_max, np.float64)
        t32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32))
        i64 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int64))
        self.h_max = float(h_max)
        self.steps = steps
        self.plan = []
        for t in range(1, steps + 1):
            rows, op = cone.rows[t], cone.ops[t]
            mat = None
            if op is not None:
                with warnings.catch_warnings():          # torch's beta / invariant-check notices for sparse CSR
                    warnings.simplefilter("ignore")
                    mat = torch.sparse_csr_tensor(i64(op.crow), i64(op.pre), t32(w[op.edges]), op.shape,
                                                  check_invariants=False)
            self.plan.append(dict(mat=mat, k=t32(ks[t]), prev_c=t32(cs[t - 1][rows]), alpha=t32(alpha[rows][:, None]),
                                  keep_next=i64(cone.keep_next[t]), keep_prev=i64(cone.keep_prev[t]),
                                  u_pos=i64(cone.u_pos[t]), u_src=i64(cone.u_src[t])))
        self.c_out = t32(cs[steps][np.asarray(out_idx, np.int64)])
        self.out_pos, self.out_src = i64(cone.out_pos), i64(cone.out_src)

    @torch.no_grad()
    def __call__(self, u_in) -> torch.Tensor:
        """u_in (I, B) float32 (numpy or torch CPU) -> outputs (O, B) float32."""
        u_in = torch.as_tensor(np.ascontiguousarray(u_in, np.float32)) if isinstance(u_in, np.ndarray) else u_in.float()
        batch = u_in.shape[1]
        h = None
        for p in self.plan:
            if p["mat"] is None:
                x = p["k"].expand(-1, batch).index_add(0, p["u_pos"], u_in[p["u_src"]])
            else:
                x = (p["mat"] @ h).add_(p["k"])
                x.index_add_(0, p["u_pos"], u_in[p["u_src"]])
            x.clamp_(0, self.h_max)
            prev = p["prev_c"].expand(-1, batch)
            if len(p["keep_next"]):
                prev = prev.index_copy(0, p["keep_next"], h[p["keep_prev"]])
            h = torch.lerp(prev, x, p["alpha"])
        return self.c_out.expand(-1, batch).index_copy(0, self.out_pos, h[self.out_src])
