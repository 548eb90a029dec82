"""Connectome-constrained rate RNN on B200: the module API of chessfly/brain.py over libafb.so.

    h[t+1] = (1 - alpha) * h[t] + alpha * clamp(W h[t] + b + u, 0, h_max)

W is the fixed signed wiring (Dale's law) with a learnable positive gain per synapse; alpha (leak)
and b (bias) are learnable per neuron.  ``ConnectomeRNN`` keeps the reference's constructor,
parameters, buffers and methods (chessfly/brain.py:176-329), so checkpoints, ``FlyChessNet`` and the
search / training callers use it unchanged.  The work runs in the CUDA library:

* ``light_cone``  builds the per-step row sets, sub-matrices and maps on the GPU (``afb_cone_create``);
* ``forward_io``  (no grad) runs the fused SpMM step kernel once per step, float32 state for float32
  input, float16 deviation from the resting trajectory for float16 input (``afb_cone_forward``);
  with autograd it runs the float32 training forward and the library's backward (``_ConeTrain``);
* ``forward``     (no grad) runs the literal recurrence over all neurons (``afb_graph_forward``); with
  autograd, the same training path over the cone whose inputs and outputs are all neurons.

There is no CPU path: on CPU tensors these methods raise ``RuntimeError``.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch
from torch import nn

from . import _lib
from .connectome import Connectome

CHUNK_ELEMS = 1 << 26      # kept for API compatibility (chessfly/brain.py:25)
SAMPLED_ADDMM = True       # kept for API compatibility (chessfly/brain.py:62)
SDDMM_COLS = 64            # kept for API compatibility (chessfly/brain.py:63)


class _NativeKernel:
    """Stands where the reference keeps its jiterator kernels (chessfly/brain.py:37-58): the update
    they compute is fused into libafb's step kernel, so these are descriptions, not callables."""

    def __init__(self, what: str):
        self.what = what

    def __repr__(self) -> str:
        return f"<libafb fused step: {self.what}>"


FUSED_UPDATE = _NativeKernel("float32 state, p + a (clamp(y + k, 0, h_max) - p)")
FUSED_DEVIATION = _NativeKernel("float16 deviation, p + a (clamp(s, lo, hi) + e - p)")


def _stream(dev: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"alphafly_b200 runs on CUDA devices only ({what} is on {t.device}); there is no CPU path")


def _crow(sorted_rows: torch.Tensor, n: int) -> torch.Tensor:
    """CSR row pointer of sorted row indices (chessfly/brain.py:28-31)."""
    counts = np.bincount(sorted_rows.cpu().numpy(), minlength=n)
    crow = np.zeros(n + 1, np.int64)
    np.cumsum(counts, out=crow[1:])
    return torch.from_numpy(crow).to(sorted_rows.device)


def _t_order(rows: torch.Tensor, cols: torch.Tensor, n_rows: int) -> torch.Tensor:
    """Edge permutation into the CSR order of the transpose: stable argsort of col * n_rows + row."""
    key = cols.cpu().numpy().astype(np.int64) * n_rows + rows.cpu().numpy()
    return torch.from_numpy(np.argsort(key, kind="stable")).to(rows.device)


class _SubMatrix:
    """W[R_t, R_{t-1}] as built by the library, with the reference's fields (chessfly/brain.py:102-123):
    ``edges`` (into W's edge list), local ``post`` / ``pre``, ``crow``, and the transpose's ``t_order``,
    ``t_crow``, ``t_col``, each an int64 tensor on the cone's device, exported on first access."""

    _FIELDS = ("edges", "post", "pre", "crow", "t_order", "t_crow", "t_col")

    def __init__(self, cone: "LightCone", t: int, n_rows: int, n_cols: int, nnz: int):
        self._cone, self._t, self._nnz = cone, t, nnz
        self.shape = (n_rows, n_cols)
        self._cache: dict[str, torch.Tensor] = {}

    def __getattr__(self, name):
        if name in _SubMatrix._FIELDS:
            if name not in self._cache:
                size = {"crow": self.shape[0] + 1, "t_crow": self.shape[1] + 1}.get(name, self._nnz)
                self._cache[name] = self._cone._export(name, self._t, size)
            return self._cache[name]
        raise AttributeError(name)

    def csr(self, w):
        return torch.sparse_csr_tensor(self.crow, self.pre, w, self.shape, check_invariants=False)

    def csr_t(self, w):
        return torch.sparse_csr_tensor(self.t_crow, self.t_col, w[self.t_order], self.shape[::-1], check_invariants=False)


class LightCone:
    """Rows per step that can differ between positions and can still reach an output (the reference's
    LightCone, chessfly/brain.py:126-173), built on the GPU by ``afb_cone_create``.

    Fields, as in the reference: ``rows[t]``, ``ops[t]`` (a _SubMatrix or None), ``carried[t]`` (bool,
    (|R_t|, 1)), ``keep_next[t]``, ``keep_prev[t]``, ``prev_row[t]``, ``u_pos[t]``, ``u_src[t]``,
    ``out_pos``, ``out_src``, ``out_idx``, ``edge_visits``, ``steps``; index 0 of the per-step lists
    is None (``rows[0]`` is the empty R_0)."""

    def __init__(self, rnn: "ConnectomeRNN", in_idx: torch.Tensor, out_idx: torch.Tensor, steps: int):
        dev = rnn.pre.device
        _require_cuda(rnn.pre, "the wiring")
        self.device, self.steps = dev, steps
        in_idx = in_idx.to(dev, torch.long).contiguous()
        out_idx = out_idx.to(dev, torch.long).contiguous()
        handle = ctypes.c_void_p()
        with torch.cuda.device(dev):
            lib = _lib.load()
            _lib.check(lib.afb_cone_create(ctypes.byref(handle), rnn.n, rnn.pre.numel(), _ptr(rnn.pre), _ptr(rnn.post),
                                           _ptr(in_idx), in_idx.numel(), _ptr(out_idx), out_idx.numel(), steps,
                                           _stream(dev)))
        self._h = handle
        self._lib = lib
        t1 = steps + 1
        rows_len, nnz, n_keep, n_fed = ((ctypes.c_int64 * t1)() for _ in range(4))
        n_hit, visits = ctypes.c_int64(), ctypes.c_int64()
        _lib.check(lib.afb_cone_sizes(handle, rows_len, nnz, n_keep, n_fed, ctypes.byref(n_hit), ctypes.byref(visits)))
        self.rows_len = list(rows_len)
        self.nnz = [0 if x < 0 else x for x in nnz]
        self.edge_visits = int(visits.value)
        self.rows = [self._export("rows", t, rows_len[t]) for t in range(t1)]
        self.ops, self.carried, self.keep_next, self.keep_prev = [None], [None], [None], [None]
        self.prev_row, self.u_pos, self.u_src = [None], [None], [None]
        for t in range(1, t1):
            self.ops.append(_SubMatrix(self, t, rows_len[t], rows_len[t - 1], nnz[t]) if nnz[t] >= 0 else None)
            self.carried.append(self._export("carried", t, rows_len[t]).bool().unsqueeze(1))
            self.keep_next.append(self._export("keep_next", t, n_keep[t]))
            self.keep_prev.append(self._export("keep_prev", t, n_keep[t]))
            self.prev_row.append(self._export("prev_row", t, rows_len[t]))
            self.u_pos.append(self._export("u_pos", t, n_fed[t]))
            self.u_src.append(self._export("u_src", t, n_fed[t]))
        self.out_pos = self._export("out_pos", 0, n_hit.value)
        self.out_src = self._export("out_src", 0, n_hit.value)
        self.out_idx = out_idx
        self.n_in, self.n_out = in_idx.numel(), out_idx.numel()
        self.n = rnn.n
        self._weights: dict[int, tuple] = {}
        self.generation = {}                  # mode -> count of set_weight_tensors calls (which constants are live)

    def _export(self, field: str, t: int, size: int) -> torch.Tensor:
        out = torch.empty(int(size), dtype=torch.long, device=self.device)
        if size:
            with torch.cuda.device(self.device):
                _lib.check(self._lib.afb_cone_export(self._h, _lib.FIELDS[field], t, _ptr(out), _stream(self.device)))
        return out

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                torch.cuda.synchronize(self.device)
            except Exception:
                pass
            self._lib.afb_cone_destroy(h)
            self._h = None

    # -- native forward -------------------------------------------------------------------------
    def set_weights(self, rnn: "ConnectomeRNN", mode: int, key) -> None:
        """(Re)compute the weight-dependent constants of ``mode`` unless ``key`` is unchanged."""
        if self._weights.get(mode) == key:
            return
        with torch.no_grad():
            self.set_weight_tensors(mode, rnn.edge_weights(), rnn.bias, rnn.alpha_logit, rnn.h_max)
        self._weights[mode] = key

    def set_weight_tensors(self, mode: int, w, bias, alpha_logit, h_max) -> None:
        """Constants of ``mode`` from explicit edge weights, bias and alpha logits (``afb_cone_set_weights``)."""
        self._weights.pop(mode, None)
        self.generation[mode] = self.generation.get(mode, 0) + 1
        with torch.cuda.device(self.device):
            w = w.detach().float().contiguous()
            bias = bias.detach().float().contiguous()
            alpha_logit = alpha_logit.detach().float().contiguous()
            h = float("inf") if h_max is None else float(h_max)
            _lib.check(self._lib.afb_cone_set_weights(self._h, mode, _ptr(w), _ptr(bias), _ptr(alpha_logit), h,
                                                      _stream(self.device)))

    def resting(self, t: int) -> torch.Tensor:
        """c_t, the resting trajectory (no position's input) after t steps, (N,) float32, for the weights of
        the last ``set_weights`` (``afb_cone_resting``)."""
        out = torch.empty(self.n, dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            _lib.check(self._lib.afb_cone_resting(self._h, int(t), _ptr(out), _stream(self.device)))
        return out

    def status(self, reset: bool = True) -> int:
        """Device status word of this cone's step kernels (``afb_cone_status``): 0 = ok; non-zero would
        mean that a forward since the last reset produced invalid output.  Synchronises the current
        stream."""
        st = ctypes.c_int(0)
        with torch.cuda.device(self.device):
            _lib.check(self._lib.afb_cone_status(self._h, ctypes.byref(st), int(reset), _stream(self.device)))
        return st.value

    def forward(self, mode: int, u_in: torch.Tensor, events=None) -> torch.Tensor:
        """Native forward; ``events`` (steps + 2 recorded torch.cuda.Event objects with timing) brackets
        each step's kernel and the output kernel for per-step timing."""
        batch = u_in.shape[1]
        out = torch.empty(self.n_out, batch, dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            ws_bytes = self._lib.afb_cone_forward_workspace(self._h, mode, batch)
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=self.device)
            ev = None
            if events is not None:
                assert len(events) == self.steps + 2
                ev = (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])
            _lib.check(self._lib.afb_cone_forward_timed(self._h, mode, _ptr(u_in), u_in.stride(0), batch, _ptr(out), batch,
                                                        _ptr(ws), ws_bytes, ev, _stream(self.device)))
        return out


class _Graph:
    """The whole wiring as one CSR matrix for the literal recurrence (``afb_graph_create``)."""

    def __init__(self, rnn: "ConnectomeRNN"):
        self.device = rnn.pre.device
        self._lib = _lib.load()
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(self._lib.afb_graph_create(ctypes.byref(h), rnn.n, rnn.pre.numel(), _ptr(rnn.pre), _ptr(rnn.post),
                                                  _stream(self.device)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                torch.cuda.synchronize(self.device)
            except Exception:
                pass
            self._lib.afb_graph_destroy(h)
            self._h = None

    def status(self, reset: bool = True) -> int:
        st = ctypes.c_int(0)
        with torch.cuda.device(self.device):
            _lib.check(self._lib.afb_graph_status(self._h, ctypes.byref(st), int(reset), _stream(self.device)))
        return st.value

    def forward(self, rnn: "ConnectomeRNN", u: torch.Tensor, steps: int) -> torch.Tensor:
        batch = u.shape[1]
        h = torch.empty(rnn.n, batch, dtype=torch.float32, device=self.device)
        with torch.no_grad(), torch.cuda.device(self.device):
            w = rnn.edge_weights().float().contiguous()
            bias = rnn.bias.detach().float().contiguous()
            alpha_logit = rnn.alpha_logit.detach().float().contiguous()
            h_max = float("inf") if rnn.h_max is None else float(rnn.h_max)
            ws_bytes = self._lib.afb_graph_forward_workspace(self._h, batch)
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=self.device)
            _lib.check(self._lib.afb_graph_forward(self._h, _ptr(w), _ptr(bias), _ptr(alpha_logit), h_max, _ptr(u),
                                                   u.stride(0), batch, steps, _ptr(h), batch, _ptr(ws), ws_bytes,
                                                   _stream(self.device)))
        return h


class _EdgeWeights(torch.autograd.Function):
    """w = sign * w0 * exp(log_gain) in the library; dL/dlog_gain = dL/dw * w."""

    @staticmethod
    def forward(ctx, log_gain, sign, w0):
        lg = log_gain.detach().float().contiguous()
        w = torch.empty_like(lg)
        with torch.cuda.device(lg.device):
            _lib.call("afb_edge_weights", lg.numel(), _ptr(sign.float().contiguous()), _ptr(w0.float().contiguous()),
                      _ptr(lg), _ptr(w), _stream(lg.device))
        ctx.save_for_backward(w)
        return w.to(log_gain.dtype)

    @staticmethod
    def backward(ctx, grad_w):
        (w,) = ctx.saved_tensors
        return grad_w * w.to(grad_w.dtype), None, None


class _ConeTrain(torch.autograd.Function):
    """forward_io with autograd (chessfly/brain.py:289-294, 315-329): the library's float32 training
    forward keeps every step's state, and its backward returns dL/du_in, dL/dw, dL/db and dL/dalpha in
    one pass (``afb_cone_backward``).  Inputs: u_in (I, B) float32, w (E) = edge weights (autograd links
    them to log_gain), bias (N), alpha_logit (N)."""

    @staticmethod
    def forward(ctx, u_in, w, bias, alpha_logit, cone, h_max):
        dev = cone.device
        batch = u_in.shape[1]
        u_in = u_in.contiguous()
        cone.set_weight_tensors(_lib.MODE_F32, w, bias, alpha_logit, h_max)
        lib = cone._lib
        with torch.cuda.device(dev):
            saved_bytes = lib.afb_cone_train_workspace(cone._h, batch)
            saved = torch.empty(saved_bytes, dtype=torch.uint8, device=dev)
            out = torch.empty(cone.n_out, batch, dtype=torch.float32, device=dev)
            _lib.check(lib.afb_cone_forward_train(cone._h, _ptr(u_in), u_in.stride(0), batch, _ptr(out), batch,
                                                  _ptr(saved), saved_bytes, _stream(dev)))
        ctx.cone, ctx.h_max, ctx.batch, ctx.n_in, ctx.saved_state = cone, h_max, batch, u_in.shape[0], saved
        ctx.generation = cone.generation[_lib.MODE_F32]
        ctx.save_for_backward(w.detach(), bias.detach(), alpha_logit.detach())
        return out

    @staticmethod
    def backward(ctx, g_out):
        cone, batch = ctx.cone, ctx.batch
        w, bias, alpha_logit = ctx.saved_tensors
        dev = cone.device
        lib = cone._lib
        # the cone's constants must be those of this forward's weights: set again if another call replaced them
        if cone.generation.get(_lib.MODE_F32) != ctx.generation:
            cone.set_weight_tensors(_lib.MODE_F32, w, bias, alpha_logit, ctx.h_max)
        g_out = g_out.float().contiguous()
        with torch.cuda.device(dev):
            ws_bytes = lib.afb_cone_backward_workspace(cone._h, batch)
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
            g_u = torch.empty(ctx.n_in, batch, dtype=torch.float32, device=dev)
            g_w = torch.empty_like(w, dtype=torch.float32)
            g_b = torch.empty_like(bias, dtype=torch.float32)
            g_a = torch.empty_like(alpha_logit, dtype=torch.float32)
            saved = ctx.saved_state
            _lib.check(lib.afb_cone_backward(cone._h, _ptr(g_out), g_out.stride(0), batch, _ptr(saved), saved.numel(),
                                             _ptr(g_u), batch, _ptr(g_w), _ptr(g_b), _ptr(g_a), _ptr(ws), ws_bytes,
                                             _stream(dev)))
        ctx.saved_state = None
        alpha = torch.sigmoid(alpha_logit.float())
        g_logit = g_a * alpha * (1 - alpha)
        return (g_u if ctx.needs_input_grad[0] else None, g_w.to(w.dtype), g_b.to(bias.dtype),
                g_logit.to(alpha_logit.dtype), None, None)


class ConnectomeRNN(nn.Module):
    def __init__(self, conn: Connectome, alpha_init: float = 0.5, bias_init: float = 0.0,
                 global_scale: float = 1.0, h_max: float | None = 10.0):
        """
        global_scale multiplier on the normalised connectome weights
        h_max        activity is clamped to [0, h_max]
        """
        super().__init__()
        self.n = conn.n_neurons
        self.h_max = h_max
        # the wiring is rebuilt from the connectome, never stored in checkpoints (chessfly/brain.py:186-195)
        self.register_buffer("pre", conn.pre, persistent=False)
        self.register_buffer("post", conn.post, persistent=False)
        self.register_buffer("sign", conn.sign, persistent=False)
        self.register_buffer("w0", conn.weight * global_scale, persistent=False)
        self.register_buffer("crow", _crow(conn.post, self.n), persistent=False)
        t_order = _t_order(conn.post, conn.pre, self.n)
        self.register_buffer("t_order", t_order, persistent=False)
        self.register_buffer("t_crow", _crow(conn.pre[t_order], self.n), persistent=False)
        self.register_buffer("t_col", conn.post[t_order], persistent=False)
        self.log_gain = nn.Parameter(torch.zeros(conn.n_edges))
        self.bias = nn.Parameter(torch.full((self.n,), float(bias_init)))
        a = torch.full((self.n,), float(alpha_init))
        self.alpha_logit = nn.Parameter(torch.log(a / (1 - a)))

    def edge_weights(self) -> torch.Tensor:
        _require_cuda(self.log_gain, "log_gain")
        return _EdgeWeights.apply(self.log_gain, self.sign, self.w0)

    def csr(self, w: torch.Tensor) -> torch.Tensor:
        return torch.sparse_csr_tensor(self.crow, self.pre, w, (self.n, self.n), check_invariants=False)

    def csr_t(self, w: torch.Tensor) -> torch.Tensor:
        return torch.sparse_csr_tensor(self.t_crow, self.t_col, w[self.t_order], (self.n, self.n), check_invariants=False)

    def __deepcopy__(self, memo):
        """A copy without the native handles (light cone, whole-graph CSR): the copy builds its own on first
        use, on whatever device it is moved to."""
        import copy
        new = self.__class__.__new__(self.__class__)
        memo[id(self)] = new
        for k, v in self.__dict__.items():
            new.__dict__[k] = None if k in ("_cone", "_graph_cache", "_all_idx", "_cached_f32") else copy.deepcopy(v, memo)
        return new

    # -- the literal recurrence ---------------------------------------------------------------------
    def _graph(self) -> _Graph:
        key = (self.pre.data_ptr(), str(self.pre.device))
        if getattr(self, "_graph_cache", None) is None or self._graph_cache[0] != key:
            self._graph_cache = (key, _Graph(self))
        return self._graph_cache[1]

    def forward(self, u: torch.Tensor, steps: int) -> torch.Tensor:
        """u: (N, B) contiguous constant external drive.  Returns the state after ``steps`` updates, (N, B).
        Computed in float32 (float16 input gives a float16 result).  Unlike the reference's no-grad branch
        (chessfly/brain.py:218), ``u`` is not modified."""
        assert u.is_contiguous()
        if u.dim() != 2 or u.shape[0] != self.n:
            raise ValueError(f"u must be (N, B) = ({self.n}, B), got {tuple(u.shape)}")
        _require_cuda(u, "u")
        if u.device != self.pre.device:
            raise RuntimeError(f"u must be on the module's device {self.pre.device}")
        if u.dtype not in (torch.float32, torch.float16):
            raise TypeError(f"alphafly_b200 computes in float32 or float16, got {u.dtype}")
        if torch.is_grad_enabled() and (u.requires_grad or any(p.requires_grad for p in self.parameters())):
            # the literal recurrence is the light cone with every neuron an input and an output
            everyone = self._everyone()
            cone = self.light_cone(everyone, everyone, steps)
            h = _ConeTrain.apply(u.float(), self.edge_weights(), self.bias, self.alpha_logit, cone, self.h_max)
            return h.to(u.dtype)
        h = self._graph().forward(self, u.float().contiguous(), steps)
        return h.to(u.dtype)

    def _everyone(self) -> torch.Tensor:
        if getattr(self, "_all_idx", None) is None or self._all_idx.device != self.pre.device:
            self._all_idx = torch.arange(self.n, device=self.pre.device)
        return self._all_idx

    def device_status(self, reset: bool = True) -> int:
        """0 if every native kernel since the last reset completed normally, else the library's status
        code (see ``afb_cone_status``).  Synchronises the device's current stream."""
        st = 0
        for cache in (getattr(self, "_cone", None), getattr(self, "_graph_cache", None)):
            if cache is not None:
                st = st or cache[1].status(reset)
        return st

    # -- the same function through the light cone ---------------------------------------------------
    def light_cone(self, in_idx: torch.Tensor, out_idx: torch.Tensor, steps: int) -> LightCone:
        key = (steps, in_idx.data_ptr(), out_idx.data_ptr(), str(self.pre.device))
        if getattr(self, "_cone", None) is None or self._cone[0] != key:
            self._cone = (key, LightCone(self, in_idx, out_idx, steps))
        return self._cone[1]

    @property
    def _cached(self):
        """The float32 path's weight-dependent constants in the reference's layout, (key, (cs, ks, mats, alpha,
        fused)), for diagnostics that read them (scripts/profile_gpu.py:27; built by chessfly/brain.py:296-305):
        cs[t] the resting trajectory (N, 1), ks[t] the constant drive of R_t (|R_t|, 1), mats[t] the sub-matrix
        W[R_t, R_{t-1}] as a sparse CSR tensor (None where the step has none), alpha (N, 1), fused[t] =
        (carried, c_{t-1}[R_t], alpha[R_t]).  Made on demand for the light cone last used (the native
        forward keeps its own constants); None before any light-cone forward."""
        cone = getattr(self, "_cone", None)
        if cone is None:
            return None
        cone = cone[1]
        key = (self.log_gain._version, self.bias._version, self.alpha_logit._version, torch.float32, id(cone))
        hit = getattr(self, "_cached_f32", None)
        if hit is not None and hit[0] == key:
            return hit
        with torch.no_grad():
            w = self.edge_weights()
            cone.set_weights(self, _lib.MODE_F32, self._weight_key(_lib.MODE_F32, cone))
            alpha = torch.sigmoid(self.alpha_logit).unsqueeze(1)
            cs = [cone.resting(t).unsqueeze(1) for t in range(cone.steps + 1)]
            full = self.csr(w)
            ks, mats, fused = [None], [None], [None]
            for t in range(1, cone.steps + 1):
                rows, op = cone.rows[t], cone.ops[t]
                drive = (full @ cs[t - 1] if t > 1 else torch.zeros_like(cs[0])) + self.bias.unsqueeze(1)
                k = drive[rows]
                mat = None
                if op is not None:
                    mat = op.csr(w[op.edges])
                    k = k - mat @ cs[t - 1][cone.rows[t - 1]]
                ks.append(k)
                mats.append(mat)
                fused.append((cone.carried[t].float(), cs[t - 1][rows].contiguous(), alpha[rows].contiguous()))
        self._cached_f32 = (key, (cs, ks, mats, alpha, fused))
        return self._cached_f32

    def _weight_key(self, mode, cone):
        return (self.log_gain._version, self.bias._version, self.alpha_logit._version, self.log_gain.data_ptr(),
                self.bias.data_ptr(), self.alpha_logit.data_ptr(), mode, id(cone))

    def forward_io(self, u_in: torch.Tensor, in_idx: torch.Tensor, out_idx: torch.Tensor, steps: int) -> torch.Tensor:
        """u_in: (len(in_idx), B) drive of the input neurons.  Returns the output neurons after ``steps``
        updates, (len(out_idx), B): exactly forward(u, steps)[out_idx] with u zero outside in_idx.
        float16 input runs the float16-deviation path and returns float32 (chessfly/brain.py:287-288)."""
        if u_in.dim() != 2 or u_in.shape[0] != in_idx.numel():
            raise ValueError(f"u_in must be (len(in_idx), B) = ({in_idx.numel()}, B), got {tuple(u_in.shape)}")
        _require_cuda(u_in, "u_in")
        if u_in.device != self.pre.device or in_idx.device != self.pre.device or out_idx.device != self.pre.device:
            raise RuntimeError(f"u_in, in_idx and out_idx must be on the module's device {self.pre.device}")
        if u_in.dtype not in (torch.float32, torch.float16):
            raise TypeError(f"alphafly_b200 computes in float32 or float16, got {u_in.dtype}")
        cone = self.light_cone(in_idx, out_idx, steps)
        if torch.is_grad_enabled():
            out = _ConeTrain.apply(u_in.float(), self.edge_weights(), self.bias, self.alpha_logit, cone, self.h_max)
            return out.to(u_in.dtype)
        mode = _lib.MODE_DEV16 if u_in.dtype == torch.float16 else _lib.MODE_F32
        cone.set_weights(self, mode, self._weight_key(mode, cone))
        u_in = u_in if u_in.stride(1) == 1 else u_in.contiguous()
        return cone.forward(mode, u_in)
