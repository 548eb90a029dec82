"""Policy/value network whose only hidden computation is the connectome (chessfly/model.py).

    board features --dense map--> sensory neurons --T steps of the wiring--> output neurons
    --RunningNorm--> dense readouts --> move logits, win/draw/loss logits

``FlyChessNet``, ``RunningNorm``, ``Evaluator``, ``ModelConfig``, ``load_weights`` and ``load_net`` keep the
reference's names, parameters, buffers and state_dict keys (chessfly/model.py:26-161), so checkpoints
load unchanged.  The recurrence runs in ``alphafly_b200.brain`` (libafb).  The input map writes the
(sensory neurons, batch) layout the recurrence reads in one GEMM (W x^T scaled by the input gain),
instead of x W^T followed by a transpose copy: for float16 inference in libafb's tensor-core kernel
(``input_map_f16``), in float32 (training, the float32 path) through cuBLAS.  In inference the normaliser
and the heads are one tensor-core readout in libafb (``FlyChessNet.heads``: the factorised from/to terms
folded into the policy rows, float32 accuracy from split float16 operands); training keeps the float32
layers, whose gradients autograd takes.
"""

from __future__ import annotations

import dataclasses
from collections import OrderedDict

import numpy as np
import torch
from torch import nn

from . import _lib
from .brain import ConnectomeRNN
from .connectome import Connectome
from .encoding import N_BASE, N_FEATURES, N_MOVES, move_squares
from .gemm import affine, status_word

READOUT_SUPERCLASSES = ("descending_neuron",)   # plus every efferent neuron (chessfly/model.py:23)


@dataclasses.dataclass
class ModelConfig:
    steps: int = 4
    min_syn: int = 3
    shuffled: bool = False
    attack_planes: bool = False
    input_gain: float = 5.0
    weight_scale: float = 2.0
    bias_init: float = 0.1


class RunningNorm(nn.Module):
    """Per-neuron standardisation with running statistics in both modes (chessfly/model.py:37-58): in
    training the first batch sets mean and variance, later ones move them by ``momentum``; the output is
    (r - mean) / sqrt(var + eps), clipped to +-clip."""

    def __init__(self, n: int, momentum: float = 0.05, eps: float = 1e-8, clip: float = 8.0):
        super().__init__()
        self.momentum, self.eps, self.clip = momentum, eps, clip
        self.register_buffer("mean", torch.zeros(n))
        self.register_buffer("var", torch.ones(n))
        self.register_buffer("initialised", torch.tensor(False))
        # data-parallel training: callable r -> (mean, unbiased variance) of the batch of all ranks
        self.batch_sync = None

    def forward(self, r: torch.Tensor) -> torch.Tensor:
        if self.training and r.shape[0] > 1:
            with torch.no_grad():
                # weight 1 for the first batch, else momentum; chosen on the device (no host read-back)
                m = torch.where(self.initialised, self.momentum, 1.0).to(self.mean.dtype)
                mean, var = self.batch_sync(r) if self.batch_sync is not None else (r.mean(0), r.var(0))
                self.mean.lerp_(mean, m)
                self.var.lerp_(var, m)
                self.initialised.fill_(True)
        return ((r - self.mean) / (self.var + self.eps).sqrt()).clamp(-self.clip, self.clip)


class FlyChessNet(nn.Module):
    def __init__(self, conn: Connectome, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        # float16 inference is the deviation form (brain.forward_io with float16 input), as in the reference
        self.infer_dtype = torch.float16
        if cfg.shuffled:
            conn = conn.shuffled()
        self.brain = ConnectomeRNN(conn, bias_init=cfg.bias_init, global_scale=cfg.weight_scale)
        self.register_buffer("in_idx", conn.nodes("afferent"), persistent=False)
        out = torch.cat([conn.nodes("efferent"), conn.nodes_of_superclass(*READOUT_SUPERCLASSES)]).unique()
        self.register_buffer("out_idx", out, persistent=False)
        self.encoder = nn.Linear(N_FEATURES, len(self.in_idx))
        self.norm = RunningNorm(len(out))
        self.policy = nn.Linear(len(out), N_MOVES)
        self.value = nn.Linear(len(out), 3)
        self.policy_from, self.policy_to = nn.Linear(len(out), 64), nn.Linear(len(out), 64)
        frm, to = move_squares()
        self.register_buffer("move_from", torch.as_tensor(frm), persistent=False)
        self.register_buffer("move_to", torch.as_tensor(to), persistent=False)
        # [from; to] squares -> moves as a 0/1 matrix (128, N_MOVES): the factorised terms of the training
        # heads become one GEMM, whose backward is a GEMM too (a column gather's backward is a sorted
        # scatter-add, 1.1 ms per head at B = 2,048)
        sel = torch.zeros(128, N_MOVES)
        sel[torch.as_tensor(frm).long(), torch.arange(N_MOVES)] = 1.0
        sel[64 + torch.as_tensor(to).long(), torch.arange(N_MOVES)] = 1.0
        self.register_buffer("move_select", sel, persistent=False)
        for layer in (self.policy_from, self.policy_to):
            nn.init.zeros_(layer.weight)
            nn.init.zeros_(layer.bias)
        nn.init.zeros_(self.policy.weight)
        nn.init.zeros_(self.value.weight)

    def drive(self, x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        """u_in (sensory neurons, batch) = input_gain * (W x^T + b), over the first N_BASE features unless
        the attack planes are switched on (chessfly/model.py:98-102).  For the float16 inference path the
        product runs on the tensor cores (``input_map_f16``): float16 weights (a copy refreshed when the
        encoder changes) times the float16 features (board bits, exact), accumulated in float32 and rounded
        once to the float16 drive the deviation path reads; everything else is float32 as in the reference."""
        k = N_FEATURES if self.cfg.attack_planes else N_BASE
        g = self.cfg.input_gain
        if dtype == torch.float16 and x.is_cuda and not torch.is_grad_enabled():
            w16, b16 = self.half_encoder()
            return input_map_f16(w16, b16, x[:, :k], g, self._map_status(x.device))
        w, b = self.encoder.weight[:, :k], self.encoder.bias
        if x.is_cuda and torch.is_grad_enabled():      # training: the product on the tensor cores, float32-accurate
            u = affine(w, x[:, :k].float(), b, 1, alpha=g, beta=g)
        else:
            u = torch.addmm(b.unsqueeze(1), w, x[:, :k].float().T, beta=g, alpha=g)
        return u.to(dtype).contiguous()

    @torch.no_grad()
    def half_encoder(self) -> tuple[torch.Tensor, torch.Tensor]:
        """The float16 copy of the encoder's weight (first k columns) and bias, rewritten in place when a
        parameter changed (so a captured CUDA graph reading it stays valid)."""
        k = N_FEATURES if self.cfg.attack_planes else N_BASE
        w, b = self.encoder.weight, self.encoder.bias
        key = (w._version, b._version)
        where = (w.data_ptr(), b.data_ptr(), k)
        c = getattr(self, "_enc16", None)
        if c is None or c[1] != where:
            w16 = torch.zeros(w.shape[0], -(-k // 8) * 8, dtype=torch.float16, device=w.device)[:, :k]   # rows on 16 B
            w16.copy_(w[:, :k])
            c = [key, where, w16, b.half()]
            self._enc16 = c
        elif c[0] != key:
            c[2].copy_(w[:, :k])
            c[3].copy_(b)
            c[0] = key
        return c[2], c[3]

    def _map_status(self, device) -> torch.Tensor:
        """The input map's device status word on ``device`` (0 = ok; set when a bounded wait gave up)."""
        st = getattr(self, "_status", None)
        if st is None or st.device != device:
            st = self._status = torch.zeros(1, dtype=torch.int32, device=device)
        return st

    def device_status(self, reset: bool = True) -> int:
        """0 if every library kernel this network ran on its device since the last reset completed
        normally: the light-cone step kernels (``brain.device_status``), the input map and the readout, and
        the training products (``gemm.affine``).  Otherwise the first non-zero code: a bounded wait in a
        kernel gave up and that call's output is not valid.  Reads device words, so it synchronises the
        device's current stream; ``reset`` clears them."""
        st = self.brain.device_status(reset)
        dev = self.brain.pre.device
        for word in (getattr(self, "_status", None), status_word(dev)):
            if word is not None and word.device == dev:
                v = int(word.item())
                if reset and v:
                    word.zero_()
                st = st or v
        return st

    def brain_output(self, x: torch.Tensor) -> torch.Tensor:
        """x: (B, N_FEATURES) -> the output neurons after the recurrence, (len(out_idx), B) float32
        (chessfly/model.py:97-103 up to the normaliser)."""
        dtype = self.infer_dtype if x.is_cuda and not torch.is_grad_enabled() else torch.float32
        u_in = self.drive(x, dtype)
        return self.brain.forward_io(u_in, self.in_idx, self.out_idx, self.cfg.steps)

    def readout(self, x: torch.Tensor) -> torch.Tensor:
        """x: (B, N_FEATURES) -> the normalised output-neuron state r (B, len(out_idx)) the heads read
        (chessfly/model.py:97-103)."""
        return self.norm(self.brain_output(x).T.float())

    def forward(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """x: (B, N_FEATURES) -> policy logits (B, N_MOVES), WDL logits (B, 3).  Inference on a GPU with the
        normaliser in eval mode runs the normaliser and the heads as one tensor-core readout (``heads``);
        training (and a normaliser still collecting statistics) keeps the float32 layers."""
        if x.is_cuda and not torch.is_grad_enabled() and not self.norm.training:
            return self.heads(self.brain_output(x))
        return self.dense_heads(self.readout(x))

    def dense_heads(self, r: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """The heads as the reference's float32 layers on the normalised state r (B, len(out_idx))
        (chessfly/model.py:104-105); the training path, through which autograd runs.  The from/to terms
        F[:, move_from[m]] + T[:, move_to[m]] are taken as [F, T] @ move_select, the same sums (each column
        of move_select holds two ones).  In training (autograd on, CUDA) the policy and from/to products and
        their gradients run on the tensor cores at float32 accuracy (``gemm.affine``, libafb's afb_gemm_f32)."""
        w_ft = torch.cat([self.policy_from.weight, self.policy_to.weight])
        b_ft = torch.cat([self.policy_from.bias, self.policy_to.bias])
        if r.is_cuda and torch.is_grad_enabled():
            policy = affine(r, self.policy.weight, self.policy.bias, 2)
            ft = affine(r, w_ft, b_ft, 2)
        else:
            policy = self.policy(r)
            ft = torch.addmm(b_ft, r, w_ft.T)
        logits = torch.addmm(policy, ft, self.move_select)
        return logits, self.value(r)

    @torch.no_grad()
    def folded_heads(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(W_hi, W_lo, bias) of the tensor-core readout: the policy rows with the factorised from/to terms
        folded in (W[m] = Wp[m] + Wf[move_from[m]] + Wt[move_to[m]], exact by linearity), then the value
        rows, as float16 hi / scaled lo parts (``afb_heads_split``) with 16-byte rows, and the float32 bias.
        Rewritten in place when a head parameter changed, so a captured CUDA graph reading them stays valid."""
        layers = (self.policy, self.policy_from, self.policy_to, self.value)
        params = [t for layer in layers for t in (layer.weight, layer.bias)]
        key = tuple(t._version for t in params)
        where = tuple(t.data_ptr() for t in params)
        c = getattr(self, "_heads16", None)
        if c is not None and c[0] == key and c[1] == where:
            return c[2], c[3], c[4]
        w = torch.cat([self.policy.weight + self.policy_from.weight[self.move_from] + self.policy_to.weight[self.move_to],
                       self.value.weight]).float().contiguous()
        b = torch.cat([self.policy.bias + self.policy_from.bias[self.move_from] + self.policy_to.bias[self.move_to],
                       self.value.bias]).float().contiguous()
        rows, n_out = w.shape
        ldw = -(-n_out // 8) * 8
        if c is None or c[1] != where or c[2].shape != (rows, ldw):
            hi = torch.empty(rows, ldw, dtype=torch.float16, device=w.device)
            lo = torch.empty_like(hi)
            bias = torch.empty(rows, dtype=torch.float32, device=w.device)
        else:
            hi, lo, bias = c[2], c[3], c[4]
        bias.copy_(b)
        with torch.cuda.device(w.device):
            _lib.call("afb_heads_split", rows, n_out, w.data_ptr(), n_out, hi.data_ptr(), lo.data_ptr(), ldw,
                      torch.cuda.current_stream(w.device).cuda_stream)
        self._heads16 = (key, where, hi, lo, bias)
        return hi, lo, bias

    @torch.no_grad()
    def heads(self, out: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """The readout on the tensor cores: out (len(out_idx), B) float32, the recurrence's output, ->
        policy logits (B, N_MOVES) and WDL logits (B, 3), float32 (``afb_readout_heads``: RunningNorm with
        the running statistics, then the folded heads at float32 accuracy)."""
        hi, lo, bias = self.folded_heads()
        n_out, batch = out.shape
        out = out if out.dtype == torch.float32 and out.stride(1) == 1 else out.float().contiguous()
        dev = out.device
        logits = torch.empty(batch, N_MOVES, dtype=torch.float32, device=dev)
        wdl = torch.empty(batch, 3, dtype=torch.float32, device=dev)
        lib = _lib.load()
        ws = torch.empty(lib.afb_readout_workspace(batch, n_out), dtype=torch.uint8, device=dev)
        norm = self.norm
        with torch.cuda.device(dev):
            _lib.check(lib.afb_readout_heads(n_out, batch, out.data_ptr(), out.stride(0), norm.mean.data_ptr(),
                                             norm.var.data_ptr(), float(norm.eps), float(norm.clip), hi.shape[0], N_MOVES,
                                             hi.data_ptr(), lo.data_ptr(), hi.shape[1], bias.data_ptr(), logits.data_ptr(),
                                             N_MOVES, 0, wdl.data_ptr(), 3, ws.data_ptr(), ws.numel(),
                                             self._map_status(dev).data_ptr(), torch.cuda.current_stream(dev).cuda_stream))
        return logits, wdl

    @staticmethod
    def expected_value(wdl_logits: torch.Tensor) -> torch.Tensor:
        p = wdl_logits.softmax(-1)
        return p[..., 0] - p[..., 2]


def input_map_f16(w16: torch.Tensor, b16: torch.Tensor, x: torch.Tensor, gain: float,
                  status: torch.Tensor | None = None) -> torch.Tensor:
    """u (n_in, B) float16 = fp16(gain * (w16 x^T + b16)) by the library's tensor-core kernel
    (``afb_input_map_f16``; chessfly/model.py:101-102 with the float16 cast).  w16 (n_in, k) and x (B, k)
    float16 with unit column stride; rows of x that do not start on 16 bytes are copied first.  The result
    is a view with a row stride rounded up to 8 positions (the light-cone forward reads it as it is)."""
    n_in, k = w16.shape
    if not (w16.device == b16.device == x.device) or (status is not None and status.device != x.device):
        raise RuntimeError("input_map_f16: w16, b16, x and status must be on one device")
    if w16.dtype != torch.float16 or b16.dtype != torch.float16 or b16.shape != (n_in,):
        raise ValueError("input_map_f16: w16 (n_in, k) and b16 (n_in,) must be float16")
    if w16.stride(1) != 1 or w16.stride(0) % 8 or w16.data_ptr() % 16:
        raise ValueError("w16 rows must be contiguous and start on 16-byte boundaries")
    if x.shape[1] != k:
        raise ValueError(f"x has {x.shape[1]} features, the map takes {k}")
    if x.dtype != torch.float16 or x.stride(1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
        xp = torch.empty(x.shape[0], -(-k // 8) * 8, dtype=torch.float16, device=x.device)[:, :k]
        xp.copy_(x)
        x = xp
    batch = x.shape[0]
    ldu = -(-batch // 8) * 8
    u = torch.empty(n_in, ldu, dtype=torch.float16, device=x.device)[:, :batch]
    lib = _lib.load()
    with torch.cuda.device(x.device):                 # the launch goes to the device of the operands
        _lib.check(lib.afb_input_map_f16(n_in, batch, k, w16.data_ptr(), w16.stride(0), x.data_ptr(), x.stride(0),
                                         b16.data_ptr(), float(gain), u.data_ptr(), ldu,
                                         status.data_ptr() if status is not None else None,
                                         torch.cuda.current_stream(x.device).cuda_stream))
    return u


class _Handle:
    """One submitted evaluation: its device results, the pinned buffers they are copied into, and the event
    that marks the copies done.  ``get`` waits once and keeps the host arrays."""

    def __init__(self, event, n_out, n_val, out_host, val_host, lazy):
        self.event, self.n_out, self.n_val, self.out_host, self.val_host, self.lazy = event, n_out, n_val, out_host, val_host, lazy
        self.value = None

    def get(self):
        if self.value is None:
            self.event.synchronize()
            out = self.out_host[:self.n_out].numpy().copy()
            self.value = (out.reshape(self.n_val, N_MOVES) if self.lazy else out, self.val_host[:self.n_val].numpy().copy())
            self.out_host = self.val_host = None
        return self.value


class Evaluator:
    """The ``evaluate`` callable of the search: numpy in, numpy out (chessfly/model.py:113-135): ``submit``
    launches an evaluation and returns at once, ``result`` waits for it; legal-move logits (float32) when
    ``rows``/``cols`` are given, else the whole policy (float16, the lazy search), and the values.

    The B200 pipeline behind the same contract:
      - features, legal indices and results go through pinned host buffers, two sets used in turn, so
        the copies are asynchronous and a round can be submitted while the previous one runs (the
        self-play loop keeps one round in flight, chessfly/workers.py:118-167);
      - with ``graphs`` the network up to its readout, values and from/to terms runs as one CUDA graph,
        captured once per batch bucket (multiples of 256 positions, the step kernel's batch tile; at most
        ``max_graphs`` kept); the weight-dependent constants are refreshed before a replay when a
        parameter changed, so training between rounds is seen;
      - the readout is libafb's tensor-core kernel (``FlyChessNet.heads``, part of the graph): the dense
        (B, 4168) logits at float32 accuracy, from which the legal entries are gathered, or which are
        rounded to float16 for the lazy search.
    """

    BUCKET = 256

    def __init__(self, net: FlyChessNet, device, graphs: bool = True, max_graphs: int = 4):
        self.net, self.device = net, torch.device(device)
        self.graphs = graphs and self.device.type == "cuda"
        self.max_graphs = max_graphs
        self._graphs: "OrderedDict[int, tuple]" = OrderedDict()
        self._slots = [dict(), dict()]
        self._pending: list = [None, None]
        self._turn = 0

    # -- pinned staging --------------------------------------------------------------------------------
    def _pinned(self, slot: int, name: str, n: int, dtype) -> torch.Tensor:
        buf = self._slots[slot].get(name)
        if buf is None or buf.numel() < n:
            buf = torch.empty(max(n, 1024), dtype=dtype)
            if self.device.type == "cuda":
                buf = buf.pin_memory()
            self._slots[slot][name] = buf
        return buf

    def _stage(self, slot: int, name: str, a: np.ndarray, dtype) -> torch.Tensor:
        """``a`` copied into this slot's pinned buffer and sent to the device (asynchronously)."""
        flat = np.ascontiguousarray(a).reshape(-1)
        buf = self._pinned(slot, name, flat.size, dtype)
        buf[:flat.size].numpy()[:] = flat
        return buf[:flat.size].to(self.device, non_blocking=True)

    # -- the network -------------------------------------------------------------------------------------
    def _trunk(self, x: torch.Tensor):
        """Features -> (policy logits (B, N_MOVES) float32, values (B,)): the recurrence and the tensor-core
        readout."""
        net = self.net
        logits, wdl = net.heads(net.brain_output(x))
        return logits, net.expected_value(wdl)

    def _refresh_constants(self) -> None:
        net, brain = self.net, self.net.brain
        mode = _lib.MODE_DEV16 if net.infer_dtype == torch.float16 else _lib.MODE_F32
        if mode == _lib.MODE_DEV16:
            net.half_encoder()
        net.folded_heads()
        cone = brain.light_cone(net.in_idx, net.out_idx, net.cfg.steps)
        cone.set_weights(brain, mode, brain._weight_key(mode, cone))

    def _graph(self, bucket: int):
        key = (bucket, self.net.infer_dtype)
        entry = self._graphs.get(key)
        if entry is not None:
            self._graphs.move_to_end(key)
            return entry
        while len(self._graphs) >= self.max_graphs:
            self._graphs.popitem(last=False)
        # rows padded to 16 bytes, so the input map's TMA reads them in place
        x = torch.zeros(bucket, -(-N_FEATURES // 8) * 8, dtype=torch.float16, device=self.device)[:, :N_FEATURES]
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):                  # warm-up: cone, constants, library handles
            for _ in range(2):
                self._trunk(x)
        torch.cuda.current_stream(self.device).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        # capture on a stream of this device (torch's default capture stream belongs to the device that
        # was current when it was first made)
        with torch.cuda.graph(g, stream=torch.cuda.Stream(self.device)):
            outs = self._trunk(x)
        entry = (g, x, outs)
        self._graphs[key] = entry
        return entry

    @torch.no_grad()
    def submit(self, x, rows, cols):
        """Launch the evaluation and return at once; ``result`` waits for it."""
        if self.device.type != "cuda":
            return self._submit(x, rows, cols)
        with torch.cuda.device(self.device):       # the library, the graphs and the events use the current device
            return self._submit(x, rows, cols)

    def _submit(self, x, rows, cols):
        net = self.net
        net.eval()
        slot = self._turn
        self._turn ^= 1
        if self._pending[slot] is not None:            # its pinned buffers are about to be reused
            self._pending[slot].get()
        b = len(x)
        if b == 0:
            handle = _Handle(_Done(), 0, 0, torch.empty(0, dtype=torch.float16 if rows is None else torch.float32),
                             torch.empty(0), rows is None)
            self._pending[slot] = handle
            return handle
        x_dev = self._stage(slot, "x", np.asarray(x, np.float16), torch.float16).view(b, -1)
        if self.graphs and x_dev.is_cuda and b > 0:
            self._refresh_constants()
            g, x_static, (logits, values) = self._graph((b + self.BUCKET - 1) // self.BUCKET * self.BUCKET)
            x_static[:b].copy_(x_dev)
            g.replay()
            logits, values = logits[:b], values[:b]
        else:
            logits, values = self._trunk(x_dev)
        if rows is None:
            out = logits.half().reshape(-1)
        else:
            if len(rows) != len(cols):
                raise ValueError("rows and cols must have the same length")
            if len(rows) and (np.min(rows) < 0 or np.max(rows) >= b or np.min(cols) < 0 or np.max(cols) >= N_MOVES):
                raise ValueError(f"legal-move indices out of range: rows in [0, {b}), cols in [0, {N_MOVES})")
            rows_dev = self._stage(slot, "rows", np.asarray(rows, np.int64), torch.int64)
            cols_dev = self._stage(slot, "cols", np.asarray(cols, np.int64), torch.int64)
            out = logits[rows_dev, cols_dev]
        out_host = self._pinned(slot, "out_half" if rows is None else "out", out.numel(), out.dtype)
        val_host = self._pinned(slot, "values", b, torch.float32)
        out_host[:out.numel()].copy_(out, non_blocking=True)
        val_host[:b].copy_(values.float(), non_blocking=True)
        ev = torch.cuda.Event() if out.is_cuda else None
        if ev is not None:
            ev.record(torch.cuda.current_stream(self.device))
        handle = _Handle(ev if ev is not None else _Done(), out.numel(), b, out_host, val_host, rows is None)
        self._pending[slot] = handle
        return handle

    def result(self, handle):
        return handle.get()

    def __call__(self, x, rows, cols):
        return self.result(self.submit(x, rows, cols))


class _Done:
    @staticmethod
    def synchronize():
        pass


class _ShardedHandle:
    def __init__(self, parts, n_legal, lazy):
        self.parts, self.n_legal, self.lazy = parts, n_legal, lazy    # [(handle, lo, hi, legal positions)]
        self.value = None

    def get(self):
        if self.value is None:
            vals = [h.get() for h, _, _, _ in self.parts]
            values = np.concatenate([v for _, v in vals]) if vals else np.zeros(0, np.float32)
            if self.lazy:
                out = np.concatenate([o for o, _ in vals]) if vals else np.zeros((0, N_MOVES), np.float16)
            else:
                out = np.empty(self.n_legal, np.float32)
                for (o, _), (_, _, _, sel) in zip(vals, self.parts):
                    out[sel] = o
            self.value = (out, values)
        return self.value


class ShardedEvaluator:
    """The Evaluator contract over several GPUs of one process (the MCTS leaf batch of chessfly/mcts.py:
    263-301 spread across devices): a round's positions are split into contiguous shares, one per device,
    each evaluated by an ``Evaluator`` on that device's replica of the network, concurrently (every
    share's work is queued before any result is waited for); legal-move logits come back in the order
    of the request's (rows, cols), values in position order.

    The replicas copy the primary network at construction; after a training phase changes it, ``sync``
    copies its parameters and buffers into them in place (so their captured graphs stay valid)."""

    def __init__(self, net: FlyChessNet, devices, graphs: bool = True, max_graphs: int = 4):
        import copy
        self.net = net
        self.devices = [torch.device(d) for d in devices]
        self.replicas = []
        for d in self.devices:
            r = copy.deepcopy(net).to(d)
            r.infer_dtype = net.infer_dtype
            self.replicas.append(r)
        self.evaluators = [Evaluator(r, d, graphs=graphs, max_graphs=max_graphs) for r, d in zip(self.replicas, self.devices)]

    @torch.no_grad()
    def sync(self) -> None:
        src = dict(self.net.state_dict(keep_vars=True))
        for r in self.replicas:
            for k, t in r.state_dict(keep_vars=True).items():
                s = src[k]
                if not torch.equal(t.detach(), s.detach().to(t.device)):
                    t.detach().copy_(s.detach())
            r.infer_dtype = self.net.infer_dtype

    def submit(self, x, rows, cols):
        b = len(x)
        g = len(self.evaluators)
        bounds = [b * k // g for k in range(g + 1)]
        rows_np = None if rows is None else np.asarray(rows, np.int64)
        cols_np = None if cols is None else np.asarray(cols, np.int64)
        parts = []
        for ev, lo, hi in zip(self.evaluators, bounds[:-1], bounds[1:]):
            if hi == lo:
                continue
            if rows_np is None:
                parts.append((ev.submit(x[lo:hi], None, None), lo, hi, None))
            else:
                sel = np.flatnonzero((rows_np >= lo) & (rows_np < hi))
                parts.append((ev.submit(x[lo:hi], rows_np[sel] - lo, cols_np[sel]), lo, hi, sel))
        return _ShardedHandle(parts, 0 if rows_np is None else len(rows_np), rows is None)

    def result(self, handle):
        return handle.get()

    def __call__(self, x, rows, cols):
        return self.result(self.submit(x, rows, cols))


NEW_HEADS = ("policy_from.", "policy_to.")


def load_weights(net: FlyChessNet, state: dict) -> None:
    """Checkpoints from before the factorised policy head lack its zero-initialised terms; an encoder saved
    before the attack planes is padded with zero columns; nothing else may be missing
    (chessfly/model.py:141-151)."""
    state = dict(state)
    w = state.get("encoder.weight")
    if w is not None and w.shape[1] < net.encoder.weight.shape[1]:
        pad = w.new_zeros(w.shape[0], net.encoder.weight.shape[1] - w.shape[1])
        state["encoder.weight"] = torch.cat([w, pad], dim=1)
    missing, unexpected = net.load_state_dict(state, strict=False)
    bad = [k for k in missing if not k.startswith(NEW_HEADS)] + list(unexpected)
    if bad:
        raise RuntimeError(f"checkpoint does not match the network: {bad}")


def load_net(path, conn: Connectome, device="cuda") -> FlyChessNet:
    """The network of a checkpoint, ready to evaluate (chessfly/model.py:154-161).  The reference loads the
    MaleCNS connectome itself; here the caller passes the ``Connectome`` (this package does not download)."""
    ck = torch.load(path, map_location=device, weights_only=False)
    cfg = ModelConfig(**ck["config"])
    net = FlyChessNet(conn, cfg).to(device)
    load_weights(net, ck["model"])
    return net.eval()
