"""Policy/value network whose only hidden computation is the connectome (chessfly/model.py).

    board features --dense map--> sensory neurons --T steps of the wiring--> output neurons
    --RunningNorm--> dense readouts --> move logits, win/draw/loss logits

``FlyChessNet``, ``RunningNorm``, ``Evaluator``, ``ModelConfig``, ``load_weights`` and ``load_net`` keep the
reference's names, parameters, buffers and state_dict keys (chessfly/model.py:26-161), so checkpoints
load unchanged.  The recurrence runs in ``alphafly_b200.brain`` (libafb); the dense maps are plain
GEMMs in cuBLAS through torch.  The input map writes the (sensory neurons, batch) layout the
recurrence reads in one GEMM (W x^T scaled by the input gain), instead of x W^T followed by a
transpose copy.
"""

from __future__ import annotations

import dataclasses

import torch
from torch import nn

from .brain import ConnectomeRNN
from .connectome import Connectome
from .encoding import N_BASE, N_FEATURES, N_MOVES, move_squares

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
                m = 1.0 if not self.initialised else self.momentum
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
        for layer in (self.policy_from, self.policy_to):
            nn.init.zeros_(layer.weight)
            nn.init.zeros_(layer.bias)
        nn.init.zeros_(self.policy.weight)
        nn.init.zeros_(self.value.weight)

    def drive(self, x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        """u_in (sensory neurons, batch) = input_gain * (W x^T + b), over the first N_BASE features unless
        the attack planes are switched on (chessfly/model.py:98-102)."""
        k = N_FEATURES if self.cfg.attack_planes else N_BASE
        g = self.cfg.input_gain
        w, b = self.encoder.weight[:, :k], self.encoder.bias
        u = torch.addmm(b.unsqueeze(1), w, x[:, :k].T, beta=g, alpha=g)
        return u.to(dtype).contiguous()

    def forward(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """x: (B, N_FEATURES) -> policy logits (B, N_MOVES), WDL logits (B, 3)."""
        dtype = self.infer_dtype if x.is_cuda and not torch.is_grad_enabled() else torch.float32
        u_in = self.drive(x.float(), dtype)
        r = self.norm(self.brain.forward_io(u_in, self.in_idx, self.out_idx, self.cfg.steps).T.float())
        logits = self.policy(r) + self.policy_from(r)[:, self.move_from] + self.policy_to(r)[:, self.move_to]
        return logits, self.value(r)

    @staticmethod
    def expected_value(wdl_logits: torch.Tensor) -> torch.Tensor:
        p = wdl_logits.softmax(-1)
        return p[..., 0] - p[..., 2]


class Evaluator:
    """The ``evaluate`` callable of the search: numpy in, numpy out (chessfly/model.py:113-135).  Legal-move
    logits are gathered on the GPU, so only those leave the card."""

    def __init__(self, net: FlyChessNet, device):
        self.net, self.device = net, device

    @torch.no_grad()
    def submit(self, x, rows, cols):
        """Launch the evaluation and return at once; ``result`` waits for it."""
        self.net.eval()
        logits, wdl = self.net(torch.from_numpy(x).to(self.device, non_blocking=True).float())
        if rows is None:
            return logits.half(), self.net.expected_value(wdl.float())
        legal = logits[torch.from_numpy(rows).to(self.device, non_blocking=True),
                       torch.from_numpy(cols).to(self.device, non_blocking=True)]
        return legal.float(), self.net.expected_value(wdl.float())

    @staticmethod
    def result(handle):
        return handle[0].cpu().numpy(), handle[1].float().cpu().numpy()

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
