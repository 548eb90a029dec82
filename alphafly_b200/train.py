"""The training step of the network (chessfly/train.py:93-151), single GPU or data parallel.

``make_optimizer``, ``collate``, ``train_step`` and ``validation_loss`` keep the reference's parameter
groups, targets and losses: masked log-softmax policy cross-entropy, WDL cross-entropy mixed with the
mean-squared error of the expected value (``q_ratio``), gradient clipping at 5, AdamW.

Data parallel (one process per GPU, NCCL): every rank evaluates its own positions; the gradients are
averaged with one all-reduce of a flat buffer before clipping, and ``RunningNorm``'s batch statistics are
combined exactly (sum and sum of squares over all ranks), so the ranks stay identical and the step
equals the single-GPU step on the concatenated batch.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import torch
import torch.nn.functional as F

from .encoding import N_MOVES
from .model import FlyChessNet


@dataclasses.dataclass
class TrainConfig:
    """The optimisation fields of the reference's TrainConfig (chessfly/train.py:41-86)."""
    batch_size: int = 256
    lr_shared: float = 3e-5
    q_ratio: float = 0.5
    policy_target_offset: float = 0.0
    lr_brain: float = 3e-3
    lr_io: float = 3e-4
    io_decay: float = 1e-2
    gain_decay: float = 1e-4


@dataclasses.dataclass
class Sample:
    """A training position (chessfly/selfplay.py:68-73)."""
    x: np.ndarray        # (N_FEATURES,) float16
    idx: np.ndarray      # (k,) policy indices of the legal moves
    pi: np.ndarray       # (k,) visit distribution
    q: float = 0.0
    wdl: int = 1


def shared_group(net: FlyChessNet, cfg: TrainConfig) -> dict:
    return {"params": [*net.policy_from.parameters(), *net.policy_to.parameters()], "lr": cfg.lr_shared,
            "weight_decay": cfg.io_decay}


def make_optimizer(net: FlyChessNet, cfg: TrainConfig, with_shared: bool = True) -> torch.optim.Optimizer:
    brain = net.brain
    return torch.optim.AdamW([
        {"params": [brain.log_gain], "lr": cfg.lr_brain, "weight_decay": cfg.gain_decay},
        {"params": [brain.bias, brain.alpha_logit], "lr": cfg.lr_brain, "weight_decay": 0.0},
        {"params": [*net.encoder.parameters(), *net.policy.parameters(), *net.value.parameters()],
         "lr": cfg.lr_io, "weight_decay": cfg.io_decay},
    ] + ([shared_group(net, cfg)] if with_shared else []))


def prune(pi: np.ndarray, offset: float) -> np.ndarray:
    """pi minus ``offset`` visits, renormalised (chessfly/train.py:105-111)."""
    pi = pi.astype(np.float32)
    if offset <= 0:
        return pi
    t = np.maximum(pi - offset * pi[pi > 0].min(), 0)
    return t / t.sum() if t.sum() > 0 else pi


def collate(batch: list[Sample], device, policy_target_offset: float = 0.0):
    x = torch.from_numpy(np.stack([s.x for s in batch]).astype(np.float32)).to(device)
    pi = np.zeros((len(batch), N_MOVES), dtype=np.float32)
    legal = np.zeros((len(batch), N_MOVES), dtype=bool)
    for i, s in enumerate(batch):
        pi[i, s.idx] = prune(s.pi, policy_target_offset)
        legal[i, s.idx] = True
    wdl = torch.tensor([s.wdl for s in batch], device=device)
    q = torch.tensor([s.q for s in batch], dtype=torch.float32, device=device)
    return x, torch.from_numpy(pi).to(device), torch.from_numpy(legal).to(device), wdl, q


def losses(net: FlyChessNet, x, pi, legal, wdl, q, q_ratio: float):
    logits, wdl_logits = net(x)
    logp = logits.masked_fill(~legal, -1e9).log_softmax(-1)
    policy_loss = -(pi * logp).sum(-1).mean()
    value_ce = F.cross_entropy(wdl_logits, wdl)
    value_loss = (1 - q_ratio) * value_ce + q_ratio * F.mse_loss(net.expected_value(wdl_logits), q)
    return policy_loss, value_loss, value_ce


def grow_optimizer_state(opt_state: dict, opt: torch.optim.Optimizer) -> dict:
    """An optimizer state saved before a parameter gained input columns (the encoder, when the attack
    planes were added) made to fit the current parameters: each 2-D moment with the parameter's rows but
    fewer columns is padded with zero columns (chessfly/train.py:211-218).  Returns the state it updated."""
    params = [p for g in opt.param_groups for p in g["params"]]
    for i, st in opt_state["state"].items():
        p = params[i]
        for k, v in list(st.items()):
            if torch.is_tensor(v) and v.ndim == 2 and p.ndim == 2 and v.shape[0] == p.shape[0] and v.shape[1] < p.shape[1]:
                st[k] = torch.cat([v, v.new_zeros(v.shape[0], p.shape[1] - v.shape[1])], dim=1)
    return opt_state


def average_gradients(params, group=None) -> None:
    """All-reduce (mean over ranks) the gradients of ``params`` through one flat buffer."""
    import torch.distributed as dist
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    flat /= dist.get_world_size(group)
    k = 0
    for g in grads:
        g.copy_(flat[k:k + g.numel()].view_as(g))
        k += g.numel()


def attach_data_parallel(net: FlyChessNet, group=None) -> None:
    """Make ``net.norm`` combine its batch statistics over the ranks of ``group`` (exactly: the statistics of
    the concatenated batch)."""
    import torch.distributed as dist
    norm = net.norm

    def sync_from_batch(r: torch.Tensor):
        n = torch.tensor([float(r.shape[0])], device=r.device, dtype=torch.float64)
        s = r.double().sum(0)
        ss = (r.double() ** 2).sum(0)
        buf = torch.cat([n, s, ss])
        dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
        total = buf[0]
        o = r.shape[1]
        mean = buf[1:1 + o] / total
        var = (buf[1 + o:] - total * mean ** 2) / (total - 1)
        return mean.to(r.dtype), var.to(r.dtype)

    norm.batch_sync = sync_from_batch


def train_step(net, opt, batch, device, q_ratio: float = 0.0, policy_target_offset: float = 0.0,
               data_parallel: bool = False, group=None) -> dict:
    """One optimisation step (chessfly/train.py:126-138); ``data_parallel`` averages the gradients over the
    process group before clipping (the batch is this rank's share)."""
    x, pi, legal, wdl, q = collate(batch, device, policy_target_offset) if not isinstance(batch, tuple) else batch
    policy_loss, value_loss, value_ce = losses(net, x, pi, legal, wdl, q, q_ratio)
    opt.zero_grad(set_to_none=True)
    (policy_loss + value_loss).backward()
    if data_parallel:
        average_gradients(net.parameters(), group)
    torch.nn.utils.clip_grad_norm_(net.parameters(), 5.0)
    opt.step()
    return {"policy_loss": policy_loss.item(), "value_loss": value_loss.item(), "value_ce": value_ce.item()}


@torch.no_grad()
def validation_loss(net, val: list[Sample], device, policy_target_offset: float = 0.0) -> dict:
    net.eval()
    tot = {"val_policy_loss": 0.0, "val_value_loss": 0.0}
    for i in range(0, len(val), 256):
        x, pi, legal, wdl, _ = collate(val[i:i + 256], device, policy_target_offset)
        logits, wdl_logits = net(x)
        logp = logits.float().masked_fill(~legal, -1e9).log_softmax(-1)
        tot["val_policy_loss"] += -(pi * logp).sum().item()
        tot["val_value_loss"] += F.cross_entropy(wdl_logits.float(), wdl, reduction="sum").item()
    return {k: round(v / len(val), 4) for k, v in tot.items()}
