"""The training step of the network (chessfly/train.py:93-151), single GPU or data parallel.

``make_optimizer``, ``collate``, ``train_step`` and ``validation_loss`` keep the reference's parameter
groups, targets and losses: masked log-softmax policy cross-entropy, WDL cross-entropy mixed with the
mean-squared error of the expected value (``q_ratio``), gradient clipping at 5, AdamW.

Data parallel (one process per GPU, NCCL): every rank evaluates its own positions; the gradients are
averaged before clipping, in buckets that are all-reduced while the backward still runs
(``BucketedAllReduce``), and ``RunningNorm``'s batch statistics are combined exactly (sum and sum of
squares over all ranks), so the ranks stay identical and the step equals the single-GPU step on the
concatenated batch.
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


class BucketedAllReduce:
    """Gradient averaging over a process group, overlapped with the backward that produces the gradients.

    ``params`` are taken in the order their gradients become ready and packed into buckets of about
    ``bucket_mb`` MB (a larger parameter gets a bucket of its own).  Between ``arm()`` and ``finish()`` a
    post-accumulate-grad hook counts each bucket's gradients; a complete bucket is flattened and all-reduced
    asynchronously, so with NCCL its transfer runs on the communicator's stream while the rest of the
    backward computes.  Buckets are launched strictly in bucket order (a complete bucket waits for the ones
    before it), so every rank issues the same collectives in the same order.  ``finish()`` launches the
    buckets the backward did not complete (parameters without a gradient take zeros and keep ``grad`` None),
    waits, and writes the mean over ranks back into each ``grad``.  Outside an armed step the hooks do
    nothing."""

    def __init__(self, params, group=None, bucket_mb: float = 25.0):
        self.group = group
        self.buckets: list[list[torch.nn.Parameter]] = []
        cap, cur, size = bucket_mb * 2**20, [], 0
        for p in params:
            nbytes = p.numel() * p.element_size()
            if cur and size + nbytes > cap:
                self.buckets.append(cur)
                cur, size = [], 0
            cur.append(p)
            size += nbytes
        if cur:
            self.buckets.append(cur)
        self._where = {id(p): k for k, b in enumerate(self.buckets) for p in b}
        self._armed = False
        self._hooks = [p.register_post_accumulate_grad_hook(self._on_grad) for b in self.buckets for p in b]
        self.launched_in_backward = 0

    def arm(self) -> None:
        self._count = [0] * len(self.buckets)
        self._pending: list = []               # (bucket, flat, work handle) in launch order
        self._next = 0
        self.launched_in_backward = 0
        self._armed = True

    def _on_grad(self, p: torch.Tensor) -> None:
        if not self._armed:
            return
        k = self._where[id(p)]
        self._count[k] += 1
        launched = self._next
        while self._next < len(self.buckets) and self._count[self._next] == len(self.buckets[self._next]):
            self._launch(self._next)
        self.launched_in_backward += self._next - launched

    def _launch(self, k: int) -> None:
        import torch.distributed as dist
        flat = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1) for p in self.buckets[k]])
        self._pending.append((k, flat, dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True)))
        self._next = k + 1

    def finish(self) -> None:
        import torch.distributed as dist
        if not self._armed:
            raise RuntimeError("finish() without arm()")
        while self._next < len(self.buckets):
            self._launch(self._next)
        world = dist.get_world_size(self.group)
        for k, flat, work in self._pending:
            work.wait()
            flat /= world
            at = 0
            for p in self.buckets[k]:
                if p.grad is not None:
                    p.grad.copy_(flat[at:at + p.numel()].view_as(p))
                at += p.numel()
        self._pending = []
        self._armed = False

    def __deepcopy__(self, memo):
        return None           # hooks are not copied with the parameters: a copied network averages unbucketed

    def remove(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []


def gradient_order(net: FlyChessNet) -> list[torch.nn.Parameter]:
    """FlyChessNet's parameters in the order its backward produces their gradients: the heads, then the
    connectome (one autograd node returns all three), then the input map."""
    heads = [*net.policy_to.parameters(), *net.policy_from.parameters(), *net.value.parameters(),
             *net.policy.parameters()]
    order = heads + [net.brain.alpha_logit, net.brain.bias, net.brain.log_gain, *net.encoder.parameters()]
    rest = [p for p in net.parameters() if all(p is not q for q in order)]
    return order + rest


def attach_data_parallel(net: FlyChessNet, group=None, bucket_mb: float = 25.0) -> None:
    """Make ``net.norm`` combine its batch statistics over the ranks of ``group`` (exactly: the statistics of
    the concatenated batch), and give ``net`` a ``BucketedAllReduce`` over its gradients, which
    ``train_step(..., data_parallel=True)`` arms for each backward."""
    import torch.distributed as dist
    if isinstance(net, torch.nn.Module):
        if getattr(net, "grad_reducer", None) is not None:
            net.grad_reducer.remove()
        order = gradient_order(net) if isinstance(net, FlyChessNet) else list(net.parameters())[::-1]
        net.grad_reducer = BucketedAllReduce(order, group, bucket_mb)
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
    reducer = getattr(net, "grad_reducer", None) if data_parallel else None
    if reducer is not None and reducer.group is group:
        reducer.arm()
        try:
            (policy_loss + value_loss).backward()
        finally:
            reducer.finish()
    else:
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
