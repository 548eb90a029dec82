"""The training step of the network, single GPU or data parallel (the step of chessfly/train.py:126-138).

The reference's optimisation contract is kept: the AdamW parameter groups of its ``make_optimizer``
(learning rates and weight decays per group, chessfly/train.py:88-102), the pruned visit distribution as
policy target (chessfly/train.py:105-111), the policy loss (cross-entropy of the target against the
softmax over the legal moves only), the value loss ((1 - q_ratio) WDL cross-entropy + q_ratio squared error
of the expected value), gradient clipping at 5 and the returned loss dictionary.

The implementation is this package's own.  A batch lives on the device as padded per-position move lists
(``Batch``: the legal moves' policy indices and target probabilities, at most K per position) instead of
dense (B, 4168) target and mask tensors, and the policy loss is a log-sum-exp over each position's gathered
legal logits, O(B K) rather than O(B 4168).

Data parallel (one process per GPU, NCCL): every rank evaluates its own positions; the gradients are
averaged before clipping, in buckets that are all-reduced while the backward still runs
(``BucketedAllReduce``), and ``RunningNorm``'s batch statistics are combined exactly (sum and sum of
squares over all ranks), so the ranks stay identical and the step equals the single-GPU step on the
concatenated batch.
"""

from __future__ import annotations

import dataclasses
from typing import NamedTuple

import numpy as np
import torch

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


# The AdamW parameter groups, in the reference's order (chessfly/train.py:88-102): the name of the group, the
# network's parameters it holds, and the TrainConfig fields of its learning rate and weight decay (None: no
# decay).  "shared" (the factorised from/to policy terms) comes last so that an optimiser saved without it
# still loads before the group is added.
PARAM_GROUPS = (
    ("gains", lambda net: [net.brain.log_gain], "lr_brain", "gain_decay"),
    ("neurons", lambda net: [net.brain.bias, net.brain.alpha_logit], "lr_brain", None),
    ("io", lambda net: [*net.encoder.parameters(), *net.policy.parameters(), *net.value.parameters()], "lr_io", "io_decay"),
    ("shared", lambda net: [*net.policy_from.parameters(), *net.policy_to.parameters()], "lr_shared", "io_decay"),
)


def _group(net: FlyChessNet, cfg: TrainConfig, name: str) -> dict:
    for gname, select, lr, decay in PARAM_GROUPS:
        if gname == name:
            return {"params": select(net), "lr": getattr(cfg, lr), "weight_decay": getattr(cfg, decay) if decay else 0.0}
    raise KeyError(name)


def shared_group(net: FlyChessNet, cfg: TrainConfig) -> dict:
    """The optimiser group of the factorised policy terms, for adding to an optimiser rebuilt without it."""
    return _group(net, cfg, "shared")


def make_optimizer(net: FlyChessNet, cfg: TrainConfig, with_shared: bool = True) -> torch.optim.Optimizer:
    """AdamW over ``PARAM_GROUPS``; ``with_shared=False`` leaves out the last group (optimiser states saved
    before the factorised policy terms existed).  A network on the GPU takes torch's fused AdamW, the same
    update (0.43 ms per configuration-5 step against 1.02 ms for the multi-tensor one)."""
    names = [g[0] for g in PARAM_GROUPS if with_shared or g[0] != "shared"]
    fused = all(p.is_cuda for p in net.parameters())
    return torch.optim.AdamW([_group(net, cfg, n) for n in names], fused=True if fused else None)


class Batch(NamedTuple):
    """A training batch on the device.  ``moves`` (B, K) int64: policy indices of each position's legal
    moves, padded with 0; ``probs`` (B, K) float32: the target distribution over them, 0 in the padding;
    ``valid`` (B, K) bool: which entries are moves; ``wdl`` (B,) int64; ``q`` (B,) float32."""
    x: torch.Tensor
    moves: torch.Tensor
    probs: torch.Tensor
    valid: torch.Tensor
    wdl: torch.Tensor
    q: torch.Tensor


def pruned_targets(probs: np.ndarray, valid: np.ndarray, offset: float) -> np.ndarray:
    """Per row: the visit distribution less ``offset`` visits (one visit = the row's smallest non-zero
    probability), floored at zero and renormalised; a row that this leaves empty keeps its distribution
    (the target pruning of chessfly/train.py:105-111, over padded rows)."""
    probs = np.where(valid, probs, 0).astype(np.float32)
    if offset <= 0:
        return probs
    one_visit = np.where(probs > 0, probs, np.inf).min(axis=1, keepdims=True)
    kept = np.maximum(probs - np.float32(offset) * one_visit, 0).astype(np.float32)
    total = kept.sum(axis=1, keepdims=True)
    return np.where(total > 0, kept / np.where(total > 0, total, 1), probs).astype(np.float32)


def make_batch(samples: list[Sample], device, policy_target_offset: float = 0.0) -> Batch:
    """Samples -> a ``Batch`` on ``device`` (K = the most legal moves of any sample)."""
    b = len(samples)
    k = max([len(s.idx) for s in samples] + [1])
    moves = np.zeros((b, k), np.int64)
    probs = np.zeros((b, k), np.float32)
    valid = np.zeros((b, k), bool)
    for i, s in enumerate(samples):
        n = len(s.idx)
        moves[i, :n] = s.idx
        probs[i, :n] = s.pi
        valid[i, :n] = True
    probs = pruned_targets(probs, valid, policy_target_offset)
    x = np.stack([np.asarray(s.x, np.float32) for s in samples])
    wdl = np.fromiter((s.wdl for s in samples), np.int64, b)
    q = np.fromiter((s.q for s in samples), np.float32, b)
    return Batch(*(torch.from_numpy(a).to(device) for a in (x, moves, probs, valid, wdl, q)))


# An illegal move's logit in the reference's masked softmax (chessfly/train.py:129); here it stands only in
# the padding of a position's move list, so that a position with no legal move gives zero loss, not NaN.
_MASKED = -1e9


def policy_cross_entropy(logits: torch.Tensor, batch: Batch, reduction: str = "mean") -> torch.Tensor:
    """Cross-entropy of the target distribution against the softmax over each position's legal moves:
    -sum_k p_k (l_k - logsumexp_legal l), from the gathered legal logits only."""
    legal = logits.float().gather(1, batch.moves).masked_fill(~batch.valid, _MASKED)
    logp = legal - torch.logsumexp(legal, dim=1, keepdim=True)
    per_pos = -(batch.probs * logp).sum(1)
    return per_pos.mean() if reduction == "mean" else per_pos.sum()


def value_losses(wdl_logits: torch.Tensor, batch: Batch, q_ratio: float, reduction: str = "mean"):
    """(value loss, WDL cross-entropy): the loss mixes the cross-entropy of the game result with the squared
    error of the expected value p(win) - p(loss) against the search value q."""
    logq = wdl_logits.float().log_softmax(-1)
    ce = -logq.gather(1, batch.wdl.unsqueeze(1)).squeeze(1)
    p = logq.exp()
    sq = (p[:, 0] - p[:, 2] - batch.q) ** 2
    red = torch.mean if reduction == "mean" else torch.sum
    ce_r = red(ce)
    return (1 - q_ratio) * ce_r + q_ratio * red(sq), ce_r


def loss_terms(net: FlyChessNet, batch: Batch, q_ratio: float):
    """The forward pass of a training step: (policy loss, value loss, WDL cross-entropy)."""
    logits, wdl_logits = net(batch.x)
    value, ce = value_losses(wdl_logits, batch, q_ratio)
    return policy_cross_entropy(logits, batch), value, ce


def grow_optimizer_state(opt_state: dict, opt: torch.optim.Optimizer) -> dict:
    """Fit an optimiser state saved before a parameter gained input columns (the encoder, when the attack
    planes were added) to the current parameters: a 2-D moment with the parameter's rows and fewer columns
    gains zero columns on the right (the state growth of chessfly/train.py:211-218).  Returns the state."""
    shapes = [tuple(p.shape) for group in opt.param_groups for p in group["params"]]
    for i, entry in opt_state["state"].items():
        rows_cols = shapes[i]
        if len(rows_cols) != 2:
            continue
        for name, moment in entry.items():
            if torch.is_tensor(moment) and moment.dim() == 2 and moment.shape[0] == rows_cols[0] \
                    and moment.shape[1] < rows_cols[1]:
                entry[name] = torch.nn.functional.pad(moment, (0, rows_cols[1] - moment.shape[1]))
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
    buckets the backward did not complete (a parameter without a gradient contributes zeros), waits, and
    writes the mean over ranks into each ``grad``; a parameter that has a gradient on some rank gets one on
    every rank, one that has none anywhere keeps ``grad`` None.  Outside an armed step the hooks do
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
        params = self.buckets[k]
        # one presence flag per parameter after its gradient: a parameter whose gradient exists on any rank
        # gets the mean on every rank (zeros stand in for the ranks without one), so the ranks agree on which
        # parameters the optimiser steps
        parts = [(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1) for p in params]
        flags = torch.tensor([p.grad is not None for p in params], dtype=parts[0].dtype, device=parts[0].device)
        flat = torch.cat(parts + [flags])
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
            params = self.buckets[k]
            n = sum(p.numel() for p in params)
            # the presence flags are read (a host synchronisation) only for a bucket in which this rank
            # has a parameter without a gradient: the others take the mean whatever the flags say
            present = flat[n:].tolist() if any(p.grad is None for p in params) else [1.0] * len(params)
            flat = flat[:n] / world
            at = 0
            for p, seen in zip(params, present):
                mean = flat[at:at + p.numel()].view_as(p)
                if p.grad is not None:
                    p.grad.copy_(mean)
                elif seen > 0:
                    p.grad = mean.clone()
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
    """One optimisation step (chessfly/train.py:126-138): losses, backward, clip at 5, AdamW.  ``batch`` is a
    list of ``Sample`` or a ``Batch`` already on the device; ``data_parallel`` averages the gradients over the
    process group before clipping (the batch is this rank's share)."""
    if not isinstance(batch, Batch):
        batch = make_batch(batch, device, policy_target_offset)
    policy_loss, value_loss, value_ce = loss_terms(net, batch, q_ratio)
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
    losses = torch.stack([policy_loss.detach(), value_loss.detach(), value_ce.detach()]).tolist()   # one read-back
    return dict(zip(("policy_loss", "value_loss", "value_ce"), losses))


@torch.no_grad()
def validation_loss(net, val: list[Sample], device, policy_target_offset: float = 0.0, chunk: int = 256) -> dict:
    """Mean held-out policy loss and WDL cross-entropy over ``val``, rounded to 4 places, in ``chunk``-position
    evaluations (the keys and rounding of chessfly/train.py:141-154)."""
    net.eval()
    sums = torch.zeros(2, dtype=torch.float64, device=device)
    for lo in range(0, len(val), chunk):
        batch = make_batch(val[lo:lo + chunk], device, policy_target_offset)
        logits, wdl_logits = net(batch.x)
        sums[0] += policy_cross_entropy(logits, batch, reduction="sum").double()
        sums[1] += value_losses(wdl_logits, batch, 0.0, reduction="sum")[1].double()
    pol, val_ce = (sums / max(len(val), 1)).tolist()
    return {"val_policy_loss": round(pol, 4), "val_value_loss": round(val_ce, 4)}
