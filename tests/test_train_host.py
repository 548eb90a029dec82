"""The training step's host-side pieces on CPU: the optimiser groups, target pruning, batch packing and the
losses, each against a dense restatement of the reference's definition (chessfly/train.py:88-138): a
(B, 4168) target and legal mask, masked log-softmax with illegal logits at -1e9, F.cross_entropy and
F.mse_loss of the expected value."""

import numpy as np
import torch
import torch.nn.functional as F

from alphafly_b200 import synth
from alphafly_b200.encoding import N_MOVES
from alphafly_b200.model import FlyChessNet, ModelConfig
from alphafly_b200.train import (Batch, Sample, TrainConfig, make_batch, make_optimizer, policy_cross_entropy,
                                 pruned_targets, shared_group, value_losses)


def _dense_prune(pi, offset):
    pi = pi.astype(np.float32)
    if offset <= 0:
        return pi
    t = np.maximum(pi - offset * pi[pi > 0].min(), 0)
    return t / t.sum() if t.sum() > 0 else pi


def _samples(n, seed, max_moves=40):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        k = int(rng.integers(1, max_moves))
        idx = rng.choice(N_MOVES, size=k, replace=False)
        visits = rng.integers(0, 20, size=k).astype(np.float32)
        visits[rng.integers(0, k)] += 1                      # at least one visited move
        out.append(Sample(rng.integers(0, 2, 967).astype(np.float16), idx.astype(np.int16),
                          (visits / visits.sum()).astype(np.float16), float(rng.uniform(-1, 1)), int(rng.integers(0, 3))))
    return out


def _dense(samples, offset):
    pi = np.zeros((len(samples), N_MOVES), np.float32)
    legal = np.zeros((len(samples), N_MOVES), bool)
    for i, s in enumerate(samples):
        pi[i, s.idx.astype(np.int64)] = _dense_prune(s.pi, offset)
        legal[i, s.idx.astype(np.int64)] = True
    return torch.from_numpy(pi), torch.from_numpy(legal)


def test_optimizer_groups_follow_the_reference():
    net = FlyChessNet(synth.tiny(60, 600), ModelConfig(steps=3))
    cfg = TrainConfig()
    opt = make_optimizer(net, cfg)
    groups = opt.param_groups
    assert [g["lr"] for g in groups] == [cfg.lr_brain, cfg.lr_brain, cfg.lr_io, cfg.lr_shared]
    assert [g["weight_decay"] for g in groups] == [cfg.gain_decay, 0.0, cfg.io_decay, cfg.io_decay]
    assert groups[0]["params"][0] is net.brain.log_gain
    assert groups[1]["params"][0] is net.brain.bias and groups[1]["params"][1] is net.brain.alpha_logit
    io = {id(p) for m in (net.encoder, net.policy, net.value) for p in m.parameters()}
    assert {id(p) for p in groups[2]["params"]} == io
    assert {id(p) for p in groups[3]["params"]} == {id(p) for p in shared_group(net, cfg)["params"]}
    every = [id(p) for g in groups for p in g["params"]]
    assert sorted(every) == sorted(id(p) for p in net.parameters())
    assert len(make_optimizer(net, cfg, with_shared=False).param_groups) == 3


def test_pruned_targets_equal_the_per_row_rule():
    rng = np.random.default_rng(3)
    for offset in (0.0, 0.5, 1.0, 3.0):
        for _ in range(20):
            k = int(rng.integers(1, 12))
            pi = rng.integers(0, 6, size=k).astype(np.float32)
            pi = pi / pi.sum() if pi.sum() > 0 else pi
            padded = np.zeros((1, 16), np.float32)
            padded[0, :k] = pi
            valid = np.zeros((1, 16), bool)
            valid[0, :k] = True
            got = pruned_targets(padded, valid, offset)[0]
            if pi.sum() > 0:
                np.testing.assert_allclose(got[:k], _dense_prune(pi, offset), rtol=1e-6, atol=1e-7)
            assert (got[k:] == 0).all()


def test_losses_equal_the_dense_masked_definition():
    samples = _samples(24, seed=5)
    for offset, q_ratio in ((0.0, 0.5), (1.0, 0.0), (0.5, 1.0)):
        batch = make_batch(samples, "cpu", offset)
        g = torch.Generator().manual_seed(1)
        logits = (torch.randn(len(samples), N_MOVES, generator=g) * 3).requires_grad_(True)
        wdl_logits = torch.randn(len(samples), 3, generator=g).requires_grad_(True)
        pol = policy_cross_entropy(logits, batch)
        val, ce = value_losses(wdl_logits, batch, q_ratio)
        (pol + val).backward()
        g_logits, g_wdl = logits.grad.clone(), wdl_logits.grad.clone()

        pi, legal = _dense(samples, offset)
        logits.grad = wdl_logits.grad = None
        logp = logits.masked_fill(~legal, -1e9).log_softmax(-1)
        pol_ref = -(pi * logp).sum(-1).mean()
        ce_ref = F.cross_entropy(wdl_logits, batch.wdl)
        p = wdl_logits.softmax(-1)
        val_ref = (1 - q_ratio) * ce_ref + q_ratio * F.mse_loss(p[:, 0] - p[:, 2], batch.q)
        (pol_ref + val_ref).backward()
        torch.testing.assert_close(pol, pol_ref, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(val, val_ref, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(ce, ce_ref, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(g_logits, logits.grad, rtol=1e-4, atol=1e-7)
        torch.testing.assert_close(g_wdl, wdl_logits.grad, rtol=1e-4, atol=1e-7)


def test_a_position_without_legal_moves_adds_no_loss_and_no_nan():
    b = Batch(torch.zeros(2, 967), torch.tensor([[5, 9], [0, 0]]), torch.tensor([[0.25, 0.75], [0.0, 0.0]]),
              torch.tensor([[True, True], [False, False]]), torch.tensor([0, 1]), torch.zeros(2))
    logits = torch.randn(2, N_MOVES).requires_grad_(True)
    loss = policy_cross_entropy(logits, b, reduction="sum")
    loss.backward()
    assert torch.isfinite(loss) and torch.isfinite(logits.grad).all()
    assert float(logits.grad[1].abs().max()) == 0.0
    only_first = policy_cross_entropy(logits[:1], Batch(*(t[:1] for t in b)), reduction="sum")
    torch.testing.assert_close(loss, only_first)


def test_make_batch_packs_moves_and_targets():
    samples = _samples(5, seed=9, max_moves=7)
    b = make_batch(samples, "cpu")
    assert b.moves.shape == b.probs.shape == b.valid.shape and b.moves.dtype == torch.int64
    for i, s in enumerate(samples):
        k = len(s.idx)
        assert b.valid[i, :k].all() and not b.valid[i, k:].any()
        assert torch.equal(b.moves[i, :k], torch.from_numpy(s.idx.astype(np.int64)))
        np.testing.assert_allclose(b.probs[i, :k].numpy(), s.pi.astype(np.float32))
    assert b.x.shape == (5, 967) and b.x.dtype == torch.float32
