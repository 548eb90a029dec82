"""Gradient parity of the CUDA training path (forward with saved state + backward) with the reference.

The reference's gradients were recorded in float64 (tests/golden/); the library computes in float32,
so the bound is relative: 1e-4 relative L2 per gradient (measured ~1e-6).  At the full graph, where
no float64 reference run fits, the gradients are checked against the pinned CPU oracle at B = 2 and
through a size-independent property (the gradient of a batch is the sum of its halves' gradients).
"""

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import oracle as orc
from alphafly_b200 import synth
from alphafly_b200.brain import ConnectomeRNN

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
GRAD_GATE = 1e-4


def grads(rnn, *extra):
    return [(t.grad if t.grad is not None else torch.zeros_like(t)).detach().double().cpu().numpy()
            for t in (*extra, rnn.log_gain, rnn.bias, rnn.alpha_logit)]


def close(a, b, gate=GRAD_GATE, what=""):
    ref = np.asarray(b, np.float64)
    if np.linalg.norm(ref) == 0:
        assert np.abs(a).max() < 1e-6, what
        return
    err = orc.rel_l2(a, ref)
    assert err < gate, (what, err)


@pytest.mark.parametrize("steps", [1, 2, 4, 6])
def test_light_cone_gradients_match_reference_tiny(steps):
    """tests/test_core.py:309-338 in float32 on the GPU: outputs and the gradients of u_in, log_gain,
    bias and alpha_logit through the light cone."""
    g = golden("tiny")
    conn = synth.tiny(120, 700, seed=3)
    rnn = ConnectomeRNN(conn, global_scale=3.0, bias_init=0.1)
    with torch.no_grad():
        rnn.log_gain.copy_(torch.from_numpy(g["cone_log_gain"]))
        rnn.bias.copy_(torch.from_numpy(g["cone_bias"]))
        rnn.alpha_logit.copy_(torch.from_numpy(g["cone_alpha_logit"]))
    rnn = rnn.to(DEV)
    in_idx, out_idx = torch.as_tensor(g["cone_in_idx"], device=DEV), torch.as_tensor(g["cone_out_idx"], device=DEV)
    p = f"s{steps}_"
    u_in = torch.tensor(g[p + "u_in"], dtype=torch.float32, device=DEV, requires_grad=True)
    target = torch.tensor(g[p + "target"], dtype=torch.float32, device=DEV)
    out = rnn.forward_io(u_in, in_idx, out_idx, steps)
    ((out - target) ** 2).sum().backward()
    close(out.detach().cpu().numpy(), g[p + "out"], 1e-6, "out")
    names = ("u_in", "log_gain", "bias", "alpha_logit")
    for name, mine in zip(names, grads(rnn, u_in)):
        close(mine, g[p + "grad_" + name], what=name)
    assert rnn.device_status() == 0


def test_literal_recurrence_gradients_match_reference_dense():
    """tests/test_core.py:30-44: the literal recurrence with autograd against the reference (float64)."""
    g = golden("tiny")
    rnn = ConnectomeRNN(synth.tiny(), global_scale=3.0).to(DEV)
    u = torch.tensor(g["dense_u"], dtype=torch.float32, device=DEV, requires_grad=True)
    target = torch.tensor(g["dense_target"], dtype=torch.float32, device=DEV)
    out = rnn(u.T.contiguous(), 5).T
    ((out - target) ** 2).sum().backward()
    close(out.detach().cpu().numpy(), g["dense_out"], 1e-6, "out")
    mine = grads(rnn, u)
    close(mine[0], g["dense_grad_u"], what="u")
    close(mine[1], g["dense_grad_log_gain"], what="log_gain")
    close(mine[2], g["dense_grad_bias"], what="bias")


def test_small_config_gradients_match_reference():
    """Configuration 1, B = 8: the reference's float64 gradients (projections of dL/dlog_gain, its norm
    and a sample; dL/dbias, dL/dalpha_logit, dL/du_in in full)."""
    g = golden("small")
    inst = synth.small()
    rnn = ConnectomeRNN(inst.conn)
    synth.apply(rnn, inst)
    rnn = rnn.to(DEV)
    u8 = torch.tensor(synth.drive(inst, 8, seed=5), device=DEV, requires_grad=True)
    tgt = torch.tensor(g["grad_target"], dtype=torch.float32, device=DEV)
    out = rnn.forward_io(u8, inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
    (out * tgt).sum().backward()
    close(out.detach().cpu().numpy(), g["grad_out"], 1e-5, "out")
    gu, glg, gb, ga = grads(rnn, u8)
    close(gu, g["grad_u_in"], what="u_in")
    close(gb, g["grad_bias"], what="bias")
    close(ga, g["grad_alpha_logit"], what="alpha_logit")
    proj = np.random.default_rng(11).standard_normal((8, inst.e))
    close(proj @ glg, g["grad_log_gain_proj"], what="log_gain projections")
    assert abs(np.linalg.norm(glg) / float(g["grad_log_gain_norm"]) - 1) < GRAD_GATE
    close(glg[g["grad_log_gain_sample_idx"]], g["grad_log_gain_sample"], what="log_gain sample")


@pytest.fixture(scope="module")
def full():
    inst = synth.full()
    rnn = ConnectomeRNN(inst.conn)
    synth.apply(rnn, inst)
    return inst, rnn.to(DEV)


def test_full_graph_gradients_match_the_oracle(full):
    """Configuration 5's graph at B = 2 against the oracle's float64 backward of the literal recurrence
    (pinned to the reference by test_oracle)."""
    inst, rnn = full
    u = synth.drive(inst, 2, seed=4)
    tgt = np.random.default_rng(3).standard_normal((len(inst.out_idx), 2))
    u_dev = torch.tensor(u, device=DEV, requires_grad=True)
    rnn.zero_grad()
    out = rnn.forward_io(u_dev, inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
    (out * torch.tensor(tgt, dtype=torch.float32, device=DEV)).sum().backward()
    gu, glg, gb, ga = grads(rnn, u_dev)
    pre, post = inst.conn.pre.numpy(), inst.conn.post.numpy()
    w = orc.edge_weights(inst.conn.sign.numpy(), inst.w0.numpy(), inst.log_gain.numpy())
    full_u = np.zeros((inst.n, 2))
    full_u[inst.in_idx.numpy()] = u
    gh = np.zeros((inst.n, 2))
    gh[inst.out_idx.numpy()] = tgt
    ref = orc.backward_full(orc.full_csr(inst.n, pre, post), pre, post, w, inst.bias.numpy().astype(np.float64),
                            inst.alpha_logit.numpy().astype(np.float64), full_u, 6, gh)
    close(gu, ref["u"][inst.in_idx.numpy()], what="u_in")
    close(glg, ref["log_gain"], what="log_gain")
    close(gb, ref["bias"], what="bias")
    close(ga, ref["alpha_logit"], what="alpha_logit")
    assert rnn.device_status() == 0


def test_full_graph_gradient_is_additive_over_the_batch(full):
    """Size-independent property at training batch size: the gradient of 512 positions equals the sum
    of the gradients of its two halves."""
    inst, rnn = full
    u = torch.tensor(synth.drive(inst, 512, seed=8), device=DEV)
    tgt = torch.randn(len(inst.out_idx), 512, generator=torch.Generator().manual_seed(2)).to(DEV)
    in_idx, out_idx = inst.in_idx.to(DEV), inst.out_idx.to(DEV)

    def g_of(cols):
        rnn.zero_grad()
        out = rnn.forward_io(u[:, cols].contiguous(), in_idx, out_idx, 6)
        (out * tgt[:, cols]).sum().backward()
        return [x.copy() for x in grads(rnn)]

    whole = g_of(slice(0, 512))
    a, b = g_of(slice(0, 256)), g_of(slice(256, 512))
    for name, w_, x, y in zip(("log_gain", "bias", "alpha_logit"), whole, a, b):
        close(w_, x + y, 1e-4, name)


def test_training_steps_reduce_a_loss(full):
    """A few SGD steps on a fixed batch lower a least-squares loss on the outputs."""
    inst, rnn = full
    u = torch.tensor(synth.drive(inst, 64, seed=9), device=DEV)
    tgt = torch.rand(len(inst.out_idx), 64, generator=torch.Generator().manual_seed(4)).to(DEV)
    params = [rnn.log_gain, rnn.bias, rnn.alpha_logit]
    saved = [p.detach().clone() for p in params]
    opt = torch.optim.SGD(params, lr=1e-3)
    losses = []
    for _ in range(4):
        opt.zero_grad()
        out = rnn.forward_io(u, inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
        loss = ((out - tgt) ** 2).mean()
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    with torch.no_grad():
        for p, s in zip(params, saved):
            p.copy_(s)
    assert losses[-1] < losses[0], losses
