"""Parity at the benchmark's own configuration: configuration 3 (the full synthetic graph, B = 35,840 per
GPU, the bench's exact drive) and configuration 5 (training, B = 2,048).

- The float16 deviation path at B = 35,840 against the oracle in float64 on 72 columns taken from the start,
  the middle and the end of the batch (north-star gate: 2e-3 relative L2), and the float32 path at the same
  batch on the same columns (1e-4), plus float16 against float32 over the whole batch.
- The policy argmax gate through the real FlyChessNet (RunningNorm + heads) on 2,240 positions: float16
  inference (deviation path + the tensor-core readout) against the float32 network with the reference's
  float32 head layers (>= 99.5% agreement, logits within 2e-3 relative L2), and the tensor-core readout on
  the float32 recurrence within 1e-5 of those layers.  The float32 network is pinned to the reference's own
  run by test_gpu_model.
- Configuration 5's backward at B = 2,048: the loss weights 16 positions spread over all 16 batch tiles of
  the SDDMM partial sums, and every gradient is compared with the oracle's float64 backward of those 16
  positions (1e-4); the whole-batch gradient equals the sum of its four 512-position quarters.

The oracle restates chessfly/brain.py (forward_io, brain.py:282-329; the gradients of the recurrence,
brain.py:66-99 and tests/test_core.py:309-338) and is pinned to the reference by test_oracle.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from alphafly_b200 import synth
from alphafly_b200.brain import ConnectomeRNN

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
F32_GATE = 1e-4
F16_GATE = 2e-3
GRAD_GATE = 1e-4
BATCH3 = 35_840
BATCH5 = 2_048


@pytest.fixture(scope="module")
def full():
    inst = synth.full()
    rnn = ConnectomeRNN(inst.conn)
    synth.apply(rnn, inst)
    pre, post = inst.conn.pre.numpy(), inst.conn.post.numpy()
    cone = orc.light_cone(inst.n, pre, post, inst.in_idx.numpy(), inst.out_idx.numpy(), 6)
    w = orc.edge_weights(inst.conn.sign.numpy(), inst.w0.numpy(), inst.log_gain.numpy())
    return inst, rnn.to(DEV), (orc.full_csr(inst.n, pre, post), cone, w)


def _columns(batch, width=24):
    mid = batch // 2 - width // 2
    return np.r_[0:width, mid:mid + width, batch - width:batch]


def test_config3_full_batch_matches_the_oracle(full):
    inst, rnn, (W, cone, w) = full
    u16 = synth.config3_drive(inst, BATCH3)                      # the bench's drive, float16
    cols = _columns(BATCH3)
    assert len(set((cols % 2048).tolist())) == len(cols)         # 72 distinct positions
    in_idx, out_idx = inst.in_idx.to(DEV), inst.out_idx.to(DEV)
    u_dev = torch.from_numpy(u16).to(DEV)
    with torch.no_grad():
        out16 = rnn.forward_io(u_dev, in_idx, out_idx, 6)
        assert rnn.device_status() == 0
        out16_cols = out16[:, torch.from_numpy(cols).to(DEV)].cpu().numpy()
        out32 = rnn.forward_io(u_dev.float(), in_idx, out_idx, 6)   # float32 state at the full batch too
        whole = orc.rel_l2(out16.cpu().numpy(), out32.cpu().numpy())
        out32_cols = out32[:, torch.from_numpy(cols).to(DEV)].cpu().numpy()
        del out16, out32
    ref = orc.forward_io(W, cone, w, inst.bias.numpy().astype(np.float64),
                         orc.sigmoid(inst.alpha_logit.numpy().astype(np.float64)), u16[:, cols].astype(np.float64))
    e16, e32 = orc.rel_l2(out16_cols, ref), orc.rel_l2(out32_cols, ref)
    assert e16 < F16_GATE, e16
    assert e32 < F32_GATE, e32
    assert whole < F16_GATE, whole
    # the position-dependent part as well, not only the resting pattern it sits on
    dev_ref = ref - ref.mean(1, keepdims=True)
    assert orc.rel_l2(out16_cols - out16_cols.mean(1, keepdims=True), dev_ref) < 0.05
    assert orc.rel_l2(out32_cols - out32_cols.mean(1, keepdims=True), dev_ref) < 1e-3


def _net(inst):
    from alphafly_b200.model import FlyChessNet, ModelConfig
    net = FlyChessNet(inst.conn, ModelConfig(steps=6))
    synth.apply(net.brain, inst)
    w, b = synth.encoder_weights(len(inst.in_idx))
    g = torch.Generator().manual_seed(7)
    with torch.no_grad():
        net.encoder.weight.copy_(torch.from_numpy(w))
        net.encoder.bias.copy_(torch.from_numpy(b))
        params = dict(net.named_parameters())
        for k, v in synth.head_weights(len(inst.out_idx)).items():
            params[k].copy_(torch.from_numpy(v))
        for k in ("policy_from.weight", "policy_to.weight"):      # the factorised terms, trained-looking
            params[k].normal_(0, 0.5 / np.sqrt(len(inst.out_idx)), generator=g)
        params["policy.bias"].normal_(0, 0.1, generator=g)
    return net.to(DEV)


def test_flychessnet_float16_policy_agrees_with_float32_on_the_full_graph(full):
    """The gate of the float16 deviation path, through RunningNorm and the heads of the real network.
    The normaliser's running statistics are set as training sets them (one float32 batch in training
    mode), so the heads see the position-dependent part of the output neurons."""
    inst = full[0]
    net = _net(inst)
    net.train()
    net.infer_dtype = torch.float32
    with torch.no_grad():
        net(torch.from_numpy(synth.boards(1120, seed=31)).to(DEV))   # first batch: sets mean and variance
    net.eval()
    x = torch.from_numpy(synth.boards(2240, seed=32)).to(DEV)
    with torch.no_grad():
        l32, v32 = net.dense_heads(net.readout(x))            # float32 throughout, the reference's layers
        l32_tc, v32_tc = net(x)                                # float32 recurrence, tensor-core readout
        net.infer_dtype = torch.float16
        l16, v16 = net(x)                                      # the self-play path
    assert l16.dtype == torch.float32 and l16.shape == (2240, 4168)
    l32, l16, l32_tc = l32.cpu().numpy(), l16.cpu().numpy(), l32_tc.cpu().numpy()
    assert orc.rel_l2(l32_tc, l32) < 1e-5, orc.rel_l2(l32_tc, l32)
    assert orc.rel_l2(v32_tc.cpu().numpy(), v32.cpu().numpy()) < 1e-5
    assert orc.rel_l2(l16, l32) < F16_GATE, orc.rel_l2(l16, l32)
    agree = float((l16.argmax(1) == l32.argmax(1)).mean())
    assert agree >= 0.995, agree
    ev32 = net.expected_value(v32.float()).cpu().numpy()
    ev16 = net.expected_value(v16.float()).cpu().numpy()
    assert np.abs(ev16 - ev32).mean() < 2e-3


def _grads(rnn, u_dev):
    return (u_dev.grad.cpu().numpy(), rnn.log_gain.grad.cpu().numpy(), rnn.bias.grad.cpu().numpy(),
            rnn.alpha_logit.grad.cpu().numpy())


def test_config5_gradients_at_full_training_batch_match_the_oracle(full):
    """B = 2,048 (16 batch tiles of 128 columns): the loss weights one position per tile, so the backward
    runs every tile's SDDMM partial and the fixed-order tile sum, and the exact gradient is that of the 16
    weighted positions, which the oracle computes in float64."""
    inst, rnn, (W, _, w) = full
    u = synth.drive(inst, BATCH5, seed=41)
    picked = np.arange(16) * 128 + (np.arange(16) * 37) % 128            # one column in every tile
    tgt = np.zeros((len(inst.out_idx), BATCH5), np.float32)
    tgt[:, picked] = np.random.default_rng(6).standard_normal((len(inst.out_idx), 16))
    u_dev = torch.tensor(u, device=DEV, requires_grad=True)
    rnn.zero_grad()
    out = rnn.forward_io(u_dev, inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
    (out * torch.from_numpy(tgt).to(DEV)).sum().backward()
    gu, glg, gb, ga = _grads(rnn, u_dev)
    assert rnn.device_status() == 0
    pre, post = inst.conn.pre.numpy(), inst.conn.post.numpy()
    full_u = np.zeros((inst.n, 16))
    full_u[inst.in_idx.numpy()] = u[:, picked]
    gh = np.zeros((inst.n, 16))
    gh[inst.out_idx.numpy()] = tgt[:, picked]
    ref = orc.backward_full(W, pre, post, w, inst.bias.numpy().astype(np.float64),
                            inst.alpha_logit.numpy().astype(np.float64), full_u, 6, gh)
    for name, mine, theirs in (("u_in", gu[:, picked], ref["u"][inst.in_idx.numpy()]), ("log_gain", glg, ref["log_gain"]),
                               ("bias", gb, ref["bias"]), ("alpha_logit", ga, ref["alpha_logit"])):
        err = orc.rel_l2(mine, theirs)
        assert err < GRAD_GATE, (name, err)
    others = np.setdiff1d(np.arange(BATCH5), picked)
    assert float(np.abs(gu[:, others]).max()) == 0.0                    # unweighted positions: no gradient


def test_config5_gradient_is_the_sum_of_its_quarters(full):
    """Every position weighted at B = 2,048: the whole-batch gradient equals the sum of the gradients of its
    four 512-position quarters (linearity of the batch sum, at the training batch size)."""
    inst, rnn, _ = full
    u = torch.tensor(synth.drive(inst, BATCH5, seed=42), device=DEV)
    tgt = torch.randn(len(inst.out_idx), BATCH5, generator=torch.Generator().manual_seed(8)).to(DEV)
    in_idx, out_idx = inst.in_idx.to(DEV), inst.out_idx.to(DEV)

    def g_of(lo, hi):
        rnn.zero_grad()
        out = rnn.forward_io(u[:, lo:hi].contiguous(), in_idx, out_idx, 6)
        (out * tgt[:, lo:hi]).sum().backward()
        return [p.grad.double().cpu().numpy() for p in (rnn.log_gain, rnn.bias, rnn.alpha_logit)]

    whole = g_of(0, BATCH5)
    parts = [g_of(k * 512, (k + 1) * 512) for k in range(4)]
    for i, name in enumerate(("log_gain", "bias", "alpha_logit")):
        err = orc.rel_l2(whole[i], sum(p[i] for p in parts))
        assert err < 1e-5, (name, err)
