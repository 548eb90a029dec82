"""FlyChessNet, Evaluator and train_step on the GPU against the reference's own run (tests/golden/model.npz:
the 60-neuron test graph, chessfly/model.py + chessfly/train.py on CPU in float32)."""

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import oracle as orc
from alphafly_b200 import synth
from alphafly_b200.model import Evaluator, FlyChessNet, ModelConfig
from alphafly_b200.train import Sample, TrainConfig, make_optimizer, train_step

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def reference_net(g):
    net = FlyChessNet(synth.tiny(60, 600), ModelConfig(steps=3))
    net.load_state_dict({k[len("state_"):]: torch.from_numpy(g[k]) for k in g.files if k.startswith("state_")})
    return net.to(DEV)


def test_eval_logits_match_reference_float32_and_float16():
    g = golden("model")
    net = reference_net(g).eval()
    x = torch.from_numpy(g["x"]).to(DEV)
    net.infer_dtype = torch.float32
    with torch.no_grad():
        logits, wdl = net(x)
    assert orc.rel_l2(logits.cpu().numpy(), g["eval_logits"]) < 1e-5
    assert orc.rel_l2(wdl.cpu().numpy(), g["eval_wdl"]) < 1e-5
    net.infer_dtype = torch.float16                         # the deviation path, as self-play runs it
    with torch.no_grad():
        logits16, wdl16 = net(x)
    assert orc.rel_l2(logits16.cpu().numpy(), g["eval_logits"]) < 2e-3
    assert (logits16.argmax(1).cpu().numpy() == g["eval_logits"].argmax(1)).all()


def test_evaluator_gathers_legal_logits_and_values():
    g = golden("model")
    net = reference_net(g)
    ev = Evaluator(net, DEV)
    x = g["x"].astype(np.float16)
    rows = np.repeat(np.arange(6), 5)
    cols = np.random.default_rng(0).integers(0, 4168, 30)
    legal, values = ev(x, rows, cols)
    lazy_logits, lazy_values = ev(x, None, None)
    assert legal.dtype == np.float32 and legal.shape == (30,) and values.shape == (6,)
    assert lazy_logits.dtype == np.float16 and lazy_logits.shape == (6, 4168)
    np.testing.assert_allclose(legal, lazy_logits.astype(np.float32)[rows, cols], rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(values, lazy_values, rtol=1e-6)
    p = torch.from_numpy(g["eval_wdl"]).softmax(-1).numpy()
    np.testing.assert_allclose(values, p[:, 0] - p[:, 2], atol=5e-3)


def test_train_step_matches_reference():
    """One train_step (chessfly/train.py:126-138): losses, clipped gradients of every parameter, the
    RunningNorm statistics, and the AdamW update."""
    g = golden("model")
    net = reference_net(g).train()
    batch = [Sample(g["batch_x"][i], g["batch_idx"][i].astype(np.int64), g["batch_pi"][i], float(g["batch_q"][i]),
                    int(g["batch_wdl"][i])) for i in range(len(g["batch_x"]))]
    before = {k: p.detach().clone() for k, p in net.named_parameters()}
    opt = make_optimizer(net, TrainConfig())
    res = train_step(net, opt, batch, DEV, q_ratio=0.5)
    assert abs(res["policy_loss"] - float(g["train_policy_loss"])) < 1e-5 * abs(float(g["train_policy_loss"]))
    assert abs(res["value_loss"] - float(g["train_value_loss"])) < 1e-5 * abs(float(g["train_value_loss"]))
    for k, p in net.named_parameters():
        ref = g["grad_" + k]
        if np.abs(ref).max() == 0:
            assert float(p.grad.abs().max()) < 1e-7, k
        else:
            assert orc.rel_l2(p.grad.cpu().numpy(), ref) < 1e-4, k
        step_ref = g["after_" + k] - before[k].cpu().numpy()
        step = (p.detach() - before[k]).cpu().numpy()
        # Adam's first step is lr * sign(g) where |g| >> eps; entries with |g| near eps may differ
        assert np.mean(np.abs(step - step_ref) <= 1e-6 + 1e-3 * np.abs(step_ref)) > 0.999, k
    np.testing.assert_allclose(net.norm.mean.cpu().numpy(), g["norm_mean"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(net.norm.var.cpu().numpy(), g["norm_var"], rtol=1e-4, atol=1e-7)
