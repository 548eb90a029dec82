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


def _plain(net, x, rows, cols):
    """The reference's Evaluator.submit + result (chessfly/model.py:120-132), eager, with its float32 head
    layers (``dense_heads``)."""
    net.eval()
    with torch.no_grad():
        logits, wdl = net.dense_heads(net.readout(torch.from_numpy(x).to(DEV).float()))
        v = net.expected_value(wdl.float()).cpu().numpy()
        if rows is None:
            return logits.half().cpu().numpy(), v
        return logits[torch.from_numpy(rows).to(DEV), torch.from_numpy(cols).to(DEV)].float().cpu().numpy(), v


@pytest.fixture(scope="module")
def small_net():
    inst = synth.small()
    net = FlyChessNet(inst.conn, ModelConfig(steps=6))
    synth.apply(net.brain, inst)
    w, b = synth.encoder_weights(len(inst.in_idx))
    with torch.no_grad():
        net.encoder.weight.copy_(torch.from_numpy(w))
        net.encoder.bias.copy_(torch.from_numpy(b))
        params = dict(net.named_parameters())
        for k, v in synth.head_weights(len(inst.out_idx)).items():
            params[k].copy_(torch.from_numpy(v))
        params["policy_from.weight"].normal_(0, 0.05, generator=torch.Generator().manual_seed(3))
        params["policy_to.weight"].normal_(0, 0.05, generator=torch.Generator().manual_seed(4))
    return net.to(DEV)


def _request(batch, seed):
    rng = np.random.default_rng(seed)
    x = synth.boards(batch, seed).astype(np.float16)
    rows = np.repeat(np.arange(batch), 30)
    cols = np.concatenate([rng.choice(4168, 30, replace=False) for _ in range(batch)])
    return x, rows, cols


@pytest.mark.parametrize("graphs", [False, True])
@pytest.mark.parametrize("batch", [7, 300])
def test_pipelined_evaluator_equals_the_reference_evaluation(small_net, graphs, batch):
    """Pinned staging, CUDA-graph replay (bucket of 256 or 512 positions) and the fused legal-logit kernel
    give the reference Evaluator's results: same values, legal logits to float32 rounding."""
    ev = Evaluator(small_net, DEV, graphs=graphs)
    x, rows, cols = _request(batch, batch)
    ref_legal, ref_values = _plain(small_net, x, rows, cols)
    legal, values = ev(x, rows, cols)
    assert legal.shape == ref_legal.shape and legal.dtype == np.float32
    np.testing.assert_allclose(legal, ref_legal, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(values, ref_values, rtol=1e-5, atol=1e-6)
    lazy, lazy_values = ev(x, None, None)
    ref_lazy, _ = _plain(small_net, x, None, None)
    assert lazy.shape == (batch, 4168) and lazy.dtype == np.float16
    np.testing.assert_allclose(lazy.astype(np.float32), ref_lazy.astype(np.float32), rtol=2e-3, atol=2e-3)


def test_two_rounds_in_flight_and_weight_updates_between_rounds(small_net):
    """The self-play loop's pipelining (submit round k+1 before fetching round k), and a parameter update
    between rounds (as a training phase does) reaching the captured graph."""
    ev = Evaluator(small_net, DEV, graphs=True)
    a, b = _request(200, 1), _request(200, 2)
    ha = ev.submit(*a)
    hb = ev.submit(*b)
    ra, rb = ev.result(ha), ev.result(hb)
    np.testing.assert_allclose(ra[0], _plain(small_net, *a)[0], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(rb[0], _plain(small_net, *b)[0], rtol=1e-4, atol=1e-4)
    hc = ev.submit(*a)                                   # reuses round a's pinned buffers
    ev.submit(*b)
    ev.submit(*b)                                        # a third submit before any result: hc is kept
    np.testing.assert_array_equal(ev.result(hc)[0], ra[0])
    with torch.no_grad():
        small_net.brain.bias.add_(0.3)                   # in place: bumps the version the graph checks
        small_net.policy.bias.add_(1.0)
    try:
        moved = ev(*a)
        ref = _plain(small_net, *a)
        np.testing.assert_allclose(moved[0], ref[0], rtol=1e-4, atol=1e-4)
        np.testing.assert_allclose(moved[1], ref[1], rtol=1e-5, atol=1e-6)
        assert not np.allclose(moved[1], ra[1])
    finally:
        with torch.no_grad():
            small_net.brain.bias.sub_(0.3)
            small_net.policy.bias.sub_(1.0)


@pytest.mark.parametrize("batch", [1, 37, 300, 1120])
def test_readout_heads_kernel_against_float64(batch):
    """afb_readout_heads (RunningNorm + folded heads on the tensor cores, split float16 operands) at the real
    head sizes (2,333 output neurons, 4,168 policy rows + 3 value rows) against the normaliser and the
    dense product in float64; some entries are beyond the clip.  float32 accuracy is the bar (1e-5; the
    split is ~1e-6), and the float16 output is that result rounded once."""
    from alphafly_b200 import _lib
    g = torch.Generator(device=DEV).manual_seed(batch)
    o, n_pol, n_val = 2333, 4168, 3
    rows = n_pol + n_val
    out = 4.0 + torch.randn(o, batch, device=DEV, generator=g) * 0.3        # the forward's (n_out, batch) layout
    mean = 4.0 + torch.randn(o, device=DEV, generator=g) * 0.05
    var = (torch.rand(o, device=DEV, generator=g) * 0.1 + 0.005) ** 2           # small: many clip at +-8
    w = torch.randn(rows, o, device=DEV, generator=g) / o ** 0.5
    bias = torch.randn(rows, device=DEV, generator=g)
    ldw = -(-o // 8) * 8
    hi = torch.empty(rows, ldw, dtype=torch.float16, device=DEV)
    lo = torch.empty_like(hi)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.afb_heads_split(rows, o, w.data_ptr(), o, hi.data_ptr(), lo.data_ptr(), ldw, stream))
    ws = torch.empty(lib.afb_readout_workspace(batch, o), dtype=torch.uint8, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    res = {}
    for f16 in (0, 1):
        logits = torch.full((batch, n_pol), float("nan"), dtype=torch.float16 if f16 else torch.float32, device=DEV)
        values = torch.full((batch, n_val), float("nan"), device=DEV)
        _lib.check(lib.afb_readout_heads(o, batch, out.data_ptr(), out.stride(0), mean.data_ptr(), var.data_ptr(), 1e-8, 8.0,
                                         rows, n_pol, hi.data_ptr(), lo.data_ptr(), ldw, bias.data_ptr(), logits.data_ptr(),
                                         n_pol, f16, values.data_ptr(), n_val, ws.data_ptr(), ws.numel(), status.data_ptr(),
                                         stream))
        res[f16] = (logits, values)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    r = ((out.double().T - mean.double()) / (var.double() + 1e-8).sqrt()).clamp(-8, 8)
    assert float((r.abs() == 8).double().mean()) > 0.01                        # the clip is exercised
    dense = r @ w.double().T + bias.double()
    logits, values = res[0]
    assert torch.isfinite(logits).all() and torch.isfinite(values).all()
    err = float((logits.double() - dense[:, :n_pol]).norm() / dense[:, :n_pol].norm())
    verr = float((values.double() - dense[:, n_pol:]).norm() / dense[:, n_pol:].norm())
    assert err < 1e-5 and verr < 1e-5, (err, verr)
    torch.testing.assert_close(res[1][0], logits.half(), rtol=0, atol=0)          # one rounding of the same sums
    torch.testing.assert_close(res[1][1], values, rtol=0, atol=0)


def test_folded_heads_equal_the_factorised_heads(small_net):
    """FlyChessNet.forward in inference (the tensor-core readout with the from/to terms folded into the
    policy rows) against the float32 layers of the reference's forward on the same normalised state."""
    net = small_net.eval()
    x = torch.from_numpy(synth.boards(300, seed=12)).to(DEV)
    with torch.no_grad():
        net.infer_dtype = torch.float32
        logits, wdl = net(x)
        ref, ref_wdl = net.dense_heads(net.readout(x))
        net.infer_dtype = torch.float16
    assert orc.rel_l2(logits.cpu().numpy(), ref.cpu().numpy()) < 1e-5
    assert orc.rel_l2(wdl.cpu().numpy(), ref_wdl.cpu().numpy()) < 1e-5


def _padded_half(a: torch.Tensor) -> torch.Tensor:
    rows, k = a.shape
    out = torch.zeros(rows, -(-k // 8) * 8, dtype=torch.float16, device=DEV)[:, :k]
    out.copy_(a)
    return out


@pytest.mark.parametrize("n_in,batch,k", [(17937, 1120, 838), (300, 1, 838), (129, 257, 967), (128, 256, 64),
                                          (5, 300, 8), (200, 37, 100), (1000, 4096, 838)])
def test_input_map_kernel_against_float32(n_in, batch, k):
    """The tcgen05 input map against a float32 product of the same float16 operands: within the one
    float16 rounding of the result.  Ragged tiles in every dimension, k below, at and above one k-block."""
    from alphafly_b200.model import input_map_f16
    g = torch.Generator().manual_seed(n_in * 7 + batch * 3 + k)
    w16 = _padded_half(torch.randn(n_in, k, generator=g) * 0.05)
    b16 = (torch.randn(n_in, generator=g) * 0.3).half().to(DEV)
    feats = (torch.rand(batch, k, generator=g) < 0.06).half()       # board bits, exact in float16
    x = feats.to(DEV)                                                # row stride k: copied to 16-byte rows
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    u = input_map_f16(w16, b16, x, 5.0, status)
    ref = 5.0 * (w16.float().cpu() @ feats.float().T + b16.float().cpu()[:, None])
    assert u.shape == (n_in, batch) and u.dtype == torch.float16 and u.stride(1) == 1
    torch.testing.assert_close(u.float().cpu(), ref, rtol=2 ** -10, atol=1e-5)
    # the same through the C entry point with an unaligned row stride (scalar stores)
    from alphafly_b200 import _lib
    xp = _padded_half(x)
    u2 = torch.full((n_in, batch + 1), float("nan"), dtype=torch.float16, device=DEV)
    _lib.check(_lib.load().afb_input_map_f16(n_in, batch, k, w16.data_ptr(), w16.stride(0), xp.data_ptr(), xp.stride(0),
                                             b16.data_ptr(), 5.0, u2.data_ptr(), batch + 1, status.data_ptr(),
                                             torch.cuda.current_stream().cuda_stream))
    assert torch.equal(u2[:, :batch], u)
    assert torch.isnan(u2[:, batch]).all()                           # nothing written past the batch
    assert int(status.item()) == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_input_map_runs_on_the_operands_device():
    """Called with cuda:1 operands while cuda:0 is current, the map runs on cuda:1 and equals cuda:0's."""
    from alphafly_b200.model import input_map_f16
    g = torch.Generator().manual_seed(9)
    w = torch.randn(700, 838, generator=g) * 0.05
    b = (torch.randn(700, generator=g) * 0.3).half()
    bits = (torch.rand(300, 838, generator=g) < 0.06).half()
    outs = []
    for dev in ("cuda:0", "cuda:1"):
        w16 = torch.zeros(700, 840, dtype=torch.float16, device=dev)[:, :838]
        w16.copy_(w)
        st = torch.zeros(1, dtype=torch.int32, device=dev)
        with torch.cuda.device(0):
            outs.append(input_map_f16(w16, b.to(dev), bits.to(dev), 5.0, st).cpu())
        assert int(st.item()) == 0
    assert torch.equal(outs[0], outs[1])


def test_web_model_round_trip_evaluates_like_the_exported_network(small_net, tmp_path):
    """export_web_model -> net_from_web_model on configuration 1's network: the manifest's test vectors
    (float32 logits of legal moves and values, made on the original network) are reproduced by the rebuilt
    network within the float16 rounding of the exported synapse, encoder and policy weights."""
    from alphafly_b200 import webmodel
    net = small_net
    x, rows, cols = _request(10, 12)
    legal = [cols[rows == k] for k in range(10)]
    with torch.no_grad():
        net.norm.mean.normal_(0, 0.1, generator=torch.Generator(device=DEV).manual_seed(1))
    try:
        tests = webmodel.make_test_vectors(net, x.astype(np.float32), legal)
        webmodel.export_web_model(net, tmp_path, tests=tests)
        back = webmodel.net_from_web_model(tmp_path, device=DEV)
        again = webmodel.make_test_vectors(back, x.astype(np.float32), legal)
        for a, b in zip(tests, again):
            assert a["idx"] == b["idx"] and a["features"] == b["features"]
            np.testing.assert_allclose(b["logits"], a["logits"], rtol=0, atol=2e-2)
            assert abs(a["value"] - b["value"]) < 2e-2
        ref = np.concatenate([t["logits"] for t in tests])
        got = np.concatenate([t["logits"] for t in again])
        assert orc.rel_l2(got, ref) < 5e-3
    finally:
        with torch.no_grad():
            net.norm.mean.zero_()


@pytest.mark.parametrize("lazy", [False, True])
def test_sharded_evaluator_equals_one_evaluator(small_net, lazy):
    """ShardedEvaluator (two replicas; on a one-GPU box both live on cuda:0, which exercises the split and
    the reassembly) returns what one Evaluator returns, for a request whose (rows, cols) are not grouped
    by position; after a parameter change, sync() brings the replicas along."""
    from alphafly_b200.model import ShardedEvaluator
    devices = [f"cuda:{k % torch.cuda.device_count()}" for k in range(2)]
    x, rows, cols = _request(301, 21)
    perm = np.random.default_rng(0).permutation(len(rows))
    rows, cols = rows[perm], cols[perm]
    one = Evaluator(small_net, DEV)
    many = ShardedEvaluator(small_net, devices)
    assert [str(r.brain.pre.device) for r in many.replicas] == devices      # two GPUs: one replica on each
    req = (x, None, None) if lazy else (x, rows, cols)
    a, b = one(*req), many(*req)
    assert a[0].shape == b[0].shape and a[0].dtype == b[0].dtype
    np.testing.assert_allclose(b[0].astype(np.float32), a[0].astype(np.float32), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(b[1], a[1], rtol=1e-6, atol=1e-7)
    with torch.no_grad():
        small_net.brain.bias.add_(0.2)
    try:
        many.sync()
        c, d = one(*req), many(*req)
        np.testing.assert_allclose(d[1], c[1], rtol=1e-6, atol=1e-7)
        assert not np.allclose(c[1], a[1])
    finally:
        with torch.no_grad():
            small_net.brain.bias.sub_(0.2)


def _tiny_net(**cfg):
    return FlyChessNet(synth.tiny(60, 600), ModelConfig(steps=3, **cfg)).to(DEV)


def test_device_status_is_clear_after_inference_and_training():
    """FlyChessNet.device_status gathers the status words of every library kernel the network ran (step
    kernels, input map, readout, training products): 0 after a float16 inference forward through the
    tensor-core readout and a training step, and a planted code (written on the host into the word) is
    reported once, then cleared."""
    from alphafly_b200.encoding import N_FEATURES
    from alphafly_b200.train import Batch
    net = _tiny_net()
    g = torch.Generator().manual_seed(4)
    x = (torch.rand(40, N_FEATURES, generator=g) < 0.05).float().to(DEV)
    net.train()
    batch = Batch(x, torch.randint(0, 4168, (40, 5), generator=g).to(DEV), torch.full((40, 5), 0.2).to(DEV),
                  torch.ones(40, 5, dtype=torch.bool).to(DEV), torch.randint(0, 3, (40,), generator=g).to(DEV),
                  torch.zeros(40).to(DEV))
    train_step(net, make_optimizer(net, TrainConfig()), batch, DEV)
    net.eval()
    with torch.no_grad():
        net(x)
    assert net.device_status() == 0
    net._map_status(DEV).fill_(4)
    assert net.device_status() == 4 and net.device_status() == 0


def test_factorised_policy_head_is_a_no_op_until_trained():
    """tests/test_core.py:394-416: with the zero-initialised from/to terms the network is its dense policy
    head on the normalised readout; an old checkpoint without those terms loads."""
    from alphafly_b200.encoding import N_FEATURES
    from alphafly_b200.model import load_weights
    from alphafly_b200.encoding import N_BASE
    net = _tiny_net()
    with torch.no_grad():                                   # a trained dense head (the reference's is zero here)
        net.policy.weight.normal_(0, 0.1, generator=torch.Generator(device=DEV).manual_seed(3))
    old = {k: v for k, v in net.state_dict().items() if not k.startswith(("policy_from.", "policy_to."))}
    load_weights(net, old)
    x = torch.rand(3, N_FEATURES, generator=torch.Generator().manual_seed(0)).to(DEV)
    net.infer_dtype = torch.float32
    with torch.no_grad():
        w, b = net.encoder.weight[:, :N_BASE], net.encoder.bias
        u = ((x[:, :N_BASE] @ w.T + b) * net.cfg.input_gain).T.contiguous()
        dense = net.policy(net.norm(net.brain.forward_io(u, net.in_idx, net.out_idx, 3).T))
        assert float(dense.abs().max()) > 0
        torch.testing.assert_close(net.eval()(x)[0], dense, rtol=1e-5, atol=1e-5)


def test_attack_planes_are_invisible_unless_switched_on():
    """tests/test_core.py:474-488 on the GPU: without attack_planes the features from N_BASE on change
    nothing and their encoder columns get no gradient; with it they count."""
    from alphafly_b200.encoding import N_BASE, N_FEATURES
    g = torch.Generator().manual_seed(1)
    off, on = _tiny_net().eval(), _tiny_net(attack_planes=True).eval()
    with torch.no_grad():
        off.encoder.weight[:, N_BASE:].copy_(torch.randn(off.encoder.weight[:, N_BASE:].shape, generator=g))
        off.policy.weight.copy_(torch.randn(off.policy.weight.shape, generator=g) * 0.05)
    on.load_state_dict(off.state_dict())
    x = torch.rand(4, N_FEATURES, generator=g)
    y = x.clone()
    y[:, N_BASE:] = torch.rand(4, N_FEATURES - N_BASE, generator=g)
    x, y = x.to(DEV), y.to(DEV)
    with torch.no_grad():
        torch.testing.assert_close(off(x)[0], off(y)[0], rtol=0, atol=0)
        assert not torch.allclose(on(x)[0], on(y)[0])
    off.train()
    off(x)[0].sum().backward()
    assert float(off.encoder.weight.grad[:, N_BASE:].abs().sum()) == 0


def test_old_checkpoints_grow_the_encoder_without_changing_the_network():
    """tests/test_core.py:451-471 (the network part): an 838-column encoder loads into an attack-plane
    network as zero columns, so the new inputs change nothing until trained."""
    from alphafly_b200.encoding import N_BASE, N_FEATURES
    from alphafly_b200.model import load_weights
    net = _tiny_net()
    with torch.no_grad():
        net.policy.weight.normal_(0, 0.05)
    old = {k: (v[:, :N_BASE].clone() if k == "encoder.weight" else v.clone()) for k, v in net.state_dict().items()}
    fresh = _tiny_net(attack_planes=True)
    load_weights(fresh, old)
    assert fresh.encoder.weight.shape[1] == N_FEATURES and float(fresh.encoder.weight[:, N_BASE:].abs().sum()) == 0
    x = torch.rand(4, N_FEATURES, generator=torch.Generator().manual_seed(2)).to(DEV)
    x_old = x.clone()
    x_old[:, N_BASE:] = 0
    with torch.no_grad():
        torch.testing.assert_close(fresh.eval()(x)[0], fresh(x_old)[0])
