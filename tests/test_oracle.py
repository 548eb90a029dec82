"""Pins the CPU oracle (oracle/oracle.py) to outputs of the reference implementation itself.

The fixtures in tests/golden/ were produced by running the reference's chessfly/brain.py
(tests/golden/make_golden.py).  Index arrays must agree exactly; float64 results to 1e-9; the
reference's float32 results to the float32 tolerance of the north-star gate (1e-4 relative L2).
"""

import hashlib

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import oracle as orc
from alphafly_b200 import synth


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a).astype("<i8")).tobytes()).hexdigest()


def fsha(a):
    a = a.numpy() if isinstance(a, torch.Tensor) else np.asarray(a)
    return hashlib.sha256(np.ascontiguousarray(a.astype("<f4")).tobytes()).hexdigest()


def check_cone_arrays(cone, g, prefix):
    for t in range(cone.steps + 1):
        np.testing.assert_array_equal(cone.rows[t], g[f"{prefix}_rows{t}"])
    for t in range(1, cone.steps + 1):
        for name in ("keep_next", "keep_prev", "prev_row", "u_pos", "u_src"):
            np.testing.assert_array_equal(getattr(cone, name)[t], g[f"{prefix}_{name}{t}"], err_msg=f"{name}{t}")
        np.testing.assert_array_equal(cone.carried[t], g[f"{prefix}_carried{t}"])
        op = cone.ops[t]
        assert (op is None) == (f"{prefix}_op{t}_edges" not in g)
        if op is not None:
            for name in ("edges", "post", "pre", "crow", "t_order", "t_crow", "t_col"):
                np.testing.assert_array_equal(getattr(op, name), g[f"{prefix}_op{t}_{name}"], err_msg=f"op{t}.{name}")
    np.testing.assert_array_equal(cone.out_pos, g[f"{prefix}_out_pos"])
    np.testing.assert_array_equal(cone.out_src, g[f"{prefix}_out_src"])
    assert cone.edge_visits == int(g[f"{prefix}_edge_visits"])


def check_cone_hashes(cone, g, prefix="cone"):
    np.testing.assert_array_equal([len(r) for r in cone.rows], g[f"{prefix}_rows_len"])
    np.testing.assert_array_equal([0 if op is None else len(op.edges) for op in cone.ops], g[f"{prefix}_nnz"])
    assert cone.edge_visits == int(g[f"{prefix}_edge_visits"])
    for t in range(cone.steps + 1):
        assert sha(cone.rows[t]) == str(g[f"{prefix}_rows{t}_sha"]), f"rows{t}"
    for t in range(1, cone.steps + 1):
        for name in ("keep_next", "keep_prev", "prev_row", "u_pos", "u_src"):
            assert sha(getattr(cone, name)[t]) == str(g[f"{prefix}_{name}{t}_sha"]), f"{name}{t}"
        assert sha(cone.carried[t]) == str(g[f"{prefix}_carried{t}_sha"])
        op = cone.ops[t]
        if op is not None:
            for name in ("edges", "post", "pre", "crow", "t_crow", "t_col"):
                assert sha(getattr(op, name)) == str(g[f"{prefix}_op{t}_{name}_sha"]), f"op{t}.{name}"
            check_t_order(op.t_order, g, f"{prefix}_op{t}")
    assert sha(cone.out_pos) == str(g[f"{prefix}_out_pos_sha"])
    assert sha(cone.out_src) == str(g[f"{prefix}_out_src_sha"])


def check_t_order(t_order, g, prefix):
    """The transpose permutation is bit-exact where sort keys are distinct.  Where duplicate synapses
    tie, the reference's unstable argsort order is implementation-defined, and the stable order
    (the canonical form recorded from the reference's own permutation) must match instead."""
    if bool(g.get(f"{prefix}_t_order_ties", False)):
        assert sha(t_order) == str(g[f"{prefix}_t_order_canon_sha"]), f"{prefix}.t_order (canonical)"
    else:
        assert sha(t_order) == str(g[f"{prefix}_t_order_sha"]), f"{prefix}.t_order"


def check_graph(inst, g):
    assert inst.e == int(g["graph_e"])
    assert sha(inst.conn.pre) == str(g["graph_pre_sha"]) and sha(inst.conn.post) == str(g["graph_post_sha"])
    assert fsha(inst.conn.sign) == str(g["graph_sign_sha"]) and fsha(inst.w0) == str(g["graph_w0_sha"])
    assert fsha(inst.log_gain) == str(g["graph_log_gain_sha"]) and fsha(inst.bias) == str(g["graph_bias_sha"])
    assert fsha(inst.alpha_logit) == str(g["graph_alpha_logit_sha"])


def inst_arrays(inst):
    pre, post = inst.conn.pre.numpy(), inst.conn.post.numpy()
    w = orc.edge_weights(inst.conn.sign.numpy(), inst.w0.numpy(), inst.log_gain.numpy())
    alpha = orc.sigmoid(inst.alpha_logit.numpy().astype(np.float64))
    return pre, post, w, inst.bias.numpy().astype(np.float64), alpha


def test_dense_recurrence_and_gradients_match_reference():
    """tests/test_core.py:30-44: the literal recurrence and its gradients on the 30-neuron graph."""
    g = golden("tiny")
    n = 30
    pre, post = g["dense_pre"], g["dense_post"]
    W = orc.full_csr(n, pre, post)
    w = orc.edge_weights(g["dense_sign"], g["dense_w0"], np.zeros(len(pre)))
    alpha = orc.sigmoid(g["dense_alpha_logit"])
    u = g["dense_u"].T.copy()
    out = orc.forward(W, w, g["dense_bias"], alpha, u, 5)
    np.testing.assert_allclose(out.T, g["dense_out"], rtol=1e-12, atol=1e-14)
    grads = orc.backward_full(W, pre, post, w, g["dense_bias"], g["dense_alpha_logit"], u, 5,
                              2 * (out - g["dense_target"].T))
    np.testing.assert_allclose(grads["u"].T, g["dense_grad_u"], rtol=1e-10, atol=1e-13)
    np.testing.assert_allclose(grads["log_gain"], g["dense_grad_log_gain"], rtol=1e-10, atol=1e-13)
    np.testing.assert_allclose(grads["bias"], g["dense_grad_bias"], rtol=1e-10, atol=1e-13)


@pytest.mark.parametrize("steps", [1, 2, 4, 6])
def test_light_cone_forward_io_and_gradients_match_reference(steps):
    """tests/test_core.py:309-338: the light cone's fields, its outputs and every gradient."""
    g = golden("tiny")
    n = 120
    pre, post = g["cone_pre"], g["cone_post"]
    in_idx, out_idx = g["cone_in_idx"], g["cone_out_idx"]
    cone = orc.light_cone(n, pre, post, in_idx, out_idx, steps)
    check_cone_arrays(cone, g, f"cone{steps}")
    assert len(cone.rows[0]) == 0
    W = orc.full_csr(n, pre, post)
    w = orc.edge_weights(g["cone_sign"], g["cone_w0"], g["cone_log_gain"])
    alpha = orc.sigmoid(g["cone_alpha_logit"])
    p = f"s{steps}_"
    out = orc.forward_io(W, cone, w, g["cone_bias"], alpha, g[p + "u_in"])
    np.testing.assert_allclose(out, g[p + "out"], rtol=1e-9, atol=1e-11)
    # gradients through the literal recurrence equal the reference's light-cone gradients
    u = np.zeros((n, g[p + "u_in"].shape[1]))
    u[in_idx] = g[p + "u_in"]
    gh = np.zeros_like(u)
    gh[out_idx] = 2 * (out - g[p + "target"])
    grads = orc.backward_full(W, pre, post, w, g["cone_bias"], g["cone_alpha_logit"], u, steps, gh)
    np.testing.assert_allclose(grads["u"][in_idx], g[p + "grad_u_in"], rtol=1e-9, atol=1e-11)
    for name in ("log_gain", "bias", "alpha_logit"):
        np.testing.assert_allclose(grads[name], g[p + "grad_" + name], rtol=1e-9, atol=1e-11, err_msg=name)


def test_small_config_graph_cone_outputs_and_gradients_match_reference():
    """Configuration 1: the generator, the 6-step light cone, forward_io / forward and gradients."""
    g = golden("small")
    inst = synth.small()
    check_graph(inst, g)
    pre, post, w, bias, alpha = inst_arrays(inst)
    cone = orc.light_cone(inst.n, pre, post, inst.in_idx.numpy(), inst.out_idx.numpy(), 6)
    check_cone_hashes(cone, g)
    u = synth.drive(inst, 64, seed=0)
    assert fsha(u) == str(g["u_sha"])
    W = orc.full_csr(inst.n, pre, post)
    out = orc.forward_io(W, cone, w, bias, alpha, u.astype(np.float64))
    np.testing.assert_allclose(out, g["fwd_io_f64"], rtol=1e-9, atol=1e-11)
    assert orc.rel_l2(g["fwd_io_f32"], out) < 1e-5
    full = np.zeros((inst.n, 64))
    full[inst.in_idx.numpy()] = u
    ref_full = orc.forward(W, w, bias, alpha, full, 6)[inst.out_idx.numpy()]
    assert orc.rel_l2(g["fwd_full_f32"], ref_full) < 1e-5
    np.testing.assert_allclose(ref_full, out, rtol=1e-9, atol=1e-11)        # light cone == literal recurrence
    # gradients (float64) through the literal recurrence against the reference's light-cone gradients
    u8 = synth.drive(inst, 8, seed=5).astype(np.float64)
    full8 = np.zeros((inst.n, 8))
    full8[inst.in_idx.numpy()] = u8
    gh = np.zeros_like(full8)
    gh[inst.out_idx.numpy()] = g["grad_target"]
    grads = orc.backward_full(W, pre, post, w, bias, inst.alpha_logit.numpy().astype(np.float64), full8, 6, gh)
    np.testing.assert_allclose(grads["u"][inst.in_idx.numpy()], g["grad_u_in"], rtol=1e-8, atol=1e-12)
    np.testing.assert_allclose(grads["bias"], g["grad_bias"], rtol=1e-8, atol=1e-12)
    np.testing.assert_allclose(grads["alpha_logit"], g["grad_alpha_logit"], rtol=1e-8, atol=1e-12)
    lg = grads["log_gain"]
    proj = np.random.default_rng(11).standard_normal((8, inst.e))
    np.testing.assert_allclose(proj @ lg, g["grad_log_gain_proj"], rtol=1e-8, atol=1e-10)
    np.testing.assert_allclose(np.linalg.norm(lg), g["grad_log_gain_norm"], rtol=1e-10)
    np.testing.assert_allclose(lg[g["grad_log_gain_sample_idx"]], g["grad_log_gain_sample"], rtol=1e-8, atol=1e-12)


def test_shuffled_config_cone_and_outputs_match_reference():
    """Configuration 4 (duplicates allowed): generator, light cone and float32 forward_io."""
    g = golden("shuffled")
    inst = synth.shuffled()
    check_graph(inst, g)
    pre, post, w, bias, alpha = inst_arrays(inst)
    cone = orc.light_cone(inst.n, pre, post, inst.in_idx.numpy(), inst.out_idx.numpy(), 6)
    check_cone_hashes(cone, g)
    W = orc.full_csr(inst.n, pre, post)
    out = orc.forward_io(W, cone, w, bias, alpha, synth.drive(inst, 16, seed=3).astype(np.float64))
    assert orc.rel_l2(g["fwd_io_f32"], out) < 1e-5


@pytest.mark.slow
def test_full_config_cone_and_outputs_match_reference():
    """Configuration 2's graph: generator, 6-step light cone, forward_io and the unpruned forward."""
    g = golden("full")
    inst = synth.full()
    check_graph(inst, g)
    pre, post, w, bias, alpha = inst_arrays(inst)
    cone = orc.light_cone(inst.n, pre, post, inst.in_idx.numpy(), inst.out_idx.numpy(), 6)
    check_cone_hashes(cone, g)
    W = orc.full_csr(inst.n, pre, post)
    out = orc.forward_io(W, cone, w, bias, alpha, synth.drive(inst, 8, seed=0).astype(np.float64))
    assert orc.rel_l2(g["fwd_io_f32"], out) < 1e-5
    u4 = synth.drive(inst, 4, seed=1)
    full = np.zeros((inst.n, 4))
    full[inst.in_idx.numpy()] = u4
    ref_full = orc.forward(W, w, bias, alpha, full, 6)[inst.out_idx.numpy()]
    assert orc.rel_l2(g["fwd_full_f32"], ref_full) < 1e-5


def test_planted_mistake_in_the_oracle_is_caught():
    """The checks above are sharp: the oracle with one edge dropped from the light cone fails them."""
    g = golden("tiny")
    pre, post = g["cone_pre"], g["cone_post"]
    cone = orc.light_cone(120, pre, post, g["cone_in_idx"], g["cone_out_idx"], 4)
    cone.ops[3].edges = cone.ops[3].edges[1:]
    with pytest.raises(AssertionError):
        check_cone_arrays(cone, g, "cone4")


@pytest.mark.parametrize("config", ["small", "shuffled"])
def test_torch_cpu_restatement_matches_reference(config):
    """oracle/torch_port.py (the reference's torch CPU sparse forward_io, timed as the CPU baseline) against
    the reference's own float32 outputs."""
    from oracle.torch_port import TorchCpuForward
    g = golden(config)
    inst = synth.small() if config == "small" else synth.shuffled()
    fwd = TorchCpuForward(inst.n, inst.conn.pre.numpy(), inst.conn.post.numpy(), inst.conn.sign.numpy(), inst.w0.numpy(),
                          inst.log_gain.numpy(), inst.bias.numpy(), inst.alpha_logit.numpy(), inst.in_idx.numpy(),
                          inst.out_idx.numpy(), 6)
    batch, seed = (64, 0) if config == "small" else (16, 3)
    out = fwd(synth.drive(inst, batch, seed=seed)).numpy()
    assert out.dtype == np.float32 and out.shape == (len(inst.out_idx), batch)
    assert orc.rel_l2(out, g["fwd_io_f32"]) < 1e-5
