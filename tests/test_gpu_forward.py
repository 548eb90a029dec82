"""Parity of the CUDA forward path with the reference, through the package's module API.

Light-cone indices must be bit-exact (against the reference's own arrays or their SHA-256 in
tests/golden/).  float32 outputs must be within 1e-4 relative L2 of the reference (north-star gate;
in practice they are ~1e-7).  The float16-deviation path must be within 2e-3 relative L2 of float32
with >= 99.5% policy-argmax agreement, and within the reference's own test bound
(tests/test_core.py:491-511).
"""

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import oracle as orc
from test_oracle import check_cone_arrays, check_cone_hashes
from alphafly_b200 import synth
from alphafly_b200.brain import ConnectomeRNN

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
F32_GATE = 1e-4
F16_GATE = 2e-3


def rnn_for(inst, **kw):
    rnn = ConnectomeRNN(inst.conn, **kw)
    synth.apply(rnn, inst)
    return rnn.to(DEV)


class NpCone:
    """A LightCone's tensors as numpy arrays, in the oracle's field layout."""

    def __init__(self, cone):
        to = lambda x: None if x is None else x.cpu().numpy()
        self.steps = cone.steps
        self.rows = [to(r) for r in cone.rows]
        self.ops = [None if op is None else type("Op", (), {k: to(getattr(op, k)) for k in
                                                          ("edges", "post", "pre", "crow", "t_order", "t_crow", "t_col")})
                    for op in cone.ops]
        self.carried = [None] + [to(c).squeeze(1) for c in cone.carried[1:]]
        for name in ("keep_next", "keep_prev", "prev_row", "u_pos", "u_src"):
            setattr(self, name, [None] + [to(x) for x in getattr(cone, name)[1:]])
        self.out_pos, self.out_src, self.edge_visits = to(cone.out_pos), to(cone.out_src), cone.edge_visits


@pytest.fixture(scope="module")
def small():
    inst = synth.small()
    return inst, rnn_for(inst)


@pytest.fixture(scope="module")
def full():
    inst = synth.full()
    return inst, rnn_for(inst)


@pytest.mark.parametrize("steps", [1, 2, 4, 6])
def test_light_cone_fields_equal_the_reference_tiny(steps):
    g = golden("tiny")
    conn = synth.tiny(120, 700, seed=3)
    rnn = ConnectomeRNN(conn, global_scale=3.0, bias_init=0.1).to(DEV)
    cone = rnn.light_cone(torch.as_tensor(g["cone_in_idx"], device=DEV), torch.as_tensor(g["cone_out_idx"], device=DEV),
                          steps)
    check_cone_arrays(NpCone(cone), g, f"cone{steps}")
    assert len(cone.rows[0]) == 0


@pytest.mark.parametrize("config", ["small", "shuffled"])
def test_light_cone_hashes_equal_the_reference(config):
    g = golden(config)
    inst = synth.small() if config == "small" else synth.shuffled()
    rnn = rnn_for(inst)
    cone = rnn.light_cone(inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
    check_cone_hashes(NpCone(cone), g)


def test_light_cone_hashes_equal_the_reference_full(full):
    inst, rnn = full
    cone = rnn.light_cone(inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
    check_cone_hashes(NpCone(cone), golden("full"))


def test_tiny_forward_io_float32_matches_reference():
    """The reference's light-cone test graph (float64 there): outputs of the CUDA float32 path."""
    g = golden("tiny")
    conn = synth.tiny(120, 700, seed=3)
    rnn = ConnectomeRNN(conn, global_scale=3.0, bias_init=0.1)
    with torch.no_grad():
        rnn.log_gain.copy_(torch.from_numpy(g["cone_log_gain"]))
        rnn.bias.copy_(torch.from_numpy(g["cone_bias"]))
        rnn.alpha_logit.copy_(torch.from_numpy(g["cone_alpha_logit"]))
    rnn = rnn.to(DEV)
    in_idx, out_idx = torch.as_tensor(g["cone_in_idx"], device=DEV), torch.as_tensor(g["cone_out_idx"], device=DEV)
    with torch.no_grad():
        for steps in (1, 2, 4, 6):
            u = torch.as_tensor(g[f"s{steps}_u_in"], dtype=torch.float32, device=DEV)
            out = rnn.forward_io(u, in_idx, out_idx, steps)
            assert out.dtype == torch.float32 and out.shape == (20, 5)
            assert orc.rel_l2(out.cpu().numpy(), g[f"s{steps}_out"]) < 1e-6, steps


def test_small_forward_io_float32_matches_reference(small):
    inst, rnn = small
    g = golden("small")
    u = torch.from_numpy(synth.drive(inst, 64, seed=0)).to(DEV)
    with torch.no_grad():
        out = rnn.forward_io(u, inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6).cpu().numpy()
    err = orc.rel_l2(out, g["fwd_io_f64"])
    assert err < F32_GATE, err
    assert orc.rel_l2(out, g["fwd_io_f32"]) < F32_GATE
    assert rnn.device_status() == 0


def test_small_literal_forward_matches_reference(small):
    inst, rnn = small
    g = golden("small")
    u = torch.from_numpy(synth.drive(inst, 64, seed=0))
    full = torch.zeros(inst.n, 64).index_copy_(0, inst.in_idx, u).to(DEV)
    with torch.no_grad():
        h = rnn(full.contiguous(), 6)
    assert h.shape == (inst.n, 64)
    err = orc.rel_l2(h[inst.out_idx.to(DEV)].cpu().numpy(), g["fwd_full_f32"])
    assert err < F32_GATE, err


def test_shuffled_forward_io_float32_matches_reference():
    inst = synth.shuffled()
    rnn = rnn_for(inst)
    g = golden("shuffled")
    u = torch.from_numpy(synth.drive(inst, 16, seed=3)).to(DEV)
    with torch.no_grad():
        out = rnn.forward_io(u, inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6).cpu().numpy()
    assert orc.rel_l2(out, g["fwd_io_f32"]) < F32_GATE


def test_full_forward_io_and_literal_forward_match_reference(full):
    inst, rnn = full
    g = golden("full")
    with torch.no_grad():
        u = torch.from_numpy(synth.drive(inst, 8, seed=0)).to(DEV)
        out = rnn.forward_io(u, inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6).cpu().numpy()
        assert orc.rel_l2(out, g["fwd_io_f32"]) < F32_GATE
        u4 = torch.from_numpy(synth.drive(inst, 4, seed=1))
        fullu = torch.zeros(inst.n, 4).index_copy_(0, inst.in_idx, u4).to(DEV)
        h = rnn(fullu.contiguous(), 6)[inst.out_idx.to(DEV)].cpu().numpy()
    assert orc.rel_l2(h, g["fwd_full_f32"]) < F32_GATE


def policy_logits(out: np.ndarray, n_out: int) -> np.ndarray:
    """Random readout after per-neuron standardisation (the reference's RunningNorm in spirit)."""
    heads = synth.head_weights(n_out)
    r = out.T.astype(np.float64)
    r = np.clip((r - r.mean(0)) / np.sqrt(r.var(0) + 1e-8), -8, 8)
    return r @ heads["policy.weight"].T.astype(np.float64)


@pytest.mark.parametrize("config", ["small", "full"])
def test_float16_deviation_matches_float32(config, small, full):
    inst, rnn = small if config == "small" else full
    batch = 256
    u = torch.from_numpy(synth.drive(inst, batch, seed=7)).to(DEV)
    with torch.no_grad():
        ref = rnn.forward_io(u, inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
        half = rnn.forward_io(u.half(), inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
    assert half.dtype == torch.float32
    ref, half = ref.cpu().numpy(), half.cpu().numpy()
    err = orc.rel_l2(half, ref)
    assert err < F16_GATE, err
    # the position-dependent part too, not just the resting pattern it sits on
    dev_ref, dev_half = ref - ref.mean(1, keepdims=True), half - half.mean(1, keepdims=True)
    assert orc.rel_l2(dev_half, dev_ref) < 0.05
    agree = (policy_logits(half, len(inst.out_idx)).argmax(1) == policy_logits(ref, len(inst.out_idx)).argmax(1)).mean()
    assert agree >= 0.995, agree


def test_float16_deviation_reference_bound_with_clamped_rows():
    """tests/test_core.py:491-511: a small signal on a large resting state, rows on both clamps."""
    rnn = ConnectomeRNN(synth.tiny(400, 9000, seed=5), global_scale=2.0, bias_init=0.6)
    g = torch.Generator().manual_seed(0)
    with torch.no_grad():
        rnn.log_gain.add_(torch.randn(rnn.log_gain.shape, generator=g) * 0.8)
        rnn.bias.add_(torch.randn(rnn.bias.shape, generator=g) * 0.7)
        rnn.bias[::17] += 12.0
        rnn.alpha_logit.add_(torch.randn(rnn.alpha_logit.shape, generator=g))
    rnn = rnn.to(DEV)
    in_idx, out_idx = torch.arange(0, 40, device=DEV), torch.arange(300, 400, device=DEV)
    u = (torch.randn(40, 64, generator=g) * 0.05).to(DEV)
    with torch.no_grad():
        for steps in (1, 3, 6):
            ref = rnn.forward_io(u, in_idx, out_idx, steps)
            half = rnn.forward_io(u.half(), in_idx, out_idx, steps)
            signal = (ref - ref.mean(1, keepdim=True)).abs().mean()
            assert float((half - ref).abs().max()) < 0.02 * float(signal) + 1e-4, steps


@pytest.mark.parametrize("batch", [1, 5, 37, 128, 200])
def test_ragged_batches_match_the_oracle(small, batch):
    """Batch widths that are not a multiple of the kernel's 64/128-column tile, and B = 1."""
    inst, rnn = small
    pre, post = inst.conn.pre.numpy(), inst.conn.post.numpy()
    cone = orc.light_cone(inst.n, pre, post, inst.in_idx.numpy(), inst.out_idx.numpy(), 6)
    w = orc.edge_weights(inst.conn.sign.numpy(), inst.w0.numpy(), inst.log_gain.numpy())
    alpha = orc.sigmoid(inst.alpha_logit.numpy().astype(np.float64))
    u = synth.drive(inst, batch, seed=batch)
    ref = orc.forward_io(orc.full_csr(inst.n, pre, post), cone, w, inst.bias.numpy().astype(np.float64), alpha,
                         u.astype(np.float64))
    with torch.no_grad():
        out32 = rnn.forward_io(torch.from_numpy(u).to(DEV), inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
        out16 = rnn.forward_io(torch.from_numpy(u).to(DEV).half(), inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
    assert out32.shape == (len(inst.out_idx), batch)
    assert orc.rel_l2(out32.cpu().numpy(), ref) < F32_GATE
    assert orc.rel_l2(out16.cpu().numpy(), ref) < F16_GATE


@pytest.mark.parametrize("batch", [1, 8, 9, 16, 17, 33, 64, 65, 100, 128, 129])
def test_narrow_batches_equal_a_wide_run(small, batch):
    """Batches of at most 128 float16 / 64 float32 positions take the narrow kernel (G lanes per synapse,
    G = 1 .. 16); the same columns inside a 400-wide batch take the register kernel.  Columns are
    independent, so the two agree up to the order of the float32 sums (float32 path) and one float16
    rounding of the state (float16 path)."""
    inst, rnn = small
    u = torch.from_numpy(synth.drive(inst, 400, seed=batch + 3)).to(DEV)
    in_idx, out_idx = inst.in_idx.to(DEV), inst.out_idx.to(DEV)
    with torch.no_grad():
        for dtype, tol in ((torch.float32, 1e-5), (torch.float16, 2e-3)):
            wide = rnn.forward_io(u.to(dtype), in_idx, out_idx, 6)[:, :batch]
            narrow = rnn.forward_io(u[:, :batch].contiguous().to(dtype), in_idx, out_idx, 6)
            assert narrow.shape == (len(inst.out_idx), batch)
            assert orc.rel_l2(narrow.double().cpu().numpy(), wide.double().cpu().numpy()) < tol, dtype
    assert rnn.device_status() == 0


@pytest.fixture(scope="module")
def sparse():
    """Mean in-degree ~5: every light-cone step has short rows, so every step runs on the ring kernel."""
    inst = synth.small(seed=3, n=6000, e=30_000, n_in=700, n_out=150)
    return inst, rnn_for(inst)


@pytest.mark.parametrize("batch", [1, 37, 256, 300, 1120])
def test_short_row_steps_match_the_oracle(sparse, batch):
    inst, rnn = sparse
    pre, post = inst.conn.pre.numpy(), inst.conn.post.numpy()
    cone = orc.light_cone(inst.n, pre, post, inst.in_idx.numpy(), inst.out_idx.numpy(), 6)
    w = orc.edge_weights(inst.conn.sign.numpy(), inst.w0.numpy(), inst.log_gain.numpy())
    alpha = orc.sigmoid(inst.alpha_logit.numpy().astype(np.float64))
    u = synth.drive(inst, batch, seed=batch + 11)
    ref = orc.forward_io(orc.full_csr(inst.n, pre, post), cone, w, inst.bias.numpy().astype(np.float64), alpha,
                         u.astype(np.float64))
    with torch.no_grad():
        out16 = rnn.forward_io(torch.from_numpy(u).to(DEV).half(), inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
        out32 = rnn.forward_io(torch.from_numpy(u).to(DEV), inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
    assert orc.rel_l2(out32.cpu().numpy(), ref) < F32_GATE
    assert orc.rel_l2(out16.cpu().numpy(), ref) < F16_GATE
    assert rnn.device_status() == 0


def test_strided_input_and_weight_updates_invalidate_the_cache(small):
    inst, rnn = small
    u = torch.from_numpy(synth.drive(inst, 64, seed=1)).to(DEV)
    wide = torch.zeros(len(inst.in_idx), 96, device=DEV)
    wide[:, :64] = u
    with torch.no_grad():
        a = rnn.forward_io(u, inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
        b = rnn.forward_io(wide[:, :64], inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
        torch.testing.assert_close(a, b, rtol=0, atol=0)
        rnn.bias.add_(0.05)                                    # in-place update bumps the version
        c = rnn.forward_io(u, inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
        rnn.bias.sub_(0.05)
        d = rnn.forward_io(u, inst.in_idx.to(DEV), inst.out_idx.to(DEV), 6)
    assert not torch.allclose(a, c)
    torch.testing.assert_close(a, d, rtol=1e-5, atol=1e-5)         # b + 0.05 - 0.05 is not exact in float32


def test_columns_are_independent_at_full_batch(full):
    """Size-independent property at the benchmark's batch: each position's output depends only on its
    own column.  A 35,840-wide float16 run equals, bitwise, a 12,800-wide run of the same columns (both
    wide enough to take the same item schedules), and equals a 512-wide run (which takes the fine
    schedule on the small steps, so rows cut between warps are summed in another order) to within the
    float16 rounding of the deviation state."""
    inst, rnn = full
    u = torch.from_numpy(synth.drive(inst, 512, seed=11)).to(DEV).half()
    big = u.repeat(1, 70)                                     # 35,840 columns
    in_idx, out_idx = inst.in_idx.to(DEV), inst.out_idx.to(DEV)
    with torch.no_grad():
        wide = rnn.forward_io(big, in_idx, out_idx, 6)
        mid = rnn.forward_io(u.repeat(1, 25).contiguous(), in_idx, out_idx, 6)
        narrow = rnn.forward_io(u, in_idx, out_idx, 6)
    assert wide.shape == (len(inst.out_idx), 35840)
    torch.testing.assert_close(wide[:, :12800], mid, rtol=0, atol=0)
    for k in (0, 33, 69):
        torch.testing.assert_close(wide[:, k * 512:(k + 1) * 512], mid[:, :512], rtol=0, atol=0)
        torch.testing.assert_close(wide[:, k * 512:(k + 1) * 512], narrow, rtol=0, atol=2e-3)
    assert rnn.device_status() == 0


@pytest.mark.parametrize("batch", [1, 64, 1120, 8192, 65536])
def test_shuffled_control_batch_sweep(batch):
    """Configuration 4: the degree-preserving shuffled control (duplicate synapses allowed) at the batch
    sizes of its sweep.  float16 deviation against float32 (the north-star gate); float32 against the
    oracle where it finishes in seconds (B <= 64)."""
    inst = synth.shuffled()
    rnn = rnn_for(inst)
    u = torch.from_numpy(synth.drive(inst, min(batch, 2048), seed=batch)).repeat(1, (batch + 2047) // 2048)[:, :batch]
    u = u.contiguous().to(DEV)
    in_idx, out_idx = inst.in_idx.to(DEV), inst.out_idx.to(DEV)
    with torch.no_grad():
        out32 = rnn.forward_io(u, in_idx, out_idx, 6)
        out16 = rnn.forward_io(u.half(), in_idx, out_idx, 6)
    assert out16.shape == (len(inst.out_idx), batch) and out16.dtype == torch.float32
    assert orc.rel_l2(out16.cpu().numpy(), out32.cpu().numpy()) < F16_GATE
    if batch <= 64:
        pre, post = inst.conn.pre.numpy(), inst.conn.post.numpy()
        cone = orc.light_cone(inst.n, pre, post, inst.in_idx.numpy(), inst.out_idx.numpy(), 6)
        w = orc.edge_weights(inst.conn.sign.numpy(), inst.w0.numpy(), inst.log_gain.numpy())
        ref = orc.forward_io(orc.full_csr(inst.n, pre, post), cone, w, inst.bias.numpy().astype(np.float64),
                             orc.sigmoid(inst.alpha_logit.numpy().astype(np.float64)), u.cpu().numpy().astype(np.float64))
        assert orc.rel_l2(out32.cpu().numpy(), ref) < F32_GATE
    assert rnn.device_status() == 0


def test_cached_constants_in_the_reference_layout(small):
    """brain._cached[1] = (cs, ks, mats, alpha, fused) as the reference's diagnostics read it
    (scripts/profile_gpu.py:27): one float32 step rebuilt from them in the reference's way equals the
    light-cone forward, and the resting trajectory equals the oracle's."""
    inst, rnn = small
    in_idx, out_idx = inst.in_idx.to(DEV), inst.out_idx.to(DEV)
    u = torch.from_numpy(synth.drive(inst, 8, seed=2)).to(DEV)
    with torch.no_grad():
        out = rnn.forward_io(u, in_idx, out_idx, 6)
        cs, ks, mats, alpha, fused = rnn._cached[1]
        cone = rnn.light_cone(in_idx, out_idx, 6)
        h = None
        for t in range(1, 7):
            rows = cone.rows[t]
            x = ks[t].expand(-1, 8).clone() if mats[t] is None else mats[t] @ h + ks[t]
            x = x.index_add(0, cone.u_pos[t], u[cone.u_src[t]]).clamp(0, rnn.h_max)
            prev = cs[t - 1][rows].expand(-1, 8)
            if len(cone.keep_next[t]):
                prev = prev.index_copy(0, cone.keep_next[t], h[cone.keep_prev[t]])
            h = torch.lerp(prev, x, alpha[rows])
        rebuilt = cs[6][out_idx].expand(-1, 8).index_copy(0, cone.out_pos, h[cone.out_src])
    assert orc.rel_l2(rebuilt.cpu().numpy(), out.cpu().numpy()) < 1e-5
    pre, post = inst.conn.pre.numpy(), inst.conn.post.numpy()
    w = orc.edge_weights(inst.conn.sign.numpy(), inst.w0.numpy(), inst.log_gain.numpy())
    W = orc.full_csr(inst.n, pre, post)
    c = np.zeros(inst.n)
    a = orc.sigmoid(inst.alpha_logit.numpy().astype(np.float64))
    for t in range(1, 7):
        s = W.matmul(w, c[:, None])[:, 0] if t > 1 else np.zeros(inst.n)
        c = orc.lerp(c, np.clip(s + inst.bias.numpy(), 0, 10.0), a)
        assert orc.rel_l2(cs[t].squeeze(1).cpu().numpy(), c) < 1e-5, t
