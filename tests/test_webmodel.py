"""The browser model format (scripts/export_web.py:19-82): file naming and chunking against the reference's
own exported manifest, decoding of the reference's exported tensors (tests/golden/web, copied from its
docs/model by tests/golden/make_web_golden.py), and a writer -> reader -> FlyChessNet round trip on CPU."""

import json

import numpy as np
import pytest
import torch

from conftest import ROOT
from alphafly_b200 import synth, webmodel
from alphafly_b200.encoding import N_BASE
from alphafly_b200.model import FlyChessNet, ModelConfig




def _web_dir():
    from pathlib import Path
    return Path(ROOT) / "tests" / "golden" / "web"


def _ref_manifest():
    return json.loads((_web_dir() / "manifest.json").read_text())


def test_chunking_and_names_match_the_reference_manifest():
    m = _ref_manifest()
    for name, t in m["tensors"].items():
        assert webmodel.chunk_files(name, t["bytes"]) == t["files"], name
    assert set(m) >= {"neurons", "edges", "steps", "h_max", "input_gain", "n_base", "norm_eps", "norm_clip", "tensors"}
    assert m["n_base"] == N_BASE


def test_writer_uses_the_reference_tensor_table():
    """Same tensors, order, kinds and shape conventions as the reference's export of its trained network."""
    m = _ref_manifest()
    net = FlyChessNet(synth.tiny(60, 600), ModelConfig(steps=3))
    mine = webmodel._tensor_list(net)
    assert [n for n, _, _ in mine] == list(m["tensors"])
    for name, arr, kind in mine:
        ref = m["tensors"][name]
        assert kind == ref["kind"], name
        assert len(ref["shape"]) == (1 if kind == "u24" else arr.ndim), name
    n, e = m["neurons"], m["edges"]
    t = m["tensors"]
    assert t["crow"]["shape"] == [n + 1] and t["values"]["shape"] == [e] and t["col"]["shape"] == [3 * e]
    assert t["encoder_wT"]["shape"] == [N_BASE, len_in := t["in_idx"]["shape"][0]] and len_in == 17937
    assert t["policy_w"]["shape"] == [4168, t["out_idx"]["shape"][0]]


def test_the_reference_exported_tensors_decode():
    m, t = webmodel.read_web_model(_web_dir(), names={"in_idx", "out_idx", "encoder_b", "norm_mean", "norm_std",
                                                       "policy_b", "from_b", "to_b", "value_w", "value_b"})
    n = m["neurons"]
    for name, arr in t.items():
        assert list(arr.shape) == m["tensors"][name]["shape"], name
    for idx in (t["in_idx"], t["out_idx"]):
        assert np.all(np.diff(idx.astype(np.int64)) > 0) and idx.max() < n
    assert len(np.intersect1d(t["in_idx"], t["out_idx"])) == 0
    assert np.all(t["norm_std"] > 0) and np.all(np.isfinite(t["norm_mean"]))
    assert t["value_w"].shape == (3, len(t["out_idx"]))
    # the test positions recorded by the reference: board features inside N_BASE, legal moves inside N_MOVES
    for pos in m["tests"]:
        assert all(0 <= f < N_BASE for f in pos["features"]) and len(pos["idx"]) == len(pos["logits"])
        assert all(0 <= i < 4168 for i in pos["idx"]) and -1.0 <= pos["value"] <= 1.0


def test_u24_round_trip():
    v = np.array([0, 1, 255, 256, 65535, 65536, (1 << 24) - 1], np.uint32)
    enc = webmodel.encode_u24(v)
    assert enc.dtype == np.uint8 and enc.size == 3 * v.size
    assert np.array_equal(webmodel.decode_u24(enc), v)
    with pytest.raises(ValueError):
        webmodel.encode_u24(np.array([1 << 24], np.uint32))


def test_export_read_rebuild_round_trip(tmp_path):
    """A small network through the writer (chunks forced small), the reader and net_from_web_model: the
    rebuilt network holds exactly the exported (float16-rounded where the format is f16) parameters."""
    conn = synth.tiny(60, 600, seed=2)
    net = FlyChessNet(conn, ModelConfig(steps=4))
    g = torch.Generator().manual_seed(7)
    with torch.no_grad():
        for p in net.parameters():
            p.copy_(torch.randn(p.shape, generator=g) * 0.1)
        net.norm.mean.normal_(0, 1, generator=g)
        net.norm.var.uniform_(0.5, 2.0, generator=g)
    m = webmodel.export_web_model(net, tmp_path, checkpoint="test.pt", chunk=1000)
    assert len(m["tensors"]["values"]["files"]) == -(-m["tensors"]["values"]["bytes"] // 1000)
    m2, t = webmodel.read_web_model(tmp_path)
    assert m2 == json.loads(json.dumps(m))
    b = net.brain
    w = (b.sign * b.w0 * b.log_gain.exp()).detach()
    assert np.array_equal(t["values"], w.numpy().astype(np.float16))
    assert np.array_equal(t["col"], b.pre.numpy()) and np.array_equal(t["crow"], b.crow.numpy())
    back = webmodel.net_from_web_model(tmp_path, device="cpu")
    bb = back.brain
    assert np.array_equal(bb.pre.numpy(), b.pre.numpy()) and np.array_equal(bb.post.numpy(), b.post.numpy())
    assert np.array_equal((bb.sign * bb.w0 * bb.log_gain.exp()).detach().numpy(), w.numpy().astype(np.float16).astype(np.float32))
    np.testing.assert_allclose(torch.sigmoid(bb.alpha_logit).detach().numpy(), torch.sigmoid(b.alpha_logit).detach().numpy(),
                               rtol=1e-6)
    assert torch.equal(bb.bias, b.bias) and back.cfg.steps == 4
    assert torch.equal(back.in_idx, net.in_idx) and torch.equal(back.out_idx, net.out_idx)
    assert torch.equal(back.encoder.weight[:, :N_BASE], net.encoder.weight[:, :N_BASE].half().float())
    assert torch.equal(back.policy.weight, net.policy.weight.half().float())
    for name in ("policy_from", "policy_to", "value"):
        assert torch.equal(getattr(back, name).weight, getattr(net, name).weight), name
    np.testing.assert_allclose(back.norm.var.numpy(), net.norm.var.numpy(), rtol=1e-5)
