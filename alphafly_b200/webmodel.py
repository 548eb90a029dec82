"""The browser engine's model format (scripts/export_web.py:19-82): writer, reader, and a FlyChessNet built
from it.

A model directory holds ``manifest.json`` and ``weights/<name>.<k>.bin``: each tensor as little-endian raw
bytes split into chunks of at most 24 MiB.  The kinds are

    f16   IEEE half                       values (effective synapse weights in CSR order), encoder_wT, policy_w
    f32   IEEE single                     bias, alpha (sigmoid of alpha_logit), encoder_b, norm_mean, norm_std, heads
    u32   unsigned 32-bit                 crow (row pointer of W[post, pre]), in_idx, out_idx
    u24   3 bytes per value, low first    col (the presynaptic neuron of each synapse)

and the manifest records ``neurons``, ``edges``, ``steps``, ``h_max``, ``input_gain``, ``n_base``,
``norm_eps``, ``norm_clip``, ``checkpoint``, a ``tensors`` table (kind, shape, files, bytes) and optional
``tests`` (positions with the float32 legal-move logits and value the network must reproduce).

``net_from_web_model`` rebuilds a network that evaluates exactly the exported weights: the synapse
weights are the float16 values themselves (sign and magnitude as the wiring's sign and w0, log_gain 0),
alpha_logit = logit(alpha), and the normaliser's variance = norm_std^2 - norm_eps.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from .connectome import Connectome, neuron_table
from .encoding import N_BASE, N_FEATURES, N_MOVES
from .model import READOUT_SUPERCLASSES, FlyChessNet, ModelConfig

CHUNK = 24 * 2**20
DTYPES = {"f16": "<f2", "f32": "<f4", "u32": "<u4"}


def chunk_files(name: str, nbytes: int, chunk: int = CHUNK) -> list[str]:
    """The file names a tensor of ``nbytes`` bytes is written to (one file even when empty)."""
    return [f"weights/{name}.{k}.bin" for k in range(max(1, -(-nbytes // chunk)))]


def encode_u24(v: np.ndarray) -> np.ndarray:
    v = np.asarray(v, np.uint32)
    if v.size and int(v.max()) >= 1 << 24:
        raise ValueError("u24 holds values below 2^24")
    return (v[:, None] >> np.array([0, 8, 16], dtype=np.uint32)).astype(np.uint8).reshape(-1)


def decode_u24(raw: np.ndarray) -> np.ndarray:
    b = np.asarray(raw, np.uint8).reshape(-1, 3).astype(np.uint32)
    return b[:, 0] | (b[:, 1] << 8) | (b[:, 2] << 16)


def _tensor_list(net: FlyChessNet) -> list[tuple[str, np.ndarray, str]]:
    """(name, array, kind) in the reference's order (scripts/export_web.py:49-69)."""
    b = net.brain
    with torch.no_grad():
        f = lambda t: t.detach().float().cpu().numpy()
        return [
            ("values", f(b.sign * b.w0 * b.log_gain.exp()).astype("<f2"), "f16"),    # edge_weights (brain.py:201-202)
            ("crow", b.crow.cpu().numpy().astype("<u4"), "u32"),
            ("col", encode_u24(b.pre.cpu().numpy()), "u24"),
            ("bias", f(b.bias).astype("<f4"), "f32"),
            ("alpha", f(torch.sigmoid(b.alpha_logit)).astype("<f4"), "f32"),
            ("in_idx", net.in_idx.cpu().numpy().astype("<u4"), "u32"),
            ("out_idx", net.out_idx.cpu().numpy().astype("<u4"), "u32"),
            ("encoder_wT", np.ascontiguousarray(f(net.encoder.weight[:, :N_BASE]).T).astype("<f2"), "f16"),
            ("encoder_b", f(net.encoder.bias).astype("<f4"), "f32"),
            ("norm_mean", f(net.norm.mean).astype("<f4"), "f32"),
            ("norm_std", f((net.norm.var + net.norm.eps).sqrt()).astype("<f4"), "f32"),
            ("policy_w", f(net.policy.weight).astype("<f2"), "f16"),
            ("policy_b", f(net.policy.bias).astype("<f4"), "f32"),
            ("from_w", f(net.policy_from.weight).astype("<f4"), "f32"),
            ("from_b", f(net.policy_from.bias).astype("<f4"), "f32"),
            ("to_w", f(net.policy_to.weight).astype("<f4"), "f32"),
            ("to_b", f(net.policy_to.bias).astype("<f4"), "f32"),
            ("value_w", f(net.value.weight).astype("<f4"), "f32"),
            ("value_b", f(net.value.bias).astype("<f4"), "f32"),
        ]


def export_web_model(net: FlyChessNet, out, checkpoint: str = "", tests: list | None = None, chunk: int = CHUNK) -> dict:
    """Write ``net`` in the browser format under ``out``; returns the manifest.  ``tests`` (optional) is the
    manifest's list of test positions (see ``make_test_vectors``)."""
    out = Path(out)
    (out / "weights").mkdir(parents=True, exist_ok=True)
    b, cfg = net.brain, net.cfg
    manifest = {"neurons": b.n, "edges": int(b.pre.numel()), "steps": cfg.steps, "h_max": b.h_max,
                "input_gain": cfg.input_gain, "n_base": N_BASE, "norm_eps": net.norm.eps, "norm_clip": net.norm.clip,
                "checkpoint": checkpoint, "tensors": {}}
    for name, arr, kind in _tensor_list(net):
        raw = arr.tobytes()
        files = chunk_files(name, len(raw), chunk)
        for k, f in enumerate(files):
            (out / f).write_bytes(raw[k * chunk:(k + 1) * chunk])
        shape = [arr.size] if kind == "u24" else list(arr.shape)
        manifest["tensors"][name] = {"kind": kind, "shape": shape, "files": files, "bytes": len(raw)}
    if tests is not None:
        manifest["tests"] = tests
    (out / "manifest.json").write_text(json.dumps(manifest))
    return manifest


def read_web_model(model_dir, names=None) -> tuple[dict, dict[str, np.ndarray]]:
    """(manifest, {name: array}) of a model directory; ``names`` limits the tensors read.  u24 tensors come
    back decoded (one uint32 per value), the others in their stored dtype and shape."""
    model_dir = Path(model_dir)
    manifest = json.loads((model_dir / "manifest.json").read_text())
    out = {}
    for name, t in manifest["tensors"].items():
        if names is not None and name not in names:
            continue
        raw = bytearray(b"".join((model_dir / f).read_bytes() for f in t["files"]))   # writable arrays
        if len(raw) != t["bytes"]:
            raise ValueError(f"{name}: {len(raw)} bytes on disk, the manifest says {t['bytes']}")
        if t["kind"] == "u24":
            out[name] = decode_u24(np.frombuffer(raw, np.uint8))
        else:
            out[name] = np.frombuffer(raw, DTYPES[t["kind"]]).reshape(t["shape"])
    return manifest, out


def net_from_web_model(model_dir, device="cuda") -> FlyChessNet:
    """A FlyChessNet that evaluates the exported weights (see the module docstring)."""
    manifest, t = read_web_model(model_dir)
    n, e = int(manifest["neurons"]), int(manifest["edges"])
    crow = t["crow"].astype(np.int64)
    if crow.shape != (n + 1,) or crow[-1] != e:
        raise ValueError("crow does not match the manifest's neuron and edge counts")
    post = torch.as_tensor(np.repeat(np.arange(n, dtype=np.int64), np.diff(crow)))
    pre = torch.as_tensor(t["col"].astype(np.int64))
    w = torch.as_tensor(t["values"].astype(np.float32))
    in_idx, out_idx = t["in_idx"].astype(np.int64), t["out_idx"].astype(np.int64)
    neurons = neuron_table(n, in_idx, np.setdiff1d(out_idx, in_idx))
    both = np.intersect1d(out_idx, in_idx)
    if both.size:                                 # inputs that are also read out
        neurons.loc[both, "super_class"] = READOUT_SUPERCLASSES[0]
    conn = Connectome(neurons, pre, post, torch.ones(e), torch.sign(w))
    cfg = ModelConfig(steps=int(manifest["steps"]), input_gain=float(manifest["input_gain"]))
    net = FlyChessNet(conn, cfg)
    b = net.brain
    b.h_max = float(manifest["h_max"])
    b.w0 = w.abs()
    alpha = torch.as_tensor(t["alpha"].astype(np.float64)).clamp(1e-12, 1 - 1e-12)
    norm_std = torch.as_tensor(t["norm_std"].astype(np.float32))
    with torch.no_grad():
        b.log_gain.zero_()
        b.bias.copy_(torch.as_tensor(t["bias"]))
        b.alpha_logit.copy_(torch.log(alpha / (1 - alpha)).float())
        net.encoder.weight.zero_()
        net.encoder.weight[:, :N_BASE].copy_(torch.as_tensor(t["encoder_wT"].astype(np.float32)).T)
        net.encoder.bias.copy_(torch.as_tensor(t["encoder_b"]))
        net.norm.eps, net.norm.clip = float(manifest["norm_eps"]), float(manifest["norm_clip"])
        net.norm.mean.copy_(torch.as_tensor(t["norm_mean"]))
        net.norm.var.copy_(norm_std * norm_std - net.norm.eps)
        net.norm.initialised.fill_(True)
        for layer, wn, bn in ((net.policy, "policy_w", "policy_b"), (net.policy_from, "from_w", "from_b"),
                              (net.policy_to, "to_w", "to_b"), (net.value, "value_w", "value_b")):
            layer.weight.copy_(torch.as_tensor(t[wn].astype(np.float32)))
            layer.bias.copy_(torch.as_tensor(t[bn]))
    if not (np.array_equal(net.in_idx.numpy(), in_idx) and np.array_equal(net.out_idx.numpy(), out_idx)):
        raise ValueError("in_idx / out_idx must be sorted and unique")
    return net.to(device).eval()


@torch.no_grad()
def make_test_vectors(net: FlyChessNet, x: np.ndarray, legal: list[np.ndarray]) -> list[dict]:
    """The manifest's test positions without python-chess: for each board feature vector (N_FEATURES) and
    its legal-move indices, the float32 logits of those moves and the value (scripts/export_web.py:71-80;
    ``fen`` and ``moves`` are left out)."""
    net.eval()
    dtype = net.infer_dtype
    net.infer_dtype = torch.float32
    try:
        dev = next(net.parameters()).device
        logits, wdl = net(torch.as_tensor(np.asarray(x, np.float32), device=dev))
        value = net.expected_value(wdl)
    finally:
        net.infer_dtype = dtype
    out = []
    for k, idx in enumerate(legal):
        idx = np.asarray(idx, np.int64)
        assert idx.size == 0 or (idx.min() >= 0 and idx.max() < N_MOVES)
        out.append({"idx": idx.tolist(), "logits": [round(float(v), 4) for v in logits[k, idx].cpu()],
                    "value": round(float(value[k]), 5), "features": np.flatnonzero(np.asarray(x[k])[:N_BASE]).tolist()})
    return out
