"""Generate the golden fixtures in this folder by running the REFERENCE implementation.

Usage (needs the reference checkout; it is not present on GPU boxes, which only read the .npz):
    python tests/golden/make_golden.py /path/to/alpha-fly

It imports the reference's chessfly/brain.py unchanged (python-chess is not installed, so a stub
``chess`` module is put in ``sys.modules``; brain.py never touches it), builds each synthetic graph
with ``alphafly_b200.synth``, writes the instance's w0 and parameters into the reference's
``ConnectomeRNN`` and records, on CPU:
  * tiny.npz      the reference test graphs (tests/test_core.py:12-44, 309-338): literal recurrence
                  and light-cone outputs and all gradients in float64, the full LightCone fields
  * small.npz     configuration 1: LightCone sizes and hashes (6 steps), forward_io and forward in
                  float32 and float64 at B=64, float64 gradients of forward_io at B=8
  * shuffled.npz  configuration 4: LightCone hashes, forward_io float32 at B=16
  * full.npz      configuration 2 graph: LightCone sizes and hashes (6 steps), forward_io float32 at
                  B=8, forward (no pruning) float32 at B=4
  * model.npz     FlyChessNet on the 60-neuron test graph (tests/test_core.py:404): the initial
                  state_dict, eval-mode float32 logits, and one train_step (chessfly/train.py:126-138) with
                  its losses, clipped gradients, updated parameters and RunningNorm statistics
The reference's trainer imports modules that use python-chess at import time; a permissive stand-in
module (every attribute a neutral dummy) is installed for them.  It is never called on the network path.
Index arrays too large to store are pinned by the SHA-256 of their int64 little-endian bytes.
"""

from __future__ import annotations

import hashlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from alphafly_b200 import synth  # noqa: E402


def sha(a) -> str:
    a = a.detach().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a)
    return hashlib.sha256(np.ascontiguousarray(a.astype("<i8")).tobytes()).hexdigest()


def fsha(a) -> str:
    a = a.detach().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a)
    return hashlib.sha256(np.ascontiguousarray(a.astype("<f4")).tobytes()).hexdigest()


def cone_record(cone, prefix="cone") -> dict:
    """Sizes of every LightCone field and the hash of every index array."""
    out = {f"{prefix}_edge_visits": np.int64(cone.edge_visits),
           f"{prefix}_rows_len": np.array([len(r) for r in cone.rows], np.int64),
           f"{prefix}_nnz": np.array([0 if op is None else len(op.edges) for op in cone.ops], np.int64),
           f"{prefix}_out_pos_sha": sha(cone.out_pos), f"{prefix}_out_src_sha": sha(cone.out_src)}
    for t in range(cone.steps + 1):
        out[f"{prefix}_rows{t}_sha"] = sha(cone.rows[t])
    for t in range(1, cone.steps + 1):
        for name in ("keep_next", "keep_prev", "prev_row", "u_pos", "u_src"):
            out[f"{prefix}_{name}{t}_sha"] = sha(getattr(cone, name)[t])
        out[f"{prefix}_carried{t}_sha"] = sha(cone.carried[t].squeeze(1))
        op = cone.ops[t]
        if op is not None:
            for name in ("edges", "post", "pre", "crow", "t_order", "t_crow", "t_col"):
                out[f"{prefix}_op{t}_{name}_sha"] = sha(getattr(op, name))
            # duplicate synapses (the shuffled control) make equal sort keys, whose order in torch's
            # unstable argsort is implementation-defined: record the tie-free canonical form as well
            key = (op.pre * op.shape[0] + op.post).numpy()
            t_order = op.t_order.numpy()
            assert np.all(np.diff(key[t_order]) >= 0) and np.array_equal(np.sort(t_order), np.arange(len(key)))
            out[f"{prefix}_op{t}_t_order_ties"] = np.bool_(len(np.unique(key)) < len(key))
            out[f"{prefix}_op{t}_t_order_canon_sha"] = sha(np.argsort(key, kind="stable"))
    return out


def cone_arrays(cone, prefix="cone") -> dict:
    """Every LightCone index array in full (small graphs only)."""
    out = {}
    for t in range(cone.steps + 1):
        out[f"{prefix}_rows{t}"] = cone.rows[t].numpy()
    for t in range(1, cone.steps + 1):
        for name in ("keep_next", "keep_prev", "prev_row", "u_pos", "u_src"):
            out[f"{prefix}_{name}{t}"] = getattr(cone, name)[t].numpy()
        out[f"{prefix}_carried{t}"] = cone.carried[t].squeeze(1).numpy()
        op = cone.ops[t]
        if op is not None:
            for name in ("edges", "post", "pre", "crow", "t_order", "t_crow", "t_col"):
                out[f"{prefix}_op{t}_{name}"] = getattr(op, name).numpy()
    out[f"{prefix}_out_pos"], out[f"{prefix}_out_src"] = cone.out_pos.numpy(), cone.out_src.numpy()
    out[f"{prefix}_edge_visits"] = np.int64(cone.edge_visits)
    return out


def graph_record(inst) -> dict:
    return {"graph_pre_sha": sha(inst.conn.pre), "graph_post_sha": sha(inst.conn.post),
            "graph_sign_sha": fsha(inst.conn.sign), "graph_w0_sha": fsha(inst.w0),
            "graph_log_gain_sha": fsha(inst.log_gain), "graph_bias_sha": fsha(inst.bias),
            "graph_alpha_logit_sha": fsha(inst.alpha_logit), "graph_e": np.int64(inst.e)}


def reference_rnn(brain, inst, dtype=torch.float32):
    rnn = brain.ConnectomeRNN(inst.conn)
    synth.apply(rnn, inst)
    return rnn.to(dtype)


def make_tiny(brain) -> dict:
    rec = {}
    # the dense-restatement test graph (tests/test_core.py:30-44)
    conn = synth.tiny()
    torch.manual_seed(0)
    rnn = brain.ConnectomeRNN(conn, global_scale=3.0).double()
    u = torch.rand(4, rnn.n, dtype=torch.double, requires_grad=True)
    target = torch.rand(4, rnn.n, dtype=torch.double)
    out = rnn(u.T.contiguous(), 5).T
    ((out - target) ** 2).sum().backward()
    rec.update(dense_pre=conn.pre.numpy(), dense_post=conn.post.numpy(), dense_sign=conn.sign.numpy(),
               dense_w0=rnn.w0.numpy(), dense_u=u.detach().numpy(), dense_target=target.numpy(),
               dense_out=out.detach().numpy(), dense_grad_u=u.grad.numpy(),
               dense_grad_log_gain=rnn.log_gain.grad.numpy(), dense_grad_bias=rnn.bias.grad.numpy(),
               dense_alpha_logit=rnn.alpha_logit.detach().numpy(), dense_bias=rnn.bias.detach().numpy())
    # the light-cone test graph (tests/test_core.py:309-338), perturbations seeded here
    conn = synth.tiny(120, 700, seed=3)
    rnn = brain.ConnectomeRNN(conn, global_scale=3.0, bias_init=0.1).double()
    g = torch.Generator().manual_seed(1)
    with torch.no_grad():
        rnn.bias.add_(torch.randn(rnn.n, dtype=torch.double, generator=g) * 0.2)
        rnn.alpha_logit.add_(torch.randn(rnn.n, dtype=torch.double, generator=g))
        rnn.log_gain.add_(torch.randn(conn.n_edges, dtype=torch.double, generator=g) * 0.3)
    in_idx, out_idx = torch.arange(0, 9), torch.arange(100, 120)
    rec.update(cone_pre=conn.pre.numpy(), cone_post=conn.post.numpy(), cone_sign=conn.sign.numpy(),
               cone_w0=rnn.w0.numpy(), cone_log_gain=rnn.log_gain.detach().numpy(),
               cone_bias=rnn.bias.detach().numpy(), cone_alpha_logit=rnn.alpha_logit.detach().numpy(),
               cone_in_idx=in_idx.numpy(), cone_out_idx=out_idx.numpy())
    for steps in (1, 2, 4, 6):
        u_in = torch.randn(9, 5, dtype=torch.double, generator=g, requires_grad=True)
        target = torch.randn(20, 5, dtype=torch.double, generator=g)
        rnn.zero_grad()
        out = rnn.forward_io(u_in, in_idx, out_idx, steps)
        ((out - target) ** 2).sum().backward()
        p = f"s{steps}_"
        grad = lambda t: (t.grad if t.grad is not None else torch.zeros_like(t)).detach().numpy()
        rec.update({p + "u_in": u_in.detach().numpy(), p + "target": target.numpy(), p + "out": out.detach().numpy(),
                    p + "grad_u_in": grad(u_in), p + "grad_log_gain": grad(rnn.log_gain),
                    p + "grad_bias": grad(rnn.bias), p + "grad_alpha_logit": grad(rnn.alpha_logit)})
        rec.update(cone_arrays(rnn.light_cone(in_idx, out_idx, steps), prefix=f"cone{steps}"))
    return rec


def make_small(brain) -> dict:
    inst = synth.small()
    rec = graph_record(inst)
    rnn = reference_rnn(brain, inst)
    cone = rnn.light_cone(inst.in_idx, inst.out_idx, 6)
    rec.update(cone_record(cone))
    u64 = synth.drive(inst, 64, seed=0)
    rec["u_sha"] = fsha(u64)
    with torch.no_grad():
        u = torch.from_numpy(u64)
        rec["fwd_io_f32"] = rnn.forward_io(u, inst.in_idx, inst.out_idx, 6).numpy()
        full = torch.zeros(inst.n, 64).index_copy_(0, inst.in_idx, u)
        rec["fwd_full_f32"] = rnn(full.contiguous(), 6)[inst.out_idx].numpy()
        rnn64 = reference_rnn(brain, inst, torch.float64)
        rec["fwd_io_f64"] = rnn64.forward_io(u.double(), inst.in_idx, inst.out_idx, 6).numpy()
    # float64 gradients of forward_io at B=8 against a fixed projection of the output
    u8 = torch.from_numpy(synth.drive(inst, 8, seed=5)).double().requires_grad_(True)
    tgt = torch.from_numpy(np.random.default_rng(9).standard_normal((len(inst.out_idx), 8)))
    rnn64.zero_grad()
    out = rnn64.forward_io(u8, inst.in_idx, inst.out_idx, 6)
    (out * tgt).sum().backward()
    proj = np.random.default_rng(11).standard_normal((8, inst.e))
    sample = np.random.default_rng(12).choice(inst.e, 4096, replace=False)
    lg = rnn64.log_gain.grad.numpy()
    rec.update(grad_target=tgt.numpy(), grad_out=out.detach().numpy(), grad_u_in=u8.grad.numpy(),
               grad_bias=rnn64.bias.grad.numpy(), grad_alpha_logit=rnn64.alpha_logit.grad.numpy(),
               grad_log_gain_proj=proj @ lg, grad_log_gain_norm=np.linalg.norm(lg),
               grad_log_gain_sample_idx=sample, grad_log_gain_sample=lg[sample])
    return rec


def make_shuffled(brain) -> dict:
    inst = synth.shuffled()
    rec = graph_record(inst)
    rnn = reference_rnn(brain, inst)
    cone = rnn.light_cone(inst.in_idx, inst.out_idx, 6)
    rec.update(cone_record(cone))
    with torch.no_grad():
        u = torch.from_numpy(synth.drive(inst, 16, seed=3))
        rec["fwd_io_f32"] = rnn.forward_io(u, inst.in_idx, inst.out_idx, 6).numpy()
    return rec


def make_full(brain) -> dict:
    inst = synth.full()
    rec = graph_record(inst)
    rnn = reference_rnn(brain, inst)
    cone = rnn.light_cone(inst.in_idx, inst.out_idx, 6)
    rec.update(cone_record(cone))
    with torch.no_grad():
        u = torch.from_numpy(synth.drive(inst, 8, seed=0))
        rec["fwd_io_f32"] = rnn.forward_io(u, inst.in_idx, inst.out_idx, 6).numpy()
        u4 = torch.from_numpy(synth.drive(inst, 4, seed=1))
        full = torch.zeros(inst.n, 4).index_copy_(0, inst.in_idx, u4)
        rec["fwd_full_f32"] = rnn(full.contiguous(), 6)[inst.out_idx].numpy()
    return rec


class _Dummy:
    """A neutral stand-in value for python-chess attributes used at import time by the reference's
    search modules; the network and trainer never call them."""

    def __getattr__(self, k):
        return _Dummy()

    def __call__(self, *a, **k):
        return _Dummy()

    def __iter__(self):
        return iter(())

    def __int__(self):
        return 0

    def __index__(self):
        return 0

    def __hash__(self):
        return 0

    def __eq__(self, o):
        return False

    def __bool__(self):
        return False

    def __len__(self):
        return 0

    def __getitem__(self, k):
        return _Dummy()

    def __mro_entries__(self, bases):
        return (object,)

    __add__ = __radd__ = __sub__ = __rsub__ = __mul__ = __rmul__ = __or__ = __ror__ = __and__ = __rand__ = \
        __xor__ = __lshift__ = __rshift__ = __mod__ = __floordiv__ = __truediv__ = __neg__ = __invert__ = \
        lambda self, *a: _Dummy()


class _DummyModule(types.ModuleType):
    def __getattr__(self, k):
        if k.startswith("__"):
            raise AttributeError(k)
        return _Dummy()


def install_chess_stand_in():
    chess = _DummyModule("chess")
    chess.__path__ = []
    sys.modules["chess"] = chess
    for sub in ("pgn", "engine", "polyglot", "svg"):
        m = _DummyModule("chess." + sub)
        sys.modules["chess." + sub] = m
        setattr(chess, sub, m)


def make_model(brain) -> dict:
    import chessfly.model as M
    import chessfly.selfplay as SP
    import chessfly.train as TR
    conn = synth.tiny(60, 600)
    torch.manual_seed(0)
    net = M.FlyChessNet(conn, M.ModelConfig(steps=3))
    g = torch.Generator().manual_seed(5)
    with torch.no_grad():
        for layer in (net.policy, net.value, net.policy_from, net.policy_to):
            layer.weight.copy_(torch.randn(layer.weight.shape, generator=g) * 0.05)
            layer.bias.copy_(torch.randn(layer.bias.shape, generator=g) * 0.05)
        net.brain.log_gain.add_(torch.randn(net.brain.log_gain.shape, generator=g) * 0.2)
    rec = {"state_" + k: v.detach().numpy().copy() for k, v in net.state_dict().items()}
    x = synth.boards(6, seed=1)
    net.eval()
    with torch.no_grad():
        logits, wdl = net(torch.from_numpy(x))
    rec.update(x=x, eval_logits=logits.numpy(), eval_wdl=wdl.numpy())
    rng = np.random.default_rng(2)
    batch, idxs, pis, qs, wdls = [], [], [], [], []
    for i in range(8):
        idx = np.sort(rng.choice(4168, 30, replace=False)).astype(np.int16)
        z = rng.standard_normal(30)
        pi = (np.exp(z) / np.exp(z).sum()).astype(np.float16)
        q = float(rng.uniform(-1, 1))
        w = int(rng.choice(3, p=[0.45, 0.10, 0.45]))
        batch.append(SP.Sample(synth.boards(1, seed=10 + i)[0].astype(np.float16), idx, pi, q, w))
        idxs.append(idx), pis.append(pi), qs.append(q), wdls.append(w)
    rec.update(batch_x=np.stack([s.x for s in batch]), batch_idx=np.stack(idxs), batch_pi=np.stack(pis),
               batch_q=np.array(qs), batch_wdl=np.array(wdls))
    net.train()
    opt = TR.make_optimizer(net, TR.TrainConfig())
    res = TR.train_step(net, opt, batch, "cpu", q_ratio=0.5)
    rec.update(train_policy_loss=res["policy_loss"], train_value_loss=res["value_loss"], train_value_ce=res["value_ce"])
    for k, p in net.named_parameters():
        rec["grad_" + k] = p.grad.detach().numpy().copy()
        rec["after_" + k] = p.detach().numpy().copy()
    rec["norm_mean"], rec["norm_var"] = net.norm.mean.numpy().copy(), net.norm.var.numpy().copy()
    return rec


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ALPHAFLY_REFERENCE")
    if not ref:
        sys.exit("usage: make_golden.py /path/to/reference/checkout")
    sys.path.insert(0, ref)
    install_chess_stand_in()
    import chessfly.brain as brain
    torch.set_num_threads(os.cpu_count() or 1)
    which = sys.argv[2:] or ["tiny", "small", "shuffled", "full", "model"]
    for name in which:
        rec = {"tiny": make_tiny, "small": make_small, "shuffled": make_shuffled, "full": make_full,
               "model": make_model}[name](brain)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **rec)
        print(name, "written:", len(rec), "arrays")


if __name__ == "__main__":
    main()
