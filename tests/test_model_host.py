"""The model layer's host-side contract (chessfly/model.py): checkpoint keys identical to the reference's,
load_weights' tolerance for old checkpoints, move squares.  No GPU needed (construction only)."""

import numpy as np
import pytest
import torch

from conftest import golden
from alphafly_b200 import synth
from alphafly_b200.encoding import N_BASE, N_FEATURES, N_MOVES, move_squares
from alphafly_b200.model import FlyChessNet, ModelConfig, load_weights


def test_state_dict_keys_and_shapes_match_the_reference():
    g = golden("model")
    ref = {k[len("state_"):]: g[k].shape for k in g.files if k.startswith("state_")}
    net = FlyChessNet(synth.tiny(60, 600), ModelConfig(steps=3))
    mine = {k: tuple(v.shape) for k, v in net.state_dict().items()}
    assert mine == {k: tuple(v) for k, v in ref.items()}


def test_constants_and_move_squares():
    assert (N_BASE, N_FEATURES, N_MOVES) == (838, 967, 4168)
    frm, to = move_squares()
    assert frm.shape == to.shape == (N_MOVES,)
    assert frm[64 * 12 + 28] == 12 and to[64 * 12 + 28] == 28
    assert frm[4096] == 48 and to[4096] == 56 and to[4096 + 3] == 56 and to[4096 + 6] == 57
    assert frm.max() < 64 and to.max() < 64


def test_load_weights_accepts_old_checkpoints_and_rejects_incomplete_ones():
    """tests/test_core.py:394-471: missing factorised heads load; a narrower encoder is zero-padded; a
    genuinely missing tensor is an error."""
    net = FlyChessNet(synth.tiny(60, 600), ModelConfig(steps=3))
    old = {k: v.clone() for k, v in net.state_dict().items() if not k.startswith(("policy_from.", "policy_to."))}
    old["encoder.weight"] = old["encoder.weight"][:, :N_BASE].clone()
    load_weights(net, old)
    assert float(net.encoder.weight[:, N_BASE:].abs().sum()) == 0
    with pytest.raises(RuntimeError, match="does not match"):
        load_weights(net, {k: v for k, v in old.items() if k != "value.bias"})


def test_deepcopy_drops_native_handles_and_copies_parameters():
    """ShardedEvaluator replicates the network with copy.deepcopy: the cached light cone (a native handle)
    is not copied, parameters and buffers are (new storage, same values)."""
    import copy
    net = FlyChessNet(synth.tiny(60, 600), ModelConfig(steps=3))
    net.brain._cone = ("key", object())
    c = copy.deepcopy(net)
    assert c.brain._cone is None and net.brain._cone is not None
    for (k, a), (_, b) in zip(net.state_dict().items(), c.state_dict().items()):
        assert torch.equal(a, b) and (a.numel() == 0 or a.data_ptr() != b.data_ptr()), k


def test_grow_optimizer_state_pads_the_encoder_moments():
    """tests/test_core.py:451-471 (the optimizer part): Adam moments saved for an 838-column encoder are
    padded with zero columns to the 967-column encoder, and the state loads."""
    from alphafly_b200.train import TrainConfig, grow_optimizer_state, make_optimizer
    fresh = FlyChessNet(synth.tiny(60, 600), ModelConfig(steps=3, attack_planes=True))
    opt = make_optimizer(fresh, TrainConfig())
    params = [p for g in opt.param_groups for p in g["params"]]
    i = next(k for k, p in enumerate(params) if p is fresh.encoder.weight)
    old_shape = (fresh.encoder.weight.shape[0], N_BASE)
    state = {"state": {i: {"step": torch.tensor(5.0), "exp_avg": torch.ones(old_shape), "exp_avg_sq": torch.ones(old_shape)}},
             "param_groups": opt.state_dict()["param_groups"]}
    grown = grow_optimizer_state(state, opt)
    st = grown["state"][i]
    assert st["exp_avg"].shape == fresh.encoder.weight.shape and st["exp_avg_sq"].shape == fresh.encoder.weight.shape
    assert float(st["exp_avg"][:, N_BASE:].abs().sum()) == 0 and float(st["exp_avg"][:, :N_BASE].sum()) == old_shape[0] * N_BASE
    opt.load_state_dict(grown)
