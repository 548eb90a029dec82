"""afb_cone_forward_noalloc, the forward for callers that cannot allocate device memory at evaluation
time (their memory belongs to another framework's pool, or their serving loop cannot take the implicit
synchronisation of cudaMalloc): it must give the same output as afb_cone_forward with a workspace, on
consecutive calls that reuse its built-in 32 MiB scratch, and refuse batches whose state does not fit.

Collected last on purpose, so that a run stopping at its first failure has run every other test."""

import ctypes

import pytest
import torch

from oracle import oracle as orc
from alphafly_b200 import _lib, synth
from alphafly_b200.brain import ConnectomeRNN

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SCRATCH = 32 << 20


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.fixture(scope="module")
def cone_and_inputs():
    inst = synth.small()
    rnn = ConnectomeRNN(inst.conn)
    synth.apply(rnn, inst)
    rnn = rnn.to(DEV)
    in_idx, out_idx = inst.in_idx.to(DEV), inst.out_idx.to(DEV)
    u = torch.from_numpy(synth.drive(inst, 300, seed=21)).to(DEV)
    with torch.no_grad():                                  # builds the cone and sets the weights of both modes
        ref32 = rnn.forward_io(u, in_idx, out_idx, 6)
        ref16 = rnn.forward_io(u.half(), in_idx, out_idx, 6)
    return rnn.light_cone(in_idx, out_idx, 6), u, {_lib.MODE_F32: ref32, _lib.MODE_DEV16: ref16}


def noalloc(cone, mode, u):
    out = torch.full((cone.n_out, u.shape[1]), float("nan"), device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(_lib.load().afb_cone_forward_noalloc(cone._h, mode, _ptr(u), u.stride(0), u.shape[1], _ptr(out),
                                                    out.stride(0), stream))
    return out


@pytest.mark.parametrize("mode", [_lib.MODE_F32, _lib.MODE_DEV16])
def test_noalloc_forward_matches_the_workspace_forward_twice(cone_and_inputs, mode):
    cone, u, refs = cone_and_inputs
    x = u if mode == _lib.MODE_F32 else u.half()
    assert _lib.load().afb_cone_forward_workspace(cone._h, mode, x.shape[1]) <= SCRATCH
    with torch.no_grad():
        first = noalloc(cone, mode, x)
        second = noalloc(cone, mode, x)                   # the scratch keeps the last call's contents
        workspace = cone.forward(mode, x)                 # afb_cone_forward with a torch-allocated workspace
    torch.cuda.synchronize()
    ref = refs[mode].cpu().numpy()
    for out in (first, second):
        assert torch.isfinite(out).all()
        assert orc.rel_l2(out.cpu().numpy(), workspace.cpu().numpy()) < 1e-6
        assert orc.rel_l2(out.cpu().numpy(), ref) < 1e-6
    assert cone.status() == 0


def test_noalloc_forward_refuses_a_batch_beyond_its_scratch(cone_and_inputs):
    cone, u, _ = cone_and_inputs
    lib = _lib.load()
    big = 4096
    assert lib.afb_cone_forward_workspace(cone._h, _lib.MODE_F32, big) > SCRATCH
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.afb_cone_forward_noalloc(cone._h, _lib.MODE_F32, _ptr(u), big, big, _ptr(u), big, stream)
    assert rc == _lib.EINVAL
    assert b"built-in scratch" in lib.afb_last_error()


def test_noalloc_forward_allocates_nothing(cone_and_inputs):
    """Warm calls change neither the device's free memory (no cudaMalloc behind the caller's back) nor
    torch's allocator statistics."""
    cone, u, _ = cone_and_inputs
    x = u.half()
    out = torch.empty(cone.n_out, x.shape[1], device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    lib = _lib.load()
    _lib.check(lib.afb_cone_forward_noalloc(cone._h, _lib.MODE_DEV16, _ptr(x), x.stride(0), x.shape[1], _ptr(out),
                                            out.stride(0), stream))
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    stats_before = torch.cuda.memory_stats()
    for _ in range(5):
        _lib.check(lib.afb_cone_forward_noalloc(cone._h, _lib.MODE_DEV16, _ptr(x), x.stride(0), x.shape[1], _ptr(out),
                                                out.stride(0), stream))
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    stats_after = torch.cuda.memory_stats()
    assert free_after == free_before
    for key in ("allocation.all.allocated", "segment.all.allocated", "allocated_bytes.all.current"):
        assert stats_after.get(key) == stats_before.get(key), key


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_noalloc_forward_on_a_second_device_and_device_checks():
    """A cone on cuda:1 runs against cuda:1's copy of the scratch; called with another device current, or
    with another device's stream, it is refused before any launch."""
    inst = synth.small()
    rnn = ConnectomeRNN(inst.conn)
    synth.apply(rnn, inst)
    dev1 = torch.device("cuda", 1)
    rnn = rnn.to(dev1)
    in_idx, out_idx = inst.in_idx.to(dev1), inst.out_idx.to(dev1)
    u = torch.from_numpy(synth.drive(inst, 200, seed=5)).to(dev1).half()
    lib = _lib.load()
    with torch.no_grad(), torch.cuda.device(dev1):
        ref = rnn.forward_io(u, in_idx, out_idx, 6)
        cone = rnn.light_cone(in_idx, out_idx, 6)
        out = torch.full((cone.n_out, u.shape[1]), float("nan"), device=dev1)
        s1 = ctypes.c_void_p(torch.cuda.current_stream(dev1).cuda_stream)
        _lib.check(lib.afb_cone_forward_noalloc(cone._h, _lib.MODE_DEV16, _ptr(u), u.stride(0), u.shape[1], _ptr(out),
                                                out.stride(0), s1))
        torch.cuda.synchronize(dev1)
        assert orc.rel_l2(out.cpu().numpy(), ref.cpu().numpy()) < 1e-6
        other = torch.cuda.Stream(device=torch.device("cuda", 0))          # a created stream: the legacy default
        s0 = ctypes.c_void_p(other.cuda_stream)                            # stream's handle names no device
        rc = lib.afb_cone_forward_noalloc(cone._h, _lib.MODE_DEV16, _ptr(u), u.stride(0), u.shape[1], _ptr(out),
                                          out.stride(0), s0)
        assert rc == _lib.EINVAL and b"stream belongs to device 0" in lib.afb_last_error()
    with torch.cuda.device(0):
        rc = lib.afb_cone_forward_noalloc(cone._h, _lib.MODE_DEV16, _ptr(u), u.stride(0), u.shape[1], _ptr(out),
                                          out.stride(0), s1)
        assert rc == _lib.EINVAL and b"is not the cone's device" in lib.afb_last_error()
