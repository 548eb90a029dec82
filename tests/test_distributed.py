"""Data-parallel host logic on CPU with the gloo backend, world size 2 (processes started with spawn):
gradient averaging (flat, and bucketed during the backward), RunningNorm statistics combined exactly over ranks, and a rank that leaves between
steps surfacing as an error on the other rank instead of a hang."""

import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _grads_and_stats(rank, world, port, out):
    _init(rank, world, port)
    from alphafly_b200.train import attach_data_parallel, average_gradients

    class Norm:   # RunningNorm's data-parallel hook only needs the attribute slot
        batch_sync = None

    class Net:
        norm = Norm()

    g = torch.Generator().manual_seed(10 + rank)
    params = [torch.nn.Parameter(torch.zeros(5)), torch.nn.Parameter(torch.zeros(3, 2))]
    for p in params:
        p.grad = torch.randn(p.shape, generator=g)
    local = [p.grad.clone() for p in params]
    average_gradients(params)
    net = Net()
    attach_data_parallel(net)
    r = torch.randn(4 + rank, 7, generator=g)          # unequal shares
    mean, var = net.norm.batch_sync(r)
    out[rank] = {"local": local, "avg": [p.grad.clone() for p in params], "r": r, "mean": mean, "var": var}
    dist.destroy_process_group()


def test_gradient_average_and_exact_batch_statistics():
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.start_processes(_grads_and_stats, args=(2, port, out), nprocs=2, start_method="spawn")
        res = dict(out)
    for k in range(2):
        exp = (res[0]["local"][k] + res[1]["local"][k]) / 2
        torch.testing.assert_close(res[0]["avg"][k], exp)
        torch.testing.assert_close(res[1]["avg"][k], exp)
    r = torch.cat([res[0]["r"], res[1]["r"]])
    for rank in range(2):
        torch.testing.assert_close(res[rank]["mean"], r.mean(0), rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(res[rank]["var"], r.var(0), rtol=1e-5, atol=1e-6)


def _bucketed(rank, world, port, out):
    _init(rank, world, port)
    from alphafly_b200.train import BucketedAllReduce
    torch.manual_seed(0)                                  # the same model on both ranks
    net = torch.nn.Sequential(torch.nn.Linear(6, 40), torch.nn.Tanh(), torch.nn.Linear(40, 30), torch.nn.Tanh(),
                              torch.nn.Linear(30, 2))
    unused = torch.nn.Parameter(torch.zeros(4))           # takes no gradient on any rank
    sometimes = torch.nn.Parameter(torch.ones(3))         # takes a gradient on rank 0 only
    params = [p for m in reversed(net) for p in reversed(list(m.parameters()))] + [sometimes, unused]
    x = torch.randn(8, 6, generator=torch.Generator().manual_seed(20 + rank))
    net(x).square().sum().backward()
    local = [p.grad.clone() for p in params[:-2]]
    for p in params[:-2]:
        p.grad = None
    red = BucketedAllReduce(params, bucket_mb=0.003)        # ~3 KB: several buckets
    red.arm()
    loss = net(x).square().sum()
    if rank == 0:
        loss = loss + (sometimes * torch.arange(3.0)).sum()
    loss.backward()
    in_backward = red.launched_in_backward
    red.finish()
    out[rank] = {"local": local, "avg": [p.grad.clone() for p in params[:-2]], "unused": unused.grad,
                 "sometimes": sometimes.grad, "buckets": len(red.buckets), "in_backward": in_backward}
    dist.destroy_process_group()


def test_bucketed_all_reduce_overlaps_the_backward_and_averages():
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.start_processes(_bucketed, args=(2, port, out), nprocs=2, start_method="spawn")
        res = dict(out)
    for rank in range(2):
        r = res[rank]
        assert r["buckets"] >= 3 and r["in_backward"] >= r["buckets"] - 1, r   # all but the unused one
        assert r["unused"] is None
        # a gradient present on one rank only: both ranks step it with the mean (zeros for the other rank)
        torch.testing.assert_close(r["sometimes"], torch.arange(3.0) / 2)
        for k, g in enumerate(r["avg"]):
            torch.testing.assert_close(g, (res[0]["local"][k] + res[1]["local"][k]) / 2)


def test_gradient_order_covers_every_parameter_once():
    from alphafly_b200 import synth
    from alphafly_b200.model import FlyChessNet, ModelConfig
    from alphafly_b200.train import gradient_order
    net = FlyChessNet(synth.tiny(60, 600), ModelConfig(steps=3))
    order = gradient_order(net)
    assert len(order) == len(list(net.parameters()))
    assert {id(p) for p in order} == {id(p) for p in net.parameters()}
    assert order[-1] is net.encoder.bias or order[-1] is net.encoder.weight


def _leaver(rank, world, port, out):
    _init(rank, world, port, timeout_s=5)
    t = torch.ones(3)
    dist.all_reduce(t)                                  # a completed step
    if rank == 1:
        out[rank] = "left"
        os._exit(0)                                     # leaves between steps, nothing in flight
    try:
        dist.all_reduce(t)
        out[rank] = "completed"
    except Exception as e:                              # gloo reports the lost peer / timeout
        out[rank] = "error: " + type(e).__name__
    os._exit(0)


def test_a_rank_leaving_between_steps_is_reported_not_hung():
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        ctx = mp.start_processes(_leaver, args=(2, port, out), nprocs=2, start_method="spawn", join=False)
        deadline = time.time() + 60
        while any(p.is_alive() for p in ctx.processes) and time.time() < deadline:
            time.sleep(0.2)
        for p in ctx.processes:
            if p.is_alive():
                p.kill()
        res = dict(out)
    assert res.get(1) == "left"
    assert str(res.get(0, "")).startswith("error"), res
