"""Data-parallel training over NCCL (configuration 5's scheme) on the GPUs the box has: the gradients
after one data-parallel step over 2 ranks equal the single-process gradients of the concatenated batch.
Skipped when fewer than 2 GPUs are visible.  Launched as child processes (spawn), 127.0.0.1 rendezvous,
NVLS off, a short process-group timeout."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dp_rank(rank, world, port, out, bucketed):
    import torch.distributed as dist
    from conftest import golden
    from alphafly_b200 import synth
    from alphafly_b200.model import FlyChessNet, ModelConfig
    from alphafly_b200.train import Sample, attach_data_parallel, average_gradients, loss_terms, make_batch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    g = golden("model")
    net = FlyChessNet(synth.tiny(60, 600), ModelConfig(steps=3))
    net.load_state_dict({k[len("state_"):]: torch.from_numpy(g[k]) for k in g.files if k.startswith("state_")})
    net = net.cuda().train()
    attach_data_parallel(net, bucket_mb=0.02)    # ~20 KB buckets: several on the tiny network
    n = len(g["batch_x"])
    share = range(rank * n // world, (rank + 1) * n // world)
    batch = [Sample(g["batch_x"][i], g["batch_idx"][i].astype(np.int64), g["batch_pi"][i], float(g["batch_q"][i]),
                    int(g["batch_wdl"][i])) for i in share]
    pl, vl, _ = loss_terms(net, make_batch(batch, "cuda"), 0.5)
    if bucketed:                                  # train_step's path: buckets all-reduced during the backward
        red = net.grad_reducer
        red.arm()
        (pl + vl).backward()
        out[f"in_backward{rank}"] = red.launched_in_backward
        red.finish()
    else:
        (pl + vl).backward()
        average_gradients(net.parameters())
    if rank == 0:
        out["grads"] = {k: p.grad.cpu() for k, p in net.named_parameters()}
        out["mean"], out["var"] = net.norm.mean.cpu(), net.norm.var.cpu()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("bucketed", [False, True], ids=["flat", "bucketed"])
def test_two_rank_gradients_equal_the_concatenated_batch(bucketed):
    from conftest import golden
    with mp.Manager() as m:
        out = m.dict()
        mp.start_processes(_dp_rank, args=(2, _port(), out, bucketed), nprocs=2, start_method="spawn")
        res = dict(out)
    if bucketed:                                  # the heads' and the connectome's buckets left before finish()
        assert res["in_backward0"] >= 2 and res["in_backward1"] == res["in_backward0"], res
    g = golden("model")
    # the RunningNorm statistics equal the single-process statistics of the whole batch
    np.testing.assert_allclose(res["mean"].numpy(), g["norm_mean"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(res["var"].numpy(), g["norm_var"], rtol=1e-4, atol=1e-7)
    # the reference's gradients are clipped to norm 5 (chessfly/train.py:135): apply the same clip
    total = float(np.sqrt(sum(float((gr.double() ** 2).sum()) for gr in res["grads"].values())))
    scale = min(1.0, 5.0 / (total + 1e-6))
    for k, gr in res["grads"].items():
        ref = g["grad_" + k]
        mine = gr.numpy() * scale
        if np.abs(ref).max() > 0:
            assert np.linalg.norm(mine - ref) / np.linalg.norm(ref) < 1e-4, k
