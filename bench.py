"""Benchmark of the connectome recurrence on B200: 6-step light-cone forward, float16 deviation.

    python bench.py [--gpus N --steps K --warmup W] [--batch B] [--impl ours|reference]

Workload (configuration 3): the full-scale synthetic connectome (166,700 neurons, ~10.5M synapses;
``alphafly_b200.synth.full``), inputs = 17,937 sensory neurons, outputs = 2,333, 6 steps, light-cone
pruned, float16 deviation from the float32 resting trajectory, B = 35,840 positions per GPU.
A "step" is one ``ConnectomeRNN.forward_io`` over the batch.  With N GPUs (torchrun, one process
per GPU) every rank evaluates its own 35,840 positions with the wiring replicated: no collective on
the data path, weak scaling.  ``value`` = positions evaluated by all ranks / max-over-ranks device
time of the K timed steps (inputs resident in HBM); ``e2e`` = the same through the public call with
the drive in pinned host memory and the output copied back inside the timed region.

``--impl reference`` times the reference's CPU implementation of the path (its torch CPU sparse forward_io,
restated with the same calls in oracle/torch_port.py, all host threads) on 256-position samples of the
same workload and prints the same line.
``--train`` times configuration 5 instead (FlyChessNet train_step, B = 2,048 per GPU, data parallel over
NCCL under torchrun); ``--probe`` prints the device's gather ceiling against warps per SM; ``--evaluator``
times self-play evaluation rounds (B = 1,120 positions) through three implementations of the Evaluator.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "connectome evals/sec (6-step fwd) at 1/2/4/8 B200; % of HBM roofline"
UNIT = "positions/s"
STEPS_T = 6


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=None,
                    help="positions per GPU (default 35,840; 2,048 with --train; 1,120 per round with --evaluator)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--train", action="store_true",
                    help="time the training step instead (configuration 5: FlyChessNet train_step, B = 2,048 per GPU)")
    ap.add_argument("--probe", action="store_true", help="print the gather ceiling of the step kernel's load path and exit")
    ap.add_argument("--configs", action="store_true",
                    help="time configurations 1, 2 and 4 (the other workloads of the scope; one JSON line each)")
    ap.add_argument("--evaluator", action="store_true",
                    help="time the self-play Evaluator (FlyChessNet rounds of --batch positions, 30 legal moves each)")
    ap.add_argument("--inmap", action="store_true",
                    help="time the float16 input map (tcgen05 kernel) against cuBLAS on the same operands")
    args = ap.parse_args()
    if args.batch is None:
        args.batch = 2048 if args.train else 1120 if args.evaluator else 35_840
    return args


def peaks():
    path = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError, TypeError):
        return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16 (= float16) tensor throughput in TFLOP/s: the burst figure of MEASURED_PEAKS.json, else the
    earlier measurement on this pool."""
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, ValueError, KeyError, TypeError):
        return 1590.0, "fallback"


def measured_traffic():
    """Per-launch DRAM bytes of the step kernel from the committed ncu capture (profiles/), or None."""
    path = os.path.join(HERE, "profiles", "step_kernel_traffic_config3.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("bytes_per_launch"):
            return int(line.split("=")[1])
    return None


def gather_ceiling(dev, slab_rows, n_rows=1 << 25, reps=5, blocks_per_sm=0):
    """Device ceiling of the step kernel's dominant access: n_rows random 512-byte rows of a slab of
    ``slab_rows`` rows gathered by the probe kernel of libafb_probe.so (include/afb_probe.h: 16-byte loads into
    registers, 8 rows in flight per lane, ``blocks_per_sm`` CTAs of 8 warps per SM, 0 = 8); GB/s (median of
    reps)."""
    from alphafly_b200 import _lib
    lib = _lib.load_probe()
    g = torch.Generator(device=dev).manual_seed(5)
    slab = torch.randint(0, 1 << 30, (slab_rows, 128), dtype=torch.int32, device=dev, generator=g)
    rows = torch.randint(0, slab_rows, (n_rows,), dtype=torch.int32, device=dev, generator=g)
    words = lib.afb_probe_gather_sink_words()
    if words < 0:
        raise RuntimeError("afb_probe_gather_sink_words failed")
    sink = torch.empty(words, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    args = (blocks_per_sm, slab.data_ptr(), slab_rows, rows.data_ptr(), n_rows, sink.data_ptr(), words, stream.cuda_stream)
    times = []
    for k in range(3 + reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        rc = lib.afb_probe_gather(*args)
        if rc != 0:
            raise RuntimeError(f"afb_probe_gather failed with code {rc}")
        b.record(stream)
        b.synchronize()
        if k >= 3:
            times.append(a.elapsed_time(b))
    return n_rows * 512 / (statistics.median(times) / 1000.0) / 1e9


def workload(seed=0):
    from alphafly_b200 import synth
    return synth.full(seed)


def algorithmic_bytes(rows_len, nnz, n_fed, batch, n_out, s_state=2, s_val=2, s_idx=4, row_const=10):
    """Compulsory HBM bytes of one 6-step forward of ``batch`` positions: per step t the sub-matrix
    (nnz_t (index + value) + row pointer), the gathered state R_{t-1} x B read once, the new state R_t x B
    written once, the fed input rows U_t x B read once, the per-row constants; plus the float32 output."""
    per_step = []
    for t in range(1, len(rows_len)):
        b = nnz[t] * (s_idx + s_val) + 4 * (rows_len[t] + 1) + batch * s_state * (rows_len[t - 1] + rows_len[t] + n_fed[t]) \
            + row_const * rows_len[t]
        per_step.append(b)
    return per_step, sum(per_step) + n_out * batch * 4


class Clocks:
    """nvidia-smi samples of the SM clock and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            for k, name in enumerate(names):
                if len(r) > 5 + k and r[5 + k].lower().startswith("active"):
                    reasons.add(name)
        loaded = sorted(sm)[len(sm) // 2:] if sm else []
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


def init_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    return rank, world, local


CPU_BATCH = 256


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def torch_cpu_forward(inst):
    """The reference's CPU path for configuration 3's graph: its torch CPU sparse forward_io, restated with the
    same torch calls in oracle/torch_port.py (the reference's own source does not travel to the GPU box), on
    every host thread."""
    from oracle.torch_port import TorchCpuForward
    torch.set_num_threads(host_threads())
    return TorchCpuForward(inst.n, inst.conn.pre.numpy(), inst.conn.post.numpy(), inst.conn.sign.numpy(),
                           inst.w0.numpy(), inst.log_gain.numpy(), inst.bias.numpy(), inst.alpha_logit.numpy(),
                           inst.in_idx.numpy(), inst.out_idx.numpy(), STEPS_T)


def cpu_sample(inst, seconds, batch=CPU_BATCH):
    """The reference's CPU forward (torch CPU sparse, all host threads) on ``batch`` positions of the bench's
    drive, repeated for about ``seconds``; and, beside it, the oracle's C/OpenMP float32 port on the same
    positions for a third of the time.  Returns the cpu_baseline object."""
    from alphafly_b200 import synth
    from oracle import oracle as orc
    u = synth.config3_drive(inst, batch).astype(np.float32)

    def rate(fn, budget):
        fn(u)                                                 # warm-up
        reps, t0 = 0, time.perf_counter()
        while True:
            fn(u)
            reps += 1
            el = time.perf_counter() - t0
            if el >= budget:
                return reps * batch / el, reps, el

    ref = torch_cpu_forward(inst)
    v, reps, el = rate(ref, seconds)
    port = orc.CpuForward(inst.n, inst.conn.pre.numpy(), inst.conn.post.numpy(), inst.conn.sign.numpy(), inst.w0.numpy(),
                          inst.log_gain.numpy(), inst.bias.numpy(), inst.alpha_logit.numpy(), inst.in_idx.numpy(),
                          inst.out_idx.numpy(), STEPS_T, cone=ref.cone)
    v_port, _, _ = rate(port, seconds / 3)
    return {"value": v, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{reps} x {batch} positions of the bench drive of configuration 3, float32 light-cone forward_io "
                      f"through torch CPU sparse CSR (the reference's CPU path, restated in oracle/torch_port.py), {el:.1f} s",
            "c_openmp_port": {"value": v_port, "unit": UNIT, "threads": orc.lib().ref_num_threads(),
                              "what": "oracle/csr_ref.c fused float32 step (OpenMP), same positions"}}


def reference_arm(args, rank, world):
    """The reference's CPU implementation of the path (torch CPU sparse forward_io, oracle/torch_port.py) on
    the host cores: one step = one forward of CPU_BATCH positions of the bench drive.  Rank 0 only."""
    if rank != 0:
        return
    from alphafly_b200 import synth
    inst = workload()
    fwd = torch_cpu_forward(inst)
    u = synth.config3_drive(inst, CPU_BATCH).astype(np.float32)
    for _ in range(args.warmup):
        fwd(u)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fwd(u)
    el = time.perf_counter() - t0
    value = args.steps * CPU_BATCH / el
    threads = torch.get_num_threads()
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * el / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config3: full-scale synthetic connectome, 6-step light-cone forward",
                       "batch_per_step": CPU_BATCH,
                       "note": "each step is a bounded sample of the GPU arm's 35,840-position batch"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{CPU_BATCH} positions per step, float32, the reference's torch CPU sparse "
                                       "forward_io restated with the same torch calls (oracle/torch_port.py)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def probe_arm(args):
    """Gather ceiling of the step kernel's load path (include/afb_probe.h) on configuration 3's widest slab,
    against warps per SM, then against the slab's size."""
    dev = torch.device("cuda", 0)
    rows = 166_688
    for bps in (2, 3, 4, 5, 6, 8):
        print(json.dumps({"probe": "ldg 16 B per lane, 8 rows in flight", "warps_per_sm": 8 * bps, "slab_rows": rows,
                          "gbs": round(gather_ceiling(dev, rows, blocks_per_sm=bps), 1)}), flush=True)
    # the slab against the L2: 12 MB .. 164 MB at the step kernel's 40 warps per SM and at 64
    for sr in (24_000, 48_000, 72_000, 96_000, 120_000, 144_000, 166_688, 200_000, 240_000, 320_000):
        print(json.dumps({"probe": "ldg 16 B per lane, 8 rows in flight", "slab_rows": sr, "slab_mb": round(sr * 512 / 1e6, 1),
                          "gbs_40_warps": round(gather_ceiling(dev, sr, blocks_per_sm=5), 1),
                          "gbs_64_warps": round(gather_ceiling(dev, sr, blocks_per_sm=8), 1)}), flush=True)


def inmap_arm(args):
    """The float16 input map alone: afb_input_map_f16 (tcgen05 + TMA) against torch's cuBLAS addmm on the
    same float16 operands, u = 5 (W x^T + b) for 17,937 sensory neurons from 838 board features, at the
    Evaluator's round (1,120 positions) and up to configuration 3's batch.  L2 is flushed (a 256 MB write)
    before every timed launch; each launch is timed alone with CUDA events on the launching stream."""
    from alphafly_b200 import _lib
    from alphafly_b200.model import input_map_f16
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n_in, k, gain = 17_937, 838, 5.0
    g = torch.Generator().manual_seed(5)
    w16 = torch.zeros(n_in, 840, dtype=torch.float16, device=dev)[:, :k]
    w16.copy_(torch.randn(n_in, k, generator=g) * 0.05)
    b16 = (torch.randn(n_in, generator=g) * 0.3).half().to(dev)
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    peak, peak_kind = tensor_peak()
    stream = torch.cuda.current_stream(dev)

    def timed(fn, reps):
        total = 0.0
        for _ in range(reps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            b.synchronize()
            total += a.elapsed_time(b)
        return total / reps

    for batch in sorted({1120, 8192, args.batch}):
        x = torch.zeros(batch, 840, dtype=torch.float16, device=dev)[:, :k]
        x.copy_((torch.rand(batch, k, generator=g) < 0.06).half())
        out = {}
        fns = {"tcgen05": lambda: out.__setitem__("ours", input_map_f16(w16, b16, x, gain, status)),
               "cublas": lambda: out.__setitem__("cublas", torch.addmm(b16.unsqueeze(1), w16, x.T, beta=gain, alpha=gain))}
        for fn in fns.values():
            for _ in range(args.warmup):
                fn()
        ms = {name: timed(fn, max(args.steps, 3)) for name, fn in fns.items()}
        torch.cuda.synchronize(dev)
        _lib.check(0 if int(status.item()) == 0 else _lib.ECUDA)
        flops = 2.0 * n_in * k * batch
        diff = float((out["ours"].float() - out["cublas"].float()).abs().max())
        print(json.dumps({"kernel": "input_map_kernel (tcgen05.mma 128x256x16 f16->f32, TMA SWIZZLE_128B)",
                          "workload": f"drive of {n_in} sensory neurons from {k} features", "batch": batch,
                          "ms": round(ms["tcgen05"], 4), "tflops": round(flops / ms["tcgen05"] / 1e9, 1),
                          "frac": round(flops / ms["tcgen05"] / 1e9 / peak, 3), "peak_tflops": peak, "peak": peak_kind,
                          "cublas_ms": round(ms["cublas"], 4), "cublas_tflops": round(flops / ms["cublas"] / 1e9, 1),
                          "max_abs_diff_vs_cublas": diff, "l2": "flushed before every launch"}), flush=True)


def train_batch(inst, batch, seed):
    """Configuration 5's synthetic batch: boards, policy targets softmax(N(0, 1)) over 30 random legal moves of
    the 4,168, WDL one-hots drawn 0.45 / 0.10 / 0.45, q uniform in [-1, 1]; as pinned host tensors in the
    order of ``alphafly_b200.train.Batch`` (x, moves, probs, valid, wdl, q)."""
    from alphafly_b200 import synth
    from alphafly_b200.encoding import N_MOVES
    rng = np.random.default_rng(seed)
    x = synth.boards(batch, seed)
    moves = np.stack([rng.choice(N_MOVES, size=30, replace=False) for _ in range(batch)]).astype(np.int64)
    z = np.exp(rng.standard_normal((batch, 30)))
    probs = (z / z.sum(1, keepdims=True)).astype(np.float32)
    valid = np.ones((batch, 30), bool)
    wdl = rng.choice(3, size=batch, p=[0.45, 0.10, 0.45])
    q = rng.uniform(-1, 1, batch).astype(np.float32)
    return tuple(torch.from_numpy(a).pin_memory() for a in (x, moves, probs, valid, wdl, q))


def train_arm(args, rank, world, local):
    """Configuration 5: one FlyChessNet train_step (forward through the light cone, backward, gradient clip,
    AdamW; with N GPUs the gradients are averaged over NCCL) per step on B positions per GPU."""
    from alphafly_b200 import synth
    from alphafly_b200.model import FlyChessNet, ModelConfig
    from alphafly_b200.train import Batch, TrainConfig, attach_data_parallel, make_optimizer, train_step
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    inst = workload()
    net = FlyChessNet(inst.conn, ModelConfig(steps=STEPS_T))
    synth.apply(net.brain, inst)
    w, b = synth.encoder_weights(len(inst.in_idx))
    with torch.no_grad():
        net.encoder.weight.copy_(torch.from_numpy(w))
        net.encoder.bias.copy_(torch.from_numpy(b))
        for k, v in synth.head_weights(len(inst.out_idx)).items():
            dict(net.named_parameters())[k].copy_(torch.from_numpy(v))
    net = net.to(dev).train()
    if world > 1:
        attach_data_parallel(net)
    opt = make_optimizer(net, TrainConfig())
    host = train_batch(inst, args.batch, seed=77 + rank)
    stream = torch.cuda.current_stream(dev)

    def step():
        batch = Batch(*(t.to(dev, non_blocking=True) for t in host))    # the batch arrives from pinned host memory
        return train_step(net, opt, batch, dev, q_ratio=0.5, data_parallel=world > 1)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            res = step()
        stop.record(stream)
        barrier()
    ms = start.elapsed_time(stop)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    value = world * args.batch * args.steps / (ms / 1000.0)
    if rank == 0:
        h2d = sum(a.numel() * a.element_size() for a in host)
        print(json.dumps({"metric": "connectome training positions/sec (6-step light-cone forward + backward + AdamW)",
                          "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "f32", "data": "synthetic",
                          "config": {"workload": "config5: FlyChessNet train_step on the full-scale synthetic connectome",
                                     "positions_per_gpu": args.batch, "global_positions": args.batch * world,
                                     "parallelism": f"data parallel over {world} GPU(s), NCCL gradient all-reduce"},
                          "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 12,
                                  "note": "the timed steps include the batch copy from pinned memory and the loss read-back"},
                          "last_losses": res, "clocks": clocks.summary()}), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def configs_arm(args):
    """The other configurations of the workload, one JSON line each, device time per forward (CUDA events,
    median of ``--steps`` after ``--warmup``):
      1  small synthetic graph (8,192 neurons, 400k synapses), float32 light-cone forward, B = 64;
      2  full-scale graph, float32 literal recurrence over all 166,700 neurons (no pruning), B = 1,120;
      4  shuffled control of configuration 1, float16 deviation, B = 1, 64, 1,120, 8,192, 65,536."""
    from alphafly_b200 import synth
    from alphafly_b200.brain import ConnectomeRNN
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        with torch.no_grad():
            for _ in range(args.warmup):
                fn()
            times = []
            for _ in range(args.steps):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                fn()
                b.record(stream)
                b.synchronize()
                times.append(a.elapsed_time(b))
        return statistics.median(times)

    def line(config, workload, batch, ms, dtype):
        print(json.dumps({"metric": "connectome evals/sec (6-step fwd)", "config": config, "workload": workload,
                          "batch": batch, "dtype": dtype, "ms_per_forward": round(ms, 4),
                          "value": round(batch / (ms / 1000.0), 1), "unit": UNIT, "steps": args.steps,
                          "warmup": args.warmup}), flush=True)

    for name, inst in (("1", synth.small()), ("4", synth.shuffled())):
        rnn = ConnectomeRNN(inst.conn)
        synth.apply(rnn, inst)
        rnn = rnn.to(dev)
        in_idx, out_idx = inst.in_idx.to(dev), inst.out_idx.to(dev)
        batches = (64,) if name == "1" else (1, 64, 1120, 8192, 65536)
        for batch in batches:
            u = torch.from_numpy(synth.drive(inst, min(batch, 2048), seed=7)).repeat(1, (batch + 2047) // 2048)[:, :batch]
            u = u.contiguous().to(dev)
            if name == "4":
                u = u.half()
            ms = timed(lambda: rnn.forward_io(u, in_idx, out_idx, STEPS_T))
            line(name, "small synthetic, float32 light cone" if name == "1" else "shuffled control, float16 deviation",
                 batch, ms, "f32" if name == "1" else "f16")
        del rnn
    inst = workload()
    rnn = ConnectomeRNN(inst.conn)
    synth.apply(rnn, inst)
    rnn = rnn.to(dev)
    u4 = torch.from_numpy(synth.drive(inst, 1120, seed=3))
    full_u = torch.zeros(inst.n, 1120).index_copy_(0, inst.in_idx, u4).to(dev)
    ms = timed(lambda: rnn(full_u, STEPS_T))
    line("2", "full-scale graph, float32 literal recurrence (all neurons, no pruning)", 1120, ms, "f32")


def evaluator_arm(args):
    """Self-play evaluation rounds (chessfly/workers.py:118-167): B positions per round with 30 legal moves
    each, one round in flight while the next is submitted.  Three implementations of the same contract:
    the reference's eager Evaluator logic (dense logits, gather, blocking copies), and this package's
    Evaluator without and with CUDA graphs (pinned staging, fused legal-move logits)."""
    from alphafly_b200 import synth
    from alphafly_b200.model import Evaluator, FlyChessNet, ModelConfig
    dev = torch.device("cuda", 0)
    inst = workload()
    net = FlyChessNet(inst.conn, ModelConfig(steps=STEPS_T))
    synth.apply(net.brain, inst)
    w, b = synth.encoder_weights(len(inst.in_idx))
    with torch.no_grad():
        net.encoder.weight.copy_(torch.from_numpy(w))
        net.encoder.bias.copy_(torch.from_numpy(b))
        params = dict(net.named_parameters())
        for k, v in synth.head_weights(len(inst.out_idx)).items():
            params[k].copy_(torch.from_numpy(v))
    net = net.to(dev).eval()
    rng = np.random.default_rng(5)
    B = args.batch
    rounds = []
    for k in range(4):
        x = synth.boards(B, 100 + k).astype(np.float16)
        rows = np.repeat(np.arange(B), 30)
        cols = np.concatenate([rng.choice(4168, 30, replace=False) for _ in range(B)])
        rounds.append((x, rows, cols))

    class Eager:                                  # chessfly/model.py:120-132, eager
        @torch.no_grad()
        def submit(self, x, rows, cols):
            logits, wdl = net.dense_heads(net.readout(torch.from_numpy(x).to(dev, non_blocking=True).float()))
            legal = logits[torch.from_numpy(rows).to(dev, non_blocking=True), torch.from_numpy(cols).to(dev, non_blocking=True)]
            return legal.float(), net.expected_value(wdl.float())

        @staticmethod
        def result(h):
            return h[0].cpu().numpy(), h[1].float().cpu().numpy()

    out = {}
    arms = [("reference_eager", Eager()), ("evaluator", Evaluator(net, dev, graphs=False)),
            ("evaluator_graphs", Evaluator(net, dev, graphs=True))]
    if args.gpus > 1:                             # one process, the round split over the visible GPUs
        from alphafly_b200.model import ShardedEvaluator
        arms.append((f"sharded_{args.gpus}_gpus", ShardedEvaluator(net, [f"cuda:{k}" for k in range(args.gpus)])))
    for name, ev in arms:
        def play(n):
            inflight = None
            for k in range(n):
                h = ev.submit(*rounds[k % len(rounds)])
                if inflight is not None:
                    ev.result(inflight)
                inflight = h
            ev.result(inflight)
        play(args.warmup + 1)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        play(args.steps)
        torch.cuda.synchronize(dev)
        el = time.perf_counter() - t0
        out[name] = {"positions_per_s": round(B * args.steps / el, 1), "ms_per_round": round(1000 * el / args.steps, 3)}
    print(json.dumps({"metric": "self-play evaluator positions/sec (FlyChessNet rounds, legal-move logits + values)",
                      "unit": UNIT, "positions_per_round": B, "legal_moves_per_position": 30, "rounds": args.steps,
                      "warmup": args.warmup, "timing": "host wall clock around whole rounds (submit .. result), "
                      "one round in flight", "results": out}), flush=True)


def main():
    args = parse()
    rank, world, local = init_dist(args)
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    if args.probe:
        return probe_arm(args)
    if args.inmap:
        return inmap_arm(args)
    if args.train:
        return train_arm(args, rank, world, local)
    if args.evaluator:
        return evaluator_arm(args)
    if args.configs:
        return configs_arm(args)
    from alphafly_b200 import synth
    from alphafly_b200.brain import ConnectomeRNN
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    inst = workload()
    rnn = ConnectomeRNN(inst.conn)
    synth.apply(rnn, inst)
    rnn = rnn.to(dev)
    in_idx, out_idx = inst.in_idx.to(dev), inst.out_idx.to(dev)
    B = args.batch
    # this rank's shard of positions: its own seed (2,048 distinct positions repeated to B columns)
    u_host = torch.from_numpy(synth.config3_drive(inst, B, rank))
    u = u_host.to(dev)
    cone = rnn.light_cone(in_idx, out_idx, STEPS_T)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        if world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    with torch.no_grad():
        for _ in range(args.warmup):
            out = rnn.forward_io(u, in_idx, out_idx, STEPS_T)
        barrier()
        # per-launch events on the launching stream: T step kernels + the output kernel, every timed step
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(STEPS_T + 2)] for _ in range(args.steps)]
        for row in ev:
            for e in row:
                e.record(stream)                               # creates the handles
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        with Clocks(local) as clocks:
            start.record(stream)
            for k in range(args.steps):
                out = cone.forward(1, u, events=ev[k])         # == rnn.forward_io(u16, ...) with the cache warm
            stop.record(stream)
            barrier()
        dev_ms = start.elapsed_time(stop)
        step_ms = [[ev[k][t].elapsed_time(ev[k][t + 1]) for t in range(STEPS_T + 1)] for k in range(args.steps)]
    ms = max_over_ranks(dev_ms)
    value = world * B * args.steps / (ms / 1000.0)

    # roofline of the step kernel: algorithmic bytes / its measured duration
    hbm, peak_kind = peaks()
    fed = [0] + [len(x) for x in cone.u_pos[1:]]
    per_step_bytes, total_bytes = algorithmic_bytes(cone.rows_len, cone.nnz, fed, B, len(inst.out_idx))
    kernel_ms = [sum(s[t] for s in step_ms) / args.steps for t in range(STEPS_T)]
    kernel_total_ms = sum(kernel_ms)
    achieved = sum(per_step_bytes) / (kernel_total_ms / 1000.0) / 1e9
    gathered = sum(cone.nnz) * B * 2                          # state bytes the SpMM pulls through L2 per forward
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4), "peak_kind": peak_kind,
                "traffic": measured_traffic() if B == 35_840 else None,
                "traffic_source": "profiles/step_kernel_traffic_config3.txt: ncu DRAM bytes of the 6 step launches at "
                                  "B = 2,048 (8 batch tiles), scaled by 17.5 to the 140 tiles of B = 35,840; per launch",
                "kernel": "step_kernel<__half,__half> (steps 3-6), step_kernel_pair<__half,__half> (step 2) and "
                          "step_kernel_nosyn<__half> (step 1): 6 launches per forward",
                "algorithmic_bytes_per_launch": int(sum(per_step_bytes) / STEPS_T),
                "launch_ms": [round(x, 3) for x in kernel_ms],
                "l2_gather_bytes_per_forward": int(gathered),
                "l2_gather_gbs": round(gathered / (kernel_total_ms / 1000.0) / 1e9, 1)}
    # the other ceiling of the sparse path: one FMA per synapse and position (float16 weight x float16 state into
    # a float32 sum), against the device's FP32 FMA issue rate at the SM clock sampled during the timed region
    clk = clocks.summary()
    sm_mhz = clk.get("sm_mhz") or clk.get("sm_max_mhz") or 1965.0
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    fma_rate = sms * 128 * sm_mhz * 1e6
    fmas = sum(cone.nnz) * B
    roofline.update({"fma_per_forward": int(fmas), "fma_gfma_s": round(fmas / (kernel_total_ms / 1000.0) / 1e9, 1),
                     "fma_pipe_frac": round(fmas / (kernel_total_ms / 1000.0) / fma_rate, 4),
                     "fma_rate_source": f"{sms} SMs x 128 FP32 FMA lanes per SM per clock x {sm_mhz:.0f} MHz "
                                        "(median SM clock sampled during the timed region)"})
    # the same 512-byte-row gather alone, over a slab as large as the widest step's state tile
    ceiling = gather_ceiling(dev, max(cone.rows_len))
    roofline.update({"l2_gather_ceiling_gbs": round(ceiling, 1),
                     "l2_gather_frac": round(roofline["l2_gather_gbs"] / ceiling, 4),
                     "l2_gather_ceiling_source": "afb_probe_gather: 2^25 uniform random rows of a "
                                                 f"{max(cone.rows_len):,} x 512 B slab, measured in this run"})

    # the weight-version precompute (brain.py:238-252, 296-306): edge weights, resting trajectory, sub-matrix
    # values and row constants, as after every training phase; events on the launching stream
    with torch.no_grad():
        w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for k in range(3):
            if k == 2:
                w0.record(stream)
            cone.set_weight_tensors(1, rnn.edge_weights(), rnn.bias, rnn.alpha_logit, rnn.h_max)
        w1.record(stream)
        torch.cuda.synchronize(dev)
        weight_version_ms = w0.elapsed_time(w1)

    e2e = None
    if not args.no_e2e:
        # Through the public call with host buffers: each step copies its drive from pinned host memory and
        # its output back, on a copy stream double-buffered against the compute stream (the reference's
        # self-play pipelines its GPU rounds the same way, chessfly/workers.py:121-124,162-164).
        pin_u = u_host.pin_memory()
        pin_out = [torch.empty(len(inst.out_idx), B, dtype=torch.float32).pin_memory() for _ in range(2)]
        u_dev = [torch.empty_like(u), torch.empty_like(u)]
        copy = torch.cuda.Stream(dev)
        h2d_done = [torch.cuda.Event() for _ in range(2)]
        out_ready = [torch.cuda.Event() for _ in range(2)]
        d2h_done = [torch.cuda.Event() for _ in range(2)]

        def run(k_steps):
            outs = [None, None]
            with torch.cuda.stream(copy):
                u_dev[0].copy_(pin_u, non_blocking=True)
                h2d_done[0].record(copy)
            for k in range(k_steps):
                i = k % 2
                if k + 1 < k_steps:                       # prefetch the next step's drive
                    with torch.cuda.stream(copy):
                        if k >= 1:
                            copy.wait_event(out_ready[(k + 1) % 2])   # its buffer's previous forward is done
                        u_dev[(k + 1) % 2].copy_(pin_u, non_blocking=True)
                        h2d_done[(k + 1) % 2].record(copy)
                stream.wait_event(h2d_done[i])
                if k >= 2:
                    stream.wait_event(d2h_done[i])        # the pinned output buffer is free again
                outs[i] = rnn.forward_io(u_dev[i], in_idx, out_idx, STEPS_T)
                out_ready[i].record(stream)
                with torch.cuda.stream(copy):
                    copy.wait_event(out_ready[i])
                    pin_out[i].copy_(outs[i], non_blocking=True)
                    d2h_done[i].record(copy)
            copy.synchronize()

        with torch.no_grad():
            run(2)
            barrier()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            run(args.steps)
            s1.record(copy)
            barrier()
        e2e_ms = max_over_ranks(s0.elapsed_time(s1))
        e2e = {"value": world * B * args.steps / (e2e_ms / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": pin_u.numel() * pin_u.element_size(),
               "d2h_bytes_per_step": pin_out[0].numel() * pin_out[0].element_size(),
               "ms_per_step": e2e_ms / args.steps, "pipelined": "copy stream, double-buffered"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_sample(inst, args.cpu_seconds)

    if world > 1:
        torch.distributed.barrier()
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16", "data": "synthetic",
                "config": {"workload": "config3: full-scale synthetic connectome (166,700 neurons, "
                                       f"{inst.e:,} synapses), 6-step light-cone forward, float16 deviation",
                           "positions_per_gpu": B, "global_positions": B * world, "l2": "inputs larger than L2",
                           "parallelism": f"positions sharded over {world} GPU(s), wiring replicated, no collective"},
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
                "gpu_launches": args.steps * (STEPS_T + 1),
                "weight_version_ms": round(weight_version_ms, 3),
                "light_cone": {"rows": cone.rows_len, "nnz": cone.nnz, "edge_visits": cone.edge_visits}}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
