"""Seeded synthetic connectomes and inputs with the shapes of the benchmark configurations.

There is no network here, so the MaleCNS data and trained checkpoints that the reference loads
(chessfly/connectome.py:302-326, chessfly/model.py:154-161) are replaced by graphs drawn from the
distributions below.  Every draw comes from one ``numpy.random.default_rng(seed)`` in a fixed order,
so the same seed gives the same graph on every machine with this numpy.

The reference derives ``w0`` from synapse counts normalised per postsynaptic neuron
(chessfly/connectome.py:231-235, chessfly/brain.py:190).  The synthetic configurations define the
magnitude directly (``log1p(count) / 8`` or ``/ 16``), so an :class:`Instance` carries the
parameter values and :func:`apply` writes them into a freshly built ``ConnectomeRNN`` (this
package's or the reference's: both expose the same buffers and parameters).

Configurations:
  ``small``     N=8,192, E=400,000, no self-loops or duplicates; pre drawn with probability
                proportional to a lognormal(0, 1) popularity, post uniform; sign per pre neuron
                (+1 w.p. 0.7); count = Geometric(0.3) on {1, 2, ...}; w0 = log1p(count)/8; gain 1;
                bias ~ N(0.5, 0.1); alpha = sigmoid(N(0, 1)); inputs 0-1,023, outputs 7,936-8,191.
  ``full``      N=166,700, ~10.5M edges from a configuration model: in- and out-degree
                lognormal(sigma=1) scaled to mean 63 and capped at 5,000, stubs paired by a random
                permutation, self-loops and duplicate pairs dropped; 60% excitatory pre neurons;
                count = Geometric(0.2); w0 = log1p(count)/16; gain ~ U(0.8, 1.2); bias and alpha as
                above; inputs 0-17,936, outputs the last 2,333 neurons.
  ``shuffled``  the small graph with its presynaptic partners permuted (``Connectome.shuffled``,
                seed 1): same in/out degrees and per-neuron signs, duplicates allowed.
  ``tiny``      the fixture graph of the reference's tests (tests/test_core.py:12-19).
"""

from __future__ import annotations

import dataclasses

import numpy as np
import torch

from .connectome import Connectome, neuron_table

N_BASE = 838
N_FEATURES = 967
N_MOVES = 4168
H_MAX = 10.0


@dataclasses.dataclass
class Instance:
    name: str
    conn: Connectome
    in_idx: torch.Tensor        # (I,) int64, sorted
    out_idx: torch.Tensor       # (O,) int64, sorted
    w0: torch.Tensor            # (E,) float32 magnitude, edge order
    log_gain: torch.Tensor      # (E,) float32
    bias: torch.Tensor          # (N,) float32
    alpha_logit: torch.Tensor   # (N,) float32

    @property
    def n(self) -> int:
        return self.conn.n_neurons

    @property
    def e(self) -> int:
        return self.conn.n_edges


def apply(rnn, inst: Instance) -> None:
    """Write the instance's w0 and parameters into a ConnectomeRNN built from ``inst.conn``."""
    with torch.no_grad():
        dev = rnn.w0.device
        rnn.w0.copy_(inst.w0.to(dev, rnn.w0.dtype))
        rnn.log_gain.copy_(inst.log_gain.to(dev, rnn.log_gain.dtype))
        rnn.bias.copy_(inst.bias.to(dev, rnn.bias.dtype))
        rnn.alpha_logit.copy_(inst.alpha_logit.to(dev, rnn.alpha_logit.dtype))


def _finish(name, n, pre, post, rng, p_exc, geom_p, w_div, gain_range, n_in, n_out) -> Instance:
    """Signs, counts, magnitudes and per-neuron parameters, drawn in a fixed order after the edges."""
    key = post.astype(np.int64) * n + pre
    if np.any(key[1:] < key[:-1]):
        order = np.argsort(key, kind="stable")
        pre, post = pre[order], post[order]
    e = len(pre)
    neuron_sign = np.where(rng.random(n) < p_exc, 1.0, -1.0).astype(np.float32)
    count = rng.geometric(geom_p, e).astype(np.float32)
    w0 = (np.log1p(count) / w_div).astype(np.float32)
    if gain_range is None:
        log_gain = np.zeros(e, np.float32)
    else:
        log_gain = np.log(rng.uniform(gain_range[0], gain_range[1], e)).astype(np.float32)
    bias = rng.normal(0.5, 0.1, n).astype(np.float32)
    alpha_logit = rng.normal(0.0, 1.0, n).astype(np.float32)
    in_idx = np.arange(n_in)
    out_idx = np.arange(n - n_out, n)
    conn = Connectome(neuron_table(n, in_idx, out_idx), torch.from_numpy(pre.astype(np.int64)),
                      torch.from_numpy(post.astype(np.int64)), torch.from_numpy(count),
                      torch.from_numpy(neuron_sign[pre]))
    return Instance(name, conn, torch.from_numpy(in_idx), torch.from_numpy(out_idx), torch.from_numpy(w0),
                    torch.from_numpy(log_gain), torch.from_numpy(bias), torch.from_numpy(alpha_logit))


def small(seed: int = 0, n: int = 8192, e: int = 400_000, n_in: int = 1024, n_out: int = 256) -> Instance:
    rng = np.random.default_rng(seed)
    pop = rng.lognormal(0.0, 1.0, n)
    p = pop / pop.sum()
    keys = np.empty(0, np.int64)
    while len(keys) < e:                                  # draw until e distinct non-loop pairs exist
        m = int((e - len(keys)) * 1.25) + 1024
        pre = rng.choice(n, size=m, p=p)
        post = rng.integers(0, n, m)
        k = (post * n + pre)[pre != post]
        keys = np.concatenate([keys, k])
        _, first = np.unique(keys, return_index=True)
        keys = keys[np.sort(first)]                       # distinct, in draw order
    keys = keys[:e]
    return _finish("small", n, keys % n, keys // n, rng, 0.7, 0.3, 8.0, None, n_in, n_out)


def _degrees(rng, n: int, total: int, mean: float, cap: int) -> np.ndarray:
    """Integer degrees ~ lognormal(0, 1) scaled to ``mean``, capped, summing to exactly ``total``."""
    x = rng.lognormal(0.0, 1.0, n)
    d = np.minimum(x / x.mean() * mean, cap)
    d = np.minimum(d * (total / d.sum()), cap)
    base = np.floor(d).astype(np.int64)
    short = total - int(base.sum())
    frac = d - base
    frac[base >= cap] = -1.0                               # never lift a capped neuron above the cap
    base[np.argsort(-frac, kind="stable")[:short]] += 1
    return base


def full(seed: int = 0, n: int = 166_700, mean_degree: float = 63.0, cap: int = 5000,
         n_in: int = 17_937, n_out: int = 2_333) -> Instance:
    rng = np.random.default_rng(seed)
    total = int(round(n * mean_degree))
    k_in = _degrees(rng, n, total, mean_degree, cap)
    k_out = _degrees(rng, n, total, mean_degree, cap)
    post = np.repeat(np.arange(n, dtype=np.int64), k_in)
    pre = np.repeat(np.arange(n, dtype=np.int64), k_out)[rng.permutation(total)]
    keys = np.sort((post * n + pre)[pre != post])
    keys = keys[np.r_[True, keys[1:] != keys[:-1]]]       # drops duplicate pairs; sorted = (post, pre) order
    return _finish("full", n, keys % n, keys // n, rng, 0.6, 0.2, 16.0, (0.8, 1.2), n_in, n_out)


def shuffled(seed: int = 0, shuffle_seed: int = 1) -> Instance:
    """The small graph with its partners permuted: degrees and per-neuron signs kept."""
    base = small(seed)
    s = base.conn.shuffled(shuffle_seed)
    return dataclasses.replace(base, name="shuffled", conn=s)


def tiny(n: int = 30, e: int = 200, seed: int = 0) -> Connectome:
    """The reference test fixture graph (tests/test_core.py:12-19): unique (post, pre) pairs from one
    ``randperm``, 60% excitatory neurons, the first 5 neurons afferent and the last 5 efferent.
    Drawn with torch's CPU generator, so it is the same graph as the reference's fixture."""
    g = torch.Generator().manual_seed(seed)
    pairs = torch.randperm(n * n, generator=g)[:e].sort().values
    post, pre = pairs // n, pairs % n
    nt_sign = torch.where(torch.rand(n, generator=g) < 0.6, 1.0, -1.0)
    neurons = neuron_table(n, np.arange(5), np.arange(n - 5, n))
    return Connectome(neurons, pre, post, torch.randint(1, 20, (e,), generator=g).float(), nt_sign[pre])


def boards(batch: int, seed: int = 0, features: int = N_FEATURES) -> np.ndarray:
    """(batch, features) float32 board-like inputs: each of the 64 squares is occupied with
    probability 24/64 by one of 12 piece planes (index plane*64 + square, ~24 ones), then 70 uniform
    {0, 1} bits (features 768-837).  Features from 838 on (the attack planes) stay zero."""
    rng = np.random.default_rng(seed)
    x = np.zeros((batch, features), np.float32)
    occupied = rng.random((batch, 64)) < 24.0 / 64.0
    plane = rng.integers(0, 12, (batch, 64))
    b, sq = np.nonzero(occupied)
    x[b, plane[b, sq] * 64 + sq] = 1.0
    x[:, 768:N_BASE] = rng.integers(0, 2, (batch, N_BASE - 768))
    return x


def encoder_weights(n_in: int, seed: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """The dense input map: weight (n_in, 967) with the first 838 columns ~ N(0, 0.02) and the attack-plane
    columns zero, bias zero."""
    rng = np.random.default_rng(seed + 1000)
    w = np.zeros((n_in, N_FEATURES), np.float32)
    w[:, :N_BASE] = rng.normal(0.0, 0.02, (n_in, N_BASE))
    return w, np.zeros(n_in, np.float32)


def head_weights(n_out: int, seed: int = 0) -> dict[str, np.ndarray]:
    """Readout weights for parity tests (the reference zero-initialises them, chessfly/model.py:90-93,
    which would make every policy argmax a tie): policy and value ~ N(0, 1/sqrt(O)), biases zero, the
    factorised from/to terms zero as in the reference."""
    rng = np.random.default_rng(seed + 2000)
    s = 1.0 / np.sqrt(n_out)
    return {"policy.weight": rng.normal(0.0, s, (N_MOVES, n_out)).astype(np.float32),
            "policy.bias": np.zeros(N_MOVES, np.float32),
            "value.weight": rng.normal(0.0, s, (3, n_out)).astype(np.float32),
            "value.bias": np.zeros(3, np.float32),
            "policy_from.weight": np.zeros((64, n_out), np.float32), "policy_from.bias": np.zeros(64, np.float32),
            "policy_to.weight": np.zeros((64, n_out), np.float32), "policy_to.bias": np.zeros(64, np.float32)}


def drive(inst: Instance, batch: int, seed: int = 0, input_gain: float = 5.0) -> np.ndarray:
    """u_in (I, batch) float32: the encoder applied to synthetic boards, times the input gain
    (chessfly/model.py:101-102)."""
    x = boards(batch, seed)
    w, b = encoder_weights(len(inst.in_idx), seed)
    enc = x[:, :N_BASE] @ w[:, :N_BASE].T + b
    return np.ascontiguousarray((enc * input_gain).T.astype(np.float32))


def config3_drive(inst: Instance, batch: int, rank: int = 0, block: int = 2048) -> np.ndarray:
    """The benchmark's float16 drive of configuration 3 for ``rank``: ``block`` distinct positions
    (``drive`` with seed 1000 + rank) repeated to ``batch`` columns, (I, batch) float16.  The step kernel's
    gathers do not depend on the values, so the repetition changes no work; column c is position c % block."""
    base = drive(inst, min(batch, block), seed=1000 + rank).astype(np.float16)
    reps = -(-batch // base.shape[1])
    return np.ascontiguousarray(np.tile(base, (1, reps))[:, :batch])


CONFIGS = {"small": small, "full": full, "shuffled": shuffled}
