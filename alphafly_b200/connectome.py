"""The wiring a ConnectomeRNN is built from.

Mirrors the data type of chessfly/connectome.py:215-255 (``Connectome``): edge arrays in
(post, pre) order, which is the CSR order of W[post, pre], a per-edge synapse count and a
per-edge sign that belongs to the presynaptic neuron (Dale's law).  The MaleCNS download
(chessfly/connectome.py:258-326) is not part of this package: graphs come from
``alphafly_b200.synth`` or from a caller that already holds the tensors.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pandas as pd
import torch


@dataclasses.dataclass
class Connectome:
    neurons: pd.DataFrame     # one row per neuron; column "flow" in {afferent, intrinsic, efferent}
    pre: torch.Tensor         # (E,) int64 presynaptic neuron
    post: torch.Tensor        # (E,) int64 postsynaptic neuron; edges sorted by (post, pre)
    syn_count: torch.Tensor   # (E,) float32
    sign: torch.Tensor        # (E,) float32, +1 / -1

    @property
    def n_neurons(self) -> int:
        return len(self.neurons)

    @property
    def n_edges(self) -> int:
        return int(self.pre.numel())

    @property
    def weight(self) -> torch.Tensor:
        """Synapse count over the postsynaptic neuron's total input (chessfly/connectome.py:231-235)."""
        total = torch.zeros(self.n_neurons).index_add_(0, self.post, self.syn_count)
        return self.syn_count / total[self.post].clamp_min(1.0)

    def nodes(self, flow: str) -> torch.Tensor:
        return torch.as_tensor(np.flatnonzero((self.neurons["flow"] == flow).to_numpy()), dtype=torch.long)

    def nodes_of_superclass(self, *names: str) -> torch.Tensor:
        return torch.as_tensor(np.flatnonzero(self.neurons["super_class"].isin(names).to_numpy()), dtype=torch.long)

    def shuffled(self, seed: int = 0) -> "Connectome":
        """Degree-preserving control (chessfly/connectome.py:243-250): the presynaptic partners are
        permuted with torch's CPU generator seeded by ``seed`` (the same draw as the reference, so the
        same graph), the edges are re-sorted into (post, pre) order, and each edge takes the sign of
        its new presynaptic neuron.  Duplicate (post, pre) pairs may appear; CSR consumers sum them."""
        g = torch.Generator().manual_seed(seed)
        pre = self.pre[torch.randperm(self.n_edges, generator=g)]
        order = torch.as_tensor(np.lexsort((pre.numpy(), self.post.numpy())))
        neuron_sign = torch.ones(self.n_neurons).index_put_((self.pre,), self.sign)
        return Connectome(self.neurons, pre[order], self.post[order], self.syn_count[order], neuron_sign[pre[order]])


def neuron_table(n: int, afferent: np.ndarray, efferent: np.ndarray) -> pd.DataFrame:
    """A neuron table with the given afferent (input) and efferent (output) neurons; the rest intrinsic."""
    flow = np.full(n, "intrinsic", dtype=object)
    flow[afferent] = "afferent"
    flow[efferent] = "efferent"
    return pd.DataFrame({"root_id": np.arange(n), "super_class": flow, "cell_type": "", "nt": "", "flow": flow})
