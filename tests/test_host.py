"""Host-side behaviour of the drop-in module that needs no GPU: constructor, buffers, parameters,
checkpoint keys, module globals, and the refusal of CPU tensors (there is no CPU path)."""

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from alphafly_b200 import brain, synth
from alphafly_b200.brain import ConnectomeRNN


@pytest.mark.parametrize("graph", ["tiny", "small"])
def test_wiring_buffers_match_the_reference_layout(graph):
    conn = synth.tiny(120, 700, seed=3) if graph == "tiny" else synth.small().conn
    rnn = ConnectomeRNN(conn, global_scale=3.0)
    pre, post = conn.pre.numpy(), conn.post.numpy()
    np.testing.assert_array_equal(rnn.crow.numpy(), orc.crow_of(post, conn.n_neurons))
    order = orc.transpose_order(post, pre, conn.n_neurons)
    np.testing.assert_array_equal(rnn.t_order.numpy(), order)
    np.testing.assert_array_equal(rnn.t_crow.numpy(), orc.crow_of(pre[order], conn.n_neurons))
    np.testing.assert_array_equal(rnn.t_col.numpy(), post[order])
    torch.testing.assert_close(rnn.w0, conn.weight * 3.0)
    assert rnn.log_gain.shape == (conn.n_edges,) and float(rnn.log_gain.abs().sum()) == 0


def test_parameters_and_checkpoint_keys_are_the_references():
    rnn = ConnectomeRNN(synth.tiny(), alpha_init=0.3, bias_init=0.2)
    assert set(rnn.state_dict()) == {"log_gain", "bias", "alpha_logit"}     # wiring buffers are non-persistent
    torch.testing.assert_close(torch.sigmoid(rnn.alpha_logit), torch.full((30,), 0.3))
    torch.testing.assert_close(rnn.bias, torch.full((30,), 0.2))
    assert rnn.h_max == 10.0


def test_module_globals_exist():
    assert brain.FUSED_UPDATE is not None and brain.FUSED_DEVIATION is not None
    assert brain.SAMPLED_ADDMM is True and brain.SDDMM_COLS == 64 and brain.CHUNK_ELEMS == 1 << 26


def test_cpu_tensors_are_rejected():
    rnn = ConnectomeRNN(synth.tiny())
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        rnn.forward_io(torch.zeros(5, 2), torch.arange(5), torch.arange(25, 30), 2)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        with torch.no_grad():
            rnn(torch.zeros(30, 2), 2)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        rnn.light_cone(torch.arange(5), torch.arange(25, 30), 2)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        rnn.edge_weights()


def test_shapes_are_checked_before_any_device_work():
    """A drive whose rows do not match in_idx (or the neuron count) is refused with ValueError, as the
    reference's own indexing would refuse it (chessfly/brain.py:214, 271-275)."""
    rnn = ConnectomeRNN(synth.tiny())
    with pytest.raises(ValueError, match="len\\(in_idx\\)"):
        rnn.forward_io(torch.zeros(4, 2), torch.arange(5), torch.arange(25, 30), 2)
    with pytest.raises(ValueError, match="len\\(in_idx\\)"):
        rnn.forward_io(torch.zeros(5), torch.arange(5), torch.arange(25, 30), 2)
    with pytest.raises(ValueError, match="\\(N, B\\)"):
        with torch.no_grad():
            rnn(torch.zeros(29, 2), 2)


def test_bench_algorithmic_bytes():
    import bench
    per_step, total = bench.algorithmic_bytes([0, 3, 4], [0, 0, 10], [0, 3, 0], batch=8, n_out=2)
    # step 1: no matrix, 3 rows all fed; step 2: 10 edges, 4 rows
    assert per_step[0] == 4 * 4 + 8 * 2 * (0 + 3 + 3) + 10 * 3
    assert per_step[1] == 10 * 6 + 4 * 5 + 8 * 2 * (3 + 4 + 0) + 10 * 4
    assert total == sum(per_step) + 2 * 8 * 4
