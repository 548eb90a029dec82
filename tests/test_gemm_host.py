"""Host side of the training products (alphafly_b200/gemm.py) on CPU: how an operand view is handed to
afb_gemm_f32 (leading dimension and transposed flag, without a copy where the library can read the view),
and the training heads' selection-matrix form of the reference's from/to gathers (chessfly/model.py:104)."""

import torch

from alphafly_b200 import synth
from alphafly_b200.gemm import _operand
from alphafly_b200.model import FlyChessNet, ModelConfig


def _element(t, ld, trans, i, k):
    """Element (i, k) of the logical matrix as the library addresses it in t's storage."""
    flat = t.as_strided((t.untyped_storage().nbytes() // t.element_size(),), (1,), 0)
    at = t.storage_offset() + (k * ld + i if trans else i * ld + k)
    return flat[at]


def test_operand_reads_row_major_and_transposed_views_in_place():
    base = torch.arange(7 * 11, dtype=torch.float32).reshape(7, 11)
    cases = [base, base[:, :5], base[2:, 3:9], base.T, base[:, :5].T, base[1:6, 2:10].T]
    for v in cases:
        t, ld, trans = _operand(v)
        assert t.data_ptr() == v.data_ptr()                       # no copy
        for i in range(v.shape[0]):
            for k in range(v.shape[1]):
                assert float(_element(t, ld, trans, i, k)) == float(v[i, k])


def test_operand_copies_what_the_library_cannot_read():
    base = torch.arange(8 * 9, dtype=torch.float32).reshape(8, 9)
    v = base[::2, ::3]                                            # neither dimension contiguous
    t, ld, trans = _operand(v)
    assert trans == 0 and t.is_contiguous() and torch.equal(t, v) and ld == v.shape[1]


def test_selection_matrix_heads_equal_the_gathered_from_to_terms():
    net = FlyChessNet(synth.tiny(60, 600), ModelConfig(steps=3))
    g = torch.Generator().manual_seed(3)
    for m in (net.policy, net.policy_from, net.policy_to, net.value):
        m.weight.data.normal_(0, 0.1, generator=g)
        m.bias.data.normal_(0, 0.1, generator=g)
    sel = net.move_select
    assert sel.shape == (128, len(net.move_from)) and torch.equal(sel.sum(0), torch.full((sel.shape[1],), 2.0))
    r = torch.randn(23, len(net.out_idx), generator=g, requires_grad=True)
    logits, _ = net.dense_heads(r)
    ref = net.policy(r) + net.policy_from(r)[:, net.move_from] + net.policy_to(r)[:, net.move_to]
    torch.testing.assert_close(logits, ref, rtol=1e-6, atol=1e-6)
    w = torch.randn(logits.shape, generator=g)
    got = torch.autograd.grad((logits * w).sum(), [r, net.policy_from.weight, net.policy_to.bias])
    want = torch.autograd.grad((ref * w).sum(), [r, net.policy_from.weight, net.policy_to.bias])
    for a, b in zip(got, want):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)
