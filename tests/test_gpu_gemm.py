"""The training path's float32 products on the tensor cores (afb_gemm_f32 through alphafly_b200.gemm) against
float64: plain and transposed operand layouts, ragged sizes, both bias forms, operands far from 1 in
magnitude, the autograd backward, and configuration 5's layer shapes."""

import pytest
import torch

from alphafly_b200 import gemm

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rel(x, ref):
    return float((x.double() - ref).norm() / ref.norm())


def _rand(*shape, scale=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(*shape, device=DEV, generator=g) * scale


@pytest.mark.parametrize("p,q,k", [(1, 1, 1), (37, 5, 3), (129, 257, 65), (300, 130, 1000), (2048, 4168, 2333),
                                   (17937, 2048, 838)])
def test_gemm_equals_float64(p, q, k):
    x, y = _rand(p, k, seed=p), _rand(q, k, seed=q + 1)
    ref = x.double() @ y.double().T
    got = gemm.gemm(x, y)
    plain = x @ y.T                                     # cuBLAS float32 (TF32 off by default)
    assert got.shape == (p, q)
    assert _rel(got, ref) < 4e-6 and _rel(got, ref) < 8 * _rel(plain, ref) + 1e-7, (_rel(got, ref), _rel(plain, ref))
    assert int(gemm._device_status(DEV)) == 0


@pytest.mark.parametrize("xt,yt", [(0, 1), (1, 0), (1, 1)])
def test_gemm_reads_transposed_operands(xt, yt):
    p, q, k = 300, 200, 517
    xs = _rand(k, p, seed=1) if xt else _rand(p, k, seed=1)
    ys = _rand(k, q, seed=2) if yt else _rand(q, k, seed=2)
    x, y = (xs.T if xt else xs), (ys.T if yt else ys)
    got = gemm.gemm(x, y)
    assert _rel(got, x.double() @ y.double().T) < 4e-6


@pytest.mark.parametrize("bias_dim", [1, 2])
def test_gemm_alpha_beta_and_bias(bias_dim):
    p, q, k = 333, 190, 222
    x, y = _rand(p, k, seed=3), _rand(q, k, seed=4)
    bias = _rand(p if bias_dim == 1 else q, seed=5)
    got = gemm.gemm(x, y, alpha=5.0, bias=bias, bias_dim=bias_dim, beta=-0.5)
    b = bias.double().view(-1, 1) if bias_dim == 1 else bias.double().view(1, -1)
    ref = 5.0 * (x.double() @ y.double().T) - 0.5 * b
    assert _rel(got, ref) < 4e-6


@pytest.mark.parametrize("sx,sy", [(1e-12, 1.0), (1e15, 1e-20), (3e-30, 7e25)])
def test_gemm_scales_operands_of_any_magnitude(sx, sy):
    x, y = _rand(200, 300, scale=sx, seed=6), _rand(150, 300, scale=sy, seed=7)
    ref = x.double() @ y.double().T
    assert _rel(gemm.gemm(x, y), ref) < 4e-6


def test_affine_backward_equals_float64():
    p, q, k = 512, 333, 700
    x = _rand(p, k, scale=0.3, seed=8).requires_grad_(True)
    w = _rand(q, k, seed=9).requires_grad_(True)
    b = _rand(q, seed=10).requires_grad_(True)
    gy = _rand(p, q, seed=11)
    out = gemm.affine(x, w, b, 2, alpha=2.0, beta=3.0)
    gx, gw, gb = torch.autograd.grad((out * gy).sum(), [x, w, b])
    x64, w64, b64 = (t.detach().double().requires_grad_(True) for t in (x, w, b))
    ref = 2.0 * x64 @ w64.T + 3.0 * b64
    rx, rw, rb = torch.autograd.grad((ref * gy.double()).sum(), [x64, w64, b64])
    assert _rel(out, ref.detach()) < 4e-6
    for got, r in ((gx, rx), (gw, rw), (gb, rb)):
        assert _rel(got, r) < 4e-6


def test_affine_per_row_bias_gradient():
    x, y = _rand(64, 50, seed=12).requires_grad_(True), _rand(40, 50, seed=13)
    b = _rand(64, seed=14).requires_grad_(True)
    out = gemm.affine(x, y, b, 1, alpha=5.0, beta=5.0)
    gb, = torch.autograd.grad(out.sum(), [b])
    torch.testing.assert_close(gb, torch.full_like(gb, 5.0 * 40), rtol=1e-6, atol=1e-5)
