"""Float32 products of the training path on the tensor cores (``afb_gemm_f32``).

The reference trains FlyChessNet's encoder and heads as float32 layers (chessfly/model.py:95-105); cuBLAS
runs their products, and the gradients' products, as float32 SIMT GEMMs.  ``affine`` computes

    R (p, q) = alpha X Y^T + beta bias        X (p, k), Y (q, k), bias (p,) per row or (q,) per column

through libafb's split-float16 tensor-core GEMM (float32 accuracy, see include/afb.h) and carries its own
backward, which is two more such products.  Operands may be transposed views: the library reads either
layout, so no transposed copy is made here.
"""

from __future__ import annotations

import torch

from . import _lib

_status: dict = {}


def _device_status(dev: torch.device) -> torch.Tensor:
    st = _status.get(dev)
    if st is None:
        st = _status[dev] = torch.zeros(1, dtype=torch.int32, device=dev)
    return st


def status_word(dev: torch.device) -> torch.Tensor | None:
    """The device status word ``gemm`` passes to the library on ``dev`` (0 = ok; non-zero when a bounded
    wait of the kernel gave up), or None before the first product on that device."""
    return _status.get(dev)


def _operand(t: torch.Tensor) -> tuple[torch.Tensor, int, int]:
    """(tensor, leading dimension, transposed) of a logical (rows, k) float32 matrix as the library reads it."""
    if t.stride(1) == 1 and t.stride(0) >= max(t.shape[1], 1):
        return t, t.stride(0), 0
    if t.stride(0) == 1 and t.stride(1) >= max(t.shape[0], 1):
        return t, t.stride(1), 1
    t = t.contiguous()
    return t, max(t.shape[1], 1), 0


def gemm(x: torch.Tensor, y: torch.Tensor, alpha: float = 1.0, bias: torch.Tensor | None = None, bias_dim: int = 0,
         beta: float = 1.0) -> torch.Tensor:
    """alpha x y^T + beta bias, float32 (p, q), without autograd."""
    p, k = x.shape
    q = y.shape[0]
    if y.shape[1] != k:
        raise ValueError(f"inner dimensions differ: {tuple(x.shape)} and {tuple(y.shape)}^T")
    dev = x.device
    if x.dtype != torch.float32 or y.dtype != torch.float32 or not x.is_cuda or y.device != dev:
        raise TypeError("gemm takes float32 CUDA tensors on one device")
    r = torch.empty(p, q, dtype=torch.float32, device=dev)
    if p == 0 or q == 0:
        return r
    if k == 0:
        r.zero_()
        if bias_dim:
            r.add_(bias.view(-1, 1) if bias_dim == 1 else bias.view(1, -1), alpha=beta)
        return r
    xt, ldx, tx = _operand(x)
    yt, ldy, ty = _operand(y)
    b = None
    if bias_dim:
        b = bias.detach().float().contiguous()
        if b.numel() != (p if bias_dim == 1 else q):
            raise ValueError("bias length does not match")
    lib = _lib.load()
    ws = torch.empty(lib.afb_gemm_workspace(p, q, k), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(lib.afb_gemm_f32(p, q, k, float(alpha), xt.data_ptr(), ldx, tx, yt.data_ptr(), ldy, ty,
                                    b.data_ptr() if b is not None else None, bias_dim, float(beta), r.data_ptr(), q,
                                    ws.data_ptr(), ws.numel(), _device_status(dev).data_ptr(),
                                    torch.cuda.current_stream(dev).cuda_stream))
    return r


class _Affine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, y, bias, bias_dim, alpha, beta):
        ctx.save_for_backward(x if ctx.needs_input_grad[1] else None, y if ctx.needs_input_grad[0] else None)
        ctx.bias_dim, ctx.alpha, ctx.beta = bias_dim, alpha, beta
        return gemm(x.detach(), y.detach(), alpha, bias, bias_dim, beta)

    @staticmethod
    def backward(ctx, g):
        x, y = ctx.saved_tensors
        g_x = g_y = g_b = None
        if ctx.needs_input_grad[0]:                     # alpha g Y        (p, k)
            g_x = gemm(g, y.T, ctx.alpha)
        if ctx.needs_input_grad[1]:                     # alpha g^T X      (q, k)
            g_y = gemm(g.T, x.T, ctx.alpha)
        if ctx.needs_input_grad[2]:
            g_b = g.sum(1 if ctx.bias_dim == 1 else 0)
            if ctx.beta != 1.0:
                g_b = g_b * ctx.beta
        return g_x, g_y, g_b, None, None, None


def affine(x: torch.Tensor, y: torch.Tensor, bias: torch.Tensor | None = None, bias_dim: int = 0, alpha: float = 1.0,
           beta: float = 1.0) -> torch.Tensor:
    """alpha x y^T + beta bias with autograd: x (p, k), y (q, k) float32 on one GPU; bias (p,) with bias_dim 1
    or (q,) with bias_dim 2.  nn.Linear(x) = affine(x, weight, bias, 2)."""
    return _Affine.apply(x, y, bias if bias_dim else None, int(bias_dim), float(alpha), float(beta))
