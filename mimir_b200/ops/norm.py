"""Weightless RMSNorm: ``y = x * rsqrt(mean(x^2) + eps)`` over the last dim.

Reference: ``F.rms_norm(x, (d,), eps)`` at ``src/mimir/model/transformer.py:96,225``.
CUDA: one warp per row, fp32 statistics, bf16/fp32 I/O; backward reuses the saved
per-row ``rstd``: ``dx = rstd * (dy - y * mean(dy * y))``.

:func:`add_rms_norm` fuses the pre-norm residual add that precedes a norm: ``h = x + delta``
(rounded to the tensor dtype exactly as the separate add stores it) and ``rmsnorm(h)`` in one
pass; its backward adds the residual stream's gradient inside the norm backward, so neither
direction launches a separate elementwise add.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from mimir_b200.ops._ext import ext, kernels_enabled


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, eps):
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        y, rstd = ext().rmsnorm_fwd(x2, float(eps))
        ctx.save_for_backward(x2, rstd)
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, rstd = ctx.saved_tensors
        dx = ext().rmsnorm_bwd(dy.reshape(x2.shape).contiguous(), x2, rstd)
        return dx.view(dy.shape), None


def rms_norm(x: torch.Tensor, eps: float) -> torch.Tensor:
    if kernels_enabled(x) and x.dtype in (torch.bfloat16, torch.float32) and x.shape[-1] % 8 == 0:
        return _RMSNormFn.apply(x, eps)
    return F.rms_norm(x, (x.shape[-1],), eps=eps)


class _AddRMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, delta, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        d2 = delta.reshape(-1, shape[-1]).contiguous()
        h, y, rstd = ext().add_rmsnorm_fwd(x2, d2, float(eps))
        ctx.save_for_backward(h, rstd)
        return h.view(shape), y.view(shape)

    @staticmethod
    def backward(ctx, dh, dy):
        h, rstd = ctx.saved_tensors
        dy2 = dy.reshape(h.shape).contiguous() if dy is not None else torch.zeros_like(h)
        if dh is None:
            dx = ext().rmsnorm_bwd(dy2, h, rstd)
        else:
            dx = ext().rmsnorm_bwd_res(dy2, h, rstd, dh.reshape(h.shape).contiguous())
        dx = dx.view(dy.shape if dy is not None else dh.shape)
        return dx, dx, None


def add_rms_norm(x: torch.Tensor, delta: torch.Tensor, eps: float):
    """``(h, rmsnorm(h))`` with ``h = x + delta``."""
    if (kernels_enabled(x) and x.dtype in (torch.bfloat16, torch.float32) and delta.dtype == x.dtype
            and delta.shape == x.shape and x.shape[-1] % 8 == 0):
        return _AddRMSNormFn.apply(x, delta, eps)
    h = x + delta
    return h, rms_norm(h, eps)
