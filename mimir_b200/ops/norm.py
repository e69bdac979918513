"""Weightless RMSNorm: ``y = x * rsqrt(mean(x^2) + eps)`` over the last dim.

Reference: ``F.rms_norm(x, (d,), eps)`` at ``src/mimir/model/transformer.py:96,225``.
CUDA: one warp per row, fp32 statistics, bf16/fp32 I/O; backward reuses the saved
per-row ``rstd``: ``dx = rstd * (dy - y * mean(dy * y))``.
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
