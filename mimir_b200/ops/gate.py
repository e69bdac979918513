"""Invocation gate ``injection * (1 + alpha * tanh(W [hidden; injection] + b))`` on the GPU.

Semantics: :class:`mimir_b200.models.mimir2.InvocationGate` (reference
``src/mimir/model/mimir2.py:135-141``).  The projection runs on the tcgen05 dense GEMM
(:func:`mimir_b200.ops.gemm.linear`, forward and both gradients); bias, tanh and the gating run
in one fused kernel (``csrc/gate.cu``) whose backward returns the projection's gradient, the
injection's gradient and the bias gradient (a fixed-order sum over token tiles).  ``alpha`` is a
model buffer, read on the device, without gradient.
"""
from __future__ import annotations

import torch

from mimir_b200.ops import gemm as G
from mimir_b200.ops._ext import ext, kernels_enabled


class _GateFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pre, injection, bias, alpha):
        ctx.save_for_backward(pre, injection, bias, alpha)
        return ext().invocation_gate_fwd(pre, injection, bias, alpha)

    @staticmethod
    def backward(ctx, dout):
        pre, injection, bias, alpha = ctx.saved_tensors
        dpre, dinj, dbias = ext().invocation_gate_bwd(dout.contiguous(), pre, injection, bias, alpha)
        return dpre, dinj, dbias, None


def supported(hidden: torch.Tensor, injection: torch.Tensor, alpha: torch.Tensor) -> bool:
    return (kernels_enabled(hidden) and hidden.dtype in (torch.bfloat16, torch.float32)
            and injection.dtype == hidden.dtype and alpha.numel() == 1 and not alpha.requires_grad)


def invocation_gate(hidden, injection, weight, bias, alpha):
    hidden, injection = torch.broadcast_tensors(hidden, injection)
    shape = injection.shape
    x = torch.cat((hidden, injection), dim=-1).reshape(-1, 2 * shape[-1])
    pre = G.linear(x, weight.to(x.dtype)).reshape(-1, shape[-1]).contiguous()
    inj = injection.reshape(-1, shape[-1]).contiguous()
    out = _GateFn.apply(pre, inj, bias.float(), alpha.detach().float().reshape(1).contiguous())
    return out.view(shape)
