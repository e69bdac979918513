"""Fused residual-branch mixes (``csrc/branches.cu``) with autograd.

Semantics: :class:`mimir_b200.models.branches.ResidualConnection` (reference
``src/mimir/model/residual_branches.py:27-40``): per channel, softmax over the branch axis of
``alpha * (logits + tanh(streams) * gain)`` in fp32;

* ``branch_read(streams, logits, gain, alpha)``  -> ``sum_b w_b streams_b``            ``[..., d]``
* ``branch_write(streams, update, logits, gain, alpha)`` -> ``streams + B w update``   ``[..., B, d]``

One kernel per direction replaces the eager chain (casts, tanh, softmax, products, sums and
their fp32 ``[..., B, d]`` temporaries).  ``alpha`` (a model buffer) is read on the device and
gets no gradient; ``logits`` / ``gain`` gradients are summed over tokens in a fixed order.
"""
from __future__ import annotations

import torch

from mimir_b200.ops._ext import ext, kernels_enabled


def _flat(streams: torch.Tensor) -> torch.Tensor:
    return streams.reshape(-1, streams.shape[-2], streams.shape[-1])


class _ReadFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, streams, logits, gain, alpha):
        s = _flat(streams)
        ctx.save_for_backward(s, logits, gain, alpha)
        ctx.shape = streams.shape
        return ext().branch_read(s, logits, gain, alpha).view(*streams.shape[:-2], streams.shape[-1])

    @staticmethod
    def backward(ctx, dx):
        s, logits, gain, alpha = ctx.saved_tensors
        ds, _, dl, dg = ext().branch_mix_bwd(dx.contiguous(), s, None, logits, gain, alpha)
        return ds.view(ctx.shape), dl, (dg if gain is not None else None), None


class _WriteFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, streams, update, logits, gain, alpha):
        s = _flat(streams)
        u = update.reshape(-1, update.shape[-1]).contiguous()
        ctx.save_for_backward(s, u, logits, gain, alpha)
        ctx.shapes = (streams.shape, update.shape)
        return ext().branch_write(s, u, logits, gain, alpha).view(streams.shape)

    @staticmethod
    def backward(ctx, do):
        s, u, logits, gain, alpha = ctx.saved_tensors
        ds, du, dl, dg = ext().branch_mix_bwd(do.contiguous(), s, u, logits, gain, alpha)
        return ds.view(ctx.shapes[0]), du.view(ctx.shapes[1]), dl, (dg if gain is not None else None), None


def fused_supported(streams: torch.Tensor, alpha: torch.Tensor) -> bool:
    return (kernels_enabled(streams) and streams.dtype in (torch.bfloat16, torch.float32) and streams.dim() >= 3
            and streams.shape[-2] <= 8 and streams.stride(-1) == 1 and alpha.numel() == 1
            and not alpha.requires_grad)


def _params(logits, gain, alpha):
    return (logits.float().contiguous(), None if gain is None else gain.float().contiguous(),
            alpha.detach().float().reshape(1).contiguous())


def branch_read(streams, logits, gain, alpha):
    return _ReadFn.apply(streams, *_params(logits, gain, alpha))


def branch_write(streams, update, logits, gain, alpha):
    return _WriteFn.apply(streams, update.to(streams.dtype), *_params(logits, gain, alpha))
