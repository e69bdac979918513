"""A list of equally shaped parameters used as one stacked matrix, without a copy when possible.

The MoE router keeps one parameter per expert row and per bias (the checkpoint layout of the
reference, ``src/mimir/model/expert_mixtures.py``), and ``torch.stack`` of them costs a copy in
the forward and one gradient-accumulation kernel (plus one hook) per parameter in the backward:
thousands of tiny launches per step for a 64-expert, 16-layer model.  Under the replicated engine
the parameters are consecutive, equally strided views of one flat weight buffer and their
gradients views of one flat gradient buffer (announced through ``_mimir_grad_sink``).  Then
:func:`stacked` copies the strided weights once (as ``torch.stack`` would), and the backward adds
the stacked gradient into the gradient buffer with one kernel and announces every parameter,
with the values ``torch.stack``'s per-parameter accumulations would give.  Otherwise it is
``torch.stack``.
"""
from __future__ import annotations

import torch


def _strided_view(tensors: list) -> torch.Tensor | None:
    """``[len(tensors), *shape]`` view over the storage of equally strided, same-shape tensors."""
    first = tensors[0]
    if not first.is_contiguous() or any(t.shape != first.shape or t.dtype != first.dtype or not t.is_contiguous()
                                        or t.untyped_storage().data_ptr() != first.untyped_storage().data_ptr()
                                        for t in tensors):
        return None
    if len(tensors) == 1:
        return first.unsqueeze(0)
    step = tensors[1].storage_offset() - first.storage_offset()
    if step < first.numel() or any(t.storage_offset() != first.storage_offset() + i * step
                                   for i, t in enumerate(tensors)):
        return None
    return first.as_strided((len(tensors), *first.shape), (step, *first.stride()), first.storage_offset())


class _StackedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, weight_view, grad_view, *params):
        ctx.grad_view = grad_view
        ctx.params = params
        return weight_view.clone()

    @staticmethod
    def backward(ctx, grad):
        ctx.grad_view.add_(grad.to(ctx.grad_view.dtype))
        for p in ctx.params:  # announced after the kernel that writes them is enqueued
            p._mimir_grad_sink(p)
        return (None, None) + (None,) * len(ctx.params)


def stacked(params) -> torch.Tensor:
    params = list(params)
    grads = [p.grad for p in params]
    if (all(getattr(p, "_mimir_grad_sink", None) is not None and p.requires_grad for p in params)
            and all(g is not None for g in grads)):
        weights, grad_view = _strided_view([p.detach() for p in params]), _strided_view(grads)
        if weights is not None and grad_view is not None and torch.is_grad_enabled():
            return _StackedFn.apply(weights, grad_view, *params)
    return torch.stack(params)
