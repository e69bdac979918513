"""Scaled token embedding ``scale * E[ids]`` (reference ``src/mimir/model/layers.py:103-104``).

CUDA: one fused gather-and-scale kernel (``csrc/embedding.cu``) forward; backward sorts the token
ids stably and sums each id's rows in fp32 in position order (deterministic, no atomics), adding
``scale * sum`` to the weight's gradient.  When the replicated engine owns the gradient (a view
of its flat buffer, announced by ``_mimir_grad_sink``) the rows are added in place; otherwise a
zero gradient of the weight's dtype is allocated.  CPU and fp16 weights use the PyTorch
formulation, which is also the numerical oracle.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from mimir_b200.ops._ext import ext, kernels_enabled


class _ScaledEmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, weight, scale):
        ctx.save_for_backward(ids)
        ctx.weight = weight
        ctx.scale = scale
        return ext().embed_fwd(ids, weight, scale)

    @staticmethod
    def backward(ctx, dout):
        (ids,) = ctx.saved_tensors
        w = ctx.weight
        if not ctx.needs_input_grad[1]:
            return None, None, None
        sorted_ids, order = torch.sort(ids.reshape(-1).to(torch.int64), stable=True)
        sink = getattr(w, "_mimir_grad_sink", None)
        target = w.grad if sink is not None and w.grad is not None and w.grad.is_contiguous() else None
        fresh = target is None
        if fresh:
            target = torch.zeros_like(w)
        ext().embed_bwd(dout.reshape(-1, w.shape[1]).contiguous(), sorted_ids, order, target, ctx.scale)
        if not fresh:
            sink(w)
            return None, None, None
        return None, target, None


def scaled_embedding(ids: torch.Tensor, weight: torch.Tensor, scale: float) -> torch.Tensor:
    if (kernels_enabled(weight) and weight.dtype in (torch.bfloat16, torch.float32) and weight.dim() == 2
            and weight.shape[1] % 8 == 0 and weight.is_contiguous()):
        return _ScaledEmbeddingFn.apply(ids, weight, float(scale))
    return scale * F.embedding(ids, weight)
