"""Fused LM-head projection + fp32 cross entropy + argmax accuracy.

Reference: ``src/mimir/model/lm_head.py:65-106`` — ``logits = lm_head(h)`` in the compute
dtype, ``F.cross_entropy(logits.float(), labels, ignore_index=-100, reduction='sum')`` and
``argmax(logits) == labels``.

CUDA path: the projection is one tcgen05 GEMM (``ops.gemm``) into a bf16 logits buffer; a row kernel then
computes the row max, first-index argmax and log-sum-exp in fp32 in one read (online
softmax) and emits the per-row loss.  The fp32 ``[T, V]`` logits the reference
materialises never exist.  The backward kernel turns the same buffer into
``g * (softmax - onehot)`` in place (zero on ignored rows) before the two GEMMs.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from mimir_b200.ops import gemm as G
from mimir_b200.ops._ext import ext, kernels_enabled

IGNORE_INDEX = -100


class _LinearCEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, weight, labels):
        C = ext()
        h2 = h.reshape(-1, h.shape[-1])
        w = weight if weight.dtype == h2.dtype else weight.to(h2.dtype)
        logits = G.mm_nt(h2, w) if G.supported(h2, w) else torch.mm(h2, w.t())
        loss_rows, lse, correct = C.ce_fwd(logits, labels.reshape(-1).to(torch.int64).contiguous())
        ctx.save_for_backward(h2, w, logits, lse, labels)
        ctx.weight_dtype = weight.dtype
        ctx.h_shape = h.shape
        ctx.mark_non_differentiable(correct)
        return loss_rows.sum(), correct.view(labels.shape)

    @staticmethod
    def backward(ctx, g, _unused):
        h2, w, logits, lse, labels = ctx.saved_tensors
        C = ext()
        C.ce_bwd_inplace(logits, lse, labels.reshape(-1).to(torch.int64).contiguous(), g.float().reshape(1).contiguous())
        if G.supported(h2, w):
            dh = G.mm_nn(logits, w).view(ctx.h_shape)
            dw = G.weight_grad(w, logits, h2) if ctx.weight_dtype == w.dtype else G.mm_tn(logits, h2).to(ctx.weight_dtype)
        else:
            dh = torch.mm(logits, w).view(ctx.h_shape)
            dw = torch.mm(logits.t(), h2).to(ctx.weight_dtype)
        return dh, dw, None


def linear_cross_entropy_reference(h, weight, labels):
    logits = F.linear(h, weight.to(h.dtype) if weight.dtype != h.dtype else weight)
    loss = F.cross_entropy(logits.reshape(-1, logits.shape[-1]).to(torch.float32), labels.reshape(-1).to(torch.long),
                           ignore_index=IGNORE_INDEX, reduction="sum")
    correct = torch.argmax(logits, dim=-1) == labels
    return loss, correct


def linear_cross_entropy(h: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor):
    """Return ``(sum of fp32 CE over non-ignored tokens, per-token argmax-correct mask)``."""
    if kernels_enabled(h) and h.dtype in (torch.bfloat16,) and weight.shape[0] % 8 == 0:
        return _LinearCEFn.apply(h, weight, labels)
    return linear_cross_entropy_reference(h, weight, labels)
