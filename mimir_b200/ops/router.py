"""MoE router logits ``x.float() @ w.float().T + b`` with fp32 results on the tensor cores.

The reference scores experts in fp32 (``src/mimir/model/expert_mixtures.py``: ``F.linear`` of the
fp32-cast hidden state and router rows), which on a GPU is a SIMT fp32 GEMM: about a third of a
millisecond per layer for 16384 tokens x 2048 x 64 experts, forward, and twice that backward.
When the hidden state and the router rows are bf16 (the compute dtype), every product of the fp32
GEMM is a product of two bf16 numbers, which is exact in fp32, so the tcgen05 bf16 GEMM with fp32
accumulation and fp32 output (``csrc/gemm.cu``) computes the same sums (in another order).

Backward: the logits' gradient is fp32, so it is split into two bf16 terms ``hi + lo`` (16
significant bits together) placed side by side as a ``[T, 2n]`` operand; the input gradient is
one GEMM against the rows stacked twice, the row gradient one GEMM whose two halves are added in
fp32, and the bias gradient a column sum.

Anything else (CPU, fp32 weights, an expert count that is not a multiple of 32) runs the
reference's fp32 ``F.linear``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from mimir_b200.ops._ext import ext, kernels_enabled


class _RouterLogitsFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b):
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous() or x2.data_ptr() % 16:
            x2 = x2.contiguous()
        n = w.shape[0]
        s = torch.empty(x2.shape[0], n, dtype=torch.float32, device=x.device)
        if x2.shape[0]:
            ext().gemm(x2, False, w, False, s)
        s += b.float()
        ctx.save_for_backward(x2, w)
        ctx.x_shape = x.shape
        ctx.b_dtype = b.dtype
        return s.view(*x.shape[:-1], n)

    @staticmethod
    def backward(ctx, ds):
        x2, w = ctx.saved_tensors
        n = w.shape[0]
        ds2 = ds.reshape(-1, n).float()
        hi = ds2.to(torch.bfloat16)
        split = torch.cat([hi, (ds2 - hi.float()).to(torch.bfloat16)], dim=1)  # [T, 2n]: hi | lo
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = ext().gemm(split, False, torch.cat([w, w], dim=0), True).view(ctx.x_shape)
        if ctx.needs_input_grad[1]:
            both = torch.empty(2 * n, x2.shape[1], dtype=torch.float32, device=x2.device)
            ext().gemm(split, True, x2, True, both)
            dw = (both[:n] + both[n:]).to(w.dtype)
        db = ds2.sum(0).to(ctx.b_dtype) if ctx.needs_input_grad[2] else None
        return dx, dw, db


def tensor_core_path(x: torch.Tensor, w: torch.Tensor) -> bool:
    return (kernels_enabled(x) and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and w.dim() == 2
            and w.shape[0] % 32 == 0 and w.shape[1] % 8 == 0 and w.shape[1] == x.shape[-1] and w.is_contiguous()
            and w.data_ptr() % 16 == 0)


def router_logits(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """fp32 ``x @ w^T + b`` for the router rows ``w`` [n, d] and biases ``b`` [n]."""
    if tensor_core_path(x, w):
        return _RouterLogitsFn.apply(x, w, b)
    return F.linear(x.float(), w.float(), b.float())
