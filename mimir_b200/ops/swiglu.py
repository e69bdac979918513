"""SwiGLU activation on a packed ``[gate | up]`` projection: ``silu(gate) * up``.

Reference: ``src/mimir/model/layers.py:270-271``.  The CUDA kernel reads the packed
projection once and writes the product (bf16); the backward recomputes ``silu`` from the
saved projection and writes ``[dgate | dup]`` in one pass.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from mimir_b200.ops._ext import ext, kernels_enabled


class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        gu2 = gu.reshape(-1, gu.shape[-1]).contiguous()
        out = ext().swiglu_fwd(gu2)
        ctx.save_for_backward(gu2)
        ctx.shape = gu.shape
        return out.view(*gu.shape[:-1], gu.shape[-1] // 2)

    @staticmethod
    def backward(ctx, dp):
        (gu2,) = ctx.saved_tensors
        dgu = ext().swiglu_bwd(dp.reshape(gu2.shape[0], gu2.shape[1] // 2).contiguous(), gu2)
        return dgu.view(ctx.shape)


def swiglu_reference(gu: torch.Tensor) -> torch.Tensor:
    gate, up = gu.chunk(2, dim=-1)
    return F.silu(gate) * up


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    if kernels_enabled(gu) and gu.dtype in (torch.bfloat16, torch.float32) and gu.shape[-1] % 16 == 0:
        return _SwiGLUFn.apply(gu)
    return swiglu_reference(gu)
