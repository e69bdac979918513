"""Fused n-gram hash + table gather + validity mask + order sum (CUDA) with scatter-add backward.

Semantics: :class:`mimir_b200.models.ngram.NGramMemory` (reference
``src/mimir/model/ngram_memory.py:52-65``).  One thread block handles a group of tokens;
for each (order, head) it recomputes the polynomial hash of the previous ``order`` tokens,
checks that they are consecutive positions, and accumulates the gathered row.
"""
from __future__ import annotations

import torch

from mimir_b200.ops._ext import ext


class _NGramFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, positions, orders, heads, buckets, dtype, *tables):
        out = ext().ngram_fwd(ids, positions, list(tables), list(orders), heads, buckets, dtype)
        ctx.save_for_backward(ids, positions)
        ctx.info = (orders, heads, buckets, [t.shape for t in tables], [t.dtype for t in tables])
        return out

    @staticmethod
    def backward(ctx, dout):
        ids, positions = ctx.saved_tensors
        orders, heads, buckets, shapes, dtypes = ctx.info
        grads = [torch.zeros(s, dtype=torch.float32, device=dout.device) for s in shapes]
        ext().ngram_bwd(dout.contiguous(), ids, positions, grads, list(orders), heads, buckets)
        grads = [g.to(d) for g, d in zip(grads, dtypes)]
        return (None, None, None, None, None, None, *grads)


def ngram_lookup(ids, positions, tables, orders, heads, buckets, dtype):
    if not hasattr(ext(), "ngram_fwd"):
        raise RuntimeError("n-gram kernel missing from mimir_b200._C")
    return _NGramFn.apply(ids.to(torch.int64).contiguous(), positions.to(torch.int64).contiguous(), tuple(orders),
                          heads, buckets, dtype, *tables)
