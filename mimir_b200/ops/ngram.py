"""Fused n-gram hash + table gather + validity mask + order sum (CUDA) and its sparse backward.

Semantics: :class:`mimir_b200.models.ngram.NGramMemory` (reference
``src/mimir/model/ngram_memory.py:52-65``).  Forward: one warp per token recomputes, for each
(order, head), the polynomial hash of the previous ``order`` tokens, checks that they are
consecutive positions, and accumulates the gathered row.

Backward: a key per (token, order, head) names the table row it read; after a stable sort, one
warp per run of equal keys sums the run's output-gradient slices in fp32 and adds the sum to that
row once.  Deterministic, and only hashed rows are touched: when the replicated engine owns the
tables' gradients (views into its flat buffer, announced by ``_mimir_grad_sink``) the rows are
accumulated there in place and nothing table-sized is allocated; otherwise the gradient is a
zero tensor in the table's dtype with the hashed rows filled in.
"""
from __future__ import annotations

import torch

from mimir_b200.ops._ext import ext


class _NGramFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, positions, orders, heads, buckets, dtype, *tables):
        out = ext().ngram_fwd(ids, positions, list(tables), list(orders), heads, buckets, dtype)
        ctx.save_for_backward(ids, positions)
        ctx.info = (orders, heads, buckets)
        ctx.tables = tables
        return out

    @staticmethod
    def backward(ctx, dout):
        ids, positions = ctx.saved_tensors
        orders, heads, buckets = ctx.info
        tables = ctx.tables
        C = ext()
        keys = C.ngram_keys(ids, positions, list(orders), heads, buckets, tables[0].shape[1])
        sorted_keys, order = torch.sort(keys, stable=True)
        sinks = [getattr(t, "_mimir_grad_sink", None) for t in tables]
        in_place = all(sink is not None and t.grad is not None and t.grad.is_contiguous()
                       and t.grad.dtype in (torch.bfloat16, torch.float32) for sink, t in zip(sinks, tables)) \
            and len({t.grad.dtype for t in tables}) == 1
        grads = [t.grad for t in tables] if in_place else [torch.zeros_like(t) for t in tables]
        C.ngram_bwd(dout.contiguous(), ids, positions, sorted_keys, order, grads, list(orders), heads, buckets)
        if in_place:
            for sink, t in zip(sinks, tables):
                sink(t)
            grads = [None] * len(tables)
        return (None, None, None, None, None, None, *grads)


def ngram_lookup(ids, positions, tables, orders, heads, buckets, dtype):
    if not hasattr(ext(), "ngram_fwd"):
        raise RuntimeError("n-gram kernel missing from mimir_b200._C")
    return _NGramFn.apply(ids.to(torch.int64).contiguous(), positions.to(torch.int64).contiguous(), tuple(orders),
                          heads, buckets, dtype, *tables)
