"""Hashed causal n-gram memory (Engram-like) added to the token embeddings.

Reference behaviour: ``src/mimir/model/ngram_memory.py:11-90``.  For every order ``n``
and head ``h`` the last ``n`` tokens are hashed with the polynomial
``v <- (v * (65599 + 2h) + token + 1) mod buckets`` (newest token first), the bucket's
row of table ``(n, h)`` is gathered, and rows are concatenated across heads and summed
across orders.  An n-gram only counts when its tokens are consecutive positions of one
packed sequence (``position[t] - position[t-o] == o`` for every offset).  The sum is
optionally gated by ``sigmoid(Wq rms(x) + Wk rms(mem))`` and added as ``x + alpha * mem``.

On CUDA the hash, gather, validity mask and order sum run in one kernel
(:func:`mimir_b200.ops.ngram_lookup`), with a deterministic backward that touches only the hashed rows.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from mimir_b200 import ops


def ngram_hashes(ids: torch.Tensor, positions: torch.Tensor, orders, heads: int, buckets: int):
    """Return ``{order: (hash[heads, *ids.shape], valid[*ids.shape])}`` for ``ids`` of shape [B, S]."""
    out = {}
    hashed = [torch.zeros_like(ids) for _ in range(heads)]
    valid = torch.ones_like(ids, dtype=torch.bool)
    index = torch.arange(ids.shape[-1], device=ids.device)
    for offset in range(max(orders)):
        shifted = ids.roll(offset, dims=-1)
        valid = valid & (index >= offset) & (positions - positions.roll(offset, dims=-1) == offset)
        hashed = [(v * (65599 + 2 * h) + shifted + 1).remainder(buckets) for h, v in enumerate(hashed)]
        if offset + 1 in orders:
            out[offset + 1] = (torch.stack(hashed), valid)
    return out


class NGramMemory(nn.Module):
    def __init__(self, hidden_size, orders=(2, 3), buckets=4096, heads=1, contextual_gate=False):
        super().__init__()
        if not orders or min(orders) < 2 or len(set(orders)) != len(orders) or buckets < 2:
            raise ValueError("N-grams require unique orders >= 2 and at least two buckets")
        if heads < 1 or hidden_size % heads:
            raise ValueError("N-gram heads must be positive and divide hidden_size")
        self.orders = tuple(orders)
        self.buckets = buckets
        self.heads = heads
        self.tables = nn.ParameterList([nn.Parameter(torch.zeros(buckets, hidden_size // heads))
                                        for _ in orders for _ in range(heads)])
        self.contextual_gate = contextual_gate
        if contextual_gate:
            self.query = nn.Linear(hidden_size, hidden_size, bias=False)
            self.key = nn.Linear(hidden_size, hidden_size, bias=False)
            nn.init.normal_(self.query.weight, std=hidden_size ** -0.5)
            nn.init.normal_(self.key.weight, std=hidden_size ** -0.5)
        self.register_buffer("alpha", torch.tensor(0.0))

    def lookup(self, ids: torch.Tensor, positions: torch.Tensor, dtype) -> torch.Tensor:
        """Summed n-gram memory ``[B, S, hidden]`` for token ids/positions ``[B, S]``."""
        if ops.kernels_enabled(ids) and ids.shape[0] == 1:
            return ops.ngram_lookup(ids[0], positions[0], list(self.tables), self.orders, self.heads,
                                    self.buckets, dtype).unsqueeze(0)
        hidden = sum(t.shape[-1] for t in self.tables[:self.heads])
        out = torch.zeros((*ids.shape, hidden), dtype=dtype, device=ids.device)
        for order, (hashes, valid) in ngram_hashes(ids, positions, self.orders, self.heads, self.buckets).items():
            base = self.orders.index(order) * self.heads
            rows = torch.cat([F.embedding(hashes[h], self.tables[base + h]) for h in range(self.heads)], dim=-1)
            out = out + rows.to(dtype) * valid[..., None]
        return out

    def forward(self, x, tokens, position_ids=None, history=None, *, diagnostics=None):
        if tokens.shape != x.shape[:-1] or tokens.ndim not in (1, 2):
            raise ValueError("N-gram tokens must match [tokens] or [batch, tokens] embeddings")
        if history is not None and position_ids is None:
            raise ValueError("Cached n-grams require explicit position_ids for sequence resets")
        ids = tokens.long().reshape(-1, tokens.shape[-1])
        positions = (torch.arange(ids.shape[-1], device=ids.device).expand_as(ids) if position_ids is None
                     else position_ids.expand_as(ids))
        prefix = 0
        if history is not None and "tokens" in history:
            if history["tokens"].shape[0] != ids.shape[0]:
                raise ValueError("N-gram cache batch changed; create/reset cache for new requests")
            prefix = history["tokens"].shape[-1]
            ids = torch.cat((history["tokens"], ids), dim=-1)
            positions = torch.cat((history["positions"], positions), dim=-1)
        memory = self.lookup(ids, positions.long(), x.dtype)
        if history is not None:
            tail = max(self.orders) - 1
            history["tokens"] = ids[:, -tail:].detach().clone()
            history["positions"] = positions[:, -tail:].detach().clone()
        memory = memory[:, prefix:].reshape_as(x)
        if diagnostics is not None:
            diagnostics["retrieved_rms"] = memory.detach().float().square().mean().sqrt()
        if self.contextual_gate:
            ctx = F.rms_norm(x, (x.shape[-1],), eps=1e-6)
            mem = F.rms_norm(memory, (memory.shape[-1],), eps=1e-6)
            gate = torch.sigmoid(self.query(ctx) + self.key(mem))
            memory = gate.to(x.dtype) * memory
            if diagnostics is not None:
                g = gate.detach().float()
                diagnostics.update(gate_mean=g.mean(), gate_min=g.min(), gate_max=g.max(),
                                   gate_saturated_fraction=((g < .01) | (g > .99)).float().mean())
        if diagnostics is not None:
            contribution = self.alpha.to(x.dtype) * memory.detach()
            diagnostics["contribution_rms"] = contribution.float().square().mean().sqrt()
            diagnostics["input_rms"] = x.detach().float().square().mean().sqrt()
            diagnostics["contribution_input_ratio"] = diagnostics["contribution_rms"] / diagnostics["input_rms"].clamp_min(1e-12)
        return x + self.alpha.to(x.dtype) * memory
