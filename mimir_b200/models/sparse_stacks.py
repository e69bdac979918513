"""Sparse mixture-of-stacks (MoS): whole sequences are routed to L-stack experts.

Behavioural reference: ``src/mimir/model/sparse_stacks.py:9-162``.

* Routing: each sequence is routed once, from a pooled embedding — its first token
  (``first_token``) or the mean of its prompt (``prefix_mean``).  During cached decode a row is
  routed when it starts (cache length 0) and keeps that route.
* Execution: every selected expert stack runs on complete sequences only, so attention contexts
  are never pruned; its output is scattered back weighted by the sequence's routing weight.
* Participation: an expert that received no sequence still runs on a one-token dummy whose
  output enters the result multiplied by zero, so every rank runs the same modules (and issues
  the same collectives) whatever the routing.

Two layouts: ``[batch, seq, hidden]`` (``batched_sparse_stack_step``; also cached decode) and
packed varlen ``[tokens, hidden]`` with ``cu_seqlens`` (``sparse_stack_step``), where the chosen
sequences are gathered into a fresh packed batch with its own prefix-LM metadata.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from mimir_b200.data.prefixlm import compute_aux_seq_tensors_scalars
from mimir_b200.models.common import unwrap_tensor, wrap_tensor

_POLICIES = ("first_token", "prefix_mean")


def _pool_batched(x, seq_info, policy):
    if policy == "first_token":
        return x[:, 0]
    lengths = seq_info.get("prefix_lens")
    if lengths is None or bool((lengths < 1).any()) or bool((lengths > x.shape[1]).any()):
        raise ValueError("Prefix routing requires valid prefix_lens for each sequence")
    return torch.stack([seq[:int(n)].mean(0) for seq, n in zip(x, lengths, strict=True)])


def _pool_packed(x, seq_info, policy):
    count = int(unwrap_tensor(seq_info["numseqs"]))
    starts = seq_info["cu_seqlens"][:count].long()
    if policy == "first_token":
        return x.index_select(0, starts)
    lengths = seq_info["prefix_lens"][:count].tolist()
    if min(lengths, default=1) < 1:
        raise ValueError("Prefix routing requires nonempty instruction prefixes")
    return torch.stack([x[s:s + n].mean(0) for s, n in zip(starts.tolist(), lengths, strict=True)])


@torch.compiler.disable
def sequence_routes(router, x, seq_info, bias=None, policy="first_token"):
    """Routing weights ``[sequences, experts]`` from each sequence's pooled embedding."""
    if policy not in _POLICIES:
        raise ValueError(f"Unknown sparse routing policy: {policy}")
    if x.ndim == 3:
        return router(_pool_batched(x, seq_info, policy), bias)
    if x.ndim != 2 or "cu_seqlens" not in seq_info:
        raise ValueError("Sparse MoS requires packed sequences with cu_seqlens/numseqs")
    return router(_pool_packed(x, seq_info, policy), bias)


@torch.compiler.disable
def cached_sequence_routes(model, x, cache, seq_info, bias=None):
    """Decode: route the rows that start now (cache length 0); every other row keeps its route."""
    if x.ndim != 3:
        raise ValueError("Cached sparse MoS expects batch x sequence x hidden")
    routes = cache["mos_routes"][:x.shape[0]]
    starting = (seq_info["cache_lengths"] == 0).nonzero().flatten()
    if len(starting) == 0:
        return routes
    info = dict(seq_info)
    prefix = info.get("prefix_lens", torch.full((x.shape[0],), x.shape[1], device=x.device))
    info["prefix_lens"] = prefix.index_select(0, starting)
    row_bias = bias.index_select(0, starting) if bias is not None and bias.ndim > 1 else bias
    new = sequence_routes(model.L_level.stack_router, x.index_select(0, starting), info, row_bias,
                          model.gate_config.mos_sparse_routing)
    routes.index_copy_(0, starting, new.detach())
    return routes


def _experts(model):
    return (model.L_level.core, *model.L_level.stack_experts)


def _rows_info(seq_info, rows, cache):
    """Per-row inputs restricted to the selected batch rows."""
    info = dict(seq_info)
    pos = info.get("position_ids")
    if pos is not None and pos.ndim > 1:
        info["position_ids"] = pos.index_select(0, rows)
    if cache is not None:
        info["cache_lengths"] = info["cache_lengths"].index_select(0, rows)
        info["cache_batch_indices"] = rows
    return info


@torch.compiler.disable
def batched_sparse_stack_step(model, z_l, z_h, states, invocation, diagnostics, seq_info, weights, cache=None,
                              expert_outputs=None):
    """MoS step on ``[batch, seq, hidden]``: expert ``e`` runs on the batch rows routed to it."""
    mixed = torch.zeros_like(z_h)
    updated = [] if states is not None else None
    for e, core in enumerate(_experts(model)):
        start = (z_l if states is None else states[e]).expand_as(z_h)
        rows = (weights[:, e] != 0).nonzero().flatten()
        kept = start
        contribution = None if expert_outputs is None else torch.zeros_like(z_h)
        stack_input = start + model._inject(model.L_level, invocation, start, z_h)
        if len(rows):
            scope = f"L/cycle_{invocation:03d}/expert_{e}" if diagnostics else None
            y = core(stack_input.index_select(0, rows), cache=None if cache is None else cache[e],
                     **_rows_info(seq_info, rows, cache), stability_diagnostics=diagnostics, stability_scope=scope)
            mixed = mixed.index_add(0, rows, y * weights[rows, e, None, None].to(y.dtype))
            kept = start.index_copy(0, rows, y)
            if contribution is not None:
                contribution = contribution.index_copy(0, rows, y)
        elif cache is None and model.training:  # keep the expert in the step: zero-weighted dummy
            info = dict(seq_info)
            pos = info.get("position_ids")
            if pos is not None and pos.ndim > 1:
                info["position_ids"] = pos[:1]
            zero = core(stack_input[:1], **info).sum() * 0
            mixed = mixed + zero
            if contribution is not None:
                contribution = contribution + zero
        if contribution is not None:
            expert_outputs.append((contribution, weights[:, e, None, None]))
        if updated is not None:
            updated.append(kept)
    return mixed, updated


class _PackedChoice:
    """The sequences of a packed batch routed to one expert, re-packed as a batch of their own
    (or a one-token dummy when none were): token index, inputs, positions and prefix-LM metadata."""

    def __init__(self, chosen, bounds, prefix, causal, stack_input, positions, device):
        self.chosen = chosen
        if chosen:
            self.index = torch.cat([torch.arange(bounds[s], bounds[s + 1], device=device) for s in chosen])
            tokens, pos = stack_input.index_select(0, self.index), positions.index_select(0, self.index)
            p, c = [prefix[s] for s in chosen], [causal[s] for s in chosen]
        else:
            self.index = torch.zeros(1, dtype=torch.long, device=device)
            tokens, pos, p, c = stack_input[:1], positions[:1], [1], [0]
        self.valid = len(tokens)
        size = max(len(p) + 1, self.valid)  # room for the padding sequence the metadata expects
        if size > self.valid:
            tokens = F.pad(tokens, (0, 0, 0, size - self.valid))
            pos = F.pad(pos, (0, size - self.valid))
        self.tokens, self.positions = tokens, pos
        tensors, scalars = compute_aux_seq_tensors_scalars(np.array(p, np.int32), np.array(c, np.int32), size)
        self.meta = ({k: torch.from_numpy(v).to(device) for k, v in tensors.items()}
                     | {k: wrap_tensor(torch.tensor(v)) for k, v in scalars.items()})

    def token_weights(self, weights, e, bounds):
        return torch.cat([weights[s, e].expand(bounds[s + 1] - bounds[s]) for s in self.chosen])


@torch.compiler.disable
def sparse_stack_step(model, z_l, z_h, states, invocation, diagnostics, seq_info, weights, expert_outputs=None):
    """MoS step on a packed varlen batch: expert ``e`` runs on a re-packed batch of the sequences
    routed to it."""
    n = int(unwrap_tensor(seq_info["numseqs"]))
    bounds = seq_info["cu_seqlens"][:n + 1].tolist()
    prefix, causal = seq_info["prefix_lens"][:n].tolist(), seq_info["causal_lens"][:n].tolist()
    mixed = torch.zeros_like(z_h)
    updated = [] if states is not None else None
    for e, core in enumerate(_experts(model)):
        start = (z_l if states is None else states[e]).expand_as(z_h)
        stack_input = start + model._inject(model.L_level, invocation, start, z_h)
        pick = _PackedChoice((weights[:, e] != 0).nonzero().flatten().tolist(), bounds, prefix, causal, stack_input,
                             seq_info["position_ids"], z_h.device)
        if "routing_bias" in seq_info:
            pick.meta["routing_bias"] = seq_info["routing_bias"]
        live = bool(pick.chosen)
        y = core(pick.tokens, position_ids=pick.positions, **pick.meta,
                 stability_diagnostics=diagnostics if live else None,
                 stability_scope=f"L/cycle_{invocation:03d}/expert_{e}" if diagnostics and live else None)[:pick.valid]
        if expert_outputs is not None:
            contribution = torch.zeros_like(z_h) + y.sum() * 0
            contribution_w = weights.new_zeros(z_h.shape[0], 1)
        if live:
            w = pick.token_weights(weights, e, bounds)
            mixed = mixed.index_add(0, pick.index, y * w[:, None].to(y.dtype))
            if expert_outputs is not None:
                contribution = contribution.index_copy(0, pick.index, y)
                contribution_w = contribution_w.index_copy(0, pick.index, w[:, None])
            if updated is not None:
                updated.append(start.index_copy(0, pick.index, y))
        else:
            mixed = mixed + y.sum() * 0
            if updated is not None:
                updated.append(start)
        if expert_outputs is not None:
            expert_outputs.append((contribution, contribution_w))
    return mixed, updated
