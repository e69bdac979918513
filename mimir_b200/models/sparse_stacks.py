"""Sparse mixture-of-stacks (MoS): route whole sequences to L-stack experts.

Reference: ``src/mimir/model/sparse_stacks.py:9-162``.  A sequence is routed once, from
its first token embedding or from the mean of its prompt embeddings, and each selected
expert stack runs on complete sequences only (attention contexts are never pruned).
Experts with no sequences still run on a one-token dummy whose output is multiplied by
zero, so every rank issues the same collectives in the same order.
"""
from __future__ import annotations

import numpy as np
import torch

from mimir_b200.data.prefixlm import compute_aux_seq_tensors_scalars
from mimir_b200.models.common import unwrap_tensor, wrap_tensor


@torch.compiler.disable
def sequence_routes(router, x, seq_info, bias=None, policy="first_token"):
    if x.ndim == 3:
        if policy == "first_token":
            pooled = x[:, 0]
        elif policy == "prefix_mean":
            lengths = seq_info.get("prefix_lens")
            if lengths is None or (lengths < 1).any() or (lengths > x.shape[1]).any():
                raise ValueError("Prefix routing requires valid prefix_lens for each sequence")
            pooled = torch.stack([row[:int(n)].mean(0) for row, n in zip(x, lengths, strict=True)])
        else:
            raise ValueError(f"Unknown sparse routing policy: {policy}")
        return router(pooled, bias)
    if x.ndim != 2 or "cu_seqlens" not in seq_info:
        raise ValueError("Sparse MoS requires packed sequences with cu_seqlens/numseqs")
    count = int(unwrap_tensor(seq_info["numseqs"]))
    starts = seq_info["cu_seqlens"][:count].long()
    if policy == "prefix_mean":
        lengths = seq_info["prefix_lens"][:count].tolist()
        if any(n < 1 for n in lengths):
            raise ValueError("Prefix routing requires nonempty instruction prefixes")
        pooled = torch.stack([x[s:s + n].mean(0) for s, n in zip(starts.tolist(), lengths, strict=True)])
    elif policy == "first_token":
        pooled = x.index_select(0, starts)
    else:
        raise ValueError(f"Unknown sparse routing policy: {policy}")
    return router(pooled, bias)


@torch.compiler.disable
def cached_sequence_routes(model, x, cache, seq_info, bias=None):
    if x.ndim != 3:
        raise ValueError("Cached sparse MoS expects batch x sequence x hidden")
    fresh_rows = (seq_info["cache_lengths"] == 0).nonzero().flatten()
    routes = cache["mos_routes"][:x.shape[0]]
    if len(fresh_rows):
        info = dict(seq_info)
        lengths = info.get("prefix_lens", torch.full((x.shape[0],), x.shape[1], device=x.device))
        info["prefix_lens"] = lengths.index_select(0, fresh_rows)
        row_bias = bias.index_select(0, fresh_rows) if bias is not None and bias.ndim > 1 else bias
        fresh = sequence_routes(model.L_level.stack_router, x.index_select(0, fresh_rows), info, row_bias,
                                model.gate_config.mos_sparse_routing)
        routes.index_copy_(0, fresh_rows, fresh.detach())
    return routes


def _stack_cores(model):
    return [model.L_level.core, *model.L_level.stack_experts]


@torch.compiler.disable
def batched_sparse_stack_step(model, z_l, z_h, states, invocation, diagnostics, seq_info, weights, cache=None,
                              expert_outputs=None):
    output, next_states = torch.zeros_like(z_h), []
    for e, core in enumerate(_stack_cores(model)):
        rows = (weights[:, e] != 0).nonzero().flatten()
        prev = (states[e] if states is not None else z_l).expand_as(z_h)
        candidate = prev
        expert_value = torch.zeros_like(z_h) if expert_outputs is not None else None
        if len(rows):
            info = dict(seq_info)
            pos = info.get("position_ids")
            if pos is not None and pos.ndim > 1:
                info["position_ids"] = pos.index_select(0, rows)
            if cache is not None:
                info["cache_lengths"] = info["cache_lengths"].index_select(0, rows)
                info["cache_batch_indices"] = rows
            inj = model._inject(model.L_level, invocation, prev, z_h)
            value = core((prev + inj).index_select(0, rows), cache=cache[e] if cache is not None else None, **info,
                         stability_diagnostics=diagnostics,
                         stability_scope=f"L/cycle_{invocation:03d}/expert_{e}" if diagnostics else None)
            output = output.index_add(0, rows, value * weights[rows, e, None, None].to(value.dtype))
            candidate = prev.index_copy(0, rows, value)
            if expert_outputs is not None:
                expert_value = expert_value.index_copy(0, rows, value)
        elif cache is None and model.training:
            info = dict(seq_info)
            if info.get("position_ids") is not None and info["position_ids"].ndim > 1:
                info["position_ids"] = info["position_ids"][:1]
            inj = model._inject(model.L_level, invocation, prev, z_h)
            dummy = core((prev + inj)[:1], **info)
            output = output + dummy.sum() * 0
            if expert_outputs is not None:
                expert_value = expert_value + dummy.sum() * 0
        if expert_outputs is not None:
            expert_outputs.append((expert_value, weights[:, e, None, None]))
        if states is not None:
            next_states.append(candidate)
    return output, (next_states if states is not None else None)


@torch.compiler.disable
def sparse_stack_step(model, z_l, z_h, states, invocation, diagnostics, seq_info, weights, expert_outputs=None):
    nseq = int(unwrap_tensor(seq_info["numseqs"]))
    bounds = seq_info["cu_seqlens"][:nseq + 1].tolist()
    prefix = seq_info["prefix_lens"][:nseq].tolist()
    causal = seq_info["causal_lens"][:nseq].tolist()
    output, next_states = torch.zeros_like(z_h), []
    for e, core in enumerate(_stack_cores(model)):
        chosen = (weights[:, e] != 0).nonzero().flatten().tolist()
        prev = (states[e] if states is not None else z_l).expand_as(z_h)
        inj = model._inject(model.L_level, invocation, prev, z_h)
        if chosen:
            idx = torch.cat([torch.arange(bounds[s], bounds[s + 1], device=z_h.device) for s in chosen])
            p, c = [prefix[s] for s in chosen], [causal[s] for s in chosen]
            gathered = (prev + inj).index_select(0, idx)
            pos = seq_info["position_ids"].index_select(0, idx)
        else:
            idx = torch.zeros(1, dtype=torch.long, device=z_h.device)
            gathered, pos, p, c = (prev + inj)[:1], seq_info["position_ids"][:1], [1], [0]
        n_valid = len(gathered)
        capacity = max(len(p) + 1, n_valid)
        if capacity > n_valid:
            gathered = torch.nn.functional.pad(gathered, (0, 0, 0, capacity - n_valid))
            pos = torch.nn.functional.pad(pos, (0, capacity - n_valid))
        tensors, scalars = compute_aux_seq_tensors_scalars(np.array(p, np.int32), np.array(c, np.int32), capacity)
        info = ({k: torch.from_numpy(v).to(z_h.device) for k, v in tensors.items()}
                | {k: wrap_tensor(torch.tensor(v)) for k, v in scalars.items()})
        if "routing_bias" in seq_info:
            info["routing_bias"] = seq_info["routing_bias"]
        y = core(gathered, position_ids=pos, **info, stability_diagnostics=diagnostics if chosen else None,
                 stability_scope=f"L/cycle_{invocation:03d}/expert_{e}" if diagnostics and chosen else None)[:n_valid]
        if expert_outputs is not None:
            expert_value = torch.zeros_like(z_h) + y.sum() * 0
            expert_weight = weights.new_zeros(z_h.shape[0], 1)
        if chosen:
            tok_w = torch.cat([weights[s, e].expand(bounds[s + 1] - bounds[s]) for s in chosen])
            output = output.index_add(0, idx, y * tok_w[:, None].to(y.dtype))
            if expert_outputs is not None:
                expert_value = expert_value.index_copy(0, idx, y)
                expert_weight = expert_weight.index_copy(0, idx, tok_w[:, None])
            if states is not None:
                next_states.append(prev.index_copy(0, idx, y))
        else:
            output = output + y.sum() * 0
            if states is not None:
                next_states.append(prev)
        if expert_outputs is not None:
            expert_outputs.append((expert_value, expert_weight))
    return output, (next_states if states is not None else None)
