"""Specialist training (frozen reference expert) and strict specialist composition.

Reference: ``src/mimir/model/specialists.py:8-104``.  A specialist run trains only the
non-reference experts (and their router rows) of a two-expert MoE or MoS model;
:func:`compose_specialists` assembles the shared reference plus one specialist per source
model into an ``1 + len(sources)`` expert model, refusing any drift in shared weights or
optimizer state.
"""
from __future__ import annotations

import copy
import re

import torch

_ROUTER = re.compile(r"(?:router|stack_router)\.(?:rows|biases)\.([0-9]+)$")
_EXPERT = re.compile(r"\.experts\.([0-9]+)\.")


def configure_specialist(model, router_only=False):
    cfg = getattr(model, "model", model).gate_config
    if (cfg.moe_num_experts > 1) == (cfg.mos_num_experts > 1):
        raise ValueError("Independent specialist composition supports MoE or MoS, not nested mixtures")
    model.requires_grad_(False)
    trainable = []
    for name, p in model.named_parameters():
        router = _ROUTER.search(name)
        expert = _EXPERT.search(name)
        on = bool(router and int(router[1]) > 0)
        if not router_only:
            on |= bool(expert and int(expert[1]) > 0) or (".stack_experts." in name and not router)
        p.requires_grad_(on)
        if on:
            trainable.append(name)
    if not trainable:
        raise ValueError("No specialist parameters found")
    return trainable


def _owner(name):
    """(source index, key in a two-expert source) for an expert-specific key, else (None, name)."""
    for pattern, shift in ((r"\.experts\.(\d+)\.", 0), (r"\.stack_experts\.(\d+)\.", 1),
                           (r"\.(?:router|stack_router)\.(?:rows|biases)\.(\d+)$", 0)):
        m = re.search(pattern, name)
        if m:
            expert = int(m[1]) + shift
            if expert > 0:
                a, b = m.span(1)
                return expert - 1, name[:a] + str(1 - shift) + name[b:]
    return None, name


@torch.no_grad()
def compose_specialists(destination, sources, optimizer=None, source_optimizers=None):
    if not sources:
        raise ValueError("At least one specialist is required")
    cfg = getattr(destination, "model", destination).gate_config
    if (cfg.moe_num_experts > 1) == (cfg.mos_num_experts > 1):
        raise ValueError("Compose exactly one mixture type")
    if max(cfg.moe_num_experts, cfg.mos_num_experts) != len(sources) + 1:
        raise ValueError("Destination expert count must be one plus the number of branches")
    states = [m.state_dict() for m in sources]
    want = (2, 1) if cfg.moe_num_experts > 1 else (1, 2)
    for src in sources:
        scfg = getattr(src, "model", src).gate_config
        if (scfg.moe_num_experts, scfg.mos_num_experts) != want:
            raise ValueError("Each branch must contain the reference plus one specialist")
        for field in ("H_cycles", "L_cycles", "hidden_size", "n_layers", "H_override", "max_seq_len", "norm_type",
                      "rope_theta", "mos_state_mode"):
            if getattr(scfg, field) != getattr(cfg, field):
                raise ValueError(f"Incompatible specialist configuration: {field}")
    target = destination.state_dict()
    expected = {_owner(n)[1] for n in target}
    if any(set(s) != expected for s in states):
        raise ValueError("Specialist feature keys differ from destination")
    mapping = {}
    for name, value in target.items():
        owner, key = _owner(name)
        if name.endswith("logit_bias"):
            if any(s[name].count_nonzero() for s in states):
                raise ValueError("Remove training-only logit biases before composition")
            target[name] = torch.zeros_like(value)
            continue
        if key not in states[0]:
            raise ValueError(f"Missing specialist key: {key}")
        if owner is None:
            if any(not torch.equal(s[key], states[0][key]) for s in states[1:]):
                raise ValueError(f"Common reference drift: {key}")
            owner = 0
        if states[owner][key].shape != value.shape:
            raise ValueError(f"Specialist shape mismatch: {name}")
        target[name] = states[owner][key].clone()
        mapping[name] = (owner, key)
    destination.load_state_dict(target, strict=True)
    if optimizer is None:
        return
    if source_optimizers is None or len(source_optimizers) != len(sources):
        raise ValueError("Provide all source optimizers to retain moments/EMA")
    params = [dict(m.named_parameters()) for m in sources]
    for name, p in destination.named_parameters():
        owner, key = mapping[name]
        state = source_optimizers[owner].state[params[owner][key]]
        if set(state) != set(optimizer.state[p]):
            raise ValueError(f"Optimizer slot mismatch: {name}")
        if _owner(name)[0] is None:
            for i in range(1, len(sources)):
                other = source_optimizers[i].state[params[i][key]]
                if any((not torch.equal(v, other[k])) if torch.is_tensor(v) else v != other[k] for k, v in state.items()):
                    raise ValueError(f"Common optimizer/EMA drift: {name}")
        optimizer.state[p] = copy.deepcopy(state)
