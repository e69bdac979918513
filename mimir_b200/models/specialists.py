"""Specialist training against a frozen reference expert, and strict specialist composition.

Behavioural reference: ``src/mimir/model/specialists.py:8-104``.

* :func:`configure_specialist` freezes a two-expert MoE (or MoS) model except its specialist:
  the non-reference experts and their router rows (or only the router rows).
* :func:`compose_specialists` builds an ``1 + len(sources)``-expert model from several such
  two-expert runs that share the reference: expert ``i + 1`` (and its router row) comes from
  source ``i``, everything else must be bit-identical across the sources (weights and, when
  optimizers are given, every optimizer slot and EMA), and training-only logit biases must be
  zero.

Parameter names are the interface here.  An expert-specific name carries its expert index in
one of three places: ``.experts.<e>.`` (MoE experts, 0 = reference), ``.stack_experts.<s>.``
(MoS specialist stacks, which are experts ``s + 1``: the reference stack lives elsewhere) and
``.router|stack_router.rows|biases.<e>`` (router rows).
"""
from __future__ import annotations

import copy
import re
from dataclasses import dataclass
from typing import Optional

import torch


@dataclass(frozen=True)
class _Slot:
    kind: str     # "expert", "stack", "router"
    expert: int   # expert number in the composed model (0 = the shared reference)
    start: int    # span of the index digits inside the name
    end: int


_SLOT_PATTERNS = (("expert", re.compile(r"\.experts\.(\d+)\."), 0),
                  ("stack", re.compile(r"\.stack_experts\.(\d+)\."), 1),
                  ("router", re.compile(r"\.(?:router|stack_router)\.(?:rows|biases)\.(\d+)$"), 0))


def _slot(name: str) -> Optional[_Slot]:
    for kind, pattern, shift in _SLOT_PATTERNS:
        m = pattern.search(name)
        if m:
            return _Slot(kind, int(m.group(1)) + shift, m.start(1), m.end(1))
    return None


def _source_key(name: str) -> tuple[Optional[int], str]:
    """(index of the source model, name inside that two-expert source) for a specialist's
    parameter; (None, name) for the shared part, reference expert included."""
    s = _slot(name)
    if s is None or s.expert == 0:
        return None, name
    local = 0 if s.kind == "stack" else 1  # the specialist's index inside a two-expert source
    return s.expert - 1, f"{name[:s.start]}{local}{name[s.end:]}"


def _mixture_config(model):
    return getattr(model, "model", model).gate_config


def _one_mixture(cfg) -> bool:
    return (cfg.moe_num_experts > 1) != (cfg.mos_num_experts > 1)


def configure_specialist(model, router_only: bool = False) -> list:
    """Freeze everything but the specialist; returns the trainable parameter names."""
    if not _one_mixture(_mixture_config(model)):
        raise ValueError("Independent specialist composition supports MoE or MoS, not nested mixtures")
    model.requires_grad_(False)
    chosen = []
    for name, param in model.named_parameters():
        s = _slot(name)
        if s is None:
            train = False
        elif s.kind == "router":
            train = s.expert > 0
        else:
            train = not router_only and (s.kind == "stack" or s.expert > 0)
        param.requires_grad_(train)
        if train:
            chosen.append(name)
    if not chosen:
        raise ValueError("No specialist parameters found")
    return chosen


_SHARED_FIELDS = ("H_cycles", "L_cycles", "hidden_size", "n_layers", "H_override", "max_seq_len", "norm_type",
                  "rope_theta", "mos_state_mode")


def _check_sources(cfg, sources) -> None:
    if not _one_mixture(cfg):
        raise ValueError("Compose exactly one mixture type")
    if max(cfg.moe_num_experts, cfg.mos_num_experts) != len(sources) + 1:
        raise ValueError("Destination expert count must be one plus the number of branches")
    pair = (2, 1) if cfg.moe_num_experts > 1 else (1, 2)
    for src in sources:
        scfg = _mixture_config(src)
        if (scfg.moe_num_experts, scfg.mos_num_experts) != pair:
            raise ValueError("Each branch must contain the reference plus one specialist")
        for field in _SHARED_FIELDS:
            if getattr(scfg, field) != getattr(cfg, field):
                raise ValueError(f"Incompatible specialist configuration: {field}")


def _same_slots(a: dict, b: dict) -> bool:
    if set(a) != set(b):
        return False
    return all(torch.equal(v, b[k]) if torch.is_tensor(v) else v == b[k] for k, v in a.items())


@torch.no_grad()
def compose_specialists(destination, sources, optimizer=None, source_optimizers=None):
    """Load ``destination`` (and, optionally, its optimizer state) from the specialist runs."""
    if not sources:
        raise ValueError("At least one specialist is required")
    _check_sources(_mixture_config(destination), sources)
    source_states = [src.state_dict() for src in sources]
    composed = destination.state_dict()
    wanted = {_source_key(name)[1] for name in composed}
    if any(set(state) != wanted for state in source_states):
        raise ValueError("Specialist feature keys differ from destination")

    origin = {}  # destination name -> (source index, source key)
    for name, current in composed.items():
        owner, key = _source_key(name)
        if name.endswith("logit_bias"):
            if any(bool(state[name].count_nonzero()) for state in source_states):
                raise ValueError("Remove training-only logit biases before composition")
            composed[name] = torch.zeros_like(current)
            continue
        if key not in source_states[0]:
            raise ValueError(f"Missing specialist key: {key}")
        if owner is None:
            first = source_states[0][key]
            if not all(torch.equal(state[key], first) for state in source_states[1:]):
                raise ValueError(f"Common reference drift: {key}")
            owner = 0
        value = source_states[owner][key]
        if value.shape != current.shape:
            raise ValueError(f"Specialist shape mismatch: {name}")
        composed[name] = value.clone()
        origin[name] = (owner, key)
    destination.load_state_dict(composed, strict=True)

    if optimizer is None:
        return
    if source_optimizers is None or len(source_optimizers) != len(sources):
        raise ValueError("Provide all source optimizers to retain moments/EMA")
    source_params = [dict(src.named_parameters()) for src in sources]
    for name, param in destination.named_parameters():
        owner, key = origin[name]
        slots = source_optimizers[owner].state[source_params[owner][key]]
        if set(slots) != set(optimizer.state[param]):
            raise ValueError(f"Optimizer slot mismatch: {name}")
        if _source_key(name)[0] is None:
            for i in range(1, len(sources)):
                if not _same_slots(slots, source_optimizers[i].state[source_params[i][key]]):
                    raise ValueError(f"Common optimizer/EMA drift: {name}")
        optimizer.state[param] = copy.deepcopy(slots)
