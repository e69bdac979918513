"""Per-module learning rates for the HRM components and the automatic (``lr_auto``) rates.

Behavioural reference: ``src/mimir/model/module_learning_rates.py:6-96``.  Every parameter
belongs to one component: token embeddings and n-gram tables ("embeddings"), the LM head
("head"), the H stack ("h") or the L stack ("l"); invocation gates are used once per forward
and keep scale 1.  An optimizer never gets extra parameter groups for this: the rates become a
per-parameter multiplier of the base LR (``parameter_lr_scales``), so optimizer checkpoints keep
their group layout.

With ``lr_auto`` the H and L rates are the base LR divided by the number of gradient-carrying
invocations of that stack in one forward (the truncated-BPTT window of ``bp_steps`` calls), so
the summed update a stack receives per step does not grow with ``bp_steps``.
"""
from __future__ import annotations

import math
from typing import Optional

# Module-name component -> rate category (a parameter must match exactly one).
_CATEGORY = {"embed_tokens": "embeddings", "ngram": "embeddings", "lm_head": "head", "H_level": "h",
             "L_level": "l"}
_RATE_NAMES = ("embeddings", "head", "h", "l")


def windowed_cosine_lr(base_lr, min_ratio, step, start, end):
    """Half-cosine from ``base_lr`` at ``start`` to ``base_lr * min_ratio`` at ``end`` (clamped)."""
    if start is None or end is None or not 0 <= start < end:
        raise ValueError("Cosine LR window requires 0 <= start < end")
    if not 0 <= min_ratio <= 1:
        raise ValueError("Cosine LR window requires 0 <= lr_min_ratio <= 1")
    t = (step - start) / (end - start)
    t = 0.0 if t < 0 else 1.0 if t > 1 else t
    return base_lr * (min_ratio + (1 - min_ratio) * (1 + math.cos(math.pi * t)) / 2)


def _category(param_name: str) -> Optional[str]:
    """Rate category of a parameter, or None for an invocation gate (fixed scale 1)."""
    parts = set(param_name.split("."))
    if "invocation_gates" in parts:
        return None
    hits = [comp for comp in _CATEGORY if comp in parts]
    if len(hits) != 1:
        raise ValueError(f"Cannot uniquely assign learning rate to {param_name}")
    return _CATEGORY[hits[0]]


def module_lr_scales(model, base_lr, rates):
    """Per-parameter LR multipliers for the configured per-category ``rates`` (None when no
    category has its own rate)."""
    if all(r is None for r in rates.values()):
        return None
    if base_lr <= 0:
        raise ValueError("Per-module learning rates require lr > 0")
    scales, present = {}, set()
    for name, param in model.named_parameters():
        cat = _category(name)
        if cat is None:
            scales[param] = 1.0
            continue
        present.add(cat)
        scales[param] = 1.0 if rates[cat] is None else rates[cat] / base_lr
    required = set(rates)
    if not all(getattr(m, "has_h_stack", True) for m in model.modules()):
        required.discard("h")  # a model without an H stack has no "h" parameters
    if present != required:
        raise ValueError(f"Missing HRM parameter categories: {set(rates) - present}")
    return scales


def backward_call_counts(h_cycles, l_cycles, bp_steps, *, has_h_stack=True):
    """Gradient-carrying (H, L) stack invocations in one forward: the last ``bp_steps`` calls of
    the H/L schedule, where the H stack runs once per H cycle (at least one L call stays inside
    the window) and the L stack once per L cycle of every H cycle."""
    if min(h_cycles, l_cycles) < 1 or bp_steps < 2:
        raise ValueError("Auto LR requires positive cycles and bp_steps >= 2")
    l_calls = h_cycles * l_cycles
    if not has_h_stack:
        return 0, min(l_calls, bp_steps)
    h_in_window = min(h_cycles, bp_steps - 1)
    return h_in_window, min(l_calls, bp_steps - h_in_window)


def _arch_dict(config) -> dict:
    arch = getattr(config, "arch", {})
    return arch.model_dump() if hasattr(arch, "model_dump") else dict(arch)


def configured_module_rates(config, bp_steps=None):
    """The per-category LRs: the explicit ``lr_<category>`` settings, with ``lr_auto`` filling the
    unset ones from the invocation counts."""
    explicit = {name: getattr(config, f"lr_{name}") for name in _RATE_NAMES}
    if not getattr(config, "lr_auto", False):
        return explicit
    arch = _arch_dict(config)
    if arch["name"] != "mimir2":
        raise ValueError("lr_auto requires Mimir2 recurrence semantics")
    window = arch.get("bp_min_steps", 2) if bp_steps is None else bp_steps
    h_calls, l_calls = backward_call_counts(arch["H_cycles"], arch["L_cycles"], window,
                                            has_h_stack=arch.get("H_override", {}).get("n_layers") != 0)
    lr = config.lr
    derived = {"embeddings": lr, "head": lr, "h": lr / h_calls if h_calls else None, "l": lr / l_calls}
    return {name: derived[name] if explicit[name] is None else explicit[name] for name in _RATE_NAMES}


def update_auto_module_rates(config, model, optimizer, bp_steps):
    """Recompute the optimizer's multipliers when ``lr_auto`` is on and ``bp_steps`` changed."""
    if not getattr(config, "lr_auto", False):
        return
    if bp_steps is None:
        raise ValueError("lr_auto requires the current training bp_steps")
    if getattr(optimizer, "_auto_lr_bp_steps", None) == bp_steps:
        return
    optimizer.parameter_lr_scales = module_lr_scales(model, config.lr, configured_module_rates(config, bp_steps))
    optimizer._auto_lr_bp_steps = bp_steps


def module_lr_metrics(config, lr, bp_steps=None):
    """Logged LRs per category (``train/lr_<category>``) plus the older metric names that
    existing dashboards read (``train/lr_H``, ``train/lr_L``, ``train/lr_embedding_head``)."""
    rates = configured_module_rates(config, bp_steps)
    if all(r is None for r in rates.values()):
        return {}
    out = {f"train/lr_{name}": lr * (1.0 if r is None else r / config.lr) for name, r in rates.items()}
    if _arch_dict(config).get("H_override", {}).get("n_layers") == 0:
        del out["train/lr_h"]
    else:
        out["train/lr_H"] = out["train/lr_h"]
    out["train/lr_L"] = out["train/lr_l"]
    if out["train/lr_embeddings"] == out["train/lr_head"]:
        out["train/lr_embedding_head"] = out["train/lr_embeddings"]
    return out
