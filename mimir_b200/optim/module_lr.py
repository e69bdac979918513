"""Per-module learning rates and HRM auto-LR.

Reference: ``src/mimir/model/module_learning_rates.py:6-96``.  Parameters are grouped by
component (embeddings incl. n-gram tables, head, H stack, L stack; invocation gates keep
scale 1).  With ``lr_auto`` the H/L learning rates are divided by the number of backward
invocations of that stack per step (truncated BPTT), so the summed update per step is
independent of ``bp_steps``.
"""
from __future__ import annotations

import math


def windowed_cosine_lr(base_lr, min_ratio, step, start, end):
    if start is None or end is None or start < 0 or end <= start:
        raise ValueError("Cosine LR window requires 0 <= start < end")
    if not 0 <= min_ratio <= 1:
        raise ValueError("Cosine LR window requires 0 <= lr_min_ratio <= 1")
    progress = min(1.0, max(0.0, (step - start) / (end - start)))
    return base_lr * (min_ratio + (1 - min_ratio) * 0.5 * (1 + math.cos(math.pi * progress)))


_COMPONENTS = (("embed_tokens", "embeddings"), ("ngram", "embeddings"), ("lm_head", "head"), ("H_level", "h"),
               ("L_level", "l"))


def module_lr_scales(model, base_lr, rates):
    if not any(v is not None for v in rates.values()):
        return None
    if base_lr <= 0:
        raise ValueError("Per-module learning rates require lr > 0")
    scales, seen = {}, set()
    for name, p in model.named_parameters():
        parts = name.split(".")
        if "invocation_gates" in parts:
            scales[p] = 1.0
            continue
        labels = [label for comp, label in _COMPONENTS if comp in parts]
        if len(labels) != 1:
            raise ValueError(f"Cannot uniquely assign learning rate to {name}")
        seen.add(labels[0])
        rate = rates[labels[0]]
        scales[p] = 1.0 if rate is None else rate / base_lr
    expected = set(rates)
    if any(getattr(m, "has_h_stack", True) is False for m in model.modules()):
        expected.discard("h")
    if seen != expected:
        raise ValueError(f"Missing HRM parameter categories: {set(rates) - seen}")
    return scales


def backward_call_counts(h_cycles, l_cycles, bp_steps, *, has_h_stack=True):
    """Number of H and L stack invocations that carry gradients in one forward."""
    if h_cycles < 1 or l_cycles < 1 or bp_steps < 2:
        raise ValueError("Auto LR requires positive cycles and bp_steps >= 2")
    if not has_h_stack:
        return 0, min(h_cycles * l_cycles, bp_steps)
    h = min(h_cycles, bp_steps - 1)
    return h, min(h_cycles * l_cycles, bp_steps - h)


def configured_module_rates(config, bp_steps=None):
    rates = {name: getattr(config, f"lr_{name}") for name in ("embeddings", "head", "h", "l")}
    if not getattr(config, "lr_auto", False):
        return rates
    arch = config.arch.model_dump() if hasattr(config.arch, "model_dump") else config.arch
    if arch["name"] != "mimir2":
        raise ValueError("lr_auto requires Mimir2 recurrence semantics")
    h, l = backward_call_counts(arch["H_cycles"], arch["L_cycles"],
                                arch.get("bp_min_steps", 2) if bp_steps is None else bp_steps,
                                has_h_stack=arch.get("H_override", {}).get("n_layers") != 0)
    auto = dict(embeddings=config.lr, head=config.lr, h=config.lr / h if h else None, l=config.lr / l)
    return {name: auto[name] if v is None else v for name, v in rates.items()}


def update_auto_module_rates(config, model, optimizer, bp_steps):
    if not getattr(config, "lr_auto", False):
        return
    if bp_steps is None:
        raise ValueError("lr_auto requires the current training bp_steps")
    if getattr(optimizer, "_auto_lr_bp_steps", None) != bp_steps:
        optimizer.parameter_lr_scales = module_lr_scales(model, config.lr, configured_module_rates(config, bp_steps))
        optimizer._auto_lr_bp_steps = bp_steps


def module_lr_metrics(config, lr, bp_steps=None):
    rates = configured_module_rates(config, bp_steps)
    if not any(v is not None for v in rates.values()):
        return {}
    metrics = {f"train/lr_{n}": lr * (v / config.lr if v is not None else 1.0) for n, v in rates.items()}
    arch = getattr(config, "arch", {})
    arch = arch.model_dump() if hasattr(arch, "model_dump") else arch
    if arch.get("H_override", {}).get("n_layers") == 0:
        metrics.pop("train/lr_h", None)
    else:
        metrics["train/lr_H"] = metrics["train/lr_h"]
    metrics["train/lr_L"] = metrics["train/lr_l"]
    if metrics["train/lr_embeddings"] == metrics["train/lr_head"]:
        metrics["train/lr_embedding_head"] = metrics["train/lr_embeddings"]
    return metrics
