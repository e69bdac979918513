"""Shared updates for invocation gates that receive no gradient in a step.

Reference: ``src/mimir/model/gate_updates.py:6-40``.  Gates outside the truncated-BPTT
window copy the actual parameter delta of their level's first active gate ("donor") and
track its optimizer moments, so they stay usable when the window later widens.
"""
from __future__ import annotations

import torch


@torch.no_grad()
def snapshot_donors(optimizer):
    pairs = getattr(optimizer, "shared_parameter_updates", {})
    for target, donor in pairs.items():
        if target is donor or donor in pairs:
            raise ValueError("Gate donors must be active, independent parameters")
        if donor.grad is None:
            raise RuntimeError("Gate donor mapping disagrees with gradient eligibility")
        if target.shape != donor.shape:
            raise ValueError("Gate donor and target shapes must match")
        if target not in optimizer.state or donor not in optimizer.state:
            raise ValueError("Gate parameters must belong to this optimizer")
    return {donor: donor.detach().clone() for donor in set(pairs.values())}


@torch.no_grad()
def apply_shared_updates(optimizer, before):
    pairs = getattr(optimizer, "shared_parameter_updates", {})
    deltas = {donor: donor - old for donor, old in before.items()}
    for group in optimizer.param_groups:
        for target in group["params"]:
            if target not in pairs:
                continue
            donor = pairs[target]
            target.add_(deltas[donor])
            state = optimizer.state[target]
            for key, value in optimizer.state[donor].items():
                if key != "param_ema":
                    state[key].copy_(value)
            if "param_ema" in state:
                state["param_ema"].lerp_(target.to(state["param_ema"].dtype), 1 - group["ema"])
