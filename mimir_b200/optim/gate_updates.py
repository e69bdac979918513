"""Donor updates for invocation gates that receive no gradient in a step.

Behavioural reference: ``src/mimir/model/gate_updates.py:6-40``.  A gate whose level is outside
the truncated-BPTT window this step gets no gradient.  Instead of standing still it moves by the
same amount as its level's first active gate (the "donor"), and it adopts the donor's optimizer
moments, so the update history it carries into a later, wider window is the one that moved it.
Only its parameter EMA stays its own (advanced towards the moved value).

Usage inside an optimizer's ``step``::

    with donor_updates(self) as passive:
        for p in params:
            if p in passive or p.grad is None:
                continue
            ...  # the regular update

The donors' values are recorded on entry; on a clean exit every passive gate receives its
donor's parameter change.
"""
from __future__ import annotations

from contextlib import contextmanager
from typing import Iterator

import torch


def _mapping(optimizer) -> dict:
    return getattr(optimizer, "shared_parameter_updates", None) or {}


def _check(optimizer, mapping: dict) -> None:
    donors = set(mapping.values())
    for target, donor in mapping.items():
        if donor is target or donor in mapping:
            raise ValueError("Gate donors must be active, independent parameters")
        # The invocation schedule decides which gates are passive; an FSDP zero gradient on a
        # passive gate is harmless, but a donor without a gradient means the schedule is wrong.
        if donor.grad is None:
            raise RuntimeError("Gate donor mapping disagrees with gradient eligibility")
        if donor.shape != target.shape:
            raise ValueError("Gate donor and target shapes must match")
        if any(p not in optimizer.state for p in (target, donor)):
            raise ValueError("Gate parameters must belong to this optimizer")
    del donors


def _group_ema(optimizer) -> dict:
    """EMA decay of each parameter's group, keyed by the parameter."""
    return {p: group.get("ema") for group in optimizer.param_groups for p in group["params"]}


@torch.no_grad()
def _follow_donors(optimizer, mapping: dict, before: dict) -> None:
    moved = {donor: donor - value for donor, value in before.items()}
    ema_decay = _group_ema(optimizer)
    for target, donor in mapping.items():
        if target not in ema_decay:
            continue
        target.add_(moved[donor])
        mine, theirs = optimizer.state[target], optimizer.state[donor]
        for slot, value in theirs.items():
            if slot == "param_ema":
                continue
            if torch.is_tensor(value):
                mine[slot].copy_(value)
            else:
                mine[slot] = value
        ema = mine.get("param_ema")
        if ema is not None:
            ema.lerp_(target.to(ema.dtype), 1 - ema_decay[target])


@contextmanager
def donor_updates(optimizer) -> Iterator[frozenset]:
    """Yield the passive gates (to be skipped by the regular update); move them on exit."""
    mapping = _mapping(optimizer)
    if not mapping:
        yield frozenset()
        return
    _check(optimizer, mapping)
    with torch.no_grad():
        before = {donor: donor.detach().clone() for donor in set(mapping.values())}
    yield frozenset(mapping)
    _follow_donors(optimizer, mapping, before)
