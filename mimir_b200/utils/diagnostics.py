"""Opt-in experiment telemetry: JSONL records and measured parameter updates.

Reference behaviour: ``src/mimir/model/experiment_diagnostics.py:10-68``.
``ParameterUpdateProbe`` snapshots each rank's local shard on the host before the optimizer
step and, after it, reduces only four scalars per parameter (squared sums before/after, the
squared update and the element count) with one all-reduce: no full parameter is gathered.
Replicated parameters are counted once per replica, which cancels in every ratio reported.
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import torch
import torch.distributed as dist


def _finite(value):
    if isinstance(value, float) and not math.isfinite(value):
        return None
    if isinstance(value, dict):
        return {k: _finite(v) for k, v in value.items()}
    if isinstance(value, list):
        return [_finite(v) for v in value]
    return value


def append_jsonl(path, record: dict) -> None:
    """Append one JSON line (non-finite floats become null).  Callers are rank 0."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("a") as f:
        f.write(json.dumps(_finite(record), allow_nan=False) + "\n")
        f.flush()


def _local(t):
    return t.to_local() if hasattr(t, "to_local") else t


class ParameterUpdateProbe:
    def __init__(self, model):
        self.parameters = list(model.named_parameters())
        self.before = {n: _local(p).detach().to("cpu", copy=True) for n, p in self.parameters}

    @torch.no_grad()
    def finish(self, device) -> list[dict]:
        rows = []
        for name, p in self.parameters:
            before = self.before.pop(name).double()
            after = _local(p).detach().to("cpu", torch.float64)
            rows.append([before.square().sum().item(), after.square().sum().item(),
                         (after - before).square().sum().item(), before.numel()])
        values = torch.tensor(rows, device=device, dtype=torch.float64)
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(values)
        out = []
        for (name, _), (w2, a2, u2, n) in zip(self.parameters, values.tolist()):
            out.append({"parameter": name, "weight_rms_before": math.sqrt(w2 / max(n, 1)),
                        "weight_rms_after": math.sqrt(a2 / max(n, 1)), "update_rms": math.sqrt(u2 / max(n, 1)),
                        "update_to_weight": math.sqrt(u2 / max(w2, 1e-300))})
        self.parameters.clear()
        return out
