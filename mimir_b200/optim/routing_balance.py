"""Aux-loss-free expert load balancing, one ledger per optimizer step.

Behavioural reference: ``src/mimir/model/routing_balance.py:11-61`` (the DeepSeek-V3 bias
update).  While a step's real forwards run, every balanced router adds its top-k selections to a
ledger; activation-checkpoint replays (forwards inside the backward's graph task) are not new
routing decisions and are not counted.  After a step whose optimizer update actually ran, the
counts are summed over all ranks (every rank joins, even one that routed no tokens) and each
expert's selection bias moves by ``rate * sign(mean load - its load)``.

The ledger keeps the counts of every balanced router in one flat int64 buffer, so the
cross-rank sum is a single all-reduce per step; each router reads and writes its own slice.
"""
from __future__ import annotations

import threading
from contextlib import contextmanager
from typing import Iterator, Optional

import torch
import torch.distributed as dist

_open = threading.local()  # the ledger of the step running on this thread, if any


def _replaying() -> bool:
    """True inside the backward's graph task (activation-checkpoint recomputation)."""
    return torch._C._current_graph_task_id() != -1


class RoutingLedger:
    def __init__(self, module: torch.nn.Module):
        self.routers = [m for m in module.modules() if getattr(m, "balance_enabled", False)]
        size = sum(r.n for r in self.routers)
        device = self.routers[0].selection_bias.device if self.routers else None
        self.flat = torch.zeros(size, dtype=torch.int64, device=device)
        self.slices, start = {}, 0
        for r in self.routers:
            self.slices[r] = self.flat[start:start + r.n]
            start += r.n

    def counts(self, router) -> torch.Tensor:
        return self.slices[router]

    @torch.no_grad()
    def commit(self) -> None:
        """Sum the counts over all ranks and move every balanced router's selection bias."""
        if not self.routers:
            return
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM)
        for r in self.routers:
            load = self.slices[r].to(torch.float32)
            r.selection_bias.add_(torch.sign(load.mean() - load) * r.balance_update_rate)


def _recording(router) -> Optional[RoutingLedger]:
    ledger = getattr(_open, "ledger", None)
    if ledger is None or not router.training or _replaying():
        return None
    return ledger


@contextmanager
def routing_balance(module: torch.nn.Module) -> Iterator[RoutingLedger]:
    """Open the step's ledger for the balanced routers of ``module``; the caller commits it once
    the optimizer update has run."""
    if getattr(_open, "ledger", None) is not None:
        raise RuntimeError("Nested routing balance steps are unsupported")
    ledger = RoutingLedger(module)
    _open.ledger = ledger
    try:
        yield ledger
    finally:
        _open.ledger = None


@torch.compiler.disable
@torch.no_grad()
def record_load(router, mask: torch.Tensor) -> None:
    """Add a forward's boolean selection mask ``[..., n]`` to the open ledger."""
    ledger = _recording(router)
    if ledger is not None:
        ledger.counts(router).add_(mask.detach().reshape(-1, router.n).sum(0))


def load_counter(router) -> Optional[torch.Tensor]:
    """The int64 ``[n]`` slice a fused selection kernel adds this forward's selections to, or None
    when nothing is recorded (no open step, eval mode, or an activation replay)."""
    ledger = _recording(router)
    return None if ledger is None else ledger.counts(router)


def has_balanced_routers(module: torch.nn.Module) -> bool:
    return any(getattr(m, "balance_enabled", False) for m in module.modules())
