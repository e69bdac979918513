"""Aux-loss-free expert load balancing, scoped to one optimizer step.

Reference: ``src/mimir/model/routing_balance.py:11-61`` (DeepSeek-V3 style).  During the
real forwards of a step (not activation-checkpoint replays) each balanced router's top-k
selections are counted; after a successful optimizer step the counts are summed over all
ranks (every rank participates, even with zero tokens) and each expert's selection bias
moves by ``rate * sign(mean_load - load)``.
"""
from __future__ import annotations

import inspect
from contextvars import ContextVar
from functools import wraps

import torch
import torch.distributed as dist

_ACTIVE: ContextVar = ContextVar("mimir_b200_routing_balance", default=None)


@torch.compiler.disable
@torch.no_grad()
def record_load(router, mask):
    session = _ACTIVE.get()
    if session is not None and router.training and torch._C._current_graph_task_id() == -1:
        session.counts[router].add_(mask.detach().reshape(-1, router.n).sum(0))


def load_counter(router):
    """The int64 [n] count buffer a fused selection kernel may add this forward's selections to, or
    None when nothing is being recorded (no balance step, eval mode, or an activation replay)."""
    session = _ACTIVE.get()
    if session is not None and router.training and torch._C._current_graph_task_id() == -1:
        return session.counts[router]
    return None


class BalanceStep:
    def __init__(self, model):
        self.counts = {m: torch.zeros(m.n, dtype=torch.int64, device=m.selection_bias.device)
                       for m in model.modules() if getattr(m, "balance_enabled", False)}

    def __enter__(self):
        if _ACTIVE.get() is not None:
            raise RuntimeError("Nested routing balance steps are unsupported")
        self._token = _ACTIVE.set(self)
        return self

    def __exit__(self, *exc):
        _ACTIVE.reset(self._token)

    @torch.no_grad()
    def commit(self):
        if not self.counts:
            return
        # One collective for every router's counts instead of one per router.
        routers = list(self.counts)
        flat = torch.cat([self.counts[r] for r in routers])
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(flat, op=dist.ReduceOp.SUM)
        offset = 0
        for r in routers:
            load = flat[offset:offset + r.n].to(torch.float32)
            offset += r.n
            r.selection_bias.add_(r.balance_update_rate * torch.sign(load.mean() - load))


def balanced_optimizer_step(fn):
    """Decorator: open a balance session around a train step and commit it if the step ran."""
    signature = inspect.signature(fn)

    @wraps(fn)
    def wrapped(*args, **kwargs):
        bound = signature.bind(*args, **kwargs)
        state = bound.arguments["train_state"]
        if not any(getattr(m, "balance_enabled", False) for m in state.model.modules()):
            return fn(*args, **kwargs)
        with BalanceStep(state.model) as step:
            result = fn(*args, **kwargs)
            skipped = result[1] if fn.__name__ == "train_accumulated_batches" else False
            if bound.arguments.get("optimizer_step_enabled", True) and not skipped:
                step.commit()
            return result
    return wrapped
