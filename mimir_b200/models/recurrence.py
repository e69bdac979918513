"""Hierarchical recurrent backbone (HRM v1): an H stack and an L stack applied in nested cycles.

Behavioural reference: ``src/mimir/model/recurrence.py:14-158``.  One forward is a fixed
schedule of stack invocations: for every H cycle, ``L_cycles`` calls of the L stack (input:
its own state plus the H state) followed by one call of the H stack (its state plus the L
state).  Truncated BPTT: only the last ``bp_steps`` invocations record autograd state; the H
stack gets ``min(H_cycles, bp_steps - 1)`` of them (the latest H calls) and the L stack the
rest, so at least one L call is always differentiated.

Module and buffer names (``H_level``, ``L_level``, ``core``, ``zL_init``) and the construction
order (H stack, L stack, then ``zL_init``: it fixes the RNG consumption) are the checkpoint
interface.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, Tuple

import torch
from torch import Tensor, nn

from mimir_b200.models.common import trunc_normal_init_
from mimir_b200.models.transformer import Transformer, TransformerConfig


class RecurrentConfig(TransformerConfig):
    half_layers: bool = False
    H_cycles: int
    L_cycles: int
    bp_warmup_ratio: float = 0.0
    bp_min_steps: int = 2
    bp_max_steps: int = 5
    fwd_bwd_dtype: str = "bfloat16"
    H_override: Dict[str, Any] = {}


def truncated_bptt_split(h_cycles: int, bp_steps: int) -> tuple[int, int]:
    """(H, L) invocations inside the backward window of ``bp_steps`` calls."""
    h = min(h_cycles, bp_steps - 1)
    return h, bp_steps - h


@dataclass(frozen=True)
class StackCall:
    level: str  # "H" or "L"
    slot: int   # the call's index within its level (its decode-cache slot)
    grad: bool  # inside the truncated-BPTT window


def invocation_schedule(h_cycles: int, l_cycles: int, bp_steps: int) -> list[StackCall]:
    h_window, l_window = truncated_bptt_split(h_cycles, bp_steps)
    first_l_grad, first_h_grad = h_cycles * l_cycles - l_window, h_cycles - h_window
    calls = []
    for i in range(h_cycles):
        calls.extend(StackCall("L", k, k >= first_l_grad) for k in range(i * l_cycles, (i + 1) * l_cycles))
        calls.append(StackCall("H", i, i >= first_h_grad))
    return calls


class RecurrentBlock(nn.Module):
    """A transformer stack applied to ``state + injection``."""

    def __init__(self, config: TransformerConfig) -> None:
        super().__init__()
        self.core = Transformer(config)

    def create_cache(self, **kwargs):
        return self.core.create_cache(**kwargs)

    @staticmethod
    def _record_inputs(diag, scope, state, injection, combined) -> None:
        if scope is None:
            raise ValueError("stability_scope is required when diagnostics are enabled")
        prefix = f"recurrent/{scope}"
        diag.record_tensor(f"{prefix}/hidden", state, record_gradient=True)
        diag.record_tensor(f"{prefix}/injection", injection, record_gradient=True)
        diag.record_tensor(f"{prefix}/combined", combined, record_gradient=True)
        diag.record_pair(f"{prefix}/hidden_injection", state, injection)

    def forward(self, hidden: Tensor, injection: Tensor, stability_diagnostics=None, stability_scope=None,
                **kwargs) -> Tensor:
        combined = hidden + injection
        if stability_diagnostics is not None:
            self._record_inputs(stability_diagnostics, stability_scope, hidden, injection, combined)
        out = self.core(combined, stability_diagnostics=stability_diagnostics, stability_scope=stability_scope,
                        **kwargs)
        if stability_diagnostics is not None:
            stability_diagnostics.record_tensor(f"recurrent/{stability_scope}/output",
                                                out[1] if isinstance(out, tuple) else out, record_gradient=True)
        return out


class RecurrentBackbone(nn.Module):
    def __init__(self, config_dict: dict) -> None:
        super().__init__()
        config = RecurrentConfig(**config_dict)
        if config.half_layers:
            assert config.n_layers % 2 == 0, "n_layers must be divisible by 2."
            config.n_layers //= 2
        self.H_level = RecurrentBlock(TransformerConfig(**(config.model_dump() | config.H_override)))
        self.L_level = RecurrentBlock(config)
        self.H_cycles, self.L_cycles = config.H_cycles, config.L_cycles
        self.bp_warmup_ratio = config.bp_warmup_ratio
        self.bp_min_steps, self.bp_max_steps = config.bp_min_steps, config.bp_max_steps
        self.hidden_size = config.hidden_size
        self.head_hint = self.H_level.core.head_hint
        init = torch.empty(config.hidden_size, dtype=getattr(torch, config.fwd_bwd_dtype))
        self.zL_init = nn.Buffer(trunc_normal_init_(init, std=1.0), persistent=True)

    def create_cache(self, **kwargs):
        return {"H": [self.H_level.create_cache(**kwargs) for _ in range(self.H_cycles)],
                "L": [self.L_level.create_cache(**kwargs) for _ in range(self.H_cycles * self.L_cycles)]}

    def forward(self, carry: None, x: Tensor, cache=None, bp_steps: int = 2, stability_diagnostics=None,
                **seq_info) -> Tuple[None, Tensor]:
        state = {"H": x, "L": self.zL_init}
        partner = {"H": "L", "L": "H"}
        stacks = {"H": self.H_level, "L": self.L_level}
        record = torch.is_grad_enabled()
        for call in invocation_schedule(self.H_cycles, self.L_cycles, bp_steps):
            scope = f"{call.level}/cycle_{call.slot:03d}" if stability_diagnostics is not None else None
            with torch.set_grad_enabled(record and call.grad):
                state[call.level] = stacks[call.level](
                    state[call.level], state[partner[call.level]], **seq_info,
                    cache=None if cache is None else cache[call.level][call.slot],
                    stability_diagnostics=stability_diagnostics, stability_scope=scope)
        return None, state["H"]

    def compute_train_extra_args(self, train_state: Any) -> dict[str, Any]:
        """``bp_steps`` grows linearly from ``bp_min_steps`` to ``bp_max_steps`` over the first
        ``bp_warmup_ratio`` of training (integer steps, rounded down)."""
        if self.bp_warmup_ratio == 0:
            return {"bp_steps": self.bp_max_steps}
        progress = min(1, train_state.step / (train_state.total_steps * self.bp_warmup_ratio))
        return {"bp_steps": self.bp_min_steps + int(progress * (self.bp_max_steps - self.bp_min_steps))}

    def initial_carry(self, batch_size: int, dtype: torch.dtype) -> None:
        return None
