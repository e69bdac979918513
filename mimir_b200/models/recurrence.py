"""Hierarchical recurrent backbone (HRM v1): an H stack and an L stack re-applied in nested cycles.

Reference behaviour: ``src/mimir/model/recurrence.py:14-158``.  Per forward, L runs
``H_cycles * L_cycles`` times and H runs ``H_cycles`` times; only the last ``bp_steps``
invocations record autograd state (truncated BPTT).  H receives the first
``min(H_cycles, bp_steps - 1)`` backward slots, L the remainder.
"""
from __future__ import annotations

from typing import Any, Dict, Optional, Tuple

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


class RecurrentBlock(nn.Module):
    """A stack whose input is ``hidden + injection``."""

    def __init__(self, config: TransformerConfig) -> None:
        super().__init__()
        self.core = Transformer(config)

    def create_cache(self, **kwargs):
        return self.core.create_cache(**kwargs)

    def forward(self, hidden: Tensor, injection: Tensor, stability_diagnostics=None, stability_scope=None,
                **kwargs) -> Tensor:
        combined = hidden + injection
        if stability_diagnostics is not None:
            if stability_scope is None:
                raise ValueError("stability_scope is required when diagnostics are enabled")
            for name, t in (("hidden", hidden), ("injection", injection), ("combined", combined)):
                stability_diagnostics.record_tensor(f"recurrent/{stability_scope}/{name}", t, record_gradient=True)
            stability_diagnostics.record_pair(f"recurrent/{stability_scope}/hidden_injection", hidden, injection)
        out = self.core(combined, stability_diagnostics=stability_diagnostics, stability_scope=stability_scope,
                        **kwargs)
        if stability_diagnostics is not None:
            value = out[1] if isinstance(out, tuple) else out
            stability_diagnostics.record_tensor(f"recurrent/{stability_scope}/output", value, record_gradient=True)
        return out


def truncated_bptt_split(h_cycles: int, bp_steps: int) -> tuple[int, int]:
    """(H backward invocations, L backward invocations) for the v1 backbone."""
    h = min(h_cycles, bp_steps - 1)
    return h, bp_steps - h


class RecurrentBackbone(nn.Module):
    def __init__(self, config_dict: dict) -> None:
        super().__init__()
        config = RecurrentConfig(**config_dict)
        if config.half_layers:
            assert config.n_layers % 2 == 0, "n_layers must be divisible by 2."
            config.n_layers //= 2
        # Construction order fixes RNG consumption: H stack, L stack, then zL_init.
        self.H_level = RecurrentBlock(TransformerConfig(**(config.model_dump() | config.H_override)))
        self.L_level = RecurrentBlock(config)
        self.H_cycles = config.H_cycles
        self.L_cycles = config.L_cycles
        self.bp_warmup_ratio = config.bp_warmup_ratio
        self.bp_min_steps = config.bp_min_steps
        self.bp_max_steps = config.bp_max_steps
        self.hidden_size = config.hidden_size
        self.head_hint = self.H_level.core.head_hint
        self.zL_init = nn.Buffer(trunc_normal_init_(torch.empty(config.hidden_size,
                                                                dtype=getattr(torch, config.fwd_bwd_dtype)), std=1.0),
                                 persistent=True)

    def create_cache(self, **kwargs):
        return dict(H=[self.H_level.create_cache(**kwargs) for _ in range(self.H_cycles)],
                    L=[self.L_level.create_cache(**kwargs) for _ in range(self.H_cycles * self.L_cycles)])

    def forward(self, carry: None, x: Tensor, cache=None, bp_steps: int = 2, stability_diagnostics=None,
                **seq_info) -> Tuple[None, Tensor]:
        z_H, z_L = x, self.zL_init
        h_bp, l_bp = truncated_bptt_split(self.H_cycles, bp_steps)
        total_l = self.H_cycles * self.L_cycles
        grad = torch.is_grad_enabled()
        for i in range(self.H_cycles):
            for k in range(i * self.L_cycles, (i + 1) * self.L_cycles):
                with torch.set_grad_enabled(grad and k >= total_l - l_bp):
                    z_L = self.L_level(z_L, z_H, **seq_info, cache=cache["L"][k] if cache is not None else None,
                                       stability_diagnostics=stability_diagnostics,
                                       stability_scope=f"L/cycle_{k:03d}" if stability_diagnostics is not None else None)
            with torch.set_grad_enabled(grad and i >= self.H_cycles - h_bp):
                z_H = self.H_level(z_H, z_L, **seq_info, cache=cache["H"][i] if cache is not None else None,
                                   stability_diagnostics=stability_diagnostics,
                                   stability_scope=f"H/cycle_{i:03d}" if stability_diagnostics is not None else None)
        return None, z_H

    def compute_train_extra_args(self, train_state: Any) -> dict[str, Any]:
        if self.bp_warmup_ratio == 0:
            return dict(bp_steps=self.bp_max_steps)
        progress = min(1, train_state.step / (train_state.total_steps * self.bp_warmup_ratio))
        return dict(bp_steps=self.bp_min_steps + int(progress * (self.bp_max_steps - self.bp_min_steps)))

    def initial_carry(self, batch_size: int, dtype: torch.dtype) -> None:
        return None
