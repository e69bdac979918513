"""Global-norm gradient clipping reported in mean-gradient units.

Reference: ``src/mimir/model/gradient_clipping.py:28-65``.  FSDP2 here reduces gradients
with SUM (no division), so thresholds and reported norms are divided by
``summed_gradient_scale`` (the world size) to stay comparable with DDP/single-GPU runs.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable

import torch
from torch import Tensor, nn


@dataclass(frozen=True)
class GradientClipMetrics:
    total_norm: Tensor
    clip_coefficient: Tensor
    clipped: Tensor


def _local(value: Tensor) -> Tensor:
    to_local = getattr(value, "to_local", None)
    return (to_local() if callable(to_local) else value).detach()


def clip_grad_norm_mean_units(parameters: Iterable[nn.Parameter], *, max_norm: float,
                              summed_gradient_scale: float = 1.0) -> GradientClipMetrics:
    if max_norm <= 0:
        raise ValueError("max_norm must be positive")
    if summed_gradient_scale <= 0:
        raise ValueError("summed_gradient_scale must be positive")
    raw_max = max_norm * summed_gradient_scale
    raw_norm = _local(torch.nn.utils.clip_grad_norm_(list(parameters), max_norm=raw_max, norm_type=2.0,
                                                     error_if_nonfinite=True))
    norm = raw_norm / summed_gradient_scale
    coeff = torch.clamp(raw_norm.new_tensor(raw_max) / (raw_norm + 1e-6), max=1.0)
    clipped = (norm > norm.new_tensor(max_norm)).to(norm.dtype)
    return GradientClipMetrics(total_norm=norm, clip_coefficient=coeff, clipped=clipped)
