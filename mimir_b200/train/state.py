"""Mutable training state (reference ``src/mimir/training/state.py:10-31``)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Optional

import torch
from torch import nn


@dataclass
class TrainState:
    model: nn.Module
    carry: Optional[Any]
    optim: Any
    step: int
    total_steps: int
    fwd_bwd_dtype: torch.dtype
    use_cuda_autocast: bool


@dataclass
class ResumeState:
    tag: str
    step: int
    start_epoch: int
    skip_batches: int
    start_row_cursor: Optional[int] = None
    resume_mode: str = "batch"
