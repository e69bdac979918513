"""Shared model helpers (reference: ``src/mimir/model/common.py:8-70``)."""
from __future__ import annotations

from dataclasses import dataclass

import torch.nn.functional as F
from torch import Tensor

IGNORE_LABEL_ID = -100
# Scale that restores unit variance after folding a standard normal into (-3, 3).
_FMOD3_VARIANCE_FIX = 1.014762601732121


def trunc_normal_init_(tensor: Tensor, std: float = 1.0) -> Tensor:
    """Approximately truncated normal: draw N(0,1), fold into (-3, 3) with fmod, rescale.

    The RNG consumption (one ``normal_`` per tensor) is part of the checkpoint-parity
    contract: models built from the same seed must get identical weights.
    """
    return tensor.normal_().fmod_(3.0).mul_(_FMOD3_VARIANCE_FIX * std)


def packing_sequence_sum(x: Tensor, cu_seqlens: Tensor) -> Tensor:
    """Per-sequence sums of a packed 1-D tensor given cumulative boundaries."""
    csum = F.pad(x.cumsum(0), (1, 0))
    return csum[cu_seqlens[1:]] - csum[cu_seqlens[:-1]]


@dataclass
class WrappedTensor:
    """Host scalar hidden from FSDP/DDP input casting (e.g. ``numseqs``)."""
    value: Tensor


def wrap_tensor(value: Tensor) -> WrappedTensor:
    return WrappedTensor(value)


def unwrap_tensor(value):
    return value.value if isinstance(value, WrappedTensor) else value


def find_multiple(a: int, b: int) -> int:
    return (-(a // -b)) * b
