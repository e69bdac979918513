"""Goldfish loss: deterministically drop about 1/k supervised labels by a context hash.

Reference: ``src/mimir/model/goldfish_loss.py:34-124``.  For each token the hash XORs,
over the previous ``context_width`` positions of the same packed sequence, a splitmix64
finaliser of ``token*c0 + position*c1 + seed*c2 + offset*c3``; the label is dropped when
``|hash| mod k == 0``.  The mixing constants are the public splitmix64 / golden-ratio
constants and must stay fixed for runs to be reproducible across implementations.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Literal, Optional

import torch
from torch import Tensor

from mimir_b200.models.common import IGNORE_LABEL_ID

GoldfishStrategy = Literal["hash"]

_MIX_CONSTANTS = (0x9E3779B185EBCA87, 0xC2B2AE3D27D4EB4F, 0x165667B19E3779F9, 0x85EBCA77C2B2AE63)
_SPLITMIX = (0xBF58476D1CE4E5B9, 0x94D049BB133111EB)


def _signed(v: int) -> int:
    v &= (1 << 64) - 1
    return v - (1 << 64) if v >= (1 << 63) else v


@dataclass(frozen=True)
class GoldfishLossConfig:
    strategy: Optional[GoldfishStrategy] = None
    k: int = 50
    context_width: int = 50
    seed: int = 0

    def enabled(self) -> bool:
        return self.strategy is not None

    def validate(self) -> None:
        if self.strategy is None:
            return
        if self.strategy != "hash":
            raise ValueError(f"Unsupported Goldfish strategy: {self.strategy}")
        if self.k < 2:
            raise ValueError("Goldfish k must be >= 2")
        if self.context_width < 1:
            raise ValueError("Goldfish context_width must be >= 1")


def _splitmix(x: Tensor) -> Tensor:
    x = x ^ (x >> 30)
    x = x * _signed(_SPLITMIX[0])
    x = x ^ (x >> 27)
    x = x * _signed(_SPLITMIX[1])
    return x ^ (x >> 31)


def goldfish_drop_mask(inputs: Tensor, supervised: Tensor, cu_seqlens: Tensor, k: int, context_width: int,
                       seed: int) -> Tensor:
    from mimir_b200.ops._ext import ext, kernels_enabled
    if kernels_enabled(inputs) and inputs.dim() == 1 and cu_seqlens.dtype == torch.int32:
        # One CUDA kernel (csrc/goldfish.cu): same int64 arithmetic, no host synchronisation.
        return ext().goldfish_mask(inputs.contiguous(), supervised.contiguous(), cu_seqlens.contiguous(), k,
                                   context_width, seed, [_signed(v) for v in _MIX_CONSTANTS + _SPLITMIX])
    return goldfish_drop_mask_reference(inputs, supervised, cu_seqlens, k, context_width, seed)


def goldfish_drop_mask_reference(inputs: Tensor, supervised: Tensor, cu_seqlens: Tensor, k: int,
                                 context_width: int, seed: int) -> Tensor:
    """The PyTorch formulation (one vectorised pass per context offset and sequence)."""
    c_tok, c_pos, c_seed, c_off = (torch.tensor(_signed(v), dtype=torch.int64, device=inputs.device)
                                   for v in _MIX_CONSTANTS)
    bounds = cu_seqlens.detach().cpu().tolist()
    drop = torch.zeros_like(supervised, dtype=torch.bool)
    for start, end in zip(bounds[:-1], bounds[1:]):
        if end <= start:
            continue
        n = end - start
        tok = inputs[start:end].to(torch.int64)
        pos = torch.arange(n, device=inputs.device, dtype=torch.int64)
        h = torch.zeros(n, device=inputs.device, dtype=torch.int64)
        for off in range(1, min(context_width, n) + 1):
            ctx = torch.zeros_like(h)
            ctx[off:] = tok[:-off] * c_tok + (pos[:-off] + off) * c_pos
            h ^= _splitmix(ctx + seed * c_seed + off * c_off)
        drop[start:end] = supervised[start:end] & (torch.remainder(h.abs(), k) == 0)
    return drop


def apply_goldfish_loss_mask(labels: Tensor, inputs: Tensor, cu_seqlens: Tensor, config: GoldfishLossConfig):
    """Return ``(labels with drops set to -100, supervised mask)``."""
    config.validate()
    if not config.enabled():
        return labels, labels != IGNORE_LABEL_ID
    supervised = labels != IGNORE_LABEL_ID
    out = labels.clone()
    out[goldfish_drop_mask(inputs, supervised, cu_seqlens, config.k, config.context_width, config.seed)] = IGNORE_LABEL_ID
    return out, out != IGNORE_LABEL_ID
