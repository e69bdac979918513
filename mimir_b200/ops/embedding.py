"""Scaled token embedding ``scale * E[ids]`` (reference ``src/mimir/model/layers.py:103-104``)."""
from __future__ import annotations

import torch
import torch.nn.functional as F


def scaled_embedding(ids: torch.Tensor, weight: torch.Tensor, scale: float) -> torch.Tensor:
    return scale * F.embedding(ids, weight)
