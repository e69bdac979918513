"""Token -> expert dispatch plans for sparse MoE.

Reference: ``src/mimir/model/expert_mixtures.py:92-104`` builds each expert's token list
with ``nonzero`` per expert.  Here one stable sort of the (expert, token) selections
yields every expert's list (ascending token order, as the reference's ``nonzero``) and the
per-expert counts in a single host transfer.
"""
from __future__ import annotations

import torch


class MoEPlan:
    def __init__(self, weights: torch.Tensor):
        n_experts = weights.shape[-1]
        selected = (weights != 0)
        token_ids = torch.arange(weights.shape[0], device=weights.device)
        pairs_e = torch.nonzero(selected.t(), as_tuple=False)  # [(expert, token)] sorted by expert then token
        self.tokens = pairs_e[:, 1].contiguous()
        counts = torch.bincount(pairs_e[:, 0], minlength=n_experts)
        self.offsets = [0] + torch.cumsum(counts, 0).tolist()
        del token_ids

    def indices(self, expert: int) -> torch.Tensor:
        return self.tokens[self.offsets[expert]:self.offsets[expert + 1]]


def moe_plan(weights: torch.Tensor) -> MoEPlan:
    return MoEPlan(weights)
