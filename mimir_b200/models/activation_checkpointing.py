"""Selective activation checkpointing of transformer blocks without changing parameter FQNs.

Reference: ``src/mimir/model/activation_checkpointing.py:10-36`` — modes ``full``,
``l_only`` and ``h_only``; blocks of v2 models that take non-tensor keyword inputs are
wrapped with a non-reentrant ``torch.utils.checkpoint`` call instead of the composable API.
"""
from __future__ import annotations

import functools

import torch
from torch import nn
from torch.distributed._composable import checkpoint
from torch.utils.checkpoint import checkpoint as checkpoint_fn

from mimir_b200.models.transformer import TransformerBlock


def apply_activation_checkpointing(model: nn.Module, mode: str) -> set:
    chosen = []
    for name, module in model.named_modules():
        if not isinstance(module, TransformerBlock):
            continue
        parts = name.split(".")
        if mode == "full" or (mode == "l_only" and "L_level" in parts) or (mode == "h_only" and "H_level" in parts):
            chosen.append(module)
    for block in chosen:
        if getattr(block, "_v2_explicit_checkpoint", False):
            if not getattr(block, "_v2_checkpoint_installed", False):
                block.forward = _explicit(block.forward)
                block._v2_checkpoint_installed = True
        else:
            checkpoint(block)
    return set(chosen)


def _explicit(forward):
    @functools.wraps(forward)
    def wrapped(*args, **kwargs):
        if not torch.is_grad_enabled():
            return forward(*args, **kwargs)
        return checkpoint_fn(forward, *args, use_reentrant=False, **kwargs)
    return wrapped
