"""Language-model head: scaled embedding, backbone, untied unembedding, fp32 CE and metrics.

Reference behaviour: ``src/mimir/model/lm_head.py:23-110``.  The loss is the fp32
cross-entropy *sum* divided by the (all-reduced, averaged) count of supervised tokens, so
that averaging gradients over ranks yields the global token mean.  Metrics are
``(sum, count)`` pairs: loss, accuracy, exact (whole-sequence) accuracy and the Goldfish
drop rate.

On CUDA the unembedding and the loss run as one fused op
(:func:`mimir_b200.ops.linear_cross_entropy`) that never materialises fp32 logits.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
from pydantic import BaseModel
from torch import nn

from mimir_b200 import ops
from mimir_b200.models.common import packing_sequence_sum
from mimir_b200.models.goldfish import GoldfishLossConfig, GoldfishStrategy, apply_goldfish_loss_mask
from mimir_b200.models.layers import LinearInit, ScaledEmbeddingInit


class LMHeadConfig(BaseModel):
    vocab_size: int
    goldfish_strategy: Optional[GoldfishStrategy] = None
    goldfish_k: int = 50
    goldfish_context_width: int = 50
    goldfish_seed: int = 0


class LMHead(nn.Module):
    def __init__(self, model: nn.Module, config_dict: dict) -> None:
        super().__init__()
        self.model = model
        cfg = LMHeadConfig(**{k: v for k, v in config_dict.items() if k in LMHeadConfig.model_fields})
        self.goldfish_config = GoldfishLossConfig(strategy=cfg.goldfish_strategy, k=cfg.goldfish_k,
                                                  context_width=cfg.goldfish_context_width, seed=cfg.goldfish_seed)
        self.goldfish_config.validate()
        hint = self.model.head_hint
        self.embed_tokens = ScaledEmbeddingInit(cfg.vocab_size, hint["in"]["dim"], init_std=hint["in"]["init_std"])
        self.lm_head = LinearInit(hint["out"]["dim"], cfg.vocab_size, bias=False, init_std=hint["out"]["init_std"])
        if config_dict.get("specialist_training", False) or config_dict.get("specialist_router_calibration", False):
            from mimir_b200.models.specialists import configure_specialist
            configure_specialist(self, router_only=config_dict.get("specialist_router_calibration", False))

    def create_cache(self, **kwargs):
        return self.model.create_cache(**kwargs)

    def compute_train_extra_args(self, train_state):
        return self.model.compute_train_extra_args(train_state)

    def forward(self, carry, batch: dict, **kwargs):
        x = self.embed_tokens(batch["inputs"])
        if getattr(self.model, "ngram_enabled", False):
            kwargs["token_ids"] = batch["inputs"]
        diag = kwargs.get("stability_diagnostics")
        if diag is not None:
            diag.record_tensor("activation/model/input_embedding", x, record_gradient=True)
        new_carry, hidden = self.model(carry, x, **{k: v for k, v in batch.items() if k not in ("inputs", "labels")},
                                       **kwargs)
        if "labels" not in batch:
            return new_carry, self.lm_head(hidden)

        raw_labels = batch["labels"]
        labels, masks = apply_goldfish_loss_mask(raw_labels, batch["inputs"], batch["cu_seqlens"], self.goldfish_config)
        if diag is not None:
            logits = self.lm_head(hidden)
            diag.record_tensor("activation/model/logits", logits, record_gradient=True)
            loss_sum, is_correct = ops.linear_cross_entropy_reference(hidden, self.lm_head.weight, labels)
        else:
            loss_sum, is_correct = ops.linear_cross_entropy(hidden, self.lm_head.weight, labels)
        divisor = masks.sum().to(torch.float32)
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(divisor, op=dist.ReduceOp.AVG)
        with torch.no_grad():
            local_valid = masks.sum()
            seq_correct = packing_sequence_sum(is_correct, batch["cu_seqlens"])
            seq_valid = packing_sequence_sum(masks, batch["cu_seqlens"])
            seq_ok = seq_valid > 0
            metrics = {
                "loss": (loss_sum.detach(), local_valid),
                "accuracy": (is_correct.sum(), local_valid),
                "exact_accuracy": (((seq_correct == seq_valid) & seq_ok).sum(), seq_ok.sum()),
            }
            if self.goldfish_config.enabled():
                raw_valid = (raw_labels != -100).sum()
                metrics["goldfish_drop_rate"] = (raw_valid - local_valid, raw_valid)
        return new_carry, loss_sum / divisor, metrics
