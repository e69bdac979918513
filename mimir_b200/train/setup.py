"""Model, optimizer and data-loader construction.

Reference behaviour: ``src/mimir/training/setup.py:27-243``: the model config is the arch
config plus dataset metadata (vocab size, max_seq_len) and the data config; the LM head
wraps Mimir2; optional activation checkpointing; FSDP2/HSDP or DDP wrapping; AdamATan2 or
MuonAdamW with per-module learning-rate scales and an EMA slot whose dtype is fp32 when
parameters are bf16.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
from torch import nn

from mimir_b200.models import LMHead, Mimir2
from mimir_b200.optim.adam_atan2 import AdamATan2
from mimir_b200.optim.module_lr import configured_module_rates, module_lr_scales
from mimir_b200.parallel.fsdp import optimizer_ema_dtype, wrap_ddp, wrap_fsdp
from mimir_b200.train.state import TrainState


def model_config_dict(config, metadata: dict) -> dict:
    """Arch config merged with dataset metadata and data config (what the model sees)."""
    return (config.arch.model_dump() | dict(metadata) | config.data.model_dump()
            | {"fwd_bwd_dtype": config.fwd_bwd_dtype, "activation_checkpointing": config.activation_checkpointing})


def create_model_and_optimizer(config, metadata: dict, device: torch.device, local_batch_size: int = 0):
    model_cfg = model_config_dict(config, metadata)
    fwd_bwd_dtype = getattr(torch, config.fwd_bwd_dtype)
    if (config.data.homogeneous_categories or config.data.routing_categories) and config.arch.name != "mimir2":
        raise ValueError("Metadata-guided routing currently requires HRM v2")
    if config.fsdp_wrap_policy == "recurrent_level" and (
            model_cfg.get("gates_enabled") or model_cfg.get("mos_num_experts", 1) > 1
            or model_cfg.get("h_memory_branches", 1) > 1 or model_cfg.get("l_memory_branches", 1) > 1):
        raise ValueError("V2 direct level parameter access requires fsdp_wrap_policy=transformer_block")
    with torch.device(device):
        backbone = Mimir2(model_cfg)
        carry = backbone.initial_carry(local_batch_size, dtype=fwd_bwd_dtype)
        model: nn.Module = LMHead(backbone, model_cfg)
    if config.initialize_from:
        from mimir_b200.ckpt.importer import initialize_weights
        initialize_weights(model, config.initialize_from, upcycle=config.arch.upcycle_from_dense)
    checkpointed: set = set()
    if config.activation_checkpointing != "none":
        from mimir_b200.models.activation_checkpointing import apply_activation_checkpointing
        checkpointed = apply_activation_checkpointing(model, config.activation_checkpointing)
        if not checkpointed:
            raise ValueError(f"activation_checkpointing={config.activation_checkpointing} found no matching blocks")
    distributed = dist.is_available() and dist.is_initialized()
    if config.distributed_strategy == "replicated":
        return _replicated_model_and_optimizer(config, model, carry, device, fwd_bwd_dtype)
    if distributed:
        if config.distributed_strategy == "fsdp":
            model = wrap_fsdp(model, config, fwd_bwd_dtype, checkpointed)
        elif config.distributed_strategy == "ddp":
            model = wrap_ddp(model, config, fwd_bwd_dtype, device)
        elif config.distributed_strategy != "none":
            raise ValueError(f"Unsupported distributed_strategy: {config.distributed_strategy}")
    elif config.distributed_strategy not in ("fsdp", "none"):
        raise RuntimeError(f"distributed_strategy={config.distributed_strategy} requires torchrun/distributed training")

    options = {}
    params = model.parameters()
    cls = AdamATan2
    if config.optimizer == "muon":
        from mimir_b200.optim.muon import MuonAdamW
        cls, params = MuonAdamW, model.named_parameters()
        options = dict(momentum=config.muon_momentum, ns_steps=config.muon_ns_steps, muon_lr_scale=config.muon_lr_scale)
    optim = cls(params, **options, lr=0.0, betas=(config.beta1, config.beta2), weight_decay=config.weight_decay,
                ema=config.ema, ema_dtype=optimizer_ema_dtype(config),
                parameter_lr_scales=module_lr_scales(model, config.lr, configured_module_rates(config)))
    return model, carry, optim


def _replicated_model_and_optimizer(config, model, carry, device, fwd_bwd_dtype):
    """Replicated bf16 weights + sharded fp32 master/optimizer, fused peer-memory step."""
    from mimir_b200.parallel.replicated import ReplicatedAdamATan2, ReplicatedMuonAdamW, wrap_replicated
    if config.optimizer not in ("adam_atan2", "muon"):
        raise ValueError(f"distributed_strategy=replicated does not implement optimizer={config.optimizer}")
    if config.arch.gates_enabled:
        raise ValueError("distributed_strategy=replicated does not implement shared gate-donor updates")
    scales = module_lr_scales(model, config.lr, configured_module_rates(config))
    engine = wrap_replicated(model, device, fwd_bwd_dtype)
    common = dict(lr=0.0, betas=(config.beta1, config.beta2), weight_decay=config.weight_decay, ema=config.ema,
                  ema_dtype=torch.float32, parameter_lr_scales=scales)
    if config.optimizer == "muon":
        optim = ReplicatedMuonAdamW(engine, momentum=config.muon_momentum, ns_steps=config.muon_ns_steps,
                                    muon_lr_scale=config.muon_lr_scale, **common)
    else:
        optim = ReplicatedAdamATan2(engine, **common)
    return model, carry, optim


def make_train_state(config, model, carry, optim, total_steps: int, device: torch.device) -> TrainState:
    fwd_bwd_dtype = getattr(torch, config.fwd_bwd_dtype)
    return TrainState(model=model, carry=carry, optim=optim, step=0, total_steps=total_steps,
                      fwd_bwd_dtype=fwd_bwd_dtype,
                      use_cuda_autocast=(config.distributed_strategy == "ddp" and device.type == "cuda"
                                         and fwd_bwd_dtype != torch.float32))


def local_batch_tokens(config, world_size: int) -> int:
    divisor = world_size * config.gradient_accumulation_steps
    if config.global_batch_size % divisor:
        raise ValueError(f"Global batch size {config.global_batch_size} must be divisible by world_size * "
                         f"gradient_accumulation_steps ({world_size} * {config.gradient_accumulation_steps}).")
    return config.global_batch_size // divisor


def create_dataloader(config, local_batch_size: int, rank: int, world_size: int, drop_last_batch: bool = True,
                      path: Optional[str] = None, seed_offset: int = 0):
    from torch.utils.data import DataLoader

    from mimir_b200.data.corpus import V1Dataset, V1DatasetConfig
    dataset = V1Dataset(V1DatasetConfig(seed=config.seed + seed_offset, dataset_path=path or config.data.path,
                                        batch_max_length=local_batch_size, drop_last_batch=drop_last_batch,
                                        target_only=config.data.target_only, rank=rank, num_replicas=world_size,
                                        homogeneous_categories=config.data.homogeneous_categories,
                                        routing_categories=config.data.routing_categories))
    generator = torch.Generator()
    generator.manual_seed(config.seed + rank)
    loader = DataLoader(dataset, batch_size=None, num_workers=1, prefetch_factor=config.dataloader_prefetch_factor,
                        pin_memory=torch.cuda.is_available(), persistent_workers=False, generator=generator)
    return loader, dataset.metadata
