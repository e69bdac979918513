"""Data-parallel wrapping: FSDP2 (ZeRO-3), HSDP (2-D mesh) and DDP.

Reference behaviour: ``src/mimir/training/distributed.py:14-125`` and
``src/mimir/training/setup.py:134-178``.  FSDP2 units are the transformer blocks (or
whole stacks with ``recurrent_level``) plus the root; parameters are gathered in the
compute dtype and gradients reduced in fp32 with SUM (divide factor 1 — the Adam-family
optimizers are scale invariant).  HSDP uses a ``(replicate, shard)`` mesh whose shard
degree must divide the world and fit in a node.

NCCL does the collectives here; this is the baseline against which the replicated-weight
engine (:mod:`mimir_b200.parallel.replicated`, one fused peer-memory update kernel per step)
is compared.
"""
from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist
from torch import nn
from torch.distributed.device_mesh import DeviceMesh, init_device_mesh
from torch.distributed.fsdp import FSDPModule, MixedPrecisionPolicy, fully_shard
from torch.nn.parallel import DistributedDataParallel

from mimir_b200.models.transformer import Transformer, TransformerBlock


def apply_fsdp(module: nn.Module, param_dtype: torch.dtype, *, mesh: Optional[DeviceMesh] = None,
               reshard_after_forward: bool = False):
    fully_shard(module, mesh=mesh,
                mp_policy=MixedPrecisionPolicy(param_dtype=param_dtype, reduce_dtype=torch.get_default_dtype()),
                reshard_after_forward=reshard_after_forward)
    assert isinstance(module, FSDPModule)
    if hasattr(module, "set_gradient_divide_factor"):
        module.set_gradient_divide_factor(1.0)
    else:  # older torch
        module.set_reduce_scatter_divide_factor(1.0)
    if hasattr(module, "set_force_sum_reduction_for_comms"):
        module.set_force_sum_reduction_for_comms(True)


def create_fsdp_mesh(config) -> Optional[DeviceMesh]:
    degree = config.fsdp_shard_degree
    if degree is None:
        return None
    if not dist.is_available() or not dist.is_initialized():
        raise RuntimeError("fsdp_shard_degree requires initialized distributed training")
    world = dist.get_world_size()
    local = int(os.environ.get("LOCAL_WORLD_SIZE", torch.cuda.device_count()))
    if degree > local:
        raise ValueError(f"fsdp_shard_degree={degree} exceeds LOCAL_WORLD_SIZE={local}")
    if world % degree:
        raise ValueError(f"WORLD_SIZE={world} must be divisible by fsdp_shard_degree={degree}")
    if degree == world:
        return None
    device_type = "cuda" if torch.cuda.is_available() else "cpu"
    return init_device_mesh(device_type, (world // degree, degree), mesh_dim_names=("replicate", "shard"))


def fsdp_reshard_after_forward(config, *, checkpointed: bool) -> bool:
    if config.fsdp_reshard_after_forward is not None:
        return config.fsdp_reshard_after_forward
    return checkpointed


def fsdp_wrap_modules(model: nn.Module, policy: str) -> list[nn.Module]:
    if policy == "transformer_block":
        return [m for m in model.modules() if isinstance(m, TransformerBlock)]
    if policy == "recurrent_level":
        return [m for m in model.modules() if isinstance(m, Transformer)]
    raise ValueError(f"Unsupported fsdp_wrap_policy: {policy}")


def contains_checkpointed_block(module: nn.Module, blocks: set) -> bool:
    return any(child in blocks for child in module.modules())


def unwrap_model(model: nn.Module) -> nn.Module:
    return model.module if isinstance(model, DistributedDataParallel) else model


def fsdp_model_dtype(config) -> torch.dtype:
    return {"fp32": torch.float32, "bf16": torch.bfloat16}[config.fsdp_params_precision]


def ddp_model_dtype(config, fwd_bwd_dtype: torch.dtype) -> torch.dtype:
    return torch.float32 if config.ddp_params_precision == "fp32" else fwd_bwd_dtype


def optimizer_ema_dtype(config) -> Optional[torch.dtype]:
    if config.distributed_strategy == "ddp" and config.ddp_params_precision == "bf16":
        return torch.float32
    if config.distributed_strategy == "fsdp" and config.fsdp_params_precision == "bf16":
        return torch.float32
    return None


def wrap_fsdp(model: nn.Module, config, fwd_bwd_dtype: torch.dtype, checkpointed: set) -> nn.Module:
    mesh = create_fsdp_mesh(config)
    model_dtype = fsdp_model_dtype(config)
    if model_dtype != torch.float32:
        model = model.to(dtype=model_dtype)
    for buf in model.buffers():
        dist.broadcast(buf, src=0)
    for module in fsdp_wrap_modules(model, config.fsdp_wrap_policy):
        apply_fsdp(module, fwd_bwd_dtype, mesh=mesh,
                   reshard_after_forward=fsdp_reshard_after_forward(
                       config, checkpointed=contains_checkpointed_block(module, checkpointed)))
    apply_fsdp(model, fwd_bwd_dtype, mesh=mesh,
               reshard_after_forward=fsdp_reshard_after_forward(config, checkpointed=bool(checkpointed)))
    return model


def wrap_ddp(model: nn.Module, config, fwd_bwd_dtype: torch.dtype, device: torch.device) -> nn.Module:
    dtype = ddp_model_dtype(config, fwd_bwd_dtype)
    if dtype != torch.float32:
        model = model.to(dtype=dtype)
    kwargs = dict(device_ids=[device.index], output_device=device.index) if device.type == "cuda" else {}
    return DistributedDataParallel(model, find_unused_parameters=config.ddp_find_unused_parameters, **kwargs)
