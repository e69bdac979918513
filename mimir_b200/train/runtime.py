"""Loop-side runtime helpers: config broadcast, devices, batch transfer, memory, state fingerprint.

Reference behaviour: ``src/mimir/training/runtime.py:27-135`` and
``src/mimir/model/accelerator.py`` (device selection).  This framework targets CUDA (sm_100a)
and keeps a CPU path for tests; other accelerator names map to CPU.
"""
from __future__ import annotations

import os
import random
from pathlib import Path

import torch
import torch.distributed as dist
from torch import Tensor

from mimir_b200.utils.trace import trace_print  # noqa: F401  (re-export for loop callers)

_ADJECTIVES = ("amber", "brisk", "calm", "deft", "eager", "fleet", "grand", "hardy", "ivory", "jolly", "keen",
               "lucid", "mellow", "noble", "quiet", "rapid", "sage", "tidy", "vivid", "witty")
_NOUNS = ("badger", "condor", "dingo", "egret", "falcon", "gecko", "heron", "ibis", "jackal", "kestrel", "lynx",
          "marten", "newt", "otter", "puffin", "quokka", "raven", "stoat", "tapir", "walrus")


def run_slug(rng: random.Random | None = None) -> str:
    """Two-word run name (``adjective-noun``) for unnamed runs."""
    rng = rng or random.Random()
    return f"{rng.choice(_ADJECTIVES)}-{rng.choice(_NOUNS)}"


def load_synced_config(config, rank: int):
    """Fill project/run/checkpoint names on rank 0 and broadcast the validated config."""
    box = [None]
    if rank == 0:
        config = config.model_copy(deep=True)
        if config.project_name is None:
            config.project_name = f"{Path(config.data.path).stem.capitalize()} HLM-torch"
        if config.run_name is None:
            config.run_name = os.environ.get("MLP_TASK_NAME", f"{config.arch.name.split('@')[-1]} {run_slug()}")
        if config.checkpoint_path is None:
            config.checkpoint_path = os.path.join("checkpoints", config.project_name, config.run_name)
        box = [config]
    if dist.is_available() and dist.is_initialized():
        dist.broadcast_object_list(box, src=0)
    return box[0]


def device_for(config, local_rank: int) -> torch.device:
    if config.accelerator_type in ("sm100", "sm90") and torch.cuda.is_available():
        return torch.device("cuda", local_rank)
    return torch.device("cpu")


def synchronize(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device)


def move_batch_to_device(batch: dict[str, Tensor], device: torch.device) -> dict[str, Tensor]:
    return {k: v.to(device, non_blocking=device.type == "cuda") for k, v in batch.items()}


def memory_stats(device: torch.device) -> dict[str, int]:
    if device.type != "cuda":
        return {}
    return {"allocated": torch.cuda.memory_allocated(device), "reserved": torch.cuda.memory_reserved(device),
            "max_allocated": torch.cuda.max_memory_allocated(device)}


def _mib(v: int) -> str:
    return f"{v / 1024 / 1024:.3f} MiB"


def maybe_log_memory(step: int, label: str, device: torch.device, enabled: bool) -> None:
    if enabled and (stats := memory_stats(device)):
        print(f"[{device.type} memory] step={step} {label}: " + " ".join(f"{k}={_mib(v)}" for k, v in stats.items()),
              flush=True)


def maybe_empty_cache(step: int, device: torch.device, interval: int) -> None:
    if interval <= 0 or step % interval or device.type != "cuda":
        return
    before = memory_stats(device)
    torch.cuda.empty_cache()
    synchronize(device)
    after = memory_stats(device)
    print(f"[{device.type} empty_cache] step={step}: " + " ".join(
        f"{k} {_mib(before.get(k, 0))}->{_mib(after.get(k, 0))}" for k in sorted(before | after)), flush=True)


@torch.no_grad()
def distributed_state_fingerprint(config, train_state, device: torch.device) -> dict[str, dict[str, float]]:
    """Sum, |sum|, sum of squares, count and max|x| of parameters and each optimizer slot, all ranks."""
    buckets: dict[str, list[Tensor]] = {"parameters": list(train_state.model.parameters())}
    for state in train_state.optim.state.values():
        for key, value in state.items():
            if torch.is_tensor(value) and value.is_floating_point():
                buckets.setdefault(f"optimizer/{key}", []).append(value)
    distributed = dist.is_available() and dist.is_initialized()
    world = dist.get_world_size() if distributed else 1
    replicas = world // config.fsdp_shard_degree if (config.fsdp_shard_degree and distributed) else 1
    out = {}
    for name, tensors in sorted(buckets.items()):
        sums = torch.zeros(4, dtype=torch.float64, device=device)
        peak = torch.zeros(1, dtype=torch.float64, device=device)
        for t in tensors:
            x = (t.to_local() if hasattr(t, "to_local") else t).to(device).double()
            sums += torch.stack([x.sum(), x.abs().sum(), x.square().sum(), x.new_tensor(float(x.numel()))])
            if x.numel():
                peak = torch.maximum(peak, x.abs().max().reshape(1))
        if distributed:
            dist.all_reduce(sums)
            dist.all_reduce(peak, op=dist.ReduceOp.MAX)
        sums /= world if name == "optimizer/step" else replicas
        out[name] = {"sum": sums[0].item(), "abs_sum": sums[1].item(), "square_sum": sums[2].item(),
                     "numel": sums[3].item(), "abs_max": peak.item()}
    return out
