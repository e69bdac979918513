"""Training checkpoints: staged save + publish, exact-continuation guards, DCP/unsharded I/O.

Reference behaviour: ``src/mimir/training/checkpoint_io.py`` (tag grammar ``:29-42``, resume
state ``:104-162``, exact-continuation guards ``:166-281``, DCP ``:306-374,434-437``,
unsharded ``:390-456``, sidecar ``:488-545``, staged save + publish ``:549-587``, ephemeral
GC ``:609-624``).  The on-disk layout is kept identical so that checkpoints move between the
two frameworks:

    <checkpoint_path>/<tag>/            tag = step_N | epoch_N | ephemeral_step_N
        fsdp2_<tag>/ (DCP: {"model": model.state_dict(), "optim": get_optimizer_state_dict})
          or unsharded_<tag>.pt
        rng.<rank>.pt, all_config.yaml, train_metadata.yaml,
        checkpoint_state_<tag>.json, manifest.json (mode, tag, step, total_steps, world_size)

Saving writes everything into ``.<tag>.<uuid>.partial`` (uuid broadcast from rank 0) and
rank 0 publishes it by one atomic rename; a crash leaves only a partial directory that no
resume accepts.
"""
from __future__ import annotations

import json
import os
import re
import shutil
import uuid
from pathlib import Path
from typing import Literal, Optional

import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp
import yaml
from torch.distributed.checkpoint.state_dict import (StateDictOptions, get_model_state_dict,
                                                     get_optimizer_state_dict, set_optimizer_state_dict,
                                                     set_state_dict)

from mimir_b200.train.state import ResumeState, TrainState
from mimir_b200.utils.trace import trace_print

_TAG = re.compile(r"(?:epoch|step|ephemeral_step)_\d+")

# Keys whose change breaks an exact continuation (reference ``checkpoint_io.py:183-189``).
PROTECTED_KEYS = ("data", "seed", "global_batch_size", "epochs", "training_total_steps", "lr", "lr_auto",
                  "lr_piecewise_points", "lr_warmup_steps", "lr_min_ratio", "lr_rewarm_steps", "lr_rewarm_stages",
                  "lr_rewarm_start_ratio", "lr_decay_start_step", "lr_decay_end_step", "lr_cooldown_checkpoint",
                  "lr_embeddings", "lr_head", "lr_h", "lr_l", "weight_decay", "beta1", "beta2", "ema", "optimizer",
                  "muon_momentum", "muon_ns_steps", "muon_lr_scale", "fwd_bwd_dtype")

# Opt-in architecture flags newer than some checkpoints; absent means disabled.
_ARCH_DEFAULTS = dict(h_residual_persistence=False, h_branch_l_mixing=False, moe_aux_loss_free=False,
                      mos_aux_loss_free=False, routing_bias_update_rate=0.001)


def _world() -> int:
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def _barrier() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def normalize_checkpoint_tag(tag: str) -> str:
    for prefix in ("fsdp2_", "unsharded_", "carry_"):
        if tag.startswith(prefix):
            tag = tag.removeprefix(prefix)
            if prefix == "unsharded_":
                tag = tag.removesuffix(".pt")
            break
    if os.path.basename(tag) != tag:
        raise ValueError(f"Checkpoint tag must be a name, not a path: {tag}")
    if not tag.startswith(("epoch_", "step_", "ephemeral_step_")):
        raise ValueError(f"Checkpoint tag must start with 'epoch_', 'step_', or 'ephemeral_step_': {tag}")
    return tag


def load_checkpoint_metadata(checkpoint_path: str, tag: str) -> dict:
    path = Path(checkpoint_path) / f"checkpoint_state_{tag}.json"
    return json.loads(path.read_text()) if path.is_file() else {}


def infer_checkpoint_world_size(checkpoint_path: str, tag: str, metadata: dict) -> Optional[int]:
    if metadata.get("world_size") is not None:
        return int(metadata["world_size"])
    pattern = re.compile(rf"^carry_{re.escape(tag)}\.(\d+)\.pt$")
    ranks = [int(m.group(1)) for name in os.listdir(checkpoint_path) if (m := pattern.fullmatch(name))]
    return max(ranks) + 1 if ranks else None


def checkpoint_carry_policy(checkpoint_path: str, tag: str, metadata: dict) -> Literal["none", "per_rank"]:
    """``carry_policy`` from the sidecar; legacy checkpoints with all-None carry files are ``none``."""
    policy = metadata.get("carry_policy")
    if policy is not None:
        if policy not in ("none", "per_rank"):
            raise ValueError(f"Unsupported carry_policy={policy!r} in checkpoint {tag}")
        return policy
    inferred = "per_rank"
    if not (dist.is_available() and dist.is_initialized()) or dist.get_rank() == 0:
        world = infer_checkpoint_world_size(checkpoint_path, tag, metadata)
        if world is not None:
            paths = [Path(checkpoint_path) / f"carry_{tag}.{r}.pt" for r in range(world)]
            if all(p.is_file() for p in paths) and all(
                    torch.load(p, map_location="cpu", weights_only=False) is None for p in paths):
                inferred = "none"
    if dist.is_available() and dist.is_initialized():
        box = [inferred]
        dist.broadcast_object_list(box, src=0)
        inferred = box[0]
    return inferred


def same_architecture(previous: Optional[dict], current: dict) -> bool:
    return previous is not None and (_ARCH_DEFAULTS | previous) == (_ARCH_DEFAULTS | current)


def resolve_resume_state(config, current_local_batch_size: int) -> Optional[ResumeState]:
    """Where to restart: epoch boundary, batch skip, or global row cursor (layout changed)."""
    path, tag = config.resume_checkpoint_path, config.resume_checkpoint_tag
    if path is None and tag is None:
        return None
    if path is None or tag is None:
        raise ValueError("Both resume_checkpoint_path and resume_checkpoint_tag must be set to resume training")
    tag = normalize_checkpoint_tag(tag)
    meta = load_checkpoint_metadata(path, tag)
    step = meta.get("step", config.resume_step)
    epoch = meta.get("epoch", config.resume_epoch)
    batch_in_epoch = meta.get("batch_in_epoch", config.resume_batch_in_epoch)
    if tag.startswith("epoch_"):
        done = int(tag.removeprefix("epoch_"))
        return ResumeState(tag=tag, step=-1 if step is None else int(step), start_epoch=done + 1, skip_batches=0)
    match = re.fullmatch(r"(?:ephemeral_)?step_(\d+)", tag)
    if match is None:
        raise ValueError(f"Unsupported checkpoint tag: {tag}")
    step = int(match.group(1)) if step is None else int(step)
    if epoch is None or batch_in_epoch is None:
        raise ValueError(f"Step checkpoint {tag} needs checkpoint_state_{tag}.json or explicit "
                         "resume_epoch and resume_batch_in_epoch overrides")
    cursor = meta.get("global_row_cursor_in_epoch")
    saved_local = meta.get("local_batch_size")
    saved_world = infer_checkpoint_world_size(path, tag, meta)
    layout_changed = saved_local is not None and (
        int(saved_local) != current_local_batch_size
        or (saved_world is not None and int(saved_world) != _world())
        or not bool(meta.get("batch_in_epoch_exact", True)))
    if cursor is not None and layout_changed:
        return ResumeState(tag=tag, step=step, start_epoch=int(epoch), skip_batches=int(batch_in_epoch),
                           start_row_cursor=int(cursor), resume_mode="row_cursor")
    return ResumeState(tag=tag, step=step, start_epoch=int(epoch), skip_batches=int(batch_in_epoch))


def _check_exact_continuation(config, resume: ResumeState, meta: dict, rank: int, local_batch_size: int) -> None:
    root = Path(config.resume_checkpoint_path)
    previous = yaml.safe_load((root / "all_config.yaml").read_text()) if (root / "all_config.yaml").is_file() else {}
    if previous:
        current = config.model_dump()
        for key in PROTECTED_KEYS:
            if previous.get(key) != current.get(key):
                raise ValueError(f"Exact continuation configuration changed: {key}")
        if not config.arch.upcycle_from_dense and not config.arch.gate_initialize_from_v1:
            if not same_architecture(previous.get("arch"), current["arch"]):
                raise ValueError("Exact continuation architecture changed")
        from mimir_b200.data.corpus import V1Dataset, V1DatasetConfig
        saved = yaml.safe_load((root / "train_metadata.yaml").read_text())
        corpus = V1Dataset(V1DatasetConfig(seed=config.seed, dataset_path=config.data.path,
                                           batch_max_length=local_batch_size, drop_last_batch=True,
                                           target_only=config.data.target_only, rank=rank, num_replicas=_world()))
        if saved != corpus.metadata.model_dump():
            raise ValueError("Corpus metadata changed during continuation")
    if meta.get("optimizer", previous.get("optimizer", "adam_atan2")) != config.optimizer:
        raise ValueError("Optimizer changes require an explicit offline state conversion")
    old_homog = meta.get("homogeneous_categories", (previous.get("data") or {}).get("homogeneous_categories", False))
    mode_changed = old_homog != config.data.homogeneous_categories
    layout_changed = old_homog and (
        infer_checkpoint_world_size(str(root), resume.tag, meta) not in (None, _world())
        or meta.get("local_batch_size", local_batch_size) != local_batch_size
        or meta.get("seed", previous.get("seed", 0)) != config.seed)
    if not resume.tag.startswith("epoch_") and (mode_changed or layout_changed):
        raise ValueError("Homogeneous sampler changes require an epoch-boundary resume")


def load_train_checkpoint(config, train_state: TrainState, rank: int, local_batch_size: int) -> Optional[ResumeState]:
    """Restore model, optimizer, step and RNG from a published checkpoint; return where to restart."""
    from mimir_b200.ckpt.contract import resolve, restore_rng, validate
    if config.resume_checkpoint_path is not None:
        config = config.model_copy(update={"resume_checkpoint_path": str(
            resolve(config.resume_checkpoint_path, config.resume_checkpoint_tag))})
    resume = resolve_resume_state(config, local_batch_size)
    if resume is None:
        return None
    root = config.resume_checkpoint_path
    meta = load_checkpoint_metadata(root, resume.tag)
    _check_exact_continuation(config, resume, meta, rank, local_batch_size)
    policy = checkpoint_carry_policy(root, resume.tag, meta)
    saved_world = infer_checkpoint_world_size(root, resume.tag, meta)
    if policy == "per_rank" and saved_world is not None and saved_world != _world():
        raise ValueError(f"Cannot resume stateful per-rank carry across a world-size change: "
                         f"checkpoint={saved_world}, current={_world()}")
    carry_path = Path(root) / f"carry_{resume.tag}.{rank}.pt"
    if policy == "per_rank" and not carry_path.is_file():
        raise ValueError(f"Carry file not found: {carry_path}")

    trace_print(config, rank, f"load_checkpoint_begin tag={resume.tag} format={config.checkpoint_format}")
    if config.checkpoint_format == "sharded":
        load_sharded_train_state(config, train_state, resume.tag)
    elif config.checkpoint_format == "unsharded":
        load_unsharded_train_state(config, train_state, resume.tag, rank)
    else:
        raise ValueError(f"Unsupported checkpoint_format: {config.checkpoint_format}")
    trace_print(config, rank, f"load_checkpoint_end tag={resume.tag}")
    if config.upcast_optimizer_state_on_resume:
        upcast_optimizer_state(train_state.optim)
    if config.reset_ema_on_resume:
        reset_optimizer_ema_to_params(train_state.optim)
    train_state.carry = None if policy == "none" else torch.load(carry_path, map_location="cuda")

    if resume.step >= 0:
        train_state.step = resume.step
    elif resume.tag.startswith("epoch_"):
        done = int(resume.tag.removeprefix("epoch_"))
        train_state.step = resume.step = int(done * train_state.total_steps // config.epochs)
    else:
        raise ValueError(f"Cannot infer resume step for checkpoint tag {resume.tag}")
    manifest = validate(root, hashes=False)
    if manifest["world_size"] != _world():
        raise ValueError("Exact RNG continuation requires unchanged world size")
    if manifest["total_steps"] != train_state.total_steps:
        raise ValueError("Total-step schedule changed; use an explicit initialization")
    restore_rng(torch.load(Path(root) / f"rng.{rank}.pt", map_location="cpu", weights_only=False))
    return resume


@torch.no_grad()
def upcast_optimizer_state(optim) -> None:
    for state in optim.state.values():
        for key, value in list(state.items()):
            if torch.is_tensor(value) and value.is_floating_point() and value.dtype != torch.float32:
                state[key] = value.float()


@torch.no_grad()
def reset_optimizer_ema_to_params(optim) -> None:
    for group in optim.param_groups:
        if group.get("ema") is None:
            continue
        for p in group["params"]:
            if "param_ema" in optim.state[p]:
                optim.state[p]["param_ema"] = p.detach().clone().float()


def sharded_checkpoint_id(checkpoint_path: str, tag: str) -> str:
    return os.path.join(checkpoint_path, f"fsdp2_{tag}")


def unsharded_checkpoint_path(checkpoint_path: str, tag: str) -> str:
    return os.path.join(checkpoint_path, f"unsharded_{tag}.pt")


def load_sharded_train_state(config, train_state: TrainState, tag: str) -> None:
    root = config.resume_checkpoint_path
    ckpt = sharded_checkpoint_id(root, tag)
    if not os.path.isdir(ckpt):
        raise ValueError(f"Checkpoint directory not found: {ckpt}")
    src_cfg = Path(root) / "all_config.yaml"
    source = yaml.safe_load(src_cfg.read_text()) if src_cfg.is_file() else {}
    if source and source.get("optimizer", "adam_atan2") != config.optimizer:
        raise ValueError("Optimizer changes require an explicit offline state conversion")
    if config.arch.upcycle_from_dense:
        from mimir_b200.ckpt.upcycle import load_upcycled_checkpoint
        load_upcycled_checkpoint(train_state.model, train_state.optim, ckpt)
        return
    if config.arch.gate_initialize_from_v1:
        src_arch = source["arch"]
        if src_arch["name"] == "legacy_v1":
            for field in ("H_cycles", "L_cycles"):
                if src_arch[field] != getattr(config.arch, field):
                    raise ValueError(f"v1 -> v2 migration must preserve {field}")
            from mimir_b200.ckpt.upcycle import load_v1_checkpoint
            if not load_v1_checkpoint(train_state.model, train_state.optim, ckpt):
                raise ValueError("Source claims v1 but contains v2 gate state")
            return
        if src_arch["name"] != config.arch.name:
            raise ValueError("Only the original HRM baseline can initialize v2 gates")
    engine = _engine(train_state)
    if engine is not None:
        _load_replicated(engine, train_state, ckpt)
        return
    model_state = train_state.model.state_dict()
    # DCP loads the requested subset only: refuse sources with modules this run disabled.
    stored = {k.removeprefix("model.") for k in dcp.FileSystemReader(ckpt).read_metadata().state_dict_metadata
              if k.startswith("model.")}
    unexpected = stored - set(model_state)
    if unexpected:
        raise ValueError("Checkpoint contains disabled or mismatched v2 features; enable the original "
                         f"gates/experts/residual branches explicitly. Unexpected model keys: {sorted(unexpected)}")
    optim_state = get_optimizer_state_dict(train_state.model, train_state.optim)
    dcp.load({"model": model_state, "optim": optim_state}, checkpoint_id=ckpt)
    if config.distributed_strategy == "ddp":
        train_state.model.load_state_dict(model_state)
        set_optimizer_state_dict(train_state.model, train_state.optim, optim_state)
        return
    set_state_dict(train_state.model, train_state.optim, model_state_dict=model_state, optim_state_dict=optim_state)


def _load_replicated(engine, train_state: TrainState, ckpt: str) -> None:
    """DCP into the engine's shard buffers in place (same keys/placements FSDP2 writes)."""
    from mimir_b200.parallel.replicated import model_dcp_state
    model_state = model_dcp_state(engine)
    stored = {k.removeprefix("model.") for k in dcp.FileSystemReader(ckpt).read_metadata().state_dict_metadata
              if k.startswith("model.")}
    known = set(model_state)
    if engine.world > 1 and any(s.local for s in engine.slots):  # other ranks own the other experts
        everyone = [None] * engine.world
        dist.all_gather_object(everyone, sorted(known), group=engine.group)
        known = set().union(*map(set, everyone))
    unexpected = stored - known
    if unexpected:
        raise ValueError(f"Checkpoint contains model keys this run does not have: {sorted(unexpected)}")
    optim_state = train_state.optim.dcp_state()
    dcp.load({"model": model_state, "optim": optim_state}, checkpoint_id=ckpt)
    train_state.optim.load_dcp_state(optim_state)
    engine.gather_weights()


def _full(value):
    return value.full_tensor() if hasattr(value, "full_tensor") else value


def _save_unsharded_replicated(engine, train_state: TrainState, path: str, rank: int) -> None:
    from mimir_b200.parallel.replicated import model_dcp_state
    model = {k: _full(v).cpu() for k, v in model_dcp_state(engine).items()}
    optim = train_state.optim.dcp_state()
    optim["state"] = {k: {n: _full(t).cpu() for n, t in slots.items()} for k, slots in optim["state"].items()}
    local = [s.fqn for s in engine.slots if s.local]
    if engine.world > 1 and local:  # expert-parallel parameters live on their owner rank only
        mine = ({k: model[k] for k in local}, {k: optim["state"][k] for k in local if k in optim["state"]})
        everyone = [None] * engine.world
        dist.all_gather_object(everyone, mine, group=engine.group)
        for m, o in everyone:
            model.update(m)
            optim["state"].update(o)
    if rank == 0:
        torch.save({"model": model, "optim": optim}, path)


@torch.no_grad()
def _load_unsharded_replicated(engine, train_state: TrainState, path: str) -> None:
    ckpt = torch.load(path, map_location="cpu", weights_only=False)
    optim = train_state.optim
    buffers = dict(engine.model.named_buffers())
    for name, value in ckpt["model"].items():
        if name in buffers:
            buffers[name].copy_(value)
    for s in engine.slots:
        sl = slice(s.shard, s.shard + s.shard_numel)
        rows = slice(s.row0, s.row0 + s.rows_mine)
        engine.master[sl] = ckpt["model"][s.fqn].reshape(s.rows, -1)[rows].reshape(-1).to(engine.master)
        saved = ckpt["optim"]["state"].get(s.fqn)
        if saved is None or not s.trainable:
            continue
        for slot, buf in optim.slot_buffers(s).items():
            if slot in saved:
                buf[sl] = saved[slot].reshape(s.rows, -1)[rows].reshape(-1).to(buf)
    optim.load_dcp_state(ckpt["optim"])
    engine.gather_weights()


def load_unsharded_train_state(config, train_state: TrainState, tag: str, rank: int) -> None:
    root = config.resume_checkpoint_path
    if config.arch.gate_initialize_from_v1:
        src = yaml.safe_load((Path(root) / "all_config.yaml").read_text())["arch"]["name"]
        if src != "mimir2":
            raise ValueError("v1 -> v2 initialization currently requires a sharded DCP checkpoint")
    path = unsharded_checkpoint_path(root, tag)
    if not os.path.isfile(path):
        raise ValueError(f"Checkpoint file not found: {path}")
    distributed = dist.is_available() and dist.is_initialized()
    if _engine(train_state) is not None:
        _load_unsharded_replicated(_engine(train_state), train_state, path)
        return
    if config.arch.upcycle_from_dense:
        from mimir_b200.ckpt.upcycle import expand_unsharded_state
        opts = StateDictOptions(full_state_dict=True, cpu_offload=True)
        target = get_model_state_dict(train_state.model, options=opts)
        optim = get_optimizer_state_dict(train_state.model, train_state.optim, options=opts)
        if not distributed or rank == 0:
            target, optim = expand_unsharded_state(target, optim, torch.load(path, map_location="cpu",
                                                                             weights_only=False))
        set_state_dict(train_state.model, train_state.optim, model_state_dict=target, optim_state_dict=optim,
                       options=StateDictOptions(full_state_dict=True, broadcast_from_rank0=distributed))
        return
    if distributed:
        ddp = config.distributed_strategy == "ddp"
        ckpt = torch.load(path, map_location="cpu", weights_only=False) if (ddp or rank == 0) else {}
        set_state_dict(train_state.model, train_state.optim, model_state_dict=ckpt.get("model", {}),
                       optim_state_dict=ckpt.get("optim", {}),
                       options=StateDictOptions(full_state_dict=True, cpu_offload=True, broadcast_from_rank0=not ddp))
        return
    ckpt = torch.load(path, map_location="cpu", weights_only=False)
    train_state.model.load_state_dict(ckpt["model"])
    set_optimizer_state_dict(train_state.model, train_state.optim, ckpt["optim"])


def _engine(train_state):
    return getattr(train_state.model, "replicated_engine", None)


def save_sharded_train_state(directory: str, train_state: TrainState, tag: str) -> None:
    engine = _engine(train_state)
    if engine is not None:
        from mimir_b200.parallel.replicated import model_dcp_state
        state = {"model": model_dcp_state(engine), "optim": train_state.optim.dcp_state()}
    else:
        state = {"model": train_state.model.state_dict(),
                 "optim": get_optimizer_state_dict(train_state.model, train_state.optim)}
    dcp.save(state, checkpoint_id=sharded_checkpoint_id(directory, tag))


def save_unsharded_train_state(directory: str, train_state: TrainState, tag: str, rank: int) -> None:
    if _engine(train_state) is not None:
        _save_unsharded_replicated(_engine(train_state), train_state, unsharded_checkpoint_path(directory, tag), rank)
        return
    if dist.is_available() and dist.is_initialized():
        opts = StateDictOptions(full_state_dict=True, cpu_offload=True)
        model_state = get_model_state_dict(train_state.model, options=opts)
        optim_state = get_optimizer_state_dict(train_state.model, train_state.optim, options=opts)
        if rank == 0:
            torch.save({"model": model_state, "optim": optim_state}, unsharded_checkpoint_path(directory, tag))
        return
    torch.save({"model": train_state.model.state_dict(),
                "optim": get_optimizer_state_dict(train_state.model, train_state.optim)},
               unsharded_checkpoint_path(directory, tag))


def save_code_and_config(config, train_metadata) -> None:
    """Run-root provenance: model source copy, ``all_config.yaml``, ``train_metadata.yaml``."""
    if config.checkpoint_path is None:
        return
    root = Path(config.checkpoint_path)
    root.mkdir(parents=True, exist_ok=True)
    import inspect
    from mimir_b200.models import mimir2
    shutil.copy(inspect.getfile(mimir2), root / os.path.basename(inspect.getfile(mimir2)))
    (root / "all_config.yaml").write_text(yaml.dump(config.model_dump()))
    meta = train_metadata.model_dump() if hasattr(train_metadata, "model_dump") else dict(train_metadata)
    (root / "train_metadata.yaml").write_text(yaml.dump(meta))


def checkpoint_metadata(config, train_state: TrainState, tag: str, epoch: int, batch_in_epoch: int,
                        checkpoint_kind: str, local_batch_size: int, resume_info: Optional[dict] = None,
                        batch_in_epoch_exact: bool = True, carry_policy: str = "none") -> dict:
    """The ``checkpoint_state_<tag>.json`` sidecar (same keys as the reference sidecar)."""
    from mimir_b200.optim.schedules import rewarm_metadata
    meta = {
        "tag": tag, "checkpoint_kind": checkpoint_kind, "checkpoint_format": config.checkpoint_format,
        "step": train_state.step, "epoch": epoch, "batch_in_epoch": batch_in_epoch,
        "batch_in_epoch_exact": batch_in_epoch_exact,
        "gradient_accumulation_steps": config.gradient_accumulation_steps,
        "global_batch_size": config.global_batch_size, "local_batch_size": local_batch_size,
        "data_path": config.data.path, "homogeneous_categories": config.data.homogeneous_categories,
        "optimizer": config.optimizer, "seed": config.seed, "world_size": _world(),
        "local_world_size": int(os.environ.get("LOCAL_WORLD_SIZE", 1)), "carry_policy": carry_policy,
        "carry_schema_version": 1, "fsdp_shard_degree": config.fsdp_shard_degree,
        "fsdp_reshard_after_forward": config.fsdp_reshard_after_forward,
        "fsdp_accumulation_sync_mode": config.fsdp_accumulation_sync_mode,
    }
    if config.lr_rewarm_steps:
        meta["lr_rewarm"] = rewarm_metadata(config)
    if config.lr_piecewise_points is not None:
        meta["lr_piecewise_points"] = config.lr_piecewise_points
    if resume_info is not None:
        meta.update({"global_row_start_in_epoch": int(resume_info["global_row_start"]),
                     "global_row_cursor_in_epoch": int(resume_info["global_row_end"]),
                     "global_numseq": int(resume_info["global_numseq"]),
                     "global_batch_totlen": int(resume_info["global_batch_totlen"])})
    return meta


def _write_json_atomic(path: Path, value: dict) -> None:
    temp = path.with_name(path.name + ".tmp")
    with open(temp, "wt") as f:
        json.dump(value, f, indent=2, sort_keys=True)
        f.write("\n")
        f.flush()
        os.fsync(f.fileno())
    os.replace(temp, path)


def save_train_checkpoint(config, train_state: TrainState, tag: str, epoch: int, batch_in_epoch: int, rank: int,
                          checkpoint_kind: str = "regular", local_batch_size: int = 0,
                          resume_info: Optional[dict] = None, batch_in_epoch_exact: bool = True) -> Optional[Path]:
    """Write ``<checkpoint_path>/<tag>`` (all ranks call this); return the published directory."""
    from mimir_b200.utils.trace import nvtx_range
    with nvtx_range("checkpoint_save"):
        return _save_train_checkpoint(config, train_state, tag, epoch, batch_in_epoch, rank, checkpoint_kind,
                                      local_batch_size, resume_info, batch_in_epoch_exact)


def _save_train_checkpoint(config, train_state, tag, epoch, batch_in_epoch, rank, checkpoint_kind, local_batch_size,
                           resume_info, batch_in_epoch_exact):
    from mimir_b200.ckpt.contract import publish, rng_state
    if config.checkpoint_path is None:
        return None
    if not _TAG.fullmatch(tag):
        raise ValueError(f"Invalid checkpoint tag: {tag}")
    if train_state.carry is not None:
        raise ValueError("Mimir2 checkpoint contract requires carry=None")
    root = Path(config.checkpoint_path)
    box = [uuid.uuid4().hex if rank == 0 else None]
    if dist.is_available() and dist.is_initialized():
        dist.broadcast_object_list(box, src=0)
    stage = root / f".{tag}.{box[0]}.partial"
    stage.mkdir(parents=True, exist_ok=True)
    if config.checkpoint_format == "sharded":
        save_sharded_train_state(str(stage), train_state, tag)
    else:
        save_unsharded_train_state(str(stage), train_state, tag, rank)
    torch.save(rng_state(), stage / f"rng.{rank}.pt")
    _barrier()
    if rank == 0:
        if (root / "train_metadata.yaml").exists():
            shutil.copy2(root / "train_metadata.yaml", stage / "train_metadata.yaml")
        (stage / "all_config.yaml").write_text(yaml.safe_dump(config.model_dump()))
        _write_json_atomic(stage / f"checkpoint_state_{tag}.json",
                           checkpoint_metadata(config, train_state, tag, epoch, batch_in_epoch, checkpoint_kind,
                                               local_batch_size, resume_info, batch_in_epoch_exact, "none"))
        publish(stage, root / tag, metadata={"mode": "exact", "tag": tag, "step": train_state.step,
                                             "total_steps": train_state.total_steps, "world_size": _world()})
    _barrier()
    return root / tag


def remove_stale_ephemeral_checkpoints(config, keep_tag: str, rank: int) -> None:
    """Delete older ``ephemeral_step_*`` directories once ``keep_tag`` validates."""
    from mimir_b200.ckpt.contract import validate
    if config.checkpoint_path is None:
        return
    root = Path(config.checkpoint_path)
    validate(root / keep_tag)
    _barrier()
    if rank == 0:
        keep = int(keep_tag.rsplit("_", 1)[1])
        for entry in root.glob("ephemeral_step_*"):
            if entry.is_dir() and entry.name != keep_tag and int(entry.name.rsplit("_", 1)[1]) < keep:
                validate(entry)
                shutil.rmtree(entry)
    _barrier()
