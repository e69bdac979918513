"""The training loop: epochs of gradient-accumulated optimizer steps with exact resume.

Reference behaviour: ``src/mimir/training/loop.py:28-521``.  Per optimizer step:

1. collect ``gradient_accumulation_steps`` microbatches (host scalars wrapped so FSDP does
   not move them);
2. advance the step, apply the LR schedule (optionally the row-anchored cooldown), compute the
   model's extra arguments (truncated-BPTT ``bp_steps``), update automatic per-module LRs and
   gate-donor updates;
3. optionally replay a bounded copy of the batch under stability diagnostics (forked RNG, no
   optimizer step);
4. run the accumulated step (clip / skip inside), track consecutive skips;
5. every ``log_interval`` steps reduce metrics to rank 0 and write ``metrics.jsonl`` and
   ``progress.json``; run validation every ``validation_interval`` steps;
6. write step / ephemeral checkpoints, then give the suspension hook its chance.

An epoch checkpoint closes every ``checkpoint_interval``-th epoch.  ``max_steps`` turns on a
benchmark summary (per-step wall times, optional state fingerprint) printed as ``[bench] {...}``.

Distributed runs start under torchrun: NCCL on CUDA; the CPU path uses Gloo so the same loop
runs as multi-process CPU tests.
"""
from __future__ import annotations

import json
import os
import random
import time
from pathlib import Path
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist

from mimir_b200.models.common import wrap_tensor
from mimir_b200.utils.trace import trace_print


def _init_distributed(config):
    if "LOCAL_RANK" not in os.environ:
        return 0, 1, 0
    local = int(os.environ["LOCAL_RANK"])
    if config.accelerator_type in ("sm100", "sm90") and torch.cuda.is_available():
        torch.cuda.set_device(local)
        dist.init_process_group(backend="nccl", device_id=torch.device("cuda", local))
    elif config.accelerator_type in ("cpu", "none"):
        dist.init_process_group(backend="gloo")
    else:
        raise RuntimeError(f"accelerator_type={config.accelerator_type} cannot run distributed here")
    return dist.get_rank(), dist.get_world_size(), local


def _seed(seed: int, rank: int) -> None:
    random.seed(seed + rank)
    np.random.seed((seed + rank) % (2 ** 32))
    torch.random.manual_seed(seed + rank)


def write_progress(path: Path, record: dict) -> None:
    """Atomically replace the monitor's ``progress.json``."""
    from mimir_b200.train.suspension.protocol import atomic_write
    atomic_write(path, json.dumps(record, allow_nan=False))


class _Bench:
    """Optional per-step wall times (only with ``max_steps``), summarised at the end."""

    def __init__(self, enabled: bool):
        self.enabled = enabled
        self.times: list[float] = []
        self.last: Optional[float] = None
        self.last_metrics: dict = {}
        self.history: list[dict] = []

    def tick(self, device) -> None:
        from mimir_b200.train.runtime import synchronize
        synchronize(device)
        now = time.perf_counter()
        if self.last is not None:
            self.times.append(now - self.last)
        self.last = now

    def summary(self, config, world: int, fingerprint) -> Optional[dict]:
        if not self.times:
            return None
        warm = min(2, len(self.times) - 1) if len(self.times) > 1 else 0
        steady = sorted(self.times[warm:])
        out = {"world_size": world, "nnodes": int(os.environ.get("NNODES", os.environ.get("SLURM_JOB_NUM_NODES", 0))),
               "global_batch_size": config.global_batch_size,
               "gradient_accumulation_steps": config.gradient_accumulation_steps,
               "measured_steps": len(self.times), "warmup_dropped": warm,
               "median_step_seconds": steady[len(steady) // 2], "mean_step_seconds": sum(steady) / len(steady),
               "min_step_seconds": steady[0], "max_step_seconds": steady[-1], "all_step_seconds": self.times,
               "last_metrics": self.last_metrics, "metric_history": self.history}
        if fingerprint is not None:
            out["state_fingerprint"] = fingerprint
        return out


def init_train(config, rank: int, world_size: int, device: torch.device):
    """Data loader, model, optimizer and train state (reference ``training/setup.py:205-243``)."""
    from mimir_b200.train.setup import create_dataloader, create_model_and_optimizer, local_batch_tokens, \
        make_train_state
    local_batch = local_batch_tokens(config, world_size)
    loader, metadata = create_dataloader(config, local_batch, rank=rank, world_size=world_size, drop_last_batch=True)
    model, carry, optim = create_model_and_optimizer(config, metadata.model_dump(), device, local_batch)
    total = config.training_total_steps or config.epochs * int(metadata.total_length // config.global_batch_size)
    return make_train_state(config, model, carry, optim, total, device), loader, metadata


def launch(config) -> None:
    """Train according to a validated ``PretrainConfig`` (one process per GPU under torchrun)."""
    from mimir_b200.ckpt.checkpoint_io import (load_checkpoint_metadata, load_train_checkpoint,
                                               remove_stale_ephemeral_checkpoints, save_code_and_config,
                                               save_train_checkpoint)
    from mimir_b200.ckpt.contract import resolve
    from mimir_b200.optim.module_lr import module_lr_metrics, update_auto_module_rates
    from mimir_b200.optim.schedules import resolve_rewarm, update_lr
    from mimir_b200.parallel.fsdp import unwrap_model
    from mimir_b200.train.runtime import (device_for, distributed_state_fingerprint, load_synced_config,
                                          maybe_empty_cache, maybe_log_memory, move_batch_to_device, synchronize)
    from mimir_b200.train.setup import create_dataloader
    from mimir_b200.train.steps import reduce_metrics, train_accumulated_batches, validate_batches
    from mimir_b200.utils.tracking import TrainingWandbLogger, wandb

    rank, world, local = _init_distributed(config)
    config = load_synced_config(config, rank)
    if config.resume_checkpoint_path:
        config.resume_checkpoint_path = str(resolve(config.resume_checkpoint_path, config.resume_checkpoint_tag))
    Path(config.checkpoint_path).mkdir(parents=True, exist_ok=True)
    wandb.path = str(Path(config.checkpoint_path) / "metrics.jsonl")
    device = device_for(config, local)

    hook = None
    if config.suspend_control_dir:
        if config.suspension_backend == "cuda":
            from mimir_b200.train.suspension.runtime import SuspendHook
            hook = SuspendHook(config.suspend_control_dir, config.suspend_after_steps, device,
                               config.suspend_poll_interval_steps, config.suspend_wait_poll_seconds)
        else:
            if world != 1:
                raise ValueError("Distributed disk suspension requires a whole-launcher controller")
            from mimir_b200.train.disk_recovery import DiskHook
            hook = DiskHook(config.suspend_control_dir, config.suspend_after_steps, config.suspend_poll_interval_steps)

    _seed(config.seed, rank)
    local_batch = config.global_batch_size // (world * config.gradient_accumulation_steps)
    trace_print(config, rank, "init_train_begin")
    state, loader, metadata = init_train(config, rank, world, device)
    trace_print(config, rank, "init_train_end")
    val_loader = val_iter = None
    if config.data.validation_path is not None and config.validation_interval > 0 and config.validation_batches > 0:
        val_loader, _ = create_dataloader(config, local_batch, rank=rank, world_size=world, drop_last_batch=False,
                                          path=config.data.validation_path)
        val_iter = iter(val_loader)

    resume = load_train_checkpoint(config, state, rank=rank, local_batch_size=local_batch)
    resolve_rewarm(config, state.step if resume is not None else None,
                   load_checkpoint_metadata(config.resume_checkpoint_path, resume.tag)
                   if resume is not None and config.lr_rewarm_steps else {})
    cooldown = None
    if config.lr_cooldown_checkpoint is not None:
        from mimir_b200.optim.cooldown import EpochLRCooldown
        cooldown = EpochLRCooldown(config.lr_cooldown_checkpoint, config.data.path, state.step, config.lr_min_ratio)
    if state.step > state.total_steps:
        raise ValueError(f"Loaded checkpoint step {state.step} exceeds training_total_steps {state.total_steps}")

    start_epoch, skip_batches, exact_batch = 1, 0, True
    if resume is not None:
        start_epoch, skip_batches = resume.start_epoch, resume.skip_batches
        exact_batch = resume.resume_mode == "batch"
        loader.dataset.set_epoch(start_epoch - 1)
        if resume.start_row_cursor is not None:
            loader.dataset.set_start_row_cursor(resume.start_row_cursor)
        else:
            loader.dataset.set_start_batch(skip_batches)
        if rank == 0:
            print(f"Resumed from {config.resume_checkpoint_path} ({config.checkpoint_format}:{resume.tag}): "
                  f"step={state.step}, start_epoch={start_epoch}, skip_batches={skip_batches}, "
                  f"resume_mode={resume.resume_mode}, row_cursor={resume.start_row_cursor}", flush=True)

    session_step, session_t0 = state.step, time.perf_counter()
    bench = _Bench(config.max_steps is not None)
    progress = logger = None
    if rank == 0:
        import tqdm
        progress = tqdm.tqdm(total=state.total_steps, initial=state.step, disable=None)
        wandb.init(project=config.project_name, name=config.run_name, id=config.wandb_run_id,
                   resume=config.wandb_resume, config=config.model_dump() | {"train_metadata": metadata.model_dump()},
                   settings=wandb.Settings(_disable_stats=True))
        logger = TrainingWandbLogger(wandb)
        n_params = sum(p.numel() for p in state.model.parameters())
        if resume is None:
            logger.log({"num_params": n_params}, state.step)
        else:
            wandb.run.summary["num_params"] = n_params
        save_code_and_config(config, metadata)

    stop_reached = config.stop_after_step is not None and state.step >= config.stop_after_step
    if stop_reached and rank == 0:
        print(f"stop_after_step={config.stop_after_step} already reached at step={state.step}; "
              "exiting without another optimizer step", flush=True)
    skips, skip_stop = 0, False

    def max_steps_reached() -> bool:
        return config.max_steps is not None and state.step >= config.max_steps

    for epoch in range(start_epoch, config.epochs + 1):
        if stop_reached or skip_stop:
            break
        print(f"[Rank {rank}, World Size {world}]: Epoch {epoch}", flush=True)
        state.model.train()
        pending: list[dict] = []
        pending_info: Optional[dict] = None
        first = skip_batches + 1 if skip_batches > 0 else 1
        for batch_in_epoch, (batch, info) in enumerate(loader, start=first):
            batch = move_batch_to_device(batch, device)
            resume_info = info.pop("resume_info", None)
            pending.append(batch | {k: wrap_tensor(torch.tensor(v, device="cpu")) for k, v in info.items()})
            if resume_info is not None:
                pending_info = resume_info
            if len(pending) < config.gradient_accumulation_steps:
                continue

            state.step += 1
            ratio = cooldown.ratio(epoch, pending_info) if cooldown is not None else None
            lr = update_lr(config, state, ratio)
            trace_print(config, rank, f"optimizer_step_start step={state.step} batch_in_epoch={batch_in_epoch} lr={lr}")
            extra = unwrap_model(state.model).compute_train_extra_args(state)
            update_auto_module_rates(config, state.model, state.optim, extra.get("bp_steps"))
            backbone = getattr(unwrap_model(state.model), "model", None)
            if hasattr(backbone, "configure_gate_updates"):
                backbone.configure_gate_updates(state.optim, extra["bp_steps"])

            diagnostics = None
            if config.stability_diagnostics_interval > 0 and state.step % config.stability_diagnostics_interval == 0:
                from mimir_b200.utils.stability import StabilityDiagnostics
                diagnostics = StabilityDiagnostics(
                    step=state.step, rank=rank,
                    output_path=config.stability_diagnostics_output or os.path.join(
                        config.checkpoint_path or "logs", "stability_diagnostics.jsonl"),
                    context={"epoch": epoch, "batch_in_epoch": batch_in_epoch, "bp_steps": extra.get("bp_steps"),
                             "lr": lr, "global_batch_size": config.global_batch_size,
                             "gradient_accumulation_steps": config.gradient_accumulation_steps,
                             "distributed_strategy": config.distributed_strategy,
                             "fwd_bwd_dtype": config.fwd_bwd_dtype, "gradient_clip_norm": config.gradient_clip_norm,
                             "gradient_skip_norm": config.gradient_skip_norm})
            timing = config.experiment_metrics_output is not None
            if timing:
                synchronize(device)
                t_probe = time.perf_counter()
            mem_due = config.memory_log_interval > 0 and state.step % config.memory_log_interval == 0
            maybe_log_memory(state.step, "before_train", device, mem_due)
            if diagnostics is not None:
                if state.carry is not None:
                    raise RuntimeError("stability diagnostics shadow replay currently requires a stateless carry")
                from mimir_b200.utils.stability import diagnostic_prefixlm_batch
                devices = [device.index] if device.type == "cuda" and device.index is not None else []
                with torch.random.fork_rng(devices=devices):
                    shadow = [diagnostic_prefixlm_batch(b, max_tokens=config.stability_diagnostics_max_tokens_per_microbatch)
                              for b in pending]
                    train_accumulated_batches(config, rank, state, shadow, use_compiled=False,
                                              optimizer_step_enabled=False, **extra,
                                              stability_diagnostics=diagnostics)
            if timing:
                synchronize(device)
                t_train = time.perf_counter()
            metrics, skipped = train_accumulated_batches(config, rank, state, pending, config.compile_train_batch,
                                                         **extra)
            pending = []
            if timing:
                synchronize(device)
                t_done = time.perf_counter()
            if diagnostics is not None and rank == 0:
                logger.log(diagnostics.wandb_summary | diagnostics.wandb_detailed, optimizer_step=state.step)
            if config.gradient_skip_norm is not None:
                skips = skips + 1 if skipped else 0
                ref = next(iter(metrics.values()))[0]
                metrics["consecutive_gradient_skips"] = (ref.new_tensor(float(skips)), ref.new_ones(()))
                skip_stop = skipped and skips >= config.gradient_skip_max_consecutive
                if skipped and rank == 0:
                    print(f"Skipped optimizer step {state.step}: gradient norm "
                          f"{float(metrics['grad_norm'][0].item()):.6g} exceeded gradient_skip_norm="
                          f"{config.gradient_skip_norm}; consecutive={skips}/{config.gradient_skip_max_consecutive}",
                          flush=True)
                if skip_stop and rank == 0:
                    print("Maximum consecutive gradient skips reached; saving a regular checkpoint and exiting "
                          "cleanly", flush=True)
            if bench.enabled and rank == 0:
                bench.tick(device)
            maybe_log_memory(state.step, "after_train", device, mem_due)
            maybe_empty_cache(state.step, device, config.empty_cache_interval)

            if state.step % config.log_interval == 0 or skipped or timing:
                if device.type == "cuda":
                    from mimir_b200.ops._ext import check_kernel_status
                    check_kernel_status(device, state.step)  # a timed-out kernel wait invalidates the step
                metrics = reduce_metrics(metrics, prefix="train/")
                if rank == 0:
                    metrics.update(module_lr_metrics(config, lr, extra.get("bp_steps")))
                    if hasattr(backbone, "gate_alpha"):
                        metrics["train/gate_alpha"] = float(backbone.gate_alpha.item())
                        metrics["train/lr_gates"] = lr
                    if timing:
                        from mimir_b200.utils.diagnostics import append_jsonl
                        append_jsonl(config.experiment_metrics_output, {
                            "step": state.step, "epoch": epoch, "batch_in_epoch": batch_in_epoch, "train/lr": lr,
                            **extra, **metrics, "training_seconds": t_done - t_train,
                            "probe_seconds": t_train - t_probe})
                    bench.last_metrics = dict(metrics)
                    if bench.enabled:
                        bench.history.append({"step": state.step, **metrics})
                    progress.update(state.step - progress.n)
                    logger.log(metrics | extra | {"train/lr": lr}, state.step)
                    write_progress(Path(config.checkpoint_path) / "progress.json", {
                        "completed": state.step - session_step, "total": state.total_steps - session_step,
                        "optimizer_step": state.step, "epoch": epoch,
                        "elapsed_seconds": time.perf_counter() - session_t0})

            if val_iter is not None and state.step % config.validation_interval == 0:
                val = validate_batches(config, rank, state, val_iter, config.validation_batches, device, local_batch,
                                       **extra)
                if val is None:
                    val_iter = iter(val_loader)
                    val = validate_batches(config, rank, state, val_iter, config.validation_batches, device,
                                           local_batch, **extra)
                if val is not None:
                    val = reduce_metrics(val, prefix="val/")
                    if rank == 0:
                        logger.log(val, state.step)
            del metrics

            stop_reached = config.stop_after_step is not None and state.step >= config.stop_after_step
            step_tag = f"step_{state.step}"
            ckpt_args = dict(local_batch_size=local_batch, resume_info=pending_info, batch_in_epoch_exact=exact_batch)
            saved_step = False
            if ((config.checkpoint_step_interval is not None and state.step % config.checkpoint_step_interval == 0)
                    or stop_reached or skip_stop):
                save_train_checkpoint(config, state, step_tag, epoch, batch_in_epoch, rank, **ckpt_args)
                saved_step = True
            if (config.ephemeral_checkpoint_step_interval is not None
                    and state.step % config.ephemeral_checkpoint_step_interval == 0):
                if saved_step:
                    remove_stale_ephemeral_checkpoints(config, step_tag, rank)
                else:
                    tag = f"ephemeral_step_{state.step}"
                    save_train_checkpoint(config, state, tag, epoch, batch_in_epoch, rank, checkpoint_kind="ephemeral",
                                          **ckpt_args)
                    remove_stale_ephemeral_checkpoints(config, tag, rank)
            if hook is not None:
                def save_for_suspend(saved=saved_step, tag=step_tag, b=batch_in_epoch, e=epoch, a=ckpt_args):
                    if not saved:
                        save_train_checkpoint(config, state, tag, e, b, rank, **a)
                    return str(Path(config.checkpoint_path) / tag / f"checkpoint_state_{tag}.json")

                hook.after_step(state.step, save_for_suspend, stopping=stop_reached or skip_stop or max_steps_reached())
            if stop_reached or skip_stop or max_steps_reached():
                break
        skip_batches = 0
        if stop_reached or skip_stop or max_steps_reached():
            break
        if epoch % config.checkpoint_interval == 0 or epoch == config.epochs:
            save_train_checkpoint(config, state, f"epoch_{epoch}", epoch, 0, rank, local_batch_size=local_batch,
                                  batch_in_epoch_exact=True)

    fingerprint = None
    if config.max_steps is not None and config.benchmark_state_fingerprint:
        fingerprint = distributed_state_fingerprint(config, state, device)
    if rank == 0 and (summary := bench.summary(config, world, fingerprint)) is not None:
        if os.environ.get("BENCH_OUTPUT"):
            Path(os.environ["BENCH_OUTPUT"]).write_text(json.dumps(summary, indent=2))
        print("[bench] " + json.dumps({k: v for k, v in summary.items() if k != "all_step_seconds"}), flush=True)
    if progress is not None:
        progress.close()
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
    wandb.finish()
