"""One optimizer step over gradient-accumulation microbatches.

Reference behaviour: ``src/mimir/training/steps.py:16-300``.  Each microbatch's loss is
weighted by its share of supervised tokens (counts all-reduced with AVG); DDP/FSDP
gradient sync happens on the last microbatch only (HSDP ``reduce_scatter`` mode keeps the
shard-local reduce-scatter per microbatch and defers the replica all-reduce); optional
global-norm clipping and anomaly skipping run before the optimizer; routing-balance
counts commit after a successful step.

torch.compile is never the hot path: the model's hot ops are already hand-written sm_100a
kernels, so microbatches run eagerly (``compile_train_batch`` is accepted for config
compatibility and uses ``torch.compile`` only when explicitly enabled).
"""
from __future__ import annotations

from contextlib import nullcontext

import torch
import torch.distributed as dist
from torch import Tensor
from torch.distributed.fsdp import FSDPModule
from torch.nn.parallel import DistributedDataParallel

from mimir_b200.models.common import IGNORE_LABEL_ID, wrap_tensor
from mimir_b200.optim.clipping import clip_grad_norm_mean_units
from mimir_b200.optim.routing_balance import has_balanced_routers, routing_balance
from mimir_b200.utils.trace import nvtx_range, trace_print


def forward_backward_batch(train_state, batch: dict, loss_scale: Tensor, **kwargs):
    device_type = batch["inputs"].device.type
    use_autocast = ((device_type in ("mps", "cpu") and train_state.fwd_bwd_dtype != torch.float32)
                    or (device_type == "cuda" and train_state.use_cuda_autocast))
    with torch.autocast(device_type=device_type, dtype=train_state.fwd_bwd_dtype, enabled=use_autocast,
                        cache_enabled=False):
        train_state.carry, loss, metrics = train_state.model(batch=batch, carry=train_state.carry, **kwargs)
    (loss * loss_scale).backward()
    return metrics


_COMPILED = {}


def compiled_forward_backward(mode: str):
    if mode not in ("default", "max-autotune-no-cudagraphs"):
        raise ValueError(f"Unsupported compile_train_batch_mode: {mode}")
    if mode not in _COMPILED:
        kw = {} if mode == "default" else {"mode": mode}
        _COMPILED[mode] = torch.compile(forward_backward_batch, dynamic=False, **kw)
    return _COMPILED[mode]


def _add_metrics(total, metrics):
    if total is None:
        return {k: (s.detach(), d.detach()) for k, (s, d) in metrics.items()}
    for k, (s, d) in metrics.items():
        ts, td = total[k]
        total[k] = (ts + s.detach(), td + d.detach())
    return total


def supervised_token_count(config, rank: int, batch: dict) -> Tensor:
    return supervised_token_counts(config, rank, [batch])[0]


def supervised_token_counts(config, rank: int, batches: list) -> list[Tensor]:
    """Supervised-token count of every micro-batch, averaged over the ranks in ONE all-reduce
    (the reference issues one per micro-batch, ``src/mimir/training/steps.py:66-76``)."""
    counts = torch.stack([(b["labels"] != IGNORE_LABEL_ID).sum().to(torch.float32) for b in batches])
    if dist.is_available() and dist.is_initialized():
        trace_print(config, rank, "supervised_count_all_reduce_begin")
        dist.all_reduce(counts, op=dist.ReduceOp.AVG)
        trace_print(config, rank, "supervised_count_all_reduce_end")
    return list(counts.unbind(0))


def train_accumulated_batches(config, rank: int, train_state, batches: list, use_compiled: bool = False,
                              zero_grad_after_step: bool = True, optimizer_step_enabled: bool = True, **kwargs):
    """One optimizer step over ``batches`` (gradient accumulation); returns ``(metrics, skipped)``.
    Models with balanced MoE routers record their selections for the whole step and move the
    selection biases only when the optimizer update ran."""
    if not has_balanced_routers(train_state.model):
        return _accumulate_and_step(config, rank, train_state, batches, use_compiled, zero_grad_after_step,
                                    optimizer_step_enabled, **kwargs)
    with routing_balance(train_state.model) as ledger:
        metrics, skipped = _accumulate_and_step(config, rank, train_state, batches, use_compiled,
                                                zero_grad_after_step, optimizer_step_enabled, **kwargs)
        if optimizer_step_enabled and not skipped:
            ledger.commit()
    return metrics, skipped


def _forward_backward_all(config, rank, train_state, batches, counts, total, step_fn, model, hsdp_rs, overlap_engine,
                          **kwargs):
    """Forward and backward of every micro-batch, summing their metrics; ``overlap_engine`` (a
    replicated engine) is armed before the last backward so that it updates buckets during it."""
    metrics = None
    for i, (batch, count) in enumerate(zip(batches, counts), start=1):
        last = i == len(batches)
        if last and overlap_engine is not None:
            overlap_engine.arm_overlap(train_state.optim)
        ctx = nullcontext()
        if isinstance(model, DistributedDataParallel) and not last:
            ctx = model.no_sync()
        elif isinstance(model, FSDPModule):
            if hsdp_rs:
                model.set_requires_gradient_sync(True, recurse=True)
                model.set_requires_all_reduce(last, recurse=True)
            else:
                model.set_requires_gradient_sync(last, recurse=True)
        with ctx, nvtx_range(f"microbatch_{i}"):
            metrics = _add_metrics(metrics, step_fn(train_state, batch, count / total, **kwargs))
        trace_print(config, rank, f"forward_backward_end step={train_state.step} microbatch={i}")
    return metrics


def _accumulate_and_step(config, rank: int, train_state, batches: list, use_compiled: bool,
                         zero_grad_after_step: bool, optimizer_step_enabled: bool, **kwargs):
    trace_print(config, rank, f"train_accumulated_begin step={train_state.step} microbatches={len(batches)}")
    if config.gradient_skip_norm is not None and train_state.carry is not None:
        raise RuntimeError("gradient_skip_norm currently supports only models with no persistent carry")
    counts = supervised_token_counts(config, rank, batches)
    total = torch.stack(counts).sum().clamp_min(1.0)
    step_fn = compiled_forward_backward(config.compile_train_batch_mode) if use_compiled else forward_backward_batch
    train_state.optim.zero_grad()
    model = train_state.model
    hsdp_rs = (isinstance(model, FSDPModule) and config.fsdp_accumulation_sync_mode == "reduce_scatter"
               and config.fsdp_shard_degree is not None and dist.is_available() and dist.is_initialized()
               and config.fsdp_shard_degree < dist.get_world_size())
    metrics = None
    engine = getattr(model, "replicated_engine", None)
    # The replicated engine may run the optimizer update bucket by bucket inside the last backward
    # when nothing between the backward and the step reads the gradients or the old weights.
    overlap = (engine is not None and optimizer_step_enabled and not use_compiled
               and config.gradient_clip_norm is None and config.gradient_skip_norm is None
               and kwargs.get("stability_diagnostics") is None and not config.experiment_update_probe_interval)
    streams = engine.compute_stream() if overlap else nullcontext()
    try:
        with streams:
            metrics = _forward_backward_all(config, rank, train_state, batches, counts, total, step_fn, model,
                                            hsdp_rs, engine if overlap else None, **kwargs)
    except BaseException:
        if engine is not None:
            engine.disarm_overlap()
        raise
    finally:
        if isinstance(model, FSDPModule):
            model.set_requires_gradient_sync(True, recurse=True)
            model.set_requires_all_reduce(True, recurse=True)

    diag = kwargs.get("stability_diagnostics")
    if diag is not None:
        from mimir_b200.parallel.fsdp import unwrap_model
        diag.record_model_state(unwrap_model(model), train_state.optim)
        diag.finalize(detailed_wandb=config.stability_diagnostics_wandb_detailed)

    if not optimizer_step_enabled:
        if zero_grad_after_step:
            train_state.optim.zero_grad()
        return metrics, False

    skipped = False
    if config.gradient_clip_norm is not None or config.gradient_skip_norm is not None:
        scale = 1.0
        if isinstance(model, FSDPModule) and dist.is_available() and dist.is_initialized():
            scale = float(dist.get_world_size())
        max_norm = config.gradient_clip_norm if config.gradient_clip_norm is not None else config.gradient_skip_norm
        engine = getattr(model, "replicated_engine", None)
        if engine is not None:
            clip = _replicated_clip(engine, train_state.optim, max_norm)
        else:
            clip = clip_grad_norm_mean_units(model.parameters(), max_norm=max_norm, summed_gradient_scale=scale)
        one = clip.total_norm.new_ones(())
        metrics["grad_norm"] = (clip.total_norm.detach(), one)
        if config.gradient_clip_norm is not None:
            metrics["grad_clip_coefficient"] = (clip.clip_coefficient.detach(), one)
            metrics["grad_clipped"] = (clip.clipped.detach(), one)
        if config.gradient_skip_norm is not None:
            flag = (clip.total_norm > clip.total_norm.new_tensor(config.gradient_skip_norm)).to(torch.int32)
            if dist.is_available() and dist.is_initialized():
                dist.all_reduce(flag, op=dist.ReduceOp.MAX)
            skipped = bool(flag.item())
            metrics["optimizer_step_skipped"] = (flag.to(clip.total_norm.dtype), one)

    probe = None
    if config.experiment_update_probe_interval and train_state.step % config.experiment_update_probe_interval == 0:
        if config.experiment_metrics_output is None:
            raise ValueError("Update probes require experiment_metrics_output")
        from mimir_b200.utils.diagnostics import ParameterUpdateProbe
        probe = ParameterUpdateProbe(model)
    if not skipped:
        trace_print(config, rank, f"optim_step_begin step={train_state.step}")
        with nvtx_range("optimizer_step"):
            train_state.optim.step()
        trace_print(config, rank, f"optim_step_end step={train_state.step}")
    elif getattr(model, "replicated_engine", None) is not None:
        model.replicated_engine.reduced = None
        train_state.optim.grad_scale = None
    if probe is not None:
        from mimir_b200.utils.diagnostics import append_jsonl
        updates = probe.finish(next(model.parameters()).device)
        if rank == 0:
            append_jsonl(str(config.experiment_metrics_output) + ".updates.jsonl",
                         {"step": train_state.step, "optimizer_step_skipped": skipped, "includes_weight_decay": True,
                          "parameters": updates})
    if zero_grad_after_step:
        train_state.optim.zero_grad()
    trace_print(config, rank, f"train_accumulated_end step={train_state.step} skipped={skipped}")
    return metrics, skipped


def _replicated_clip(engine, optim, max_norm: float):
    """Global-norm clipping for replicated weights: the norm is taken over the reduced (summed)
    gradients, computed by the engine's reduce pass; the update pass then applies the coefficient."""
    from mimir_b200.optim.clipping import GradientClipMetrics
    world = float(engine.world)
    raw = engine.reduce_for_clipping().sqrt().to(torch.float32).reshape(())
    if not bool(torch.isfinite(raw)):
        raise RuntimeError(f"The total norm of order 2.0 for gradients is non-finite ({raw.item()})")
    raw_max = max_norm * world
    coeff = torch.clamp(raw.new_tensor(raw_max) / (raw + 1e-6), max=1.0)
    optim.grad_scale = coeff.reshape(1).to(engine.device)
    norm = raw / world
    return GradientClipMetrics(total_norm=norm, clip_coefficient=coeff, clipped=(norm > max_norm).to(norm.dtype))


@torch.inference_mode()
def validate_batches(config, rank, train_state, val_iter, num_batches, device, local_batch_size, **kwargs):
    from mimir_b200.train.runtime import move_batch_to_device
    if num_batches <= 0:
        return None
    was_training = train_state.model.training
    train_state.model.eval()
    old = train_state.carry
    metrics = None
    for _ in range(num_batches):
        try:
            batch, info = next(val_iter)
        except StopIteration:
            break
        batch = move_batch_to_device(batch, device)
        info.pop("resume_info", None)
        batch = batch | {k: wrap_tensor(torch.tensor(v)) for k, v in info.items()}
        use_autocast = batch["inputs"].device.type == "cuda" and train_state.use_cuda_autocast
        with torch.autocast(device_type=batch["inputs"].device.type, dtype=train_state.fwd_bwd_dtype,
                            enabled=use_autocast, cache_enabled=False):
            train_state.carry, _, m = train_state.model(batch=batch, carry=train_state.carry, **kwargs)
        metrics = _add_metrics(metrics, m)
    train_state.carry = old
    if was_training:
        train_state.model.train()
    return metrics


@torch.inference_mode()
def reduce_metrics(local_metrics: dict, prefix: str) -> dict:
    keys = sorted(local_metrics)
    values = torch.stack([local_metrics[k][0].float() for k in keys] + [local_metrics[k][1].float() for k in keys])
    if dist.is_available() and dist.is_initialized():
        dist.reduce(values, dst=0)
    sums, divs = values.chunk(2, dim=-1)
    out = (sums / divs).cpu().numpy().tolist()
    return {prefix + k: out[i] for i, k in enumerate(keys)}
