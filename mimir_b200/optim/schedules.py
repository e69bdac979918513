"""Learning-rate schedules.

Reference: ``src/mimir/training/schedules.py:11-35`` (warmup + cosine with floor),
``src/mimir/model/lr_piecewise.py`` (absolute-step piecewise linear),
``src/mimir/model/lr_rewarm.py`` (checkpoint-anchored, optionally geometric-staged rewarm)
and ``src/mimir/model/module_learning_rates.py:6-12`` (windowed cosine).
"""
from __future__ import annotations

import math
from typing import Optional

from mimir_b200.optim.module_lr import windowed_cosine_lr


def validate_lr_points(points):
    if len(points) < 2:
        raise ValueError("lr_piecewise_points requires at least two anchors")
    prev = -1
    for step, rate in points:
        if step < 0 or int(step) != step or step <= prev:
            raise ValueError("LR anchor steps must be nonnegative and strictly increasing")
        if not math.isfinite(rate) or rate <= 0:
            raise ValueError("LR anchor rates must be finite and positive")
        prev = step


def piecewise_lr(points, step):
    if step <= points[0][0]:
        return points[0][1]
    for (s0, r0), (s1, r1) in zip(points, points[1:]):
        if step <= s1:
            return r0 + (r1 - r0) * ((step - s0) / (s1 - s0))
    return points[-1][1]


def rewarm_metadata(config):
    if not config.lr_rewarm_steps:
        return None
    out = dict(start_step=config.lr_rewarm_start_step, steps=config.lr_rewarm_steps,
               start_ratio=config.lr_rewarm_start_ratio, base_lr=config.lr)
    if getattr(config, "lr_rewarm_stages", 1) != 1:
        out["stages"] = config.lr_rewarm_stages
    return out


def resolve_rewarm(config, resume_step, metadata):
    if not config.lr_rewarm_steps:
        if config.lr_rewarm_start_step is not None:
            raise ValueError("lr_rewarm_start_step requires lr_rewarm_steps > 0")
        return
    if resume_step is None:
        raise ValueError("LR rewarm requires a resumed checkpoint")
    stages = getattr(config, "lr_rewarm_stages", 1)
    if stages < 1 or (stages > 1 and config.lr_rewarm_start_ratio <= 0):
        raise ValueError("Staged rewarm requires positive stages and starting ratio")
    saved = metadata.get("lr_rewarm")
    if config.lr_rewarm_start_step is None:
        if saved:
            want = rewarm_metadata(config)
            for key in ("steps", "start_ratio", "base_lr"):
                if saved.get(key) != want[key]:
                    raise ValueError("Rewarm settings changed; supply an explicit new lr_rewarm_start_step")
            if saved.get("stages", 1) != stages:
                raise ValueError("Rewarm stages changed; supply an explicit new lr_rewarm_start_step")
            config.lr_rewarm_start_step = saved["start_step"]
        else:
            config.lr_rewarm_start_step = resume_step
    if config.lr_rewarm_start_step is None or not 0 <= config.lr_rewarm_start_step <= resume_step:
        raise ValueError("Rewarm anchor must be at or before the resume step")
    start, end = config.lr_decay_start_step, config.lr_decay_end_step
    if start is not None or end is not None:
        windowed_cosine_lr(config.lr, config.lr_min_ratio, resume_step, start, end)
        if start < config.lr_rewarm_start_step + config.lr_rewarm_steps:
            raise ValueError("Cosine decay must start after rewarm finishes; clear stale decay bounds")
    elif config.lr_min_ratio != 1:
        raise ValueError("Rewarm without explicit decay requires lr_min_ratio=1 (hold after rewarm)")


def rewarm_lr(config, step):
    if config.lr_rewarm_start_step is None:
        raise ValueError("Rewarm anchor has not been resolved from checkpoint")
    progress = min(1.0, max(0.0, (step - config.lr_rewarm_start_step) / config.lr_rewarm_steps))
    if progress < 1:
        stages = getattr(config, "lr_rewarm_stages", 1)
        ratio = config.lr_rewarm_start_ratio
        if stages > 1:
            pos = progress * stages
            k = int(pos)
            lo, hi = ratio ** (1 - k / stages), ratio ** (1 - (k + 1) / stages)
            return config.lr * (lo + (hi - lo) * (pos - k))
        return config.lr * (ratio + (1 - ratio) * progress)
    if config.lr_decay_start_step is not None:
        return windowed_cosine_lr(config.lr, config.lr_min_ratio, step, config.lr_decay_start_step,
                                  config.lr_decay_end_step)
    return config.lr


def scheduled_lr(config, step: int, total_steps: int, cooldown_ratio: Optional[float] = None) -> float:
    if getattr(config, "lr_piecewise_points", None) is not None:
        return piecewise_lr(config.lr_piecewise_points, step)
    if cooldown_ratio is not None:
        return config.lr * cooldown_ratio
    if config.lr_rewarm_steps:
        return rewarm_lr(config, step)
    if config.lr_decay_start_step is not None or config.lr_decay_end_step is not None:
        return windowed_cosine_lr(config.lr, config.lr_min_ratio, step, config.lr_decay_start_step,
                                  config.lr_decay_end_step)
    if step < config.lr_warmup_steps:
        return config.lr * min(1.0, step / config.lr_warmup_steps)
    progress = (step - config.lr_warmup_steps) / max(1, total_steps - config.lr_warmup_steps)
    return config.lr * (config.lr_min_ratio
                        + max(0.0, (1 - config.lr_min_ratio) * 0.5 * (1.0 + math.cos(math.pi * progress))))


def update_lr(config, train_state, cooldown_ratio: Optional[float] = None) -> float:
    lr = scheduled_lr(config, train_state.step, train_state.total_steps, cooldown_ratio)
    for group in train_state.optim.param_groups:
        group["lr"] = lr
    return lr
