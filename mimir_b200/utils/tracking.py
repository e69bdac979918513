"""Metric sinks: local ``metrics.jsonl`` by default, Weights & Biases only with ``MIMIR_WANDB=1``.

Reference behaviour: ``src/mimir/training/tracking.py:5-73``.  ``TrainingWandbLogger`` keeps
the optimizer step as the ``train/step`` axis and never rewinds the tracker's history cursor
on resume (rows after a resume are offset, never overwritten).
"""
from __future__ import annotations

import json
import os
from types import SimpleNamespace


class LocalTracker:
    def __init__(self):
        self.run = None
        self.path = None
        self.remote = None

    def init(self, **kwargs):
        if os.environ.get("MIMIR_WANDB") == "1":
            import wandb as remote
            self.remote = remote
            kwargs["settings"] = remote.Settings(**kwargs.get("settings", {}))
            self.run = remote.init(**kwargs)
            return self.run
        self.run = SimpleNamespace(step=0, summary={}, log_code=lambda _path: None)
        return self.run

    @staticmethod
    def Settings(**kwargs):
        return kwargs

    def define_metric(self, *args, **kwargs):
        if self.remote is not None:
            self.remote.define_metric(*args, **kwargs)

    def log(self, metrics, step, commit=True):
        if self.remote is not None:
            self.remote.log(metrics, step=step, commit=commit)
            self.run = self.remote.run
            return
        if self.path:
            with open(self.path, "a") as f:
                f.write(json.dumps(dict(metrics), allow_nan=False) + "\n")
        self.run.step = step + 1

    def finish(self):
        if self.remote is not None:
            self.remote.finish()
        self.run = None


class TrainingWandbLogger:
    def __init__(self, tracker):
        self.tracker = tracker
        self.registered = {"train/step"}
        self.offset = None
        tracker.define_metric("train/step")

    def log(self, metrics: dict, optimizer_step: int) -> None:
        if type(optimizer_step) is not int or optimizer_step < 0:
            raise ValueError("Nonnegative integer optimizer step required")
        if "train/step" in metrics and metrics["train/step"] != optimizer_step:
            raise ValueError("Conflicting optimizer step in metrics")
        for key in sorted(metrics):
            if key not in self.registered:
                self.tracker.define_metric(key, step_metric="train/step")
                self.registered.add(key)
        run = self.tracker.run
        if run is None or type(run.step) is not int or run.step < 0:
            raise RuntimeError("An initialized tracker run with a valid history cursor is required")
        if self.offset is None:
            self.offset = max(0, run.step - optimizer_step)
        history = max(optimizer_step + self.offset, run.step)
        self.tracker.log(dict(metrics) | {"train/step": optimizer_step}, step=history, commit=True)


wandb = LocalTracker()
