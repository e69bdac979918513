"""Cosine learning-rate cooldown over what is left of an epoch, anchored at a checkpoint.

Behavioural reference: ``src/mimir/model/epoch_lr_cooldown.py:9-41``.  The anchor checkpoint's
sidecar (``checkpoint_state_<tag>.json``) fixes the step, the epoch and the global row cursor.
The LR ratio follows half a cosine from 1 at the anchor's row to ``min_ratio`` at the last row of
that epoch (the epoch's ``inst_start.npy`` row count), and stays at ``min_ratio`` in later epochs.
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass
from pathlib import Path

import numpy as np


@dataclass(frozen=True)
class _Anchor:
    step: int
    epoch: int
    row: int
    data_path: Path

    @staticmethod
    def read(sidecar) -> "_Anchor":
        fields = json.loads(Path(sidecar).read_text())
        return _Anchor(step=int(fields["step"]), epoch=int(fields["epoch"]),
                       row=int(fields["global_row_cursor_in_epoch"]), data_path=Path(fields["data_path"]))


def _half_cosine(progress: float, floor: float) -> float:
    """1 at progress 0 down to ``floor`` at progress 1."""
    return floor + (1.0 - floor) * (1.0 + math.cos(math.pi * progress)) / 2.0


def _epoch_rows(dataset_path, epoch: int) -> int:
    starts = np.load(Path(dataset_path) / f"epoch_{epoch - 1}" / "inst_start.npy", mmap_mode="r",
                     allow_pickle=False)
    return int(starts.shape[0])


class EpochLRCooldown:
    """``ratio(epoch, resume_info)`` gives the LR multiplier for the batch whose row cursor ends at
    ``resume_info["global_row_end"]``."""

    def __init__(self, checkpoint_metadata, dataset_path, resume_step: int, min_ratio: float):
        anchor = _Anchor.read(checkpoint_metadata)
        if anchor.data_path.resolve() != Path(dataset_path).resolve():
            raise ValueError("LR cooldown dataset differs from anchor checkpoint")
        if resume_step < anchor.step:
            raise ValueError("LR cooldown cannot resume before its anchor step")
        if not (math.isfinite(min_ratio) and 0.0 <= min_ratio <= 1.0):
            raise ValueError("LR cooldown min ratio must be between zero and one")
        last = _epoch_rows(dataset_path, anchor.epoch)
        if anchor.row < 0 or anchor.row >= last:
            raise ValueError("LR cooldown anchor has no remaining epoch rows")
        self.start_step, self.epoch, self.start_row, self.end_row = anchor.step, anchor.epoch, anchor.row, last
        self.min_ratio = min_ratio

    def ratio(self, epoch: int, resume_info) -> float:
        if epoch != self.epoch:
            if epoch < self.epoch:
                raise ValueError("LR cooldown epoch precedes anchor checkpoint")
            return self.min_ratio
        row = (resume_info or {}).get("global_row_end")
        if row is None:
            raise ValueError("LR cooldown requires dataset row-cursor metadata")
        row = int(row)
        if row < self.start_row or row > self.end_row:
            raise ValueError("LR cooldown row cursor outside anchored epoch interval")
        return _half_cosine((row - self.start_row) / (self.end_row - self.start_row), self.min_ratio)
