"""Cosine LR cooldown over the rest of an epoch, anchored at a checkpoint's row cursor.

Reference behaviour: ``src/mimir/model/epoch_lr_cooldown.py:9-41``.  The anchor sidecar
(``checkpoint_state_<tag>.json``) fixes the step, epoch and global row cursor; the ratio falls
from 1 to ``min_ratio`` as the row cursor moves from the anchor to the end of that epoch and
stays at ``min_ratio`` in later epochs.
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np


class EpochLRCooldown:
    def __init__(self, checkpoint_metadata, dataset_path, resume_step: int, min_ratio: float):
        meta = json.loads(Path(checkpoint_metadata).read_text())
        self.start_step, self.epoch = int(meta["step"]), int(meta["epoch"])
        self.start_row = int(meta["global_row_cursor_in_epoch"])
        if Path(meta["data_path"]).resolve() != Path(dataset_path).resolve():
            raise ValueError("LR cooldown dataset differs from anchor checkpoint")
        if resume_step < self.start_step:
            raise ValueError("LR cooldown cannot resume before its anchor step")
        if not math.isfinite(min_ratio) or not 0 <= min_ratio <= 1:
            raise ValueError("LR cooldown min ratio must be between zero and one")
        self.min_ratio = min_ratio
        rows = np.load(Path(dataset_path) / f"epoch_{self.epoch - 1}" / "inst_start.npy", mmap_mode="r",
                       allow_pickle=False)
        self.end_row = len(rows)
        if not 0 <= self.start_row < self.end_row:
            raise ValueError("LR cooldown anchor has no remaining epoch rows")

    def ratio(self, epoch: int, resume_info) -> float:
        if epoch < self.epoch:
            raise ValueError("LR cooldown epoch precedes anchor checkpoint")
        if epoch > self.epoch:
            return self.min_ratio
        if resume_info is None or "global_row_end" not in resume_info:
            raise ValueError("LR cooldown requires dataset row-cursor metadata")
        row = int(resume_info["global_row_end"])
        if not self.start_row <= row <= self.end_row:
            raise ValueError("LR cooldown row cursor outside anchored epoch interval")
        progress = (row - self.start_row) / (self.end_row - self.start_row)
        return self.min_ratio + (1 - self.min_ratio) * 0.5 * (1 + math.cos(math.pi * progress))
