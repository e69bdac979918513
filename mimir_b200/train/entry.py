"""``mimir_b200 train`` entry: compose + validate the config, then train, supervise or launch.

Reference behaviour: ``src/mimir/training/entry.py:5-34``.  ``--suspendable`` runs one
recovery controller outside torchrun: the disk supervisor (default) or the CUDA-suspension
launcher (``suspension_backend=cuda`` with ``suspension_settings``).
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path
from typing import Sequence

from mimir_b200.config.schema import PretrainConfig, load_config


def configuration(overrides: Sequence[str]) -> PretrainConfig:
    return load_config(list(overrides))


def run(overrides: Sequence[str], suspendable: bool = False):
    overrides = list(overrides)
    if suspendable and not any(o.startswith("suspend_control_dir=") for o in overrides):
        checkpoint = next((o.split("=", 1)[1] for o in overrides if o.startswith("checkpoint_path=")), None)
        if not checkpoint:
            raise ValueError("--suspendable requires checkpoint_path=<directory>")
        overrides.append(f"suspend_control_dir={Path(checkpoint).resolve() / 'control'}")
    config = configuration(overrides)
    if suspendable:
        import os
        if "LOCAL_RANK" in os.environ:
            raise ValueError("Run one suspension controller outside torchrun, not one per rank")
        if config.suspension_backend == "cuda":
            if not config.suspension_settings:
                raise ValueError("CUDA suspension requires suspension_settings=<shim/settings.json>")
            return subprocess.run([sys.executable, "-m", "mimir_b200.train.suspension.launcher", "--settings",
                                   config.suspension_settings, "--control-root", config.suspend_control_dir, "--",
                                   sys.executable, "-m", "mimir_b200", "train", *overrides], check=True)
        from mimir_b200.train.disk_recovery import supervise
        return supervise(overrides, config)
    from mimir_b200.train.loop import launch
    return launch(config)
