"""Portable suspension: checkpoint, exit with status 75, restart from the published checkpoint.

Reference behaviour: ``src/mimir/training/disk_recovery.py:10-44``.

* ``DiskHook.after_step`` stops at a configured boundary step, or at a multiple of the poll
  interval while ``<control>/suspend.request`` exists: it saves, records
  ``disk-ready.json = {step, checkpoint}`` (``checkpoint`` is the sidecar JSON inside the
  published tag directory) and raises ``SystemExit(75)``.
* ``supervise`` owns recovery under ``<control>/recovery.lock``: it waits while
  ``<control>/hold`` exists, runs the training child, and on status 75 validates the
  published checkpoint (manifest step must equal the ready step) and relaunches with
  ``resume_checkpoint_path``/``resume_checkpoint_tag`` (dropping ``initialize_from``, which only
  applies to the first start).  Status 0 ends; any other status
  raises (failures are surfaced, never retried endlessly).  A launcher child (``command=``,
  e.g. torchrun over several ranks) reports a worker's status 75 as a failure of its own, so a
  non-zero status also counts as a suspension when this attempt wrote a new
  ``disk-ready.json`` for a later step than the one it resumed from.
"""
from __future__ import annotations

import json
import subprocess
import sys
import time
from pathlib import Path
from typing import Optional, Sequence

from mimir_b200.train.suspension.protocol import atomic_write, exclusive

SUSPEND_EXIT_CODE = 75


class DiskHook:
    def __init__(self, root, boundaries, interval: int):
        self.root = Path(root)
        self.root.mkdir(parents=True, exist_ok=True)
        self.boundaries = set(boundaries)
        self.interval = max(1, int(interval))

    def after_step(self, step: int, save_checkpoint, stopping: bool = False, **_unused) -> None:
        if stopping:
            return
        request = self.root / "suspend.request"
        if step not in self.boundaries and not (step % self.interval == 0 and request.exists()):
            return
        checkpoint = save_checkpoint()
        atomic_write(self.root / "disk-ready.json", {"step": step, "checkpoint": str(checkpoint)})
        request.unlink(missing_ok=True)
        raise SystemExit(SUSPEND_EXIT_CODE)


def _ready_stamp(root: Path) -> Optional[tuple]:
    ready = root / "disk-ready.json"
    if not ready.exists():
        return None
    return ready.stat().st_mtime_ns, json.loads(ready.read_text()).get("step")


def _suspended_now(root: Path, before: Optional[tuple]) -> bool:
    """The attempt that just ended wrote a new ready record for a later step."""
    now = _ready_stamp(root)
    return now is not None and now != before and (before is None or (now[1] or 0) > (before[1] or 0))


def _child_command(args: Sequence[str]) -> list[str]:
    return [sys.executable, "-m", "mimir_b200", "train", *args]


def supervise(overrides: Sequence[str], config, command: Optional[Sequence[str]] = None,
              poll_seconds: float = 1.0) -> None:
    """Run training until it finishes, restarting after every status-75 suspension."""
    from mimir_b200.ckpt.contract import validate
    if not config.checkpoint_path:
        raise ValueError("--suspendable requires checkpoint_path=<directory>")
    root = Path(config.suspend_control_dir or Path(config.checkpoint_path) / "control").resolve()
    root.mkdir(parents=True, exist_ok=True)
    args = [a for a in overrides if not a.startswith("suspend_control_dir=")] + [f"suspend_control_dir={root}"]
    make = (lambda a: [*command, *a]) if command is not None else _child_command
    with exclusive(root / "recovery.lock"):
        while True:
            while (root / "hold").exists():
                time.sleep(poll_seconds)
            before = _ready_stamp(root)
            status = subprocess.run(make(args)).returncode
            if status == 0:
                return
            if status != SUSPEND_EXIT_CODE and not _suspended_now(root, before):
                raise RuntimeError(f"Training failed with status {status}")
            ready = json.loads((root / "disk-ready.json").read_text())
            directory = Path(ready["checkpoint"]).parent  # the sidecar JSON inside the tag directory
            manifest = validate(directory)
            if manifest["step"] != ready["step"]:
                raise ValueError("Recovery step mismatch")
            resume = {"resume_checkpoint_path": str(directory), "resume_checkpoint_tag": manifest["tag"]}
            # The checkpoint holds everything now; a first start's weight initialisation must not
            # be repeated (and the two are mutually exclusive in the config).
            dropped = set(resume) | {"initialize_from"}
            args = [a for a in args if a.split("=", 1)[0] not in dropped] + [f"{k}={v}" for k, v in resume.items()]
