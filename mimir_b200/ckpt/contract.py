"""Checkpoint publication contract: staged directory -> hashed manifest -> atomic rename.

The reference calls this module (``mimir.checkpoints.contract``) from
``src/mimir/training/checkpoint_io.py:168-171,549-587,609-624`` and
``src/mimir/training/disk_recovery.py:41-42``, but does not ship it; its behaviour is fixed by
``tests/test_contract.py:6-20`` and ``tests/test_importer.py:17-34``:

* ``publish(stage, out, metadata)`` hashes every file of a fully written staging directory,
  writes ``manifest.json`` (metadata plus ``files: {relative path: [size, sha256]}``) into it
  and renames it to ``out``.  It never replaces an existing ``out`` (``FileExistsError``).
* ``validate(directory, hashes=True)`` returns the manifest.  A directory without one is a
  partial/unpublished write (``FileNotFoundError``); a missing, resized or (with ``hashes``)
  re-hashed file is ``ValueError('Corrupt checkpoint ...')``.
* ``resolve(path, tag)`` accepts a run root (containing ``tag/``) or the tag directory itself
  and refuses ``mode == 'weights'`` publications for exact continuation.
* ``rng_state()`` / ``restore_rng(state)`` capture and restore Python, NumPy, torch CPU and
  (when present) CUDA generator states for per-rank ``rng.<rank>.pt`` files.
"""
from __future__ import annotations

import hashlib
import json
import os
import random
from pathlib import Path
from typing import Any, Optional

import numpy as np
import torch

MANIFEST = "manifest.json"
_CHUNK = 1 << 22


def _digest(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            block = f.read(_CHUNK)
            if not block:
                break
            h.update(block)
    return h.hexdigest()


def _fsync_dir(path: Path) -> None:
    fd = os.open(path, os.O_RDONLY | os.O_DIRECTORY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def _inventory(root: Path) -> dict[str, list]:
    files = {}
    for path in sorted(root.rglob("*")):
        if path.is_file() and path.name != MANIFEST:
            files[path.relative_to(root).as_posix()] = [path.stat().st_size, _digest(path)]
    return files


def publish(stage, out, metadata: Optional[dict] = None) -> dict:
    """Seal ``stage`` with a manifest and atomically rename it to ``out``; return the manifest."""
    stage, out = Path(stage), Path(out)
    if out.exists():
        raise FileExistsError(f"Refusing to replace existing checkpoint {out}")
    if not stage.is_dir():
        raise FileNotFoundError(f"Staging directory {stage} does not exist")
    manifest = dict(metadata or {})
    manifest["files"] = _inventory(stage)
    temp = stage / f".{MANIFEST}.tmp"
    with open(temp, "w") as f:
        json.dump(manifest, f, indent=2, sort_keys=True)
        f.write("\n")
        f.flush()
        os.fsync(f.fileno())
    os.replace(temp, stage / MANIFEST)
    _fsync_dir(stage)
    out.parent.mkdir(parents=True, exist_ok=True)
    # rename(2) onto an existing non-empty directory fails; an empty one would be replaced,
    # so the existence check above is what keeps a published checkpoint immutable.
    os.rename(stage, out)
    _fsync_dir(out.parent)
    return manifest


def validate(directory, hashes: bool = True) -> dict:
    """Check a published checkpoint against its manifest and return the manifest."""
    directory = Path(directory)
    path = directory / MANIFEST
    if not path.is_file():
        raise FileNotFoundError(f"No {MANIFEST} in {directory}: partial or unpublished checkpoint")
    try:
        manifest = json.loads(path.read_text())
    except json.JSONDecodeError as error:
        raise ValueError(f"Corrupt checkpoint manifest {path}: {error}") from error
    for name, (size, digest) in manifest.get("files", {}).items():
        file = directory / name
        if not file.is_file():
            raise ValueError(f"Corrupt checkpoint {directory}: missing {name}")
        if file.stat().st_size != size:
            raise ValueError(f"Corrupt checkpoint {directory}: size of {name} changed")
        if hashes and _digest(file) != digest:
            raise ValueError(f"Corrupt checkpoint {directory}: hash of {name} changed")
    return manifest


def resolve(path, tag: Optional[str] = None) -> Path:
    """Directory of a published exact checkpoint given a run root or the tag directory."""
    path = Path(path)
    candidate = path / tag if tag is not None and (path / tag / MANIFEST).is_file() else path
    manifest = validate(candidate, hashes=False)
    if manifest.get("mode") == "weights":
        raise ValueError(f"Weights-only checkpoint {candidate} cannot be resumed exactly; "
                         "use initialize_from instead")
    if tag is not None and manifest.get("tag") not in (None, tag):
        raise ValueError(f"Checkpoint {candidate} holds tag {manifest.get('tag')!r}, not {tag!r}")
    return candidate


def rng_state() -> dict[str, Any]:
    state = {"python": random.getstate(), "numpy": np.random.get_state(), "torch": torch.get_rng_state()}
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        state["cuda"] = torch.cuda.get_rng_state_all()
    return state


def restore_rng(state: dict[str, Any]) -> None:
    random.setstate(state["python"])
    np.random.set_state(state["numpy"])
    torch.set_rng_state(state["torch"])
    if "cuda" in state and torch.cuda.is_available():
        cuda = state["cuda"]
        if len(cuda) != torch.cuda.device_count():
            raise ValueError("Exact RNG continuation requires the same number of visible CUDA devices")
        torch.cuda.set_rng_state_all(cuda)
