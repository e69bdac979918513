"""One-way import of pre-contract (legacy) checkpoints and weights-only initialisation.

Behaviour follows ``tests/test_importer.py:17-34`` and the reference's CLI entry
``src/mimir/cli.py:17-21`` (the module itself is not in the reference tree):

* Only Mimir/HRM architectures are accepted (``arch.name`` names an HRM model or ``mimir2``).
* ``mode='exact'`` needs every piece of state an exact continuation restores: model and
  optimizer state, per-rank RNG files and the schedule length.  Historical checkpoints that
  lack any of them are rejected, never relabelled exact, and nothing is written.
* ``mode='weights'`` keeps only the model tensors (``weights.pt``) and records what was
  dropped: ``discarded = ['optimizer', 'EMA', 'RNG', 'cursor', 'schedules']``.  Such a
  directory initialises a run through ``initialize_from`` and is refused by ``resolve``.
* The output directory is never overwritten (staging + ``publish``).

Both DCP (``fsdp2_<tag>/``) and unsharded (``unsharded_<tag>.pt``) legacy layouts load.
"""
from __future__ import annotations

import json
import shutil
import uuid
from pathlib import Path

import torch
import yaml

from mimir_b200.ckpt.contract import publish, validate

DISCARDED_BY_WEIGHTS_IMPORT = ["optimizer", "EMA", "RNG", "cursor", "schedules"]
WEIGHTS_FILE = "weights.pt"


def _is_mimir(arch: dict) -> bool:
    name = str(arch.get("name", ""))
    return name in ("mimir2", "legacy_v1") or "hrm" in name.lower() or "mimir" in name.lower()


def _unwrapped(tensors: dict) -> dict:
    """Model keys without the DDP wrapper's ``module.`` prefix: a run under DDP checkpoints its
    wrapped model (as the reference does), and initialisation reads it into an unwrapped model."""
    if tensors and all(k.startswith("module.") for k in tensors):
        return {k.removeprefix("module."): v for k, v in tensors.items()}
    return tensors


def _load_model_tensors(source: Path, tag: str) -> dict:
    source = Path(source)
    unsharded = source / f"unsharded_{tag}.pt"
    if unsharded.is_file():
        return _unwrapped(dict(torch.load(unsharded, map_location="cpu", weights_only=False)["model"]))
    sharded = source / f"fsdp2_{tag}"
    if sharded.is_dir():
        import torch.distributed.checkpoint as dcp
        from torch.distributed.checkpoint.metadata import TensorStorageMetadata
        meta = dcp.FileSystemReader(str(sharded)).read_metadata()
        wanted = {key: torch.empty(m.size, dtype=m.properties.dtype)
                  for key, m in meta.state_dict_metadata.items()
                  if key.startswith("model.") and isinstance(m, TensorStorageMetadata)}
        dcp.load(wanted, checkpoint_id=str(sharded), no_dist=True)
        return _unwrapped({key.removeprefix("model."): value for key, value in wanted.items()})
    raise FileNotFoundError(f"No unsharded_{tag}.pt or fsdp2_{tag}/ in {source}")


def import_legacy(source, output, *, tag: str, mode: str) -> dict:
    """Import ``source`` (a legacy run directory) into a published checkpoint at ``output``."""
    source, output = Path(source), Path(output)
    if mode not in ("exact", "weights"):
        raise ValueError("mode must be 'exact' or 'weights'")
    if output.exists():
        raise FileExistsError(f"Refusing to overwrite {output}")
    config = yaml.safe_load((source / "all_config.yaml").read_text()) or {}
    if not _is_mimir(config.get("arch") or {}):
        raise ValueError(f"Only Mimir/HRM checkpoints can be imported, got arch {config.get('arch')!r}")
    state_path = source / f"checkpoint_state_{tag}.json"
    state = json.loads(state_path.read_text()) if state_path.is_file() else {}
    world = int(state.get("world_size", 1))
    if mode == "exact":
        missing = [f"rng.{r}.pt" for r in range(world) if not (source / f"rng.{r}.pt").is_file()]
        if "total_steps" not in state:
            missing.append("total_steps")
        if not ((source / f"unsharded_{tag}.pt").is_file() or (source / f"fsdp2_{tag}").is_dir()):
            missing.append("model/optimizer state")
        if missing:
            raise ValueError(f"Exact continuation unavailable: legacy checkpoint lacks {missing}")
    stage = output.parent / f".{output.name}.{uuid.uuid4().hex}.partial"
    stage.mkdir(parents=True)
    try:
        for name in ("all_config.yaml", "train_metadata.yaml"):
            if (source / name).is_file():
                shutil.copy2(source / name, stage / name)
        metadata = {"mode": mode, "tag": tag, "step": state.get("step"), "source": str(source.resolve()),
                    "world_size": world}
        if mode == "weights":
            torch.save(_load_model_tensors(source, tag), stage / WEIGHTS_FILE)
            metadata["discarded"] = list(DISCARDED_BY_WEIGHTS_IMPORT)
        else:
            for entry in source.iterdir():
                if entry.name in (f"unsharded_{tag}.pt", f"checkpoint_state_{tag}.json") or (
                        entry.name.startswith("rng.") and entry.suffix == ".pt"):
                    shutil.copy2(entry, stage / entry.name)
                elif entry.name == f"fsdp2_{tag}":
                    shutil.copytree(entry, stage / entry.name)
            metadata["total_steps"] = int(state["total_steps"])
        return publish(stage, output, metadata=metadata)
    except BaseException:
        shutil.rmtree(stage, ignore_errors=True)
        raise


def initialize_weights(model: torch.nn.Module, path, upcycle: bool = False) -> None:
    """Load model weights from a published checkpoint (weights-only or exact) into ``model``.

    Optimizer/EMA state then starts from these weights.  With ``upcycle`` a dense source
    expands into the experts/stacks of ``model`` (new v2 tensors keep their initial values).
    """
    path = Path(path)
    manifest = validate(path)
    if (path / WEIGHTS_FILE).is_file():
        tensors = torch.load(path / WEIGHTS_FILE, map_location="cpu", weights_only=True)
    else:
        tag = manifest.get("tag")
        if tag is None:
            raise ValueError(f"Checkpoint {path} names no tag")
        tensors = _load_model_tensors(path, tag)
    if upcycle:
        from mimir_b200.models.experts import upcycle_dense_weights
        upcycle_dense_weights(model, tensors)
        return
    missing, unexpected = model.load_state_dict(tensors, strict=False)
    if missing or unexpected:
        raise ValueError(f"initialize_from mismatch: missing={sorted(missing)} unexpected={sorted(unexpected)}")
