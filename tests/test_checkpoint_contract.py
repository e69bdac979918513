"""Checkpoint publication contract and legacy import (CPU).

Mirrors the behaviour fixed by the reference's ``tests/test_contract.py`` and
``tests/test_importer.py``: partial/corrupt/weights-only rejection, no overwrite, explicit
weights-only import that records what it discarded.
"""
import json

import pytest
import torch
import yaml

from mimir_b200.ckpt.contract import publish, resolve, restore_rng, rng_state, validate
from mimir_b200.ckpt.importer import import_legacy, initialize_weights


def test_partial_corrupt_and_weights_only_rejected(tmp_path):
    stage = tmp_path / "partial"
    stage.mkdir()
    (stage / "state").write_text("saved")
    with pytest.raises(FileNotFoundError):
        validate(stage)
    out = tmp_path / "step_1"
    publish(stage, out, metadata={"mode": "weights", "tag": "step_1"})
    assert not stage.exists()
    assert validate(out)["tag"] == "step_1"
    with pytest.raises(ValueError, match="Weights-only"):
        resolve(out, "step_1")
    (out / "state").write_text("wrong")
    with pytest.raises(ValueError, match="Corrupt"):
        validate(out)


def test_same_size_tamper_detected_only_with_hashes(tmp_path):
    stage = tmp_path / "s"
    stage.mkdir()
    (stage / "a").write_text("abc")
    publish(stage, tmp_path / "step_2", metadata={"mode": "exact", "tag": "step_2"})
    (tmp_path / "step_2" / "a").write_text("abd")
    validate(tmp_path / "step_2", hashes=False)
    with pytest.raises(ValueError, match="Corrupt"):
        validate(tmp_path / "step_2")


def test_publication_does_not_replace_existing_checkpoint(tmp_path):
    out = tmp_path / "step_1"
    out.mkdir()
    (out / "old").write_text("safe")
    stage = tmp_path / "partial"
    stage.mkdir()
    (stage / "new").write_text("new")
    with pytest.raises(FileExistsError):
        publish(stage, out, metadata={})
    assert (out / "old").read_text() == "safe"


def test_resolve_accepts_run_root_and_tag_dir(tmp_path):
    stage = tmp_path / "s"
    stage.mkdir()
    (stage / "x").write_text("1")
    publish(stage, tmp_path / "run" / "step_3", metadata={"mode": "exact", "tag": "step_3"})
    assert resolve(tmp_path / "run", "step_3") == tmp_path / "run" / "step_3"
    assert resolve(tmp_path / "run" / "step_3", "step_3") == tmp_path / "run" / "step_3"


def test_rng_roundtrip():
    state = rng_state()
    a = torch.rand(3)
    restore_rng(state)
    assert torch.equal(a, torch.rand(3))


def _legacy(root):
    root.mkdir()
    (root / "all_config.yaml").write_text(yaml.safe_dump({
        "arch": {"name": "baselines.hrm_nocarry_bp_warmup@HierarchicalReasoningModel", "head": "lm_head@LMHead"},
        "checkpoint_format": "unsharded", "ema": .9}))
    (root / "train_metadata.yaml").write_text(yaml.safe_dump({"vocab_size": 32, "max_seq_len": 8}))
    (root / "checkpoint_state_step_1.json").write_text(json.dumps(
        {"step": 1, "epoch": 1, "batch_in_epoch": 1, "world_size": 1, "carry_policy": "none"}))
    torch.save({"model": {"weight": torch.tensor([[3.]])},
                "optim": {"state": {0: {"step": torch.tensor(1.), "param_ema": torch.tensor([[2.]])}}}},
               root / "unsharded_step_1.pt")


def test_weights_import_is_explicit_and_exact_needs_rng(tmp_path):
    source = tmp_path / "legacy"
    _legacy(source)
    with pytest.raises(ValueError, match="Exact continuation unavailable"):
        import_legacy(source, tmp_path / "exact", tag="step_1", mode="exact")
    assert not (tmp_path / "exact").exists()
    out = tmp_path / "weights"
    import_legacy(source, out, tag="step_1", mode="weights")
    assert validate(out)["discarded"] == ["optimizer", "EMA", "RNG", "cursor", "schedules"]
    m = torch.nn.Linear(1, 1, bias=False)
    initialize_weights(m, out)
    assert m.weight.item() == 3.
    with pytest.raises(ValueError, match="Weights-only"):
        resolve(out, "step_1")


def test_exact_import_with_complete_state(tmp_path):
    source = tmp_path / "legacy"
    _legacy(source)
    state = json.loads((source / "checkpoint_state_step_1.json").read_text())
    (source / "checkpoint_state_step_1.json").write_text(json.dumps(state | {"total_steps": 10}))
    torch.save(rng_state(), source / "rng.0.pt")
    out = tmp_path / "exact"
    manifest = import_legacy(source, out, tag="step_1", mode="exact")
    assert manifest["mode"] == "exact" and manifest["total_steps"] == 10
    assert resolve(out, "step_1") == out


def test_import_rejects_other_architectures_and_never_overwrites(tmp_path):
    source = tmp_path / "legacy"
    _legacy(source)
    (source / "all_config.yaml").write_text(yaml.safe_dump({"arch": {"name": "other"}}))
    with pytest.raises(ValueError, match="Only Mimir"):
        import_legacy(source, tmp_path / "out", tag="step_1", mode="weights")
    out = tmp_path / "out"
    out.mkdir()
    with pytest.raises(FileExistsError):
        import_legacy(source, out, tag="step_1", mode="weights")
