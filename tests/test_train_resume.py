"""End-to-end CPU training: staged checkpoints, bit-exact resume, disk suspension, GC.

The reference's CPU qualification flow (``tools/qualify_cpu.py:18-53``) trains a small model,
splits the run at a checkpoint, resumes, and requires bit-identical weights, optimizer state,
EMA and RNG.  Same here, through the public ``launch``/``supervise`` entry points.
"""
import json
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed.checkpoint as dcp
from torch.distributed.checkpoint.metadata import TensorStorageMetadata

from mimir_b200.config.schema import load_config
from mimir_b200.data.synthetic import write_corpus

BASE = ["size@arch=XXS", "accelerator_type=cpu", "distributed_strategy=none", "fwd_bwd_dtype=float32",
        "global_batch_size=128", "epochs=2", "lr_warmup_steps=2", "log_interval=2", "arch.hidden_size=64",
        "arch.n_layers=2", "dataloader_prefetch_factor=2", "arch.H_cycles=2", "arch.L_cycles=2"]


@pytest.fixture(scope="module")
def corpus(tmp_path_factory):
    return write_corpus(str(tmp_path_factory.mktemp("data") / "c"), rows=64, seq_len=32, vocab=64, epochs=2)


def _train(corpus, run, *extra):
    from mimir_b200.train.loop import launch
    launch(load_config(BASE + [f"data.path={corpus}", f"checkpoint_path={run}", *extra]))


def _tensors(tag_dir: Path, tag: str) -> dict:
    ckpt = tag_dir / f"fsdp2_{tag}"
    meta = dcp.FileSystemReader(str(ckpt)).read_metadata()
    out = {k: torch.empty(m.size, dtype=m.properties.dtype) for k, m in meta.state_dict_metadata.items()
           if isinstance(m, TensorStorageMetadata)}
    dcp.load(out, checkpoint_id=str(ckpt), no_dist=True)
    return out


def _same_state(a: Path, b: Path, tag: str):
    ta, tb = _tensors(a / tag, tag), _tensors(b / tag, tag)
    assert ta.keys() == tb.keys()
    assert any(k.endswith("param_ema") for k in ta) and any(k.endswith("exp_avg_sq") for k in ta)
    for k in ta:
        assert torch.equal(ta[k], tb[k]), k
    ra = torch.load(a / tag / "rng.0.pt", weights_only=False)
    rb = torch.load(b / tag / "rng.0.pt", weights_only=False)
    assert torch.equal(ra["torch"], rb["torch"]) and ra["python"] == rb["python"]


def _losses(run: Path) -> dict:
    rows = [json.loads(line) for line in (run / "metrics.jsonl").read_text().splitlines()]
    return {r["train/step"]: r["train/loss"] for r in rows if "train/loss" in r}


def test_exact_resume_is_bit_identical(corpus, tmp_path):
    full, split = tmp_path / "full", tmp_path / "split"
    _train(corpus, full, "checkpoint_step_interval=4", "stop_after_step=8")
    manifest = json.loads((full / "step_4" / "manifest.json").read_text())
    assert manifest["mode"] == "exact" and manifest["step"] == 4 and manifest["world_size"] == 1
    _train(corpus, split, "stop_after_step=8", f"resume_checkpoint_path={full}", "resume_checkpoint_tag=step_4")
    _same_state(full, split, "step_8")
    lf, ls = _losses(full), _losses(split)
    assert lf[6] == ls[6] and lf[8] == ls[8]


def test_resume_refuses_changed_protected_config(corpus, tmp_path):
    run = tmp_path / "r"
    _train(corpus, run, "stop_after_step=2")
    with pytest.raises(ValueError, match="configuration changed: lr"):
        _train(corpus, tmp_path / "r2", "lr=1e-3", f"resume_checkpoint_path={run}", "resume_checkpoint_tag=step_2")


def test_partial_checkpoint_is_not_resumable(corpus, tmp_path):
    run = tmp_path / "r"
    _train(corpus, run, "stop_after_step=2")
    partial = run / ".step_9.deadbeef.partial"
    partial.mkdir()
    with pytest.raises(FileNotFoundError):
        _train(corpus, tmp_path / "r2", f"resume_checkpoint_path={partial}", "resume_checkpoint_tag=step_9")


def test_ephemeral_checkpoints_keep_only_latest(corpus, tmp_path):
    run = tmp_path / "e"
    _train(corpus, run, "ephemeral_checkpoint_step_interval=2", "stop_after_step=7")
    assert sorted(p.name for p in run.glob("ephemeral_step_*")) == ["ephemeral_step_6"]
    assert (run / "step_7" / "manifest.json").is_file()


def test_unsharded_checkpoint_resume(corpus, tmp_path):
    full, split = tmp_path / "full", tmp_path / "split"
    _train(corpus, full, "checkpoint_format=unsharded", "checkpoint_step_interval=3", "stop_after_step=5")
    _train(corpus, split, "checkpoint_format=unsharded", "stop_after_step=5", f"resume_checkpoint_path={full}",
           "resume_checkpoint_tag=step_3")
    a = torch.load(full / "step_5" / "unsharded_step_5.pt", weights_only=False)
    b = torch.load(split / "step_5" / "unsharded_step_5.pt", weights_only=False)
    for k, v in a["model"].items():
        assert torch.equal(v, b["model"][k]), k


def test_disk_suspension_restarts_to_identical_state(corpus, tmp_path):
    from mimir_b200.train.disk_recovery import supervise
    full, susp = tmp_path / "full", tmp_path / "susp"
    _train(corpus, full, "stop_after_step=6")
    overrides = BASE + [f"data.path={corpus}", f"checkpoint_path={susp}", "stop_after_step=6",
                        "suspend_after_steps=[3]"]
    control = (susp / "control").resolve()
    config = load_config(overrides + [f"suspend_control_dir={control}"])
    supervise(overrides, config, command=[sys.executable, "-m", "mimir_b200", "train"])
    ready = json.loads((control / "disk-ready.json").read_text())
    assert ready["step"] == 3
    _same_state(full, susp, "step_6")


# A launcher that, like torchrun, reports any non-zero worker status as its own status 1.
_MASKING_LAUNCHER = ("import subprocess, sys; "
                     "r = subprocess.run([sys.executable, '-m', 'mimir_b200', 'train', *sys.argv[1:]]).returncode; "
                     "sys.exit(1 if r else 0)")


def test_disk_suspension_through_a_launcher_that_masks_the_status(corpus, tmp_path):
    """Under a launcher the worker's status 75 arrives as 1; the new ready record tells the
    supervisor it was a suspension (two of them here), and the run ends in the same state."""
    from mimir_b200.train.disk_recovery import supervise
    full, susp = tmp_path / "full", tmp_path / "susp"
    _train(corpus, full, "stop_after_step=6")
    overrides = BASE + [f"data.path={corpus}", f"checkpoint_path={susp}", "stop_after_step=6",
                        "suspend_after_steps=[2,4]"]
    control = (susp / "control").resolve()
    config = load_config(overrides + [f"suspend_control_dir={control}"])
    supervise(overrides, config, command=[sys.executable, "-c", _MASKING_LAUNCHER])
    assert json.loads((control / "disk-ready.json").read_text())["step"] == 4
    _same_state(full, susp, "step_6")


def test_launcher_failure_without_a_new_ready_record_raises(corpus, tmp_path):
    from mimir_b200.train.disk_recovery import supervise
    run = tmp_path / "r"
    overrides = BASE + [f"data.path={corpus}", f"checkpoint_path={run}", "stop_after_step=2", "lr=-1"]
    control = (run / "control").resolve()
    config = load_config([o for o in overrides if o != "lr=-1"] + [f"suspend_control_dir={control}"])
    with pytest.raises(RuntimeError, match="Training failed with status 1"):
        supervise(overrides, config, command=[sys.executable, "-c", _MASKING_LAUNCHER])


def test_suspended_run_started_from_initialize_from_resumes(corpus, tmp_path):
    """A suspendable run that starts from ``initialize_from`` resumes from its own checkpoint
    (the initialisation is not repeated, and the config would reject both at once)."""
    from mimir_b200.train.disk_recovery import supervise
    _train(corpus, tmp_path / "src", "stop_after_step=2")
    run = tmp_path / "r"
    overrides = BASE + [f"data.path={corpus}", f"checkpoint_path={run}", "stop_after_step=4",
                        "suspend_after_steps=[3]", f"initialize_from={tmp_path / 'src' / 'step_2'}"]
    control = (run / "control").resolve()
    config = load_config(overrides + [f"suspend_control_dir={control}"])
    supervise(overrides, config, command=[sys.executable, "-m", "mimir_b200", "train"])
    assert json.loads((control / "disk-ready.json").read_text())["step"] == 3
    assert (run / "step_4").is_dir()
