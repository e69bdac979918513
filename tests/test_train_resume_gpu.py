"""Exact resume on the GPU through the public ``launch`` entry with the replicated engine.

A run trains 8 steps with a DCP checkpoint at step 4; a second run resumes from step 4 and trains
to step 8.  The fp32 master weights, AdamATan2 moments, EMA, RNG and logged losses of steps 5-8
must be bit-identical (the checkpoint contract of ``src/mimir/training/checkpoint_io.py:166-281``:
an "exact" checkpoint restores everything the next step reads).  The bf16 working weights are
recomputed from the restored fp32 master, so they match as well.
"""
import json

import pytest
import torch

from mimir_b200.config.schema import load_config
from mimir_b200.data.synthetic import write_corpus

pytestmark = pytest.mark.gpu

GPU = ["size@arch=XXS", "arch.hidden_size=256", "arch.num_heads=2", "arch.n_layers=2", "arch.H_cycles=2",
       "arch.L_cycles=2", "accelerator_type=sm100", "distributed_strategy=replicated", "fwd_bwd_dtype=bfloat16",
       "compile_train_batch=false", f"global_batch_size={256 * 8}", "epochs=1", "lr=1e-3", "lr_warmup_steps=2",
       "log_interval=1"]


def _train(corpus, run, *extra):
    from mimir_b200.train.loop import launch
    launch(load_config(GPU + [f"data.path={corpus}", f"checkpoint_path={run}", *extra]))


def test_replicated_engine_resume_is_bit_exact(tmp_path):
    from test_train_resume import _losses, _same_state
    corpus = write_corpus(str(tmp_path / "data"), rows=8 * 8, seq_len=256, vocab=512)
    full, split = tmp_path / "full", tmp_path / "split"
    _train(corpus, full, "checkpoint_step_interval=4", "stop_after_step=8")
    manifest = json.loads((full / "step_4" / "manifest.json").read_text())
    assert manifest["mode"] == "exact" and manifest["step"] == 4
    _train(corpus, split, "stop_after_step=8", f"resume_checkpoint_path={full}", "resume_checkpoint_tag=step_4")
    tag = "step_8" if (full / "step_8").is_dir() else "epoch_1"
    _same_state(full, split, tag)
    lf, ls = _losses(full), _losses(split)
    assert sorted(ls) == [s for s in sorted(lf) if s > 4] and ls, (lf, ls)
    assert all(lf[s] == ls[s] for s in ls), (lf, ls)
    assert torch.isfinite(torch.tensor(list(lf.values()))).all()
