"""BASELINE config 1 as stated: the XXS dense backbone (the ``size@arch=XXS`` preset; no gates,
experts or recurrence), CPU, fp32, no compile, synthetic uniform token ids at seq_len 512 and
micro-batch 8 (causal LM loss: a one-token prompt), AdamATan2 lr 3e-4 for 20 steps with a DCP
checkpoint at step 10; resuming from step 10 must reproduce steps 11-20 bit for bit (weights,
optimizer moments, EMA, RNG and the logged losses)."""
import json

import pytest
import torch

from mimir_b200.config.schema import load_config
from mimir_b200.data.synthetic import write_corpus

CONFIG1 = ["size@arch=XXS", "arch.recurrence_mode=looped", "+arch.H_override.n_layers=0", "arch.H_cycles=1",
           "arch.L_cycles=1", "arch.half_layers=false", "+arch.attn_type=causal", "accelerator_type=cpu",
           "distributed_strategy=none", "fwd_bwd_dtype=float32", "compile_train_batch=false",
           f"global_batch_size={512 * 8}", "epochs=1", "lr=3e-4", "lr_warmup_steps=0", "log_interval=1"]


def _train(corpus, run, *extra):
    from mimir_b200.train.loop import launch
    launch(load_config(CONFIG1 + [f"data.path={corpus}", f"checkpoint_path={run}", *extra]))


@pytest.mark.slow
def test_config1_xxs_resume_at_step_10_is_bit_exact(tmp_path):
    from test_train_resume import _losses, _same_state
    corpus = write_corpus(str(tmp_path / "data"), rows=20 * 8, seq_len=512, vocab=4096, min_prefix=1, max_prefix=1)
    full, split = tmp_path / "full", tmp_path / "split"
    _train(corpus, full, "checkpoint_step_interval=10", "stop_after_step=20")
    manifest = json.loads((full / "step_10" / "manifest.json").read_text())
    assert manifest["mode"] == "exact" and manifest["step"] == 10
    _train(corpus, split, "stop_after_step=20", f"resume_checkpoint_path={full}", "resume_checkpoint_tag=step_10")
    _same_state(full, split, "epoch_1")  # step 20 closes the epoch
    lf, ls = _losses(full), _losses(split)
    assert sorted(ls) == [s for s in sorted(lf) if s > 10] and len(ls) >= 9, (lf, ls)
    assert all(lf[s] == ls[s] for s in ls), (lf, ls)
    assert all(torch.isfinite(torch.tensor(v)) for v in lf.values())
