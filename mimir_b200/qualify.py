"""Isolated CPU qualification campaign: train, checkpoint, export, evaluate, resume, suspend.

Reference behaviour: ``tools/qualify_cpu.py:18-53``.  Everything is written under one new
output directory:

1. a 32-row synthetic corpus (prompt 3 + answer 6 tokens per row);
2. ``baseline``: 4 optimizer steps of a tiny XXS model on CPU (fp32, unsharded checkpoints);
3. ``split``: the same run stopped at step 2; its EMA weights are exported to the HF format
   and scored with the ``cpu-smoke-v1`` suite;
4. ``resumed``: continues ``split`` from ``step_2`` to step 4;
5. ``suspended``: the same 4 steps under the disk-suspension supervisor, suspending at step 2
   (status 75) and restarting from the published checkpoint.

The campaign passes only if ``resumed`` and ``suspended`` end with weights, optimizer
state, EMA, RNG state and logged losses bit-identical to ``baseline``; ``result.json``
records what was checked.  Usage: ``python -m mimir_b200 qualify-cpu OUTPUT``.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import torch

ROWS, PROMPT, ANSWER = 32, 3, 6
COMMON = ["size@arch=XXS", "accelerator_type=cpu", "distributed_strategy=none", "checkpoint_format=unsharded",
          "compile_train_batch=false", "fwd_bwd_dtype=float32", "global_batch_size=16", "epochs=1", "max_steps=4",
          "arch.hidden_size=16", "arch.num_heads=2", "arch.n_layers=2", "arch.expansion=1", "lr_warmup_steps=0",
          "log_interval=1"]


def assert_identical(a, b, where="") -> None:
    if isinstance(a, torch.Tensor):
        torch.testing.assert_close(a, b, rtol=0, atol=0, msg=where)
    elif isinstance(a, np.ndarray):
        np.testing.assert_array_equal(a, b, err_msg=where)
    elif isinstance(a, dict):
        if a.keys() != b.keys():
            raise AssertionError(f"{where}: keys differ")
        for k in a:
            assert_identical(a[k], b[k], f"{where}/{k}")
    elif isinstance(a, (list, tuple)):
        if len(a) != len(b):
            raise AssertionError(f"{where}: lengths differ")
        for i, (x, y) in enumerate(zip(a, b)):
            assert_identical(x, y, f"{where}[{i}]")
    elif a != b:
        raise AssertionError(f"{where}: {a!r} != {b!r}")


def write_corpus(root: Path) -> Path:
    data = root / "corpus"
    epoch = data / "epoch_0"
    epoch.mkdir(parents=True)
    length = PROMPT + ANSWER
    np.save(data / "tokens.npy", (np.arange(ROWS * length, dtype=np.uint32) % 31 + 1))
    starts = np.arange(ROWS) * length
    for name, arr in {"inst_start": starts, "inst_len": np.full(ROWS, PROMPT), "resp_start": starts + PROMPT,
                      "resp_len": np.full(ROWS, ANSWER)}.items():
        np.save(epoch / f"{name}.npy", arr.astype(np.int64))
    (data / "metadata.json").write_text(json.dumps({"max_seq_len": length, "total_length": ROWS * (length - 1),
                                                    "tokenizer_info": {"vocab_size": 256}}))
    return data


def write_tokenizer(path: Path) -> Path:
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    core = Tokenizer(models.WordLevel({str(i): i for i in range(256)}, unk_token="0"))
    core.pre_tokenizer = pre_tokenizers.Whitespace()
    tok = PreTrainedTokenizerFast(tokenizer_object=core, unk_token="0", bos_token="1", eos_token="2", pad_token="0")
    tok.chat_template = "{% for message in messages %}{{ message['content'] }}{% endfor %}"
    tok.save_pretrained(str(path))
    return path


class Campaign:
    def __init__(self, output):
        self.root = Path(output).resolve()
        self.root.mkdir(parents=True, exist_ok=False)
        self.data = write_corpus(self.root)

    def train(self, name: str, *extra: str) -> None:
        args = [sys.executable, "-m", "mimir_b200", "train", *COMMON, f"data.path={self.data}",
                f"checkpoint_path={self.root / name}", *extra]
        env = os.environ | {"CUDA_VISIBLE_DEVICES": "", "OMP_NUM_THREADS": "2"}
        with (self.root / f"{name}.log").open("w") as log:
            subprocess.run(args, env=env, stdout=log, stderr=subprocess.STDOUT, check=True)

    def losses(self, name: str) -> list[dict]:
        return [json.loads(s) for s in (self.root / name / "metrics.jsonl").read_text().splitlines() if "train/loss" in s]

    def compare(self, name: str, reference: str = "baseline", tag: str = "step_4") -> None:
        def load(run, file):
            return torch.load(self.root / run / tag / file, weights_only=False)
        assert_identical(load(reference, f"unsharded_{tag}.pt"), load(name, f"unsharded_{tag}.pt"), f"{name}/state")
        assert_identical(load(reference, "rng.0.pt"), load(name, "rng.0.pt"), f"{name}/rng")
        base, got = self.losses(reference), self.losses(name)
        assert_identical(base[-len(got):], got, f"{name}/losses")

    def run(self) -> Path:
        from mimir_b200.evaluation.clients import evaluate
        from mimir_b200.export.convert import export
        self.train("baseline", "stop_after_step=4")
        self.train("split", "stop_after_step=2")
        export(self.root / "split" / "step_2", self.root / "export", write_tokenizer(self.root / "tokenizer"), ema=True)
        suite = Path(__file__).resolve().parent / "evaluation" / "suites" / "cpu-smoke-v1.json"
        evaluate(str(suite), str(self.root / "export"), str(self.root / "evaluation"))
        self.train("resumed", f"resume_checkpoint_path={self.root / 'split'}", "resume_checkpoint_tag=step_2",
                   "stop_after_step=4")
        self.train("suspended", "--suspendable", "suspend_after_steps=[2]", "stop_after_step=4")
        for name in ("resumed", "suspended"):
            self.compare(name)
        result = self.root / "result.json"
        result.write_text(json.dumps({
            "status": "passed", "device": "cpu", "steps": 4,
            "exact": ["weights", "optimizer", "EMA", "RNG", "losses", "recurrence/LR schedules", "sample position"],
            "campaign": ["train", "checkpoint", "EMA export", "local evaluation", "resume", "disk suspension"]},
            indent=2) + "\n")
        return result


def main(output) -> Path:
    return Campaign(output).run()
