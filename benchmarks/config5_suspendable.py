"""BASELINE config 5 on this machine's GPUs: XXS upcycled to MoE (8 experts, top-2) with a
residual branch pair and the contextual n-gram memory (hashed 2/3-grams, 2^20 rows x 256, bf16),
DDP bf16, uniform token ids at seq_len 2048, micro-batch 8 per GPU, suspendable with
``suspend_after_steps=[50,100]`` and exact DCP resume.

    python benchmarks/config5_suspendable.py [--gpus N] [--steps 120] [--out DIR]

Stage 1 trains the dense XXS model for 20 steps and checkpoints it; stage 2 upcycles it
(``initialize_from`` + ``arch.upcycle_from_dense``) and trains under the disk-suspension
supervisor, which restarts the torchrun job from the DCP checkpoint after each suspension
(exit 75 at steps 50 and 100).  Prints one JSON line: the suspensions and resumes that
happened, the final loss, and the steady-state step time of the last segment (median of its
per-step wall times, synchronised, first two steps dropped) as tokens/s.

Reference behaviour: the config-5 recipe (``src/mimir/training/disk_recovery.py:10-44`` for the
suspension protocol, ``src/mimir/model/upcycling.py`` for upcycling).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

SEQ, MICRO, VOCAB = 2048, 8, 32768
XXS = ["size@arch=XXS", "accelerator_type=sm100", "fwd_bwd_dtype=bfloat16", "compile_train_batch=false",
       "lr=3e-4", "lr_warmup_steps=10", "log_interval=10", "epochs=1"]
CONFIG5 = ["arch.moe_num_experts=8", "arch.moe_top_k=2", "arch.moe_sparse=true", "arch.upcycle_from_dense=true",
           "arch.residual_branches=2", "arch.ngram_orders=[2,3]", "arch.ngram_buckets=1048576", "arch.ngram_heads=1",
           "arch.ngram_contextual_gate=true", "distributed_strategy=ddp"]


def torchrun(gpus: int, port: int) -> list[str]:
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={gpus}",
            "--master-addr", "127.0.0.1", f"--master-port={port}", "-m", "mimir_b200", "train"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=120)
    ap.add_argument("--out", type=Path, default=None)
    args = ap.parse_args()
    import subprocess

    from mimir_b200.config.schema import load_config
    from mimir_b200.data.synthetic import write_corpus
    from mimir_b200.train.disk_recovery import supervise
    out = args.out or Path(tempfile.mkdtemp(prefix="mimir-config5-"))
    batch = SEQ * MICRO * args.gpus
    corpus = write_corpus(str(out / "data"), rows=(args.steps + 30) * MICRO * args.gpus, seq_len=SEQ, vocab=VOCAB,
                          min_prefix=1, max_prefix=1)
    dense = out / "dense"
    base = XXS + [f"data.path={corpus}", f"global_batch_size={batch}"]
    subprocess.run(torchrun(args.gpus, 29811) + base + ["distributed_strategy=ddp", f"checkpoint_path={dense}",
                   "stop_after_step=20", "checkpoint_step_interval=20"], check=True)
    run = out / "moe"
    overrides = base + CONFIG5 + [f"initialize_from={dense / 'step_20'}", f"checkpoint_path={run}",
                                  f"stop_after_step={args.steps}", f"max_steps={args.steps}",
                                  "suspend_after_steps=[50,100]", f"suspend_control_dir={run / 'control'}"]
    os.environ["BENCH_OUTPUT"] = str(out / "last_segment_bench.json")
    t0 = time.perf_counter()
    supervise(overrides, load_config(overrides), command=torchrun(args.gpus, 29812))
    wall = time.perf_counter() - t0
    rows = [json.loads(line) for line in (run / "metrics.jsonl").read_text().splitlines()]
    losses = {r["train/step"]: r["train/loss"] for r in rows if "train/loss" in r}
    bench = json.loads((out / "last_segment_bench.json").read_text())
    resumes = sorted(p.name for p in run.glob("step_*"))
    print(json.dumps({"config": "BASELINE config 5 (XXS upcycled MoE 8e top-2 + residual branches + n-gram 2^20x256, "
                                "DDP bf16, suspendable)", "gpus": args.gpus, "steps": args.steps,
                      "suspend_after_steps": [50, 100], "checkpoints": resumes,
                      "final_step_logged": max(losses) if losses else None,
                      "final_loss": losses[max(losses)] if losses else None,
                      "last_segment_median_step_s": bench["median_step_seconds"],
                      "tokens_per_s_last_segment": round(batch / bench["median_step_seconds"], 1),
                      "wall_s_including_restarts": round(wall, 1), "out": str(out)}), flush=True)


if __name__ == "__main__":
    main()
