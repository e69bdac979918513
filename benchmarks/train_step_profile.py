"""Where one training step of a bench configuration spends its GPU time (torch.profiler, 1 GPU).

    python benchmarks/train_step_profile.py [--config dense|moe] [--optimizer adam_atan2|muon] [--rows 25]
        [--overlap-report]

Builds the same model, data and engine as ``bench.py`` (our arm), runs three warm-up steps and
profiles one more, then prints the kernels (and CPU-side ops) ranked by total CUDA time.  The
profiled step is slower than a timed one (profiler overhead); compare shares, not absolutes.
``--overlap-report`` adds one JSON line on the fused optimizer update: its kernels' device time,
the part of it during which some other kernel (the backward) was also running, and when the
last update kernel ended relative to the last other kernel.
"""
from __future__ import annotations

import argparse
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", choices=["dense", "moe"], default="dense")
    ap.add_argument("--optimizer", choices=["adam_atan2", "muon"], default="adam_atan2")
    ap.add_argument("--rows", type=int, default=25)
    ap.add_argument("--overlap-report", action="store_true")
    ap.add_argument("--shapes", action="store_true", help="also group the table by input shapes")
    args = ap.parse_args()
    import bench
    bench.CONFIG["name"] = args.config
    rank, world, local = bench.init_distributed(1)
    from mimir_b200.config.schema import PretrainConfig
    from mimir_b200.models.common import wrap_tensor
    from mimir_b200.optim.schedules import update_lr
    from mimir_b200.train.setup import create_model_and_optimizer, make_train_state
    from mimir_b200.train.steps import train_accumulated_batches

    device = torch.device("cuda", local)
    arch = bench.arch_dict(kv_heads=bench.MODEL["num_key_value_heads"])
    vocab = arch.pop("vocab_size")
    config = PretrainConfig(arch=arch, data=dict(path="synthetic"), global_batch_size=bench.SEQ_LEN * bench.SEQS_PER_GPU,
                            epochs=1, lr=3e-4, lr_warmup_steps=0, lr_min_ratio=1.0, weight_decay=0.1, beta1=0.9,
                            beta2=0.95, ema=None if args.config == "moe" else 0.9999, distributed_strategy="replicated",
                            lr_auto=False, optimizer=args.optimizer, muon_momentum=0.95, muon_ns_steps=5)
    torch.manual_seed(0)
    model, carry, optim = create_model_and_optimizer(config, {"vocab_size": vocab, "max_seq_len": bench.SEQ_LEN}, device)
    state = make_train_state(config, model, carry, optim, total_steps=10_000, device=device)
    host, scalars = bench.synthetic_batch(rank, 0)
    batch = bench.device_batch(host, scalars, device, wrap_tensor)

    def step():
        state.step += 1
        update_lr(config, state)
        train_accumulated_batches(config, rank, state, [batch])

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], record_shapes=args.shapes) as prof:
        step()
        torch.cuda.synchronize()
    table = prof.key_averages()
    print(table.table(sort_by="self_cuda_time_total", row_limit=args.rows, max_name_column_width=110))
    # the same kernels with the op that launched them (shapes show which tensors they touched)
    if args.shapes:
        shaped = prof.key_averages(group_by_input_shape=True)
        print(shaped.table(sort_by="self_cuda_time_total", row_limit=args.rows, max_name_column_width=60,
                           max_shapes_column_width=80))
    total = sum(getattr(e, "self_device_time_total", getattr(e, "self_cuda_time_total", 0)) for e in table)
    print(f"total self CUDA time of the step: {total / 1e3:.1f} ms")
    if args.overlap_report:
        print(overlap_report(prof))
    import torch.distributed as dist
    dist.destroy_process_group()


def overlap_report(prof) -> str:
    """JSON line: device time of the update kernels and the part of it shared with other kernels."""
    import json
    from torch.autograd import DeviceType
    kernels = [(e.time_range.start, e.time_range.end, e.name) for e in prof.events()
               if e.device_type == DeviceType.CUDA and e.time_range.end > e.time_range.start]
    update = sorted((a, b) for a, b, n in kernels if "dp_update" in n)
    others = sorted((a, b) for a, b, n in kernels if "dp_update" not in n)
    merged = []
    for a, b in others:  # union of the other kernels' busy intervals
        if merged and a <= merged[-1][1]:
            merged[-1][1] = max(merged[-1][1], b)
        else:
            merged.append([a, b])
    shared = sum(max(0.0, min(b, mb) - max(a, ma)) for a, b in update for ma, mb in merged)
    total = sum(b - a for a, b in update)
    return json.dumps({"update_kernels": len(update), "update_ms": round(total / 1e3, 3),
                       "update_ms_concurrent_with_other_kernels": round(shared / 1e3, 3),
                       "last_update_end_minus_last_other_end_ms":
                           round(((update[-1][1] if update else 0) - (others[-1][1] if others else 0)) / 1e3, 3),
                       "other_kernels_busy_ms": round(sum(b - a for a, b in merged) / 1e3, 3)})


if __name__ == "__main__":
    main()
