"""Micro-benchmark of the fused data-parallel step (reduce-scatter + AdamATan2 + all-gather).

    python benchmarks/dp_step.py [--params 1.3e9] [--iters 10]                      # one GPU
    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/dp_step.py        # N GPUs

A synthetic parameter set with the flagship model's total size (one [rows, 2048] matrix per
~50M parameters) is wrapped by the replicated engine; gradients are random bf16.  Each timed
iteration is one ``optimizer.step()`` (ordering all-reduce, fused kernel, ordering all-reduce),
timed with CUDA events after warm-up; the maximum over ranks is reported.  The roofline is the
slower of the HBM bytes at the measured copy bandwidth and the NVLink bytes at the measured
770 GB/s per direction.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
NVLINK_GBS = 770.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--params", type=float, default=1.3e9)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--once", action="store_true", help="one step after one warm-up (for profilers)")
    args = ap.parse_args()
    from mimir_b200.parallel.replicated import ReplicatedAdamATan2, wrap_replicated
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if "RANK" in os.environ:
        dist.init_process_group("nccl", device_id=dev)
    world = dist.get_world_size() if dist.is_initialized() else 1
    cols = 2048
    rows = 24 * 1024  # 50M parameters per matrix
    n = max(1, round(args.params / (rows * cols)))
    torch.manual_seed(0)
    model = torch.nn.ParameterList([torch.nn.Parameter(torch.randn(rows, cols, device=dev) * 0.02) for _ in range(n)])
    engine = wrap_replicated(model, dev, torch.bfloat16)
    opt = ReplicatedAdamATan2(engine, lr=1e-4, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9999)
    total = sum(p.numel() for p in model.parameters())

    def step():
        engine.touched.update(s.fqn for s in engine.slots)  # as after a backward that reached every parameter
        opt.step()

    engine.grads.normal_()
    for _ in range(1 if args.once else args.warmup):
        step()
    torch.cuda.synchronize()
    iters = 1 if args.once else args.iters
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    start.record()
    for _ in range(iters):
        step()
    end.record()
    torch.cuda.synchronize()
    seconds = start.elapsed_time(end) / 1000 / iters
    if dist.is_initialized():
        t = torch.tensor([seconds], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        seconds = float(t.item())
    shard = total / world
    hbm_bytes = shard * (2 + 16 + 16 + 2)                  # own grads in, 4 fp32 slots r/w, own weights out
    nvlink_bytes = shard * (world - 1) * 2                  # peers' grads in (= weights out to peers)
    try:
        hbm = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"]
    except (OSError, ValueError, KeyError):
        hbm = 6650.0
    roofline = max(hbm_bytes / (hbm * 1e9), nvlink_bytes / (NVLINK_GBS * 1e9))
    if not dist.is_initialized() or dist.get_rank() == 0:
        print(json.dumps({"kernel": "dp_step (fused reduce-scatter + AdamATan2 + all-gather)", "world": world,
                          "params": total, "ms": round(seconds * 1e3, 3), "roofline_ms": round(roofline * 1e3, 3),
                          "frac_of_roofline": round(roofline / seconds, 3),
                          "hbm_gbs_achieved": round(hbm_bytes / seconds / 1e9, 1),
                          "nvlink_gbs_per_direction": round(nvlink_bytes / seconds / 1e9, 1)}), flush=True)
    engine.close()
    if dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
