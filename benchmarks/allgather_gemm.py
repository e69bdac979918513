"""Fused all-gather + GEMM against NCCL all-gather followed by the GEMM, on row-sharded weights.

    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 benchmarks/allgather_gemm.py
    python benchmarks/allgather_gemm.py          # one GPU: the gather is a local copy

For each projection of the flagship model (weight [out, in] sharded by rows over the ranks, as
ZeRO-3 / FSDP2 keeps it) and ``--tokens`` rows of activations per rank, three timings (CUDA
events on the launching stream, L2 flushed before every iteration by writing 256 MB, max over
ranks of the per-rank median):

* ``fused``: one ``gemm_allgather`` launch (tcgen05 tiles + NVLink gather into a local copy);
* ``nccl``: ``all_gather_into_tensor`` of the weight, then the same tcgen05 GEMM on it;
* ``gemm``: the GEMM alone on a local full weight (no communication: the lower bound).

Roofline of the fused op: the slower of its FLOPs at the measured cuBLAS bf16 peak and the
weight bytes that must cross NVLink at the measured 770 GB/s per direction.
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
SHAPES = {"gqkv": (5120, 2048), "o": (2048, 2048), "gate_up": (11264, 2048), "down": (2048, 5632)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--shapes", default=",".join(SHAPES))
    args = ap.parse_args()
    from mimir_b200.ops._ext import ext
    from mimir_b200.ops.gemm import mm_nt, status
    from mimir_b200.parallel.sharded_linear import ShardedLinear
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if "RANK" in os.environ:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        tflops = peaks.get("bf16_tflops", 1590.0)
    except (OSError, ValueError):
        tflops = 1590.0
    C = ext()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    rows = []
    for name in args.shapes.split(","):
        N, K = SHAPES[name]
        g = torch.Generator(device=dev).manual_seed(0)
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        layer = ShardedLinear(w, device=dev)
        x = torch.randn(args.tokens, K, device=dev, dtype=torch.bfloat16)
        full = torch.empty(N, K, dtype=torch.bfloat16, device=dev)

        def fused():
            layer.calls += 1
            return C.gemm_allgather(x, layer.shard_ptrs, rank, layer.gathered, layer.flags, layer.calls)

        def nccl():
            if world > 1:
                dist.all_gather_into_tensor(full, layer.shard.detach())
            else:
                full.copy_(layer.shard.detach())
            return mm_nt(x, full)

        def gemm():
            return mm_nt(x, w)

        out = {"shape": name, "N": N, "K": K, "tokens": args.tokens}
        ref = x.float() @ w.float().t()
        for label, fn in (("fused", fused), ("nccl", nccl), ("gemm", gemm)):
            times = []
            for i in range(args.warmup + args.iters):
                flush.zero_()
                if dist.is_initialized():
                    dist.barrier()
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                y = fn()
                end.record()
                torch.cuda.synchronize()
                if i >= args.warmup:
                    times.append(start.elapsed_time(end))
            err = ((y.float() - ref).abs().max() / ref.abs().max()).item()
            ms = sorted(times)[len(times) // 2]
            if dist.is_initialized():
                t = torch.tensor([ms, err], device=dev, dtype=torch.float64)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms, err = float(t[0]), float(t[1])
            out[f"{label}_ms"] = round(ms, 4)
            out[f"{label}_max_rel_err"] = float(f"{err:.2e}")
        assert torch.equal(layer.gathered, w)
        flops = 2.0 * args.tokens * N * K
        nvlink = N * K * 2 * (world - 1) / world
        roof = max(flops / (tflops * 1e12), nvlink / (NVLINK_GBS * 1e9)) * 1e3
        out.update(roofline_ms=round(roof, 4), fused_frac_of_roofline=round(roof / out["fused_ms"], 3),
                   fused_vs_nccl=round(out["nccl_ms"] / out["fused_ms"], 3),
                   fused_tflops=round(flops / out["fused_ms"] / 1e9, 1),
                   nvlink_gbs_min_per_direction=round(nvlink / out["fused_ms"] / 1e6, 1))
        rows.append(out)
        layer.close()
    torch.cuda.synchronize()
    if status(local) != 0:
        raise RuntimeError("a GEMM kernel reported a timeout")
    if rank == 0:
        for r in rows:
            print(json.dumps({"kernel": "gemm_allgather (fused all-gather + GEMM)", "world": world, **r}), flush=True)
    if dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
