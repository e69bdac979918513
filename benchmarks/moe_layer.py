"""Micro-benchmark of one MoE MLP mixture (forward + backward) on one GPU.

    python benchmarks/moe_layer.py [--tokens 16384] [--experts 64] [--top-k 2] [--ffn 1408] [--shared 1]
                                   [--impl grouped|index] [--router-std 0.0221] [--profile]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/moe_layer.py    # expert parallel over N GPUs

Times ``iters`` forward+backward passes of the mixture of BASELINE config 3 (d 2048) with CUDA
events after warm-up and reports achieved TFLOP/s of the expert GEMMs (top-k routed + shared
experts, 3 GEMMs forward and 6 backward per expert row block).  Under torchrun the experts are
split over the ranks (expert parallelism, tokens exchanged over NVLink peer memory) and the
time is the maximum over ranks.  ``--profile`` prints the torch.profiler table of the top CUDA
and CPU consumers of one pass (rank 0) instead.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--top-k", type=int, default=2)
    ap.add_argument("--ffn", type=int, default=1408)
    ap.add_argument("--shared", type=int, default=1)
    ap.add_argument("--impl", choices=["grouped", "index"], default="grouped")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--router-std", type=float, default=2048 ** -0.5,
                    help="router row init std (0: the reference's zero rows, every token to experts 0..k-1)")
    ap.add_argument("--profile", action="store_true")
    args = ap.parse_args()
    import torch.distributed as dist
    from mimir_b200.models.experts import MLPMixture
    from mimir_b200.models.layers import SwiGLU

    local = int(os.environ.get("LOCAL_RANK", 0))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ep = "RANK" in os.environ
    if ep:
        dist.init_process_group("nccl", device_id=dev)
    rank = dist.get_rank() if ep else 0
    torch.manual_seed(0)
    d = args.hidden
    m = MLPMixture(SwiGLU(d, args.ffn), d, args.experts, args.top_k, sparse=True, grouped=args.impl == "grouped",
                   shared_experts=args.shared, expert_intermediate_size=args.ffn, expert_parallel=ep,
                   router_init_std=args.router_std or None).to(dev, torch.bfloat16)
    gen = torch.Generator(device=dev).manual_seed(100 + rank)
    x = torch.randn(args.tokens, d, device=dev, dtype=torch.bfloat16, generator=gen).requires_grad_(True)
    g = torch.randn(args.tokens, d, device=dev, dtype=torch.bfloat16, generator=gen)

    def step():
        y = m(x)
        y.backward(g)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    if args.profile:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
            step()
            torch.cuda.synchronize()
        if rank == 0:
            print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=20))
            print(prof.key_averages().table(sort_by="self_cpu_time_total", row_limit=20))
        if ep:
            dist.destroy_process_group()
        return
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.iters):
        step()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.iters
    if ep:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    rows = args.tokens * (args.top_k + args.shared)
    flops = 3 * 2.0 * rows * 3 * d * args.ffn  # forward + 2x backward, three projections (per rank)
    if rank == 0:
        print(json.dumps({"impl": args.impl, "ranks": dist.get_world_size() if ep else 1, "tokens_per_rank": args.tokens,
                          "experts": args.experts, "top_k": args.top_k, "ffn": args.ffn, "shared": args.shared,
                          "router_std": args.router_std, "ms": round(ms, 3),
                          "expert_tflops_per_rank": round(flops / ms / 1e9, 1)}))
    if ep:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
