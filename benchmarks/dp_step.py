"""Micro-benchmark of the fused data-parallel step (reduce-scatter + AdamATan2 + all-gather).

    python benchmarks/dp_step.py [--params 1.3e9] [--iters 10]                      # one GPU
    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/dp_step.py        # N GPUs
    ... benchmarks/dp_step.py --optimizer muon                                      # MuonAdamW step

A synthetic parameter set with the flagship model's total size (one [rows, 2048] matrix per
~50M parameters) is wrapped by the replicated engine; gradients are random bf16.  Each timed
iteration is one ``optimizer.step()`` (ordering all-reduce, fused kernel, ordering all-reduce),
timed with CUDA events after warm-up; the maximum over ranks is reported.  The roofline is the
slower of the HBM bytes at the measured copy bandwidth and the NVLink bytes at the measured
770 GB/s per direction.

``--optimizer muon`` builds the flagship's real matrix shapes (24 layers of gqkv 5120x2048,
o 2048x2048, gate_up 11264x2048, down 2048x5632, plus the 65536x2048 embedding and head under
Adam) and times the replicated MuonAdamW step: fused reduce + momentum + gather-to-owner,
Newton-Schulz (batched bf16 tensor-core GEMMs) on each matrix's owner only, fused scatter +
update + all-gather.  It also
reports the per-rank Newton-Schulz FLOPs against what a redundant every-rank chain would do.
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
    ap.add_argument("--optimizer", choices=["adam_atan2", "muon"], default="adam_atan2")
    args = ap.parse_args()
    from mimir_b200.parallel.replicated import ReplicatedAdamATan2, ReplicatedMuonAdamW, wrap_replicated
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if "RANK" in os.environ:
        dist.init_process_group("nccl", device_id=dev)
    world = dist.get_world_size() if dist.is_initialized() else 1
    torch.manual_seed(0)
    if args.optimizer == "muon":
        model = flagship_shapes(dev)
    else:
        cols = 2048
        rows = 24 * 1024  # 50M parameters per matrix
        n = max(1, round(args.params / (rows * cols)))
        model = torch.nn.ParameterList([torch.nn.Parameter(torch.randn(rows, cols, device=dev) * 0.02)
                                        for _ in range(n)])
    engine = wrap_replicated(model, dev, torch.bfloat16)
    hp = dict(lr=1e-4, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9999)
    opt = (ReplicatedMuonAdamW(engine, momentum=0.95, ns_steps=5, **hp) if args.optimizer == "muon"
           else ReplicatedAdamATan2(engine, **hp))
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
    if args.optimizer == "muon":
        report_muon(opt, engine, world, total, seconds)
    elif not dist.is_initialized() or dist.get_rank() == 0:
        print(json.dumps({"kernel": "dp_step (fused reduce-scatter + AdamATan2 + all-gather)", "world": world,
                          "params": total, "ms": round(seconds * 1e3, 3), "roofline_ms": round(roofline * 1e3, 3),
                          "frac_of_roofline": round(roofline / seconds, 3),
                          "hbm_gbs_achieved": round(hbm_bytes / seconds / 1e9, 1),
                          "nvlink_gbs_per_direction": round(nvlink_bytes / seconds / 1e9, 1)}), flush=True)
    engine.close()
    if dist.is_initialized():
        dist.destroy_process_group()


def flagship_shapes(dev):
    """Parameters with the flagship's names and shapes (Muon matrices are found by name)."""
    from torch import nn

    def param(*shape):
        return nn.Parameter(torch.randn(*shape, device=dev) * 0.02)

    root = nn.Module()
    root.embed_tokens = param(65536, 2048)
    root.layers = nn.ModuleList()
    for _ in range(24):
        layer = nn.Module()
        layer.attn, layer.mlp = nn.Module(), nn.Module()
        layer.attn.gqkv_proj, layer.attn.o_proj = nn.Module(), nn.Module()
        layer.mlp.gate_up_proj, layer.mlp.down_proj = nn.Module(), nn.Module()
        layer.attn.gqkv_proj.weight = param(2 * 2048 + 2 * 512, 2048)
        layer.attn.o_proj.weight = param(2048, 2048)
        layer.mlp.gate_up_proj.weight = param(2 * 5632, 2048)
        layer.mlp.down_proj.weight = param(2048, 5632)
        layer.norm = param(2048)
        root.layers.append(layer)
    root.head = param(65536, 2048)
    return root


def ns_flops(rows, cols, count, steps=5):
    r, c = rows // count, cols
    m, n = min(r, c), max(r, c)
    return count * steps * 2.0 * (2 * m * m * n + m ** 3)


def report_muon(opt, engine, world, total, seconds):
    rank = dist.get_rank() if dist.is_initialized() else 0
    per_rank = {}
    for s in engine.slots:
        if opt.splits.get(s.fqn):
            k = opt.owner[s.fqn]
            per_rank[k] = per_rank.get(k, 0.0) + ns_flops(s.rows, s.numel // s.rows, opt.splits[s.fqn])
    redundant = sum(per_rank.values())
    if rank == 0:
        print(json.dumps({"kernel": "MuonAdamW step (fused gather-to-owner, owner Newton-Schulz, fused scatter)",
                          "world": world, "params": total, "ms": round(seconds * 1e3, 3),
                          "ns_tflop_max_rank": round(max(per_rank.values()) / 1e12, 2),
                          "ns_tflop_every_rank_redundant": round(redundant / 1e12, 2),
                          "ns_dtype": ("fp32 (IEEE, as the reference)" if os.environ.get("MIMIR_MUON_NS") == "fp32"
                                       else "bf16 operands, fp32 accumulation (tensor cores)")}), flush=True)


if __name__ == "__main__":
    main()
