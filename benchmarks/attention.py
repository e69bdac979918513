"""Micro-benchmark of the prefix-LM FMHA kernels (forward and backward) on the flagship shape.

    python benchmarks/attention.py [--tokens 16384] [--seq 4096] [--heads 16] [--kv-heads 4] [--iters 20]

Times each kernel with CUDA events after warm-up and reports achieved TFLOP/s (model FLOPs of
the visible (query, key) pairs; backward counted as 2.5x forward) against the measured bf16
peak in MEASURED_PEAKS.json.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--kv-heads", type=int, default=4)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--max-prefix", type=int, default=2048)
    ap.add_argument("--causal", action="store_true")
    ap.add_argument("--once", action="store_true", help="one forward + one backward launch (for profilers)")
    args = ap.parse_args()
    from mimir_b200 import ops
    from mimir_b200.data.prefixlm import compute_aux_seq_tensors_scalars
    from mimir_b200.ops.attention import attention_plan

    torch.manual_seed(0)
    nseq = args.tokens // args.seq
    rng = np.random.default_rng(0)
    prefix = rng.integers(0, args.max_prefix + 1, size=nseq).astype(np.int32)
    causal = (args.seq - prefix).astype(np.int32)
    tensors, scalars = compute_aux_seq_tensors_scalars(prefix, causal, args.tokens)
    meta = {k: torch.from_numpy(v).cuda() for k, v in tensors.items()}
    T, H, KV = args.tokens, args.heads, args.kv_heads
    q = torch.randn(T, H * 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(T, KV * 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(T, KV * 128, device="cuda", dtype=torch.bfloat16)
    do = torch.randn(T, H * 128, device="cuda", dtype=torch.bfloat16)
    C = ops.ext()
    cu, pl = meta["cu_seqlens"], meta["prefix_lens"]
    from mimir_b200.ops.attention import forward_kernel
    fwd_kernel, kind = forward_kernel()
    tiles, ntiles = attention_plan(cu, pl, nseq, T, args.causal, kind=kind)
    kv_tiles, kv_ntiles = attention_plan(cu, pl, nseq, T, args.causal, backward=True)

    def fwd():
        return fwd_kernel(q, 0, k, 0, v, 0, None, 0, H, KV, args.causal, cu, pl, nseq, tiles, ntiles)

    out, lse = fwd()
    delta = C.attn_delta(do, out, H)

    def bwd():
        return C.fmha_bwd(q, 0, k, 0, v, 0, do, lse, delta, H, KV, args.causal, cu, pl, nseq, kv_tiles, kv_ntiles)

    if args.once:
        fwd()
        bwd()
        torch.cuda.synchronize()
        assert C.fmha_status(q.device) == 0
        return
    pairs = 0
    for p in prefix:
        p = int(p) if not args.causal else 0
        pairs += p * p + sum(r + 1 for r in range(p, args.seq))
    flops_fwd = 4.0 * 128 * H * pairs
    res = {}
    for name, fn, flops in (("fwd", fwd, flops_fwd), ("bwd", bwd, 2.5 * flops_fwd)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / args.iters
        res[name] = {"ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1)}
    try:
        peak = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"]
    except (OSError, KeyError, ValueError):
        peak = 1590.0
    for r in res.values():
        r["frac_of_measured_bf16"] = round(r["tflops"] / peak, 3)
    assert C.fmha_status(q.device) == 0
    print(json.dumps({"shape": vars(args), "pairs": pairs, **res}))


if __name__ == "__main__":
    main()
