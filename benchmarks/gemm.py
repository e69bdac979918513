"""Dense projection GEMMs of the 1.3B bench model, one at a time.

    python benchmarks/gemm.py [--impl cublas|ours|both] [--tokens 16384] [--iters 20] [--kv-heads 4]

For every projection (gqkv, o, gate_up, down, lm_head) it times the three GEMMs of a training
step: forward ``Y = X W^T`` ("nt"), input gradient ``dX = dY W`` ("nn") and weight gradient
``dW = dY^T X`` ("tn"), bf16 in / fp32 accumulate / bf16 out.  Each launch is timed with CUDA
events after a write of a 512 MB buffer that flushes the 126 MB L2, so every operand comes from
HBM; the two implementations alternate launch by launch, and the median of ``--iters`` launches
is reported with TFLOP/s and the fraction of the measured bf16 peak.  ``ours`` runs the
hand-written tcgen05 kernel (``mimir_b200.ops.gemm``).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def shapes(kv_heads: int, d: int = 2048, heads: int = 16, hd: int = 128, ffn: int = 5632, vocab: int = 65536):
    """(name, out_features, in_features) of every projection."""
    return [("gqkv", (2 * heads + 2 * kv_heads) * hd, d), ("o", d, heads * hd), ("gate_up", 2 * ffn, d),
            ("down", d, ffn), ("lm_head", vocab, d)]


def _time(fn, flush, iters):
    times = []
    for _ in range(iters + 3):
        flush.add_(1)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    return statistics.median(times[3:])


def _time_interleaved(fns, flush, iters):
    """Median time of each function, the functions alternating launch by launch so that clock
    drift and neighbours on the machine affect them alike."""
    times = [[] for _ in fns]
    for it in range(iters + 3):
        for k, fn in enumerate(fns):
            flush.add_(1)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            if it >= 3:
                times[k].append(s.elapsed_time(e))
    return [statistics.median(t) for t in times]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--impl", choices=["cublas", "ours", "both"], default="both")
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--kv-heads", type=int, default=4)
    ap.add_argument("--only", default=None, help="comma-separated projection names")
    ap.add_argument("--check", action="store_true", help="compare ours against cuBLAS")
    ap.add_argument("--fused", action="store_true", help="also time the fused SwiGLU / accumulate epilogues")
    args = ap.parse_args()
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    peak = peaks.get("bf16_tflops", 1590.0)
    impls = ["cublas", "ours"] if args.impl == "both" else [args.impl]
    if "ours" in impls:
        from mimir_b200.ops import gemm as G
    flush = torch.empty(128 * 1024 * 1024, device="cuda", dtype=torch.float32)
    torch.manual_seed(0)
    T = args.tokens
    only = set(args.only.split(",")) if args.only else None
    rows = []
    for name, n_out, n_in in shapes(args.kv_heads):
        if only and name not in only:
            continue
        x = torch.randn(T, n_in, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(n_out, n_in, device="cuda", dtype=torch.bfloat16) * n_in ** -0.5
        dy = torch.randn(T, n_out, device="cuda", dtype=torch.bfloat16)
        flops = 2.0 * T * n_out * n_in
        cases = {
            "cublas": {"nt": lambda: torch.mm(x, w.t()), "nn": lambda: torch.mm(dy, w),
                       "tn": lambda: torch.mm(dy.t(), x)},
        }
        if "ours" in impls:
            cases["ours"] = {"nt": lambda: G.mm_nt(x, w), "nn": lambda: G.mm_nn(dy, w), "tn": lambda: G.mm_tn(dy, x)}
        for kind in ("nt", "nn", "tn"):
            row = {"proj": name, "kind": kind, "M": T if kind != "tn" else n_out,
                   "N": n_out if kind == "nt" else n_in, "K": n_in if kind == "nt" else (n_out if kind == "nn" else T)}
            timed = _time_interleaved([cases[impl][kind] for impl in impls], flush, args.iters)
            for impl, ms in zip(impls, timed):
                row[f"{impl}_ms"] = round(ms, 4)
                row[f"{impl}_tflops"] = round(flops / ms / 1e9, 1)
                row[f"{impl}_frac_of_measured"] = round(flops / ms / 1e9 / peak, 3)
            if args.check and "ours" in impls:
                ref = cases["cublas"][kind]().float()
                out = cases["ours"][kind]().float()
                row["max_rel_err"] = float(((out - ref).abs().max() / ref.abs().max().clamp_min(1e-6)).item())
            rows.append(row)
            print(json.dumps(row), flush=True)
    if len(impls) == 2:
        tot = {i: sum(r[f"{i}_ms"] for r in rows) for i in impls}
        print(json.dumps({"total_ms": tot}))
    if args.fused and "ours" in impls:
        fused_rows(T, args.iters, flush, peak)


def fused_rows(T, iters, flush, peak):
    """The fused epilogues as the model uses them, against cuBLAS plus the separate kernels."""
    from mimir_b200 import ops
    C = ops.ext()
    d, F = 2048, 5632
    x = torch.randn(T, d, device="cuda", dtype=torch.bfloat16)
    w_gu = torch.randn(2 * F, d, device="cuda", dtype=torch.bfloat16) * d ** -0.5
    w_dn = torch.randn(d, F, device="cuda", dtype=torch.bfloat16) * F ** -0.5
    dy = torch.randn(T, d, device="cuda", dtype=torch.bfloat16)
    gu = torch.mm(x, w_gu.t())
    grad = torch.zeros(2 * F, d, device="cuda", dtype=torch.bfloat16)
    dgu = torch.randn(T, 2 * F, device="cuda", dtype=torch.bfloat16)
    cases = [
        ("swiglu_forward (gate_up GEMM + SwiGLU)", 2.0 * T * 2 * F * d,
         lambda: C.gemm_swiglu(x, w_gu), lambda: C.swiglu_fwd(torch.mm(x, w_gu.t()))),
        ("swiglu_backward (down input-grad GEMM + SwiGLU bwd)", 2.0 * T * F * d,
         lambda: C.gemm_swiglu_bwd(dy, w_dn, gu), lambda: C.swiglu_bwd(torch.mm(dy, w_dn), gu)),
        ("gate_up weight grad accumulated in place (bf16)", 2.0 * T * 2 * F * d,
         lambda: C.gemm(dgu, True, x, True, grad, grad, 1.0, 1.0), lambda: grad.add_(torch.mm(dgu.t(), x))),
    ]
    for name, flops, ours, ref in cases:
        o, r = _time_interleaved([ours, ref], flush, iters)
        print(json.dumps({"fused": name, "ours_ms": round(o, 4), "cublas_plus_kernel_ms": round(r, 4),
                          "ours_tflops": round(flops / o / 1e9, 1),
                          "ours_frac_of_measured": round(flops / o / 1e9 / peak, 3)}), flush=True)


if __name__ == "__main__":
    main()
