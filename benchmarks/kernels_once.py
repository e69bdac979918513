"""Launch every hand-written non-attention kernel once, forward and backward, on flagship-sized
inputs (for a one-capture ncu summary of all of them).

    python benchmarks/kernels_once.py [--tokens 65536] [--experts 64] [--buckets 1048576]

Kernels: RMSNorm and fused add+RMSNorm (forward/backward), SwiGLU (forward/backward), the fused
linear cross-entropy, the n-gram memory gather/scatter (2^20-row tables), the MoE
router top-k + load counts, the MoE dispatch / combine / combine-backward exchange, the grouped
expert GEMMs, and the multi-tensor AdamATan2 update.  Activations are 2048 wide; at the default
65536 tokens each is 256 MB of bf16, above the 126 MB L2, so DRAM figures are meaningful.
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
    ap.add_argument("--tokens", type=int, default=65536)
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--buckets", type=int, default=2 ** 20)
    args = ap.parse_args()
    from mimir_b200 import ops
    from mimir_b200.models.experts import MLPMixture
    from mimir_b200.models.layers import SwiGLU
    from mimir_b200.models.ngram import NGramMemory
    from mimir_b200.optim.adam_atan2 import AdamATan2

    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    T, d, F = args.tokens, 2048, 5632
    bf = dict(device=dev, dtype=torch.bfloat16)

    x = torch.randn(T, d, **bf, requires_grad=True)
    ops.rms_norm(x, 1e-6).backward(torch.randn(T, d, **bf))
    delta = torch.randn(T, d, **bf, requires_grad=True)
    h, n = ops.add_rms_norm(x, delta, 1e-6)
    (h.float().sum() + n.float().sum()).backward()
    del h, n, delta

    gu = torch.randn(T // 4, 2 * F, **bf, requires_grad=True)
    ops.swiglu(gu).backward(torch.randn(T // 4, F, **bf))
    del gu

    w = (torch.randn(65536, d, **bf) * 0.02).requires_grad_(True)
    hid = torch.randn(T // 4, d, **bf, requires_grad=True)
    labels = torch.randint(0, 65536, (T // 4,), device=dev)
    loss, _ = ops.linear_cross_entropy(hid, w, labels)
    loss.backward()
    del w, hid

    ng = NGramMemory(256, orders=(2, 3), buckets=args.buckets, heads=1).to(dev, torch.bfloat16)  # config 5: 256 dims
    ids = torch.randint(0, 65536, (1, T), device=dev)
    pos = torch.arange(T, device=dev).remainder(4096).unsqueeze(0)
    ng.lookup(ids, pos, torch.bfloat16).float().sum().backward()
    del ng

    moe = MLPMixture(SwiGLU(d, 1408), d, args.experts, 2, sparse=True, grouped=True, shared_experts=0,
                     expert_intermediate_size=1408, router_init_std=d ** -0.5).to(dev, torch.bfloat16)
    xm = torch.randn(T // 4, d, **bf, requires_grad=True)
    moe(xm).float().sum().backward()

    params = [torch.nn.Parameter(torch.randn(4096, d, device=dev)) for _ in range(8)]
    for p in params:
        p.grad = torch.randn_like(p)
    AdamATan2(params, lr=1e-4, ema=0.999).step()
    torch.cuda.synchronize()
    assert ops.ext().fmha_status(dev) == 0 and ops.ext().grouped_gemm_status(0) == 0
    print("kernels_once ok")


if __name__ == "__main__":
    main()
