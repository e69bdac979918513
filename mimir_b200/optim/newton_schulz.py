"""Newton–Schulz orthogonalisation for Muon on the tcgen05 tensor cores.

Behavioural reference: ``src/mimir/model/muon.py:15-24`` — five iterations of

    G = X X^T,   X <- a X + (b G + c G^2) X,   (a, b, c) = (3.4445, -4.7750, 2.0315)

on ``X = M / (||M||_F + 1e-7)`` (the wide orientation: tall matrices are transposed first), run
there in IEEE fp32 with cuBLAS.  Here every iteration is three batched GEMMs of the hand-written
CTA-pair kernel (``csrc/gemm.cu``) over all same-shape matrices of a step, each with its
combination fused into the epilogue:

    gram = X X^T                        (nt, X as both operands)
    poly = c * gram gram^T + b * gram   (nt; the Gram matrix is symmetric, so gram gram^T = gram^2)
    X'   = poly X + a * X               (nn, X read as an N-major operand)

Operands are bf16 with fp32 accumulation (the numerics change relative to the reference: the
iteration is a contraction towards the orthogonal polar factor and is commonly run in bf16; the
result differs from the fp32 chain by about 1e-2 relative, far below the update's own noise).
``MIMIR_MUON_NS=fp32`` selects the reference-exact fp32 chain.
"""
from __future__ import annotations

import os

import torch

NS_COEFFS = (3.4445, -4.7750, 2.0315)


def tensor_core_ns_enabled(t: torch.Tensor) -> bool:
    from mimir_b200.ops._ext import kernels_enabled
    return kernels_enabled(t) and os.environ.get("MIMIR_MUON_NS", "bf16") != "fp32"


def _supported_shape(m: int, n: int) -> bool:
    return m % 32 == 0 and n % 32 == 0


@torch.no_grad()
def orthogonalize_batch(matrices: torch.Tensor, steps: int = 5, coeffs=NS_COEFFS) -> torch.Tensor:
    """Newton–Schulz of a batch ``[B, rows, cols]`` (any float dtype) on the tensor cores; returns
    fp32 ``[B, rows, cols]``.  Falls back to the fp32 chain for shapes the kernel does not take."""
    from mimir_b200.optim.muon import orthogonalize
    x = matrices.float()
    tall = x.shape[-2] > x.shape[-1]
    if tall:
        x = x.mT
    m, n = x.shape[-2:]
    if not _supported_shape(m, n):
        return orthogonalize(matrices, steps)
    from mimir_b200.ops._ext import ext
    C = ext()
    a, b, c = coeffs
    x = (x / (x.norm(dim=(-2, -1), keepdim=True) + 1e-7)).to(torch.bfloat16).contiguous()
    batch = x.shape[0]
    gram = torch.empty(batch, m, m, device=x.device, dtype=torch.bfloat16)
    poly = torch.empty_like(gram)
    nxt = torch.empty_like(x)
    for _ in range(steps):
        C.gemm(x, False, x, False, gram)
        C.gemm(gram, False, gram, False, poly, gram, c, b)
        C.gemm(poly, False, x, True, nxt, x, 1.0, a)
        x, nxt = nxt, x
    out = x.float()
    return out.mT if tall else out


@torch.no_grad()
def orthogonalize_pieces_(pieces: list, steps: int, scale: float = 1.0) -> None:
    """Orthogonalise equal-shape fp32 matrices (views) in place, times ``scale``, in one batch."""
    out = orthogonalize_batch(torch.stack(pieces), steps)
    if scale != 1.0:
        out.mul_(scale)
    for piece, result in zip(pieces, out):
        piece.copy_(result)
