"""Dense projection GEMMs on the hand-written tcgen05 CTA-pair kernel (``csrc/gemm.cu``).

The reference runs every projection through ``F.linear`` (cuBLAS): ``src/mimir/model/layers.py:86-87``
(``LinearInit``), ``:246`` (``o_proj``), ``:259-271`` (SwiGLU) and ``src/mimir/model/lm_head.py:65``.
Here the three GEMMs of a linear layer are one kernel with three operand layouts:

* forward ``Y = X W^T`` (:func:`mm_nt`),
* input gradient ``dX = dY W`` (:func:`mm_nn`, the weight read as an N-major operand),
* weight gradient ``dW = dY^T X`` (:func:`mm_tn`, both operands M/N-major; it can accumulate in
  place into the replicated engine's gradient view).

:func:`linear` is the autograd op of a bias-free linear layer and :func:`swiglu_mlp` the whole
``down(silu(gate) * up)`` MLP: its forward GEMM writes ``gate|up`` and the SwiGLU product in one
epilogue, and its backward fuses the SwiGLU derivative into the down projection's input-gradient
GEMM.  Every function needs CUDA bf16 operands; :func:`supported` says when the kernel applies.
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from mimir_b200.ops._ext import ext, kernels_enabled


def _library_comparison() -> bool:
    """``MIMIR_GEMM=cublas`` routes the projections through ``F.linear`` (cuBLAS) instead of the
    tcgen05 kernel: an explicit A/B switch for benchmarks, never a fallback."""
    return os.environ.get("MIMIR_GEMM", "tcgen05") == "cublas"


def mm_nt(x: torch.Tensor, w: torch.Tensor, out=None) -> torch.Tensor:
    """``x @ w.T`` for ``x`` [M, K] and ``w`` [N, K]."""
    return ext().gemm(x, False, w, False, out)


def mm_nn(dy: torch.Tensor, w: torch.Tensor, out=None) -> torch.Tensor:
    """``dy @ w`` for ``dy`` [M, K] and ``w`` [K, N]."""
    return ext().gemm(dy, False, w, True, out)


def mm_tn(dy: torch.Tensor, x: torch.Tensor, out=None, accumulate: bool = False) -> torch.Tensor:
    """``dy.T @ x`` for ``dy`` [K, M] and ``x`` [K, N]; with ``accumulate`` the product is added to
    ``out`` in place (bf16 or fp32)."""
    if accumulate:
        return ext().gemm(dy, True, x, True, out, out, 1.0, 1.0)
    return ext().gemm(dy, True, x, True, out)


def status(device: torch.device | int = 0) -> int:
    """Read and clear the GEMM kernels' bounded-wait status of ``device`` (0 = ok)."""
    return int(ext().gemm_status(device.index if isinstance(device, torch.device) else int(device)))


def _aligned(t: torch.Tensor) -> bool:
    return t.data_ptr() % 16 == 0 and (t.dim() < 2 or (t.stride(-1) == 1 and (t.stride(-2) * 2) % 16 == 0))


def supported(x: torch.Tensor, w: torch.Tensor) -> bool:
    """True when ``linear(x, w)`` runs on the tcgen05 kernel: CUDA bf16, kernels enabled,
    16-byte aligned rows and an output width that is a multiple of 32."""
    return (kernels_enabled(x) and not _library_comparison() and x.dtype == torch.bfloat16
            and w.dtype == torch.bfloat16 and w.dim() == 2
            and w.shape[0] % 32 == 0 and w.shape[1] % 8 == 0 and w.shape[1] == x.shape[-1] and w.is_contiguous()
            and _aligned(w))


def weight_grad(w: torch.Tensor, dy2: torch.Tensor, x2: torch.Tensor):
    """Gradient ``dy2.T @ x2`` of weight ``w``.  When the replicated engine owns ``w.grad`` (a view
    into its flat buffer, announced by a ``_mimir_grad_sink`` callback), the GEMM accumulates into
    it in place and autograd gets ``None``; otherwise a new tensor is returned."""
    sink = getattr(w, "_mimir_grad_sink", None)
    if sink is not None and w.grad is not None and w.grad.dtype in (torch.bfloat16, torch.float32) \
            and w.grad.is_contiguous():
        mm_tn(dy2, x2, out=w.grad, accumulate=True)
        sink(w)
        return None
    return mm_tn(dy2, x2)


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        x2 = x.reshape(-1, x.shape[-1])
        if not _aligned(x2):
            x2 = x2.contiguous()
        ctx.save_for_backward(x2, w)
        ctx.x_shape = x.shape
        return mm_nt(x2, w).view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1])
        if not _aligned(dy2):
            dy2 = dy2.contiguous()
        dx = mm_nn(dy2, w).view(ctx.x_shape) if ctx.needs_input_grad[0] else None
        dw = weight_grad(w, dy2, x2) if ctx.needs_input_grad[1] else None
        return dx, dw


def linear(x: torch.Tensor, w: torch.Tensor, bias=None) -> torch.Tensor:
    """``F.linear(x, w, bias)`` with the forward and both gradients on the tcgen05 kernel when
    :func:`supported`; plain ``F.linear`` otherwise (CPU, fp32, odd shapes)."""
    if bias is None and supported(x, w):
        return _LinearFn.apply(x, w)
    return F.linear(x, w, bias)


class _SwiGLUMLPFn(torch.autograd.Function):
    """``down(silu(gate) * up)`` with ``gate|up`` packed in ``w_gu`` ([2F, D]) and ``w_down`` [D, F].
    Saved for backward: the input rows, ``gate|up`` (bf16) and the product ``h``."""

    @staticmethod
    def forward(ctx, x, w_gu, w_down):
        C = ext()
        x2 = x.reshape(-1, x.shape[-1])
        if not _aligned(x2):
            x2 = x2.contiguous()
        h, gu = C.gemm_swiglu(x2, w_gu)
        y = mm_nt(h, w_down)
        ctx.save_for_backward(x2, gu, h, w_gu, w_down)
        ctx.x_shape = x.shape
        return y.view(*x.shape[:-1], w_down.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, gu, h, w_gu, w_down = ctx.saved_tensors
        C = ext()
        dy2 = dy.reshape(-1, dy.shape[-1])
        if not _aligned(dy2):
            dy2 = dy2.contiguous()
        dgu = C.gemm_swiglu_bwd(dy2, w_down, gu)
        # Every read of a weight is enqueued before its gradient is announced (the replicated
        # engine may update a block's weights as soon as all of its gradients are announced).
        dx = mm_nn(dgu, w_gu).view(ctx.x_shape) if ctx.needs_input_grad[0] else None
        d_down = weight_grad(w_down, dy2, h) if ctx.needs_input_grad[2] else None
        d_gu = weight_grad(w_gu, dgu, x2) if ctx.needs_input_grad[1] else None
        return dx, d_gu, d_down


def swiglu_mlp_supported(x: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor) -> bool:
    """True when :func:`swiglu_mlp` runs on the tcgen05 kernels (F a multiple of 128)."""
    if not (kernels_enabled(x) and x.dtype == w_gu.dtype == w_down.dtype == torch.bfloat16) or _library_comparison():
        return False
    if w_gu.dim() != 2 or w_down.dim() != 2:
        return False
    d, f = w_down.shape
    return (tuple(w_gu.shape) == (2 * f, x.shape[-1]) and f % 128 == 0 and d % 32 == 0 and x.shape[-1] % 8 == 0
            and w_gu.is_contiguous() and w_down.is_contiguous() and _aligned(w_gu) and _aligned(w_down))


def swiglu_mlp(x: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    """The SwiGLU MLP ``down(silu(gate) * up)`` as two fused tcgen05 GEMMs per direction."""
    return _SwiGLUMLPFn.apply(x, w_gu, w_down)
