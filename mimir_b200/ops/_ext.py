"""Loader for the compiled sm_100a extension ``mimir_b200._C``.

On a CUDA tensor every op in :mod:`mimir_b200.ops` runs its hand-written kernel; if the
extension is missing there, the op raises instead of silently falling back to PyTorch.
``MIMIR_DISABLE_KERNELS=1`` forces the PyTorch formulation (used as the oracle in tests).
"""
from __future__ import annotations

import os

import torch

_EXT = None
_LOAD_ERROR: Exception | None = None

# Kernel launches issued by one call of each binding (for launch accounting in benchmarks).
_LAUNCHES_PER_CALL = {"fmha_status": 0, "fmha_plan": 1, "gemm_status": 0, "grouped_gemm_status": 0}


class _CountingModule:
    """Thin proxy over the compiled module that counts the kernels each binding launches."""

    def __init__(self, mod):
        self._mod = mod
        self.launches = 0

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn
        per_call = _LAUNCHES_PER_CALL.get(name, 1)

        def counted(*args, **kwargs):
            self.launches += per_call
            return fn(*args, **kwargs)
        counted.__name__ = name
        return counted


def ext():
    """Return the compiled extension module, raising a clear error if it was not built."""
    global _EXT, _LOAD_ERROR
    if _EXT is None:
        if _LOAD_ERROR is not None:
            raise RuntimeError(_missing_message()) from _LOAD_ERROR
        try:
            from mimir_b200 import _C  # type: ignore[attr-defined]
        except ImportError as exc:  # pragma: no cover - depends on the build
            _LOAD_ERROR = exc
            raise RuntimeError(_missing_message()) from exc
        _EXT = _CountingModule(_C)
    return _EXT


def launch_count() -> int:
    """Number of mimir_b200 kernels launched so far in this process."""
    return _EXT.launches if _EXT is not None else 0


def _missing_message() -> str:
    return ("mimir_b200._C (the sm_100a CUDA extension) is not built. Run "
            "`python setup.py build_ext --inplace` (or __graft_entry__.build()).")


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def kernels_enabled(t: torch.Tensor | None = None) -> bool:
    """True when ``t`` lives on a CUDA device and kernels are not disabled by the environment."""
    if os.environ.get("MIMIR_DISABLE_KERNELS", "0") == "1":
        return False
    return t is not None and t.is_cuda


class KernelTimeout(RuntimeError):
    """A hand-written kernel reported a launch whose outputs are not valid: a bounded wait ran out,
    an expert-exchange route named a rank or row outside its buffers, or a token id was outside
    the embedding table.  Raised by :func:`check_kernel_status`."""


def kernel_status(device: torch.device) -> dict:
    """Read and clear the status words of every kernel family on ``device``: the bounded-wait
    words of attention, dense GEMM and grouped GEMM (0: every wait since the last read completed),
    the expert-exchange route word and the embedding's token-id word (0: every index in range)."""
    if device.type != "cuda" or not available():
        return {}
    C = ext()
    index = device.index if device.index is not None else torch.cuda.current_device()
    return {"attention": int(C.fmha_status(device)), "gemm": int(C.gemm_status(index)),
            "grouped_gemm": int(C.grouped_gemm_status(index)), "moe_routes": int(C.moe_route_status(index)),
            "embedding_ids": int(C.embed_status(index))}


def check_kernel_status(device: torch.device, step=None) -> None:
    """Raise :class:`KernelTimeout` if any kernel on ``device`` reported a failed launch."""
    bad = {name: code for name, code in kernel_status(device).items() if code}
    if bad:
        where = "" if step is None else f" at or before step {step}"
        raise KernelTimeout(f"Kernel wait timed out or index out of range{where}: {bad} "
                            "(wait status codes from csrc/common.cuh)")
