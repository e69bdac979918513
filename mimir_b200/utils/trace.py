"""``resume_trace`` markers around collectives and phases (reference ``src/mimir/training/runtime.py:21-23``),
and NVTX ranges around the phases of a training step.

With ``resume_trace=true`` every rank prints ``[resume_trace rank=R] <event>`` (flushed)
so a hang can be localised to the last collective each rank entered.

:func:`nvtx_range` names a step's phases (``microbatch_<i>``, ``optimizer_step``,
``checkpoint_save``) on the CUDA timeline for a system profiler; without CUDA it does nothing.
"""
from __future__ import annotations

import sys
import time
from contextlib import contextmanager

import torch


def trace_print(config, rank: int, message: str) -> None:
    if getattr(config, "resume_trace", False):
        print(f"[resume_trace rank={rank} t={time.time():.3f}] {message}", file=sys.stderr, flush=True)


@contextmanager
def nvtx_range(name: str):
    if not torch.cuda.is_available():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
