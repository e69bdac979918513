"""``resume_trace`` markers around collectives and phases (reference ``src/mimir/training/runtime.py:21-23``).

With ``resume_trace=true`` every rank prints ``[resume_trace rank=R] <event>`` (flushed)
so a hang can be localised to the last collective each rank entered.
"""
from __future__ import annotations

import sys
import time


def trace_print(config, rank: int, message: str) -> None:
    if getattr(config, "resume_trace", False):
        print(f"[resume_trace rank={rank} t={time.time():.3f}] {message}", file=sys.stderr, flush=True)
