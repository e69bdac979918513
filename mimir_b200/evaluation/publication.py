"""Optional tracker publication of an evaluation record on explicit step and epoch axes.

Reference behaviour: ``src/mimir/evaluation/publication.py:3-9``.
"""
from __future__ import annotations


def publish_record(run, record: dict, *, step: int, epoch: float) -> None:
    if type(step) is not int or step < 0:
        raise ValueError("Invalid step")
    if isinstance(epoch, bool) or not isinstance(epoch, (int, float)) or epoch < 0:
        raise ValueError("Invalid epoch")
    metrics = record["metrics"]
    run.define_metric("eval/step")
    run.define_metric("eval/epoch")
    for name in metrics:
        run.define_metric(name, step_metric="eval/epoch")
    run.log(dict(metrics) | {"eval/step": step, "eval/epoch": float(epoch)}, commit=True)
