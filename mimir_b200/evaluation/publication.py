"""Publish one evaluation record to an experiment tracker run (W&B-style API).

Behavioural reference: ``src/mimir/evaluation/publication.py:3-9``.  Evaluation metrics are
plotted against the fractional training epoch, so the run gets two explicit axes,
``eval/step`` and ``eval/epoch``, every metric is bound to the epoch axis, and the record is
logged in one committed call (all of it or nothing).
"""
from __future__ import annotations

STEP_AXIS = "eval/step"
EPOCH_AXIS = "eval/epoch"


def _axes(step, epoch) -> dict:
    if isinstance(step, bool) or not isinstance(step, int) or step < 0:
        raise ValueError("Invalid step")
    if isinstance(epoch, bool) or not isinstance(epoch, (int, float)) or epoch < 0:
        raise ValueError("Invalid epoch")
    return {STEP_AXIS: step, EPOCH_AXIS: float(epoch)}


def publish_record(run, record: dict, *, step: int, epoch: float) -> None:
    axes = _axes(step, epoch)
    metrics = dict(record["metrics"])
    for axis in axes:
        run.define_metric(axis)
    for name in metrics:
        run.define_metric(name, step_metric=EPOCH_AXIS)
    run.log({**metrics, **axes}, commit=True)
