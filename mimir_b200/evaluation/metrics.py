"""Exact aggregation of per-sample, per-pass observations (never unweighted shard means).

Reference behaviour: ``src/mimir/evaluation/metrics.py:8-88``.  Sample rows are JSON lines
``{"task", "sample_id", "pass", "scores": {metric: number}}``; a task set is published only
when every declared task has exactly the declared samples in every pass.  Classification
tasks additionally report accuracy, macro-F1 and multiclass MCC per pass (averaged over
passes); ``pass@k`` uses the unbiased estimator ``1 - C(n-c, k) / C(n, k)``.
"""
from __future__ import annotations

import json
import math
import os
import tempfile
from collections import Counter, defaultdict
from pathlib import Path


def _rows(paths):
    for path in paths:
        for line in Path(path).read_text().splitlines():
            if line.strip():
                yield json.loads(line)


def merge_samples(paths) -> dict:
    seen, sums, counts, n = set(), defaultdict(float), defaultdict(int), 0
    for row in _rows(paths):
        key = (row["task"], row["sample_id"], row["pass"])
        if key in seen:
            raise ValueError(f"Duplicate observation: {key}")
        seen.add(key)
        n += 1
        for metric, value in row["scores"].items():
            if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(value):
                raise ValueError("Finite numeric sample scores required")
            sums[f"{row['task']}/{metric}"] += value
            counts[f"{row['task']}/{metric}"] += 1
    if not n:
        raise ValueError("No observations")
    return {"schema": 1, "observations": n, "metrics": {k: sums[k] / counts[k] for k in sums},
            "sums": dict(sums), "counts": dict(counts)}


def write_record(path, record) -> None:
    """Atomically replace ``path`` with ``record`` as JSON (fsync'd temp file + rename)."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, temp = tempfile.mkstemp(prefix="." + path.name, dir=path.parent)
    try:
        with os.fdopen(fd, "w") as f:
            json.dump(record, f, allow_nan=False)
            f.flush()
            os.fsync(f.fileno())
        os.replace(temp, path)
    finally:
        if os.path.exists(temp):
            os.unlink(temp)


def classification_metrics(pairs) -> dict:
    """Accuracy, macro-F1 and multiclass MCC (Gorodkin's R_K) of ``(actual, predicted)`` pairs."""
    pairs = list(pairs)
    if not pairs:
        raise ValueError("No class observations")
    labels = {x for pair in pairs for x in pair}
    actual, predicted = Counter(a for a, _ in pairs), Counter(p for _, p in pairs)
    hits = Counter(a for a, p in pairs if a == p)
    n = len(pairs)
    f1 = sum(2 * hits[c] / (actual[c] + predicted[c]) for c in labels) / len(labels)
    cov = sum(hits.values()) * n - sum(actual[c] * predicted[c] for c in labels)
    norm = math.sqrt((n * n - sum(v * v for v in actual.values())) * (n * n - sum(v * v for v in predicted.values())))
    return {"accuracy": sum(hits.values()) / n, "macro_f1": f1, "mcc": cov / norm if norm else 0.0}


def pass_at_k(successes: int, attempts: int, k: int) -> float:
    if not 0 <= successes <= attempts or not 1 <= k <= attempts:
        raise ValueError("Invalid pass statistics")
    failures = attempts - successes
    return 1.0 - math.comb(failures, k) / math.comb(attempts, k) if failures >= k else 1.0


def complete_task_set(paths, expected: dict, *, classification_tasks=(), pass_k=None) -> dict:
    rows = list(_rows(paths))
    groups = defaultdict(list)
    for row in rows:
        groups[row["task"]].append(row)
    if set(groups) != set(expected):
        raise ValueError("Incomplete or unexpected task set")
    for task, items in groups.items():
        by_pass = defaultdict(set)
        for item in items:
            if item["sample_id"] in by_pass[item["pass"]]:
                raise ValueError("Duplicate sample/pass")
            by_pass[item["pass"]].add(item["sample_id"])
        want = expected[task]
        if len(by_pass) != want["passes"] or any(len(ids) != want["samples"] for ids in by_pass.values()):
            raise ValueError(f"Incomplete sample/pass coverage: {task}")
        first = next(iter(by_pass.values()))
        if any(ids != first for ids in by_pass.values()):
            raise ValueError("Passes contain different samples")
    record = merge_samples(paths)
    for task in classification_tasks:
        per_pass = defaultdict(list)
        for row in groups[task]:
            per_pass[row["pass"]].append((row["target_class"], row["predicted_class"]))
        scored = {str(p): classification_metrics(v) for p, v in per_pass.items()}
        record.setdefault("pass_metrics", {})[task] = scored
        for key in ("accuracy", "macro_f1", "mcc"):
            record["metrics"][f"{task}/{key}"] = sum(m[key] for m in scored.values()) / len(scored)
    for task, k in (pass_k or {}).items():
        outcomes = defaultdict(list)
        for row in groups[task]:
            outcomes[row["sample_id"]].append(bool(row["success"]))
        record["metrics"][f"{task}/pass@{k}"] = sum(pass_at_k(sum(v), len(v), k) for v in outcomes.values()) / len(outcomes)
    record["expected"] = expected
    return record
