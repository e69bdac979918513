"""``evaluate(suite, model, output)``: run a frozen suite and write per-sample JSONL + a receipt.

Reference behaviour: ``src/mimir/evaluation/clients.py:14-83``.  A suite is
``{"schema": 1, "tasks": [...]}``; blocked (unqualified) protocols refuse to run.  Backends:

* ``inspect`` — the task runs through Inspect AI when it is installed; tasks registered here
  (``mimir_b200.evaluation.tasks:<name>`` or a bare registered name) otherwise run through the
  direct runner against the same OpenAI-compatible endpoint;
* ``euroeval`` — the EuroEval benchmarker (version-pinned by the suite);
* ``cpu_fixture`` — next-token cross entropy of an exported model on fixed token ids;
* ``direct`` — always the built-in runner.

Outputs: ``<id>.samples.jsonl`` (or ``<id>.jsonl`` for fixtures), opened exclusively so a
rerun never appends to an earlier result, and ``receipt.json`` with the suite's SHA-256.
"""
from __future__ import annotations

import hashlib
import importlib
import json
import os
from pathlib import Path

from mimir_b200.evaluation.metrics import write_record
from mimir_b200.evaluation.runner import BackendOOM, run_task

TASK_MODULE = "mimir_b200.evaluation.tasks"
__all__ = ["evaluate", "BackendOOM"]


def _task_name(task: str) -> str:
    if ":" in task:
        module, name = task.split(":", 1)
        if not module.startswith(TASK_MODULE):
            raise ValueError("Unregistered task module")
        return name
    return task


def _write_rows(path: Path, rows) -> None:
    with path.open("x") as f:
        for row in rows:
            f.write(json.dumps(row, ensure_ascii=False) + "\n")


def _inspect_available() -> bool:
    try:
        importlib.import_module("inspect_ai")
        return True
    except ImportError:
        return False


def _run_registered(item, model, base_url, controls, out: Path) -> dict:
    from mimir_b200.evaluation.tasks import build
    spec = build(_task_name(item["task"]), **item.get("task_args", {}))
    if item.get("samples") and len(spec.samples) != item["samples"]:
        raise ValueError(f"Dataset count drift for {item['id']}")
    rows = run_task(spec, item, model, base_url, controls.get("max_connections", 4))
    _write_rows(out / f"{item['id']}.samples.jsonl", rows)
    return {"id": item["id"], "samples": len(rows), "runner": "direct"}


def _run_inspect(item, model, base_url, controls, out: Path) -> dict:
    from inspect_ai import eval as inspect_eval
    from mimir_b200.evaluation.tasks import build, inspect_task
    task = item["task"]
    if ":" in task or task in __import__(TASK_MODULE, fromlist=["REGISTRY"]).REGISTRY:
        task = inspect_task(build(_task_name(task), **item.get("task_args", {})))
        if item.get("samples") and len(task.dataset) != item["samples"]:
            raise ValueError(f"Dataset count drift for {item['id']}")
    logs = inspect_eval(task, model=f"{item.get('provider', 'openai')}/{model}", model_base_url=base_url,
                        log_dir=str(out / item["id"]), epochs=item.get("passes", 1), limit=item.get("limit"),
                        sample_id=item.get("sample_ids"), sample_shuffle=item.get("shuffle_seed"),
                        max_connections=controls.get("max_connections", 4), **item.get("generation", {}))
    failed = [log for log in logs if log.status != "success"]
    if failed:
        errors = "\n".join(str(log.error) for log in failed)
        if "torch.OutOfMemoryError" in errors or "CUDA out of memory" in errors:
            raise BackendOOM(errors)
        raise RuntimeError(f"Inspect task failed: {item['id']}: {errors}")
    rows = []
    for log in logs:
        for sample in log.samples or []:
            numeric = {}
            for name, score in (sample.scores or {}).items():
                value = score.value
                if value in ("C", "I"):
                    value = 1.0 if value == "C" else 0.0
                if isinstance(value, (int, float)):
                    numeric[name] = value
                elif isinstance(value, dict):
                    numeric.update({f"{name}/{k}": v for k, v in value.items() if isinstance(v, (int, float))})
            rows.append({"task": item.get("aggregate_task", item["id"]), "sample_id": f"{item['id']}:{sample.id}",
                         "pass": sample.epoch, "scores": numeric, "raw": sample.model_dump(mode="json")})
    _write_rows(out / f"{item['id']}.samples.jsonl", rows)
    return {"id": item["id"], "logs": [log.location for log in logs]}


def _run_euroeval(item, model, base_url, out: Path) -> dict:
    from importlib.metadata import version
    if version("euroeval") != item["version"]:
        raise ValueError("EuroEval protocol version mismatch")
    from euroeval import Benchmarker
    bench = Benchmarker(api_base=base_url, api_key=os.environ.get("OPENAI_API_KEY"), cache_dir=str(out / item["id"]),
                        raise_errors=True, save_results=True, num_iterations=item["passes"],
                        evaluate_test_split=item["split"] == "test", few_shot=item["few_shot"])
    results = bench.benchmark(model=model, dataset=item["dataset"])
    serial = [r.model_dump(mode="json") if hasattr(r, "model_dump") else r for r in results]
    write_record(out / f"{item['id']}.json", serial)
    return {"id": item["id"], "results": serial}


def _run_fixture(item, model, out: Path) -> dict:
    import torch
    from mimir_b200.export.hf import Mimir2ForCausalLM
    native = Mimir2ForCausalLM.from_pretrained(model)
    rows = []
    for i, example in enumerate(item["examples"]):
        ids = torch.tensor([example["input_ids"]])
        logits = native(ids)
        loss = torch.nn.functional.cross_entropy(logits[:, :-1].flatten(0, 1), ids[:, 1:].flatten()).item()
        rows.append({"task": item["id"], "sample_id": i, "pass": 1, "scores": {"cross_entropy": loss}})
    (out / f"{item['id']}.jsonl").write_text("".join(json.dumps(r) + "\n" for r in rows))
    return {"id": item["id"], "samples": len(rows)}


def evaluate(suite, model, output, base_url: str = "http://127.0.0.1:8000/v1", controls=None) -> dict:
    controls = controls or {}
    path = Path(suite)
    protocol = json.loads(path.read_text())
    if protocol.get("schema") != 1:
        raise ValueError("Unsupported suite schema")
    out = Path(output)
    out.mkdir(parents=True, exist_ok=True)
    receipt = {"suite_sha256": hashlib.sha256(path.read_bytes()).hexdigest(), "model": model, "tasks": []}
    for item in protocol["tasks"]:
        if item.get("blocked"):
            raise ValueError(f"Protocol {item['id']} is not qualified: {item['blocked']}")
        backend = item["backend"]
        if backend == "inspect":
            runner = _run_inspect if _inspect_available() else _run_registered
            receipt["tasks"].append(runner(item, model, base_url, controls, out))
        elif backend == "direct":
            receipt["tasks"].append(_run_registered(item, model, base_url, controls, out))
        elif backend == "euroeval":
            receipt["tasks"].append(_run_euroeval(item, model, base_url, out))
        elif backend == "cpu_fixture":
            receipt["tasks"].append(_run_fixture(item, model, out))
        else:
            raise ValueError(f"Unsupported backend: {backend}")
    write_record(out / "receipt.json", receipt)
    return receipt
