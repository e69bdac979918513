"""Direct evaluation runner: task specs against an OpenAI-compatible chat endpoint.

Runs every sample of a :class:`~mimir_b200.evaluation.tasks.TaskSpec` for ``passes`` epochs
with up to ``max_connections`` concurrent requests (plain ``urllib``; no SDK), scores each
completion and returns sample rows in the schema ``metrics.merge_samples`` aggregates.  The
``mockllm`` provider answers ``"Default output from mockllm/model"`` without a server, for
offline wiring tests.  A server error that reports a CUDA allocation failure raises
``BackendOOM`` so the scheduler can retry with fewer connections.
"""
from __future__ import annotations

import json
import urllib.error
import urllib.request
from concurrent.futures import ThreadPoolExecutor

MOCK_COMPLETION = "Default output from mockllm/model"
_OOM_MARKERS = ("torch.OutOfMemoryError", "CUDA out of memory")


class BackendOOM(RuntimeError):
    """Confirmed CUDA allocation failure reported by an evaluation backend."""


def chat_completion(base_url: str, model: str, messages: list, generation: dict, timeout: float = 600) -> str:
    body = json.dumps({"model": model, "messages": messages, **generation}).encode()
    request = urllib.request.Request(base_url.rstrip("/") + "/chat/completions", data=body,
                                     headers={"Content-Type": "application/json"})
    try:
        with urllib.request.urlopen(request, timeout=timeout) as response:
            payload = json.loads(response.read())
    except urllib.error.HTTPError as error:
        text = error.read().decode(errors="replace")
        if any(m in text for m in _OOM_MARKERS):
            raise BackendOOM(text) from error
        raise RuntimeError(f"Backend error {error.code}: {text[:2000]}") from error
    return payload["choices"][0]["message"]["content"] or ""


def run_task(spec, item: dict, model: str, base_url: str, max_connections: int = 4) -> list[dict]:
    generation = dict(spec.generation) | item.get("generation", {})
    provider = item.get("provider", "openai")
    wanted = item.get("sample_ids")
    samples = [s for s in spec.samples if wanted is None or s["id"] in wanted]
    if item.get("limit") is not None:
        samples = samples[:item["limit"]]
    jobs = [(p, s) for p in range(1, item.get("passes", 1) + 1) for s in samples]

    def one(job):
        epoch, sample = job
        if provider == "mockllm":
            completion = MOCK_COMPLETION
        else:
            completion = chat_completion(base_url, model, sample["messages"], generation)
        scored = spec.score(completion, sample)
        row = {"task": item.get("aggregate_task", item["id"]), "sample_id": f"{item['id']}:{sample['id']}",
               "pass": epoch, "scores": scored["scores"],
               "raw": {"input": sample["messages"], "target": sample["target"], "output": {"completion": completion}}}
        row.update({k: v for k, v in scored.items() if k in ("target_class", "predicted_class", "success")})
        return row

    with ThreadPoolExecutor(max(1, max_connections)) as pool:
        return list(pool.map(one, jobs))
