"""Scheduler queue, worker, idle coordinator, evaluation metrics/clients and serving (CPU, host fakes)."""
import json
import sys
import time
from concurrent.futures import ThreadPoolExecutor

import pytest

from mimir_b200.evaluation.metrics import classification_metrics, complete_task_set, merge_samples, pass_at_k
from mimir_b200.scheduling import idle
from mimir_b200.scheduling.store import Store
from mimir_b200.scheduling.worker import run_one
from mimir_b200.serving.server import ServerSpec, command


# ------------------------------------------------------------------ store / worker
def test_failed_eval_and_merge_do_not_strand_training(tmp_path):
    store = Store(tmp_path / "queue.db")
    store.add("eval", "inference", {"command": [sys.executable, "-c", 'raise RuntimeError("bad eval")'],
                                    "resources": ["gpu:0"]})
    store.add("merge", "merge", {"inputs": ["absent"], "output": str(tmp_path / "average")}, [("eval", "success")])
    marker = tmp_path / "resumed"
    store.add("resume", "train", {"command": [sys.executable, "-c", f'open({str(marker)!r},"w").write("resumed")'],
                                  "resources": ["gpu:0"]}, [("eval", "terminal")])
    while run_one(store, tmp_path / "attempts"):
        pass
    assert marker.read_text() == "resumed"
    assert {r["id"]: r["state"] for r in store.rows()} == {"eval": "failed", "merge": "blocked", "resume": "succeeded"}


def test_claims_are_exclusive_and_snapshots_immutable(tmp_path):
    store = Store(tmp_path / "queue.db")
    store.add("a", "eval", {"controls": {"max_connections": 8}, "resources": ["gpu:0"]})
    store.add("b", "eval", {"resources": ["gpu:0"]})
    with ThreadPoolExecutor(4) as pool:
        claims = list(pool.map(lambda _: store.claim(), range(4)))
    active = [c for c in claims if c]
    assert len(active) == 1
    job = active[0]
    with pytest.raises(ValueError):
        store.edit(job["id"], {})
    store.finish(job["owner"], False, {"reason": "oom"}, oom=True)
    retry = store.claim()
    assert retry["config"]["controls"]["max_connections"] == 4
    with store.connect() as db:
        original = json.loads(db.execute("SELECT config FROM attempts WHERE token=?", (job["owner"],)).fetchone()[0])
    assert original["controls"]["max_connections"] == 8
    with pytest.raises(RuntimeError):
        store.finish(job["owner"], True, {})


def test_abandoned_lease_respects_alive_owners_and_holds(tmp_path):
    store = Store(tmp_path / "queue.db")
    store.add("a", "train", {"resources": ["gpu:0"]})
    store.claim(ttl=0.001)
    time.sleep(0.01)
    assert store.recover(lambda _: True) == []
    assert store.recover(lambda _: False) == ["a"]
    store.hold("a", True)
    assert store.claim() is None
    store.hold("a", False)
    assert store.claim()["attempt"] == 2
    store.backup(tmp_path / "backup.db")
    assert Store(tmp_path / "backup.db").rows()[0]["state"] == "running"


def test_invalid_training_handoff_is_rejected(tmp_path):
    store = Store(tmp_path / "queue.db")
    store.add("eval", "eval", {})
    with pytest.raises(ValueError, match="terminal"):
        store.add("train", "train", {}, [("eval", "success")])
    store.add("merge", "merge", {}, [("eval", "success")])
    with pytest.raises(ValueError, match="administrative"):
        store.add("train", "train", {}, [("merge", "terminal")])
    with pytest.raises(ValueError, match="safe filename"):
        store.add("../x", "train", {})
    assert len(store.rows()) == 2


def test_backend_oom_retries_with_lower_concurrency(tmp_path, monkeypatch):
    from mimir_b200.evaluation.runner import BackendOOM
    from mimir_b200.scheduling import worker
    store = Store(tmp_path / "queue.db")
    store.add("eval", "eval", {"controls": {"max_connections": 8}})

    def oom(*_a, **_k):
        raise BackendOOM("CUDA out of memory")
    monkeypatch.setattr(worker, "execute", oom)
    assert worker.run_one(store, tmp_path / "attempts")
    row = store.rows()[0]
    assert row["state"] == "pending" and json.loads(row["config"])["controls"]["max_connections"] == 4


def test_command_timeout_kills_only_owned_tree(tmp_path):
    store = Store(tmp_path / "queue.db")
    store.add("slow", "inference", {"command": [sys.executable, "-c", "import time; time.sleep(60)"], "timeout": 1},
              max_attempts=1)
    assert run_one(store, tmp_path / "attempts")
    row = store.rows()[0]
    assert row["state"] == "failed" and "timed out" in json.loads(row["result"])["error"]


# ------------------------------------------------------------------ idle coordinator
def test_external_process_blocks_even_when_idle(monkeypatch):
    monkeypatch.setattr(idle, "query", lambda f, s: [["0", "uuid", "7500", "0"]] if s == "gpu" else [["uuid", "123"]])
    assert not idle.available(["0"])[0]
    assert idle.available(["0"], {123})[0]
    assert not idle.available(["1"])[0]


def test_idle_memory_and_utilization_guard(monkeypatch):
    row = ["0", "uuid", "0", "0"]
    monkeypatch.setattr(idle, "query", lambda f, s: [row] if s == "gpu" else [])
    assert idle.available(["0"])[0]
    row[2] = "2000"
    assert not idle.available(["0"])[0]
    row[2], row[3] = "0", "90"
    assert not idle.available(["0"])[0]


def test_gpu_workers_claim_only_their_tasks(tmp_path):
    store = Store(tmp_path / "queue.sqlite")
    for g in range(8):
        store.add(f"eval{g}", "eval", {"server": {"gpus": str(g)}, "resources": [f"gpu:{g}"]})
    store.add("train", "train", {})

    def claim(g):
        return store.claim(predicate=lambda j: j["kind"] == "eval" and j["config"]["server"]["gpus"] == str(g))
    with ThreadPoolExecutor(8) as pool:
        jobs = list(pool.map(claim, range(8)))
    assert {j["id"] for j in jobs} == {f"eval{g}" for g in range(8)}
    assert next(r for r in store.rows() if r["id"] == "train")["attempt"] == 0


def test_monitor_reports_wait_reason(tmp_path):
    from mimir_b200.scheduling.monitor import render
    store = Store(tmp_path / "queue.sqlite")
    (tmp_path / "idle-status.json").write_text(json.dumps({"state": "waiting_for_gpus", "time": time.time(),
                                                           "reason": "external PIDs"}))
    assert "waiting_for_gpus" in render(store).caption


def test_backups_replace_only_after_success(tmp_path, monkeypatch):
    store = Store(tmp_path / "queue.sqlite")
    store.add("first", "train", {}, held=True)
    assert idle.refresh_backup(store)
    store.add("second", "train", {}, held=True)
    assert idle.refresh_backup(store)
    backup = tmp_path / "queue.backup.sqlite"
    assert len(Store(backup).rows()) == 2
    before = backup.read_bytes()

    def fail(path):
        path.write_text("partial")
        raise OSError("full disk")
    monkeypatch.setattr(store, "backup", fail)
    with pytest.warns(RuntimeWarning, match="previous snapshot retained"):
        assert not idle.refresh_backup(store)
    assert backup.read_bytes() == before and not list(tmp_path.glob("*.partial"))


def test_idle_run_drains_queue_when_gpus_free(tmp_path):
    store = Store(tmp_path / "queue.sqlite")
    marker = tmp_path / "ran"
    store.add("job", "train", {"command": [sys.executable, "-c", f"open({str(marker)!r},'w').write('x')"]})
    idle.run(tmp_path / "queue.sqlite", ["0"], poll=0.01, quiet_polls=1, probe=lambda g, o: (True, "free"))
    assert marker.exists()
    assert json.loads((tmp_path / "idle-status.json").read_text())["state"] == "complete"


# ------------------------------------------------------------------ metrics / clients
def test_weighted_sample_merge_and_duplicates(tmp_path):
    a, b = tmp_path / "a", tmp_path / "b"
    a.write_text(json.dumps({"task": "t", "sample_id": 0, "pass": 1, "scores": {"acc": 0}}) + "\n")
    b.write_text("".join(json.dumps({"task": "t", "sample_id": i, "pass": 1, "scores": {"acc": 1}}) + "\n"
                         for i in range(1, 4)))
    assert merge_samples([a, b])["metrics"]["t/acc"] == 0.75
    with pytest.raises(ValueError, match="Duplicate"):
        merge_samples([a, a])


def test_partial_task_set_is_not_published(tmp_path):
    path = tmp_path / "samples"
    path.write_text(json.dumps({"task": "a", "sample_id": 1, "pass": 1, "scores": {"acc": 1}}) + "\n")
    with pytest.raises(ValueError, match="Incomplete"):
        complete_task_set([path], {"a": {"samples": 2, "passes": 1}})
    assert complete_task_set([path], {"a": {"samples": 1, "passes": 1}})["metrics"]["a/acc"] == 1


def test_nonlinear_metrics_and_pass_statistics():
    s = classification_metrics([(0, 0), (0, 1), (1, 1), (1, 1)])
    assert s["accuracy"] == 0.75 and abs(s["macro_f1"] - (2 / 3 + 4 / 5) / 2) < 1e-8
    assert pass_at_k(1, 4, 2) == 0.5


def test_classification_is_aggregated_per_pass(tmp_path):
    path = tmp_path / "scores"
    rows = []
    for epoch, pairs in enumerate([[(0, 0), (1, 0)], [(0, 1), (1, 1)]], 1):
        for i, (t, p) in enumerate(pairs):
            rows.append({"task": "classes", "sample_id": i, "pass": epoch, "target_class": t, "predicted_class": p,
                         "scores": {}})
    path.write_text("".join(json.dumps(r) + "\n" for r in rows))
    rec = complete_task_set([path], {"classes": {"samples": 2, "passes": 2}}, classification_tasks=["classes"])
    assert abs(rec["metrics"]["classes/macro_f1"] - 1 / 3) < 1e-8 and len(rec["pass_metrics"]["classes"]) == 2


def test_direct_runner_records_generations_and_passes(tmp_path):
    from mimir_b200.evaluation.clients import evaluate
    suite = tmp_path / "suite.json"
    suite.write_text(json.dumps({"schema": 1, "tasks": [{"id": "smoke", "backend": "direct", "provider": "mockllm",
                                                         "task": "mimir_b200.evaluation.tasks:smoke", "samples": 1,
                                                         "passes": 2}]}))
    receipt = evaluate(suite, "model", tmp_path / "results")
    rows = [json.loads(s) for s in (tmp_path / "results/smoke.samples.jsonl").read_text().splitlines()]
    assert len(rows) == 2 and {r["pass"] for r in rows} == {1, 2}
    assert all(r["scores"]["exact"] == 1 for r in rows)
    assert all(r["raw"]["output"]["completion"] == "Default output from mockllm/model" for r in rows)
    assert len(receipt["suite_sha256"]) == 64
    with pytest.raises(FileExistsError):
        evaluate(suite, "model", tmp_path / "results")


def test_blocked_protocol_refuses(tmp_path):
    from mimir_b200.evaluation.clients import evaluate
    suite = tmp_path / "s.json"
    suite.write_text(json.dumps({"schema": 1, "tasks": [{"id": "x", "backend": "direct", "blocked": "no data"}]}))
    with pytest.raises(ValueError, match="not qualified"):
        evaluate(suite, "m", tmp_path / "o")


def test_mcq_task_with_local_dataset(tmp_path):
    from mimir_b200.evaluation.tasks import build
    data = tmp_path / "piqa.json"
    data.write_text(json.dumps([{"prompt": "p", "solution0": "x", "solution1": "y", "label": 1}]))
    spec = build("piqa", dataset_path=str(data))
    assert spec.score("B", spec.samples[0])["scores"]["accuracy"] == 1.0
    assert spec.score("zzz", spec.samples[0])["scores"]["accuracy"] == 0.0


def test_chrf_properties():
    from mimir_b200.evaluation.scorers.chrf import compute_chrf3pp
    assert compute_chrf3pp("the cat sat", ["the cat sat"]) == pytest.approx(1.0)
    assert compute_chrf3pp("", ["x"]) == 0.0
    assert compute_chrf3pp("abc", []) == 0.0
    close = compute_chrf3pp("the cat sat on the mat", ["the cat sat on a mat"])
    far = compute_chrf3pp("dogs run fast", ["the cat sat on a mat"])
    assert 0 < far < close < 1


# ------------------------------------------------------------------ serving
def test_server_compatibility_includes_template_contents(tmp_path):
    (tmp_path / "export_receipt.json").write_text("{}")
    (tmp_path / "config.json").write_text(json.dumps({"model_type": "mimir2", "mos_sparse": True}))
    template = tmp_path / "chat.jinja"
    template.write_text("first")
    spec = ServerSpec(str(tmp_path), "0", template=str(template), backend="vllm")
    before = spec.key()
    template.write_text("second")
    assert spec.key() != before
    with pytest.raises(ValueError, match="eager"):
        command(spec)
    assert "--enforce-eager" in command(ServerSpec(str(tmp_path), "0", eager=True, backend="vllm"))
    with pytest.raises(ValueError, match="GPU indices"):
        command(ServerSpec(str(tmp_path), "a", eager=True, backend="vllm"))


def test_server_pool_reuses_and_owns_processes(tmp_path):
    from mimir_b200.serving.server import ServerPool
    import socket
    (tmp_path / "m").mkdir()
    (tmp_path / "m/export_receipt.json").write_text("{}")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    server = ("import http.server,socketserver\n"
              "class H(http.server.BaseHTTPRequestHandler):\n"
              "  def do_GET(self): self.send_response(200); self.end_headers()\n"
              "  def log_message(self,*a): pass\n"
              f"socketserver.TCPServer(('127.0.0.1',{port}),H).serve_forever()\n")
    pool = ServerPool(tmp_path / "servers")
    spec = ServerSpec(str(tmp_path / "m"), "0", port=port)
    try:
        url = pool.acquire(spec, timeout=30, launch=lambda _s: [sys.executable, "-c", server])
        assert url.endswith(f":{port}/v1")
        proc = next(iter(pool.entries.values()))[0]
        assert pool.acquire(spec, timeout=30, launch=lambda _s: ["false"]) == url
        assert next(iter(pool.entries.values()))[0] is proc
    finally:
        pool.close()
    assert proc.poll() is not None and not pool.entries


# ------------------------------------------------------------------ CLI
def test_cli_doctor_and_schedule(tmp_path, capsys):
    from mimir_b200.cli import main
    main(["doctor"])
    assert "torch" in json.loads(capsys.readouterr().out)
    plan = tmp_path / "plan.json"
    plan.write_text(json.dumps({"jobs": [{"id": "a", "kind": "train", "config": {"command": ["true"]}, "held": True},
                                         {"id": "b", "kind": "merge", "config": {}, "depends": [{"id": "a"}]}]}))
    main(["schedule", str(tmp_path / "q.db"), "--plan", str(plan)])
    rows = json.loads(capsys.readouterr().out)
    assert [r["id"] for r in rows] == ["a", "b"] and rows[0]["held"] == 1
    with pytest.raises(SystemExit):
        main(["export", "x"])


def test_doctor_lists_gpus_through_nvml(monkeypatch):
    """``mimir doctor`` reads GPUs through NVML only (a fake here): name, memory, capability."""
    import types

    from mimir_b200.cli import _nvml_gpus

    class Mem:
        total = 183359 << 20

    fake = types.SimpleNamespace(
        nvmlInit=lambda: None, nvmlShutdown=lambda: None, nvmlDeviceGetCount=lambda: 2,
        nvmlDeviceGetHandleByIndex=lambda i: i, nvmlDeviceGetName=lambda h: b"NVIDIA B200",
        nvmlDeviceGetCudaComputeCapability=lambda h: (10, 0) if h == 0 else (9, 0),
        nvmlDeviceGetMemoryInfo=lambda h: Mem())
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    gpus = _nvml_gpus()
    assert gpus[0] == {"index": 0, "name": "NVIDIA B200", "memory_mib": 183359, "compute_capability": "10.0",
                       "kernels_supported": True}
    assert gpus[1]["kernels_supported"] is False
