"""Execute claimed jobs with a heartbeat, owned child processes and OOM-aware retries.

Reference behaviour: ``src/mimir/scheduling/worker.py:12-110``.  Kinds: ``checkpoint_wait``
(poll until the contract validates), ``merge``/``average`` (complete task-set aggregation),
``eval`` (suite evaluation, optionally through a pooled server) and command jobs (explicit
argv, run through ``scheduling.child`` in a new session; on timeout only that process tree
is terminated).  A heartbeat thread renews the lease every 20 s.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import psutil

HEARTBEAT_SECONDS = 20
_OOM_MARKERS = ("torch.OutOfMemoryError", "CUDA out of memory")


def owned_alive(receipt) -> bool:
    try:
        data = json.loads(Path(receipt).read_text())
        p = psutil.Process(data["pid"])
        return p.create_time() == data["created"] and p.is_running() and p.status() != psutil.STATUS_ZOMBIE
    except FileNotFoundError:
        return True  # without ownership evidence nothing is reclaimed automatically
    except (psutil.NoSuchProcess, psutil.ZombieProcess):
        return False


def _terminate_tree(pid: int) -> None:
    parent = psutil.Process(pid)
    procs = parent.children(recursive=True) + [parent]
    for p in procs:
        try:
            p.terminate()
        except psutil.NoSuchProcess:
            pass
    _, alive = psutil.wait_procs(procs, timeout=10)
    for p in alive:
        try:
            p.kill()
        except psutil.NoSuchProcess:
            pass


def execute(job: dict, output, server_pool=None) -> dict:
    cfg, kind = job["config"], job["kind"]
    output = Path(output)
    output.mkdir(parents=True, exist_ok=True)
    if kind == "checkpoint_wait":
        from mimir_b200.ckpt.contract import validate
        deadline = time.monotonic() + cfg.get("timeout", 3600)
        while time.monotonic() < deadline:
            try:
                return {"checkpoint": cfg["path"], "manifest": validate(cfg["path"])}
            except (FileNotFoundError, ValueError):
                time.sleep(1)
        raise TimeoutError("Checkpoint did not become complete")
    if kind in ("merge", "average"):
        from mimir_b200.evaluation.metrics import complete_task_set, write_record
        result = complete_task_set(cfg["inputs"], cfg["expected"], classification_tasks=cfg.get("classification_tasks", ()),
                                   pass_k=cfg.get("pass_k"))
        write_record(cfg["output"], result)
        return result
    if kind == "eval":
        from mimir_b200.evaluation.clients import evaluate
        evaluation = dict(cfg["evaluation"])
        if "server" in cfg:
            if server_pool is None:
                raise ValueError("A persistent server pool is required")
            from mimir_b200.serving.server import ServerSpec
            spec = ServerSpec(**cfg["server"])
            if spec.key() not in server_pool.entries:
                server_pool.close()
            evaluation["base_url"] = server_pool.acquire(spec)
        return evaluate(**evaluation, controls=cfg.get("controls", {}))
    command = cfg.get("command")
    if not isinstance(command, list) or not command or not all(isinstance(v, str) for v in command):
        raise ValueError("Execution requires an explicit argv list")
    env = os.environ | cfg.get("env", {})
    with (output / "stdout.log").open("wb") as out, (output / "stderr.log").open("wb") as err:
        child = subprocess.Popen([sys.executable, "-m", "mimir_b200.scheduling.child",
                                  str((output / "process.json").resolve()), str(os.getpid()),
                                  str(psutil.Process().create_time()), *command],
                                 env=env, cwd=cfg.get("cwd"), stdout=out, stderr=err, start_new_session=True)
        try:
            code = child.wait(timeout=cfg.get("timeout"))
        except subprocess.TimeoutExpired:
            _terminate_tree(child.pid)
            child.wait()
            raise TimeoutError("Owned job timed out")
    return {"returncode": code, "stderr": str(output / "stderr.log")}


def run_one(store, output, server_pool=None, predicate=None) -> bool:
    """Claim and run one job; False when nothing is runnable."""
    from mimir_b200.evaluation.metrics import write_record
    from mimir_b200.evaluation.runner import BackendOOM
    job = store.claim(predicate=predicate)
    if not job:
        return False
    if server_pool is not None and job["kind"] == "train":
        server_pool.close()  # training owns the GPUs; no resident inference servers
    directory = Path(output) / job["owner"]
    directory.mkdir(parents=True, exist_ok=True)
    write_record(directory / "owner.json", {"pid": os.getpid(), "created": psutil.Process().create_time()})
    stop, errors = threading.Event(), []

    def renew():
        while not stop.wait(HEARTBEAT_SECONDS):
            try:
                store.heartbeat(job["owner"])
            except Exception as exc:  # noqa: BLE001 - surfaced after the job
                errors.append(exc)
                return

    beat = threading.Thread(target=renew, daemon=True)
    beat.start()
    try:
        result = execute(job, directory, server_pool)
        ok = result.get("returncode", 0) == 0
        stderr = Path(result["stderr"]).read_text(errors="replace")[-65536:] if "stderr" in result else ""
        oom = not ok and any(m in stderr for m in _OOM_MARKERS)
        # only evaluation clients have controls that make an OOM retry meaningful
        store.finish(job["owner"], ok, result, oom=oom and job["kind"] == "eval")
    except Exception as exc:  # noqa: BLE001 - recorded as the attempt's failure
        store.finish(job["owner"], False, {"error": str(exc), "type": type(exc).__name__},
                     transient=isinstance(exc, (ConnectionError, TimeoutError)),
                     oom=isinstance(exc, BackendOOM) and job["kind"] == "eval")
    finally:
        stop.set()
        beat.join()
    if errors:
        raise errors[0]
    return True


def recover_abandoned(store, output) -> list[str]:
    output = Path(output)

    def alive(job) -> bool:
        owner = output / job["owner"] / "owner.json"
        child = output / job["owner"] / "process.json"
        if owner.exists() and owned_alive(owner):
            return True
        if child.exists():
            return owned_alive(child)
        ident = json.loads(job.get("worker_identity") or "{}")
        if not ident:
            return True
        try:
            p = psutil.Process(ident["pid"])
            return p.create_time() == ident["created"] and p.is_running()
        except psutil.NoSuchProcess:
            return False

    return store.recover(alive)
