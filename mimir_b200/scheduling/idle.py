"""Serial scheduler that runs queued work only while the selected GPUs are idle.

Reference behaviour: ``src/mimir/scheduling/idle.py:22-140``.  It never signals other users'
processes: a GPU counts as free when no foreign compute process uses it (or, with no
processes, when memory <= 1 GiB and utilisation <= 5 %) for ``quiet_polls`` consecutive
polls.  Non-evaluation jobs run one at a time; pending evaluations then run as one worker
process per GPU (each pinned with ``CUDA_VISIBLE_DEVICES`` and draining only jobs whose
server names that GPU), all joined before the next training job.  After each unit of work a
verified backup of the queue replaces ``queue.backup.sqlite``.  Status for the monitor goes
to ``idle-status.json``.  GPU state is only read (``nvidia-smi --query``).
"""
from __future__ import annotations

import argparse
import csv
import io
import os
import subprocess
import sys
import time
import uuid
import warnings
from pathlib import Path

import psutil

from mimir_b200.evaluation.metrics import write_record
from mimir_b200.scheduling.store import Store
from mimir_b200.scheduling.worker import recover_abandoned, run_one
from mimir_b200.serving.server import ServerPool
from mimir_b200.train.suspension.protocol import exclusive


def query(fields: str, section: str) -> list[list[str]]:
    out = subprocess.check_output(["nvidia-smi", f"--query-{section}={fields}", "--format=csv,noheader,nounits"],
                                  text=True, timeout=10)
    return list(csv.reader(io.StringIO(out), skipinitialspace=True))


def available(gpus, owned=()) -> tuple[bool, str]:
    devices = {row[0]: row for row in query("index,uuid,memory.used,utilization.gpu", "gpu")}
    if any(g not in devices for g in gpus):
        return False, "Requested GPU missing"
    apps = query("gpu_uuid,pid", "compute-apps")
    reasons = []
    for gpu in gpus:
        _, uid, memory, util = devices[gpu]
        pids = [int(pid) for dev, pid in apps if dev == uid]
        foreign = [p for p in pids if p not in owned]
        if foreign:
            reasons.append(f"GPU {gpu}: external PIDs {foreign}")
        elif not pids and (float(memory) > 1024 or float(util) > 5):
            reasons.append(f"GPU {gpu}: memory/utilization not idle")
    return not reasons, "; ".join(reasons) or "No external GPU users detected"


def refresh_backup(store: Store) -> bool:
    target = store.path.parent / "queue.backup.sqlite"
    staged = target.with_name(f".{target.name}.{uuid.uuid4().hex}.partial")
    try:
        store.backup(staged)
        staged.replace(target)
        return True
    except Exception as exc:  # noqa: BLE001 - a failed backup must not stop the queue
        warnings.warn(f"Queue backup failed; previous snapshot retained: {exc}", RuntimeWarning)
        return False
    finally:
        staged.unlink(missing_ok=True)


def run(database, gpus, poll: float = 30, quiet_polls: int = 3, probe=available) -> None:
    database = Path(database)
    store = Store(database)
    status = database.parent / "idle-status.json"
    with exclusive(database.with_suffix(".runner.lock")):
        pool = ServerPool(database.parent / "servers")
        stable = 0
        try:
            recover_abandoned(store, database.parent / "attempts")
            while True:
                if not any(r["state"] in ("pending", "running") for r in store.rows()):
                    write_record(status, {"state": "complete", "pid": os.getpid(), "time": time.time()})
                    return
                owned = {p.pid for p in psutil.Process().children(recursive=True)}
                try:
                    free, reason = probe(gpus, owned)
                except Exception as exc:  # noqa: BLE001 - treated as busy
                    free, reason = False, f"GPU probe failed: {exc}"
                stable = stable + 1 if free else 0
                write_record(status, {"state": "waiting_for_gpus" if stable < quiet_polls else "ready",
                                      "pid": os.getpid(), "gpus": gpus, "reason": reason, "quiet_polls": stable,
                                      "time": time.time()})
                if stable >= quiet_polls:
                    if run_one(store, database.parent / "attempts", pool, predicate=lambda j: j["kind"] != "eval"):
                        refresh_backup(store)
                        stable = 0
                        continue
                    workers = [subprocess.Popen([sys.executable, "-m", "mimir_b200.scheduling.idle", str(database),
                                                 "--gpus", g, "--eval-worker"],
                                                env=os.environ | {"CUDA_VISIBLE_DEVICES": g}) for g in gpus]
                    if any(w.wait() for w in workers):
                        raise RuntimeError("Evaluation worker exited unexpectedly; inspect runner log")
                    refresh_backup(store)
                    stable = 0
                time.sleep(poll)
        finally:
            pool.close()


def evaluate_assigned(database, gpu: str, probe=available) -> None:
    database = Path(database)
    store = Store(database)
    pool = ServerPool(database.parent / "servers" / f"gpu-{gpu}")
    try:
        while True:
            owned = {p.pid for p in psutil.Process().children(recursive=True)}
            try:
                free, _ = probe([gpu], owned)
            except Exception:  # noqa: BLE001
                free = False
            if not free:
                time.sleep(30)
                continue
            if not run_one(store, database.parent / "attempts", pool,
                           predicate=lambda j: j["kind"] == "eval" and j["config"].get("server", {}).get("gpus") == gpu):
                return
    finally:
        pool.close()


def main(argv=None) -> None:
    parser = argparse.ArgumentParser(description="Idle-GPU scheduler")
    parser.add_argument("database", type=Path)
    parser.add_argument("--gpus", required=True)
    parser.add_argument("--poll", type=float, default=30)
    parser.add_argument("--eval-worker", action="store_true", help=argparse.SUPPRESS)
    args = parser.parse_args(argv)
    gpus = args.gpus.split(",")
    if not gpus or any(not g.isdigit() for g in gpus) or len(set(gpus)) != len(gpus):
        parser.error("Provide distinct numeric GPU indices")
    if args.poll <= 0:
        parser.error("poll must be positive")
    if args.eval_worker:
        if len(gpus) != 1:
            parser.error("Evaluation worker requires exactly one GPU")
        evaluate_assigned(args.database, gpus[0])
    else:
        run(args.database, gpus, args.poll)


if __name__ == "__main__":
    main()
