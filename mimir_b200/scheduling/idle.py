"""Serial scheduler that runs queued work only while the chosen GPUs are idle.

Behavioural reference: ``src/mimir/scheduling/idle.py:22-140``.  It never signals other users'
processes and only reads GPU state (``nvidia-smi --query-*``).  A GPU is free when no foreign
compute process uses it, or, when no compute process is listed at all, when it holds at most
1 GiB and is at most 5 % busy; work starts after ``quiet_polls`` consecutive free polls.
Training-type jobs run one at a time; pending evaluations then run as one worker process per
GPU (each pinned with ``CUDA_VISIBLE_DEVICES`` and draining only the jobs whose server names
that GPU), and all workers are joined before the next training job.  After every unit of work
a verified copy of the queue replaces ``queue.backup.sqlite``; the monitor reads
``idle-status.json``.
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
from dataclasses import dataclass
from pathlib import Path
from typing import Callable

import psutil

from mimir_b200.evaluation.metrics import write_record
from mimir_b200.scheduling.store import Store
from mimir_b200.scheduling.worker import recover_abandoned, run_one
from mimir_b200.serving.server import ServerPool
from mimir_b200.train.suspension.protocol import exclusive

IDLE_MEMORY_MIB = 1024.0
IDLE_UTILIZATION_PCT = 5.0


def query(fields: str, section: str) -> list[list[str]]:
    """Rows of ``nvidia-smi --query-<section>=<fields>`` (CSV, no header, no units)."""
    text = subprocess.check_output(["nvidia-smi", f"--query-{section}={fields}", "--format=csv,noheader,nounits"],
                                   text=True, timeout=10)
    return list(csv.reader(io.StringIO(text), skipinitialspace=True))


@dataclass
class _Gpu:
    index: str
    uuid: str
    memory_mib: float
    utilization: float
    pids: list

    def verdict(self, owned) -> str | None:
        """None when free for us, else why not."""
        strangers = [pid for pid in self.pids if pid not in owned]
        if strangers:
            return f"GPU {self.index}: external PIDs {strangers}"
        if not self.pids and (self.memory_mib > IDLE_MEMORY_MIB or self.utilization > IDLE_UTILIZATION_PCT):
            return f"GPU {self.index}: memory/utilization not idle"
        return None


def _read_gpus() -> dict[str, _Gpu]:
    gpus = {row[0]: _Gpu(row[0], row[1], float(row[2]), float(row[3]), [])
            for row in query("index,uuid,memory.used,utilization.gpu", "gpu")}
    by_uuid = {g.uuid: g for g in gpus.values()}
    for gpu_uuid, pid in query("gpu_uuid,pid", "compute-apps"):
        if gpu_uuid in by_uuid:
            by_uuid[gpu_uuid].pids.append(int(pid))
    return gpus


def available(gpus, owned=()) -> tuple[bool, str]:
    """(free, reason) for the GPU indices ``gpus``; processes in ``owned`` are our own."""
    state = _read_gpus()
    if not all(g in state for g in gpus):
        return False, "Requested GPU missing"
    problems = [v for v in (state[g].verdict(set(owned)) for g in gpus) if v is not None]
    return (False, "; ".join(problems)) if problems else (True, "No external GPU users detected")


def refresh_backup(store: Store) -> bool:
    """Replace ``queue.backup.sqlite`` with a fresh verified copy; a failure keeps the old copy
    (and is only warned about: a backup problem must not stop the queue)."""
    final = store.path.parent / "queue.backup.sqlite"
    partial = final.with_name(f".{final.name}.{uuid.uuid4().hex}.partial")
    ok = False
    try:
        store.backup(partial)
        partial.replace(final)
        ok = True
    except Exception as exc:  # noqa: BLE001
        warnings.warn(f"Queue backup failed; previous snapshot retained: {exc}", RuntimeWarning)
    finally:
        partial.unlink(missing_ok=True)
    return ok


def _own_pids() -> set:
    return {child.pid for child in psutil.Process().children(recursive=True)}


class IdleCoordinator:
    def __init__(self, database, gpus, poll: float, quiet_polls: int, probe: Callable):
        self.database = Path(database)
        self.root = self.database.parent
        self.store = Store(self.database)
        self.gpus, self.poll, self.quiet_polls, self.probe = gpus, poll, quiet_polls, probe
        self.status_file = self.root / "idle-status.json"
        self.quiet = 0

    def _status(self, **fields) -> None:
        write_record(self.status_file, {"pid": os.getpid(), "time": time.time()} | fields)

    def _queue_empty(self) -> bool:
        return all(row["state"] not in ("pending", "running") for row in self.store.rows())

    def _observe(self) -> None:
        try:
            free, reason = self.probe(self.gpus, _own_pids())
        except Exception as exc:  # noqa: BLE001 - an unreadable GPU counts as busy
            free, reason = False, f"GPU probe failed: {exc}"
        self.quiet = self.quiet + 1 if free else 0
        self._status(state="ready" if self.quiet >= self.quiet_polls else "waiting_for_gpus", gpus=self.gpus,
                     reason=reason, quiet_polls=self.quiet)

    def _evaluate_on_every_gpu(self) -> None:
        workers = [subprocess.Popen([sys.executable, "-m", "mimir_b200.scheduling.idle", str(self.database), "--gpus",
                                     gpu, "--eval-worker"], env=os.environ | {"CUDA_VISIBLE_DEVICES": gpu})
                   for gpu in self.gpus]
        codes = [w.wait() for w in workers]
        if any(codes):
            raise RuntimeError("Evaluation worker exited unexpectedly; inspect runner log")

    def serve(self, pool: ServerPool) -> None:
        recover_abandoned(self.store, self.root / "attempts")
        while not self._queue_empty():
            self._observe()
            if self.quiet >= self.quiet_polls:
                ran_training = run_one(self.store, self.root / "attempts", pool, predicate=lambda j: j["kind"] != "eval")
                if not ran_training:
                    self._evaluate_on_every_gpu()
                refresh_backup(self.store)
                self.quiet = 0
                if ran_training:
                    continue
            time.sleep(self.poll)
        self._status(state="complete")


def run(database, gpus, poll: float = 30, quiet_polls: int = 3, probe=available) -> None:
    coordinator = IdleCoordinator(database, gpus, poll, quiet_polls, probe)
    with exclusive(coordinator.database.with_suffix(".runner.lock")):
        pool = ServerPool(coordinator.root / "servers")
        try:
            coordinator.serve(pool)
        finally:
            pool.close()


def evaluate_assigned(database, gpu: str, probe=available) -> None:
    """Evaluation worker for one GPU: drain the eval jobs whose server is pinned to ``gpu``."""
    database = Path(database)
    store = Store(database)
    pool = ServerPool(database.parent / "servers" / f"gpu-{gpu}")

    def mine(job) -> bool:
        return job["kind"] == "eval" and job["config"].get("server", {}).get("gpus") == gpu

    try:
        while True:
            try:
                free = probe([gpu], _own_pids())[0]
            except Exception:  # noqa: BLE001
                free = False
            if not free:
                time.sleep(30)
            elif not run_one(store, database.parent / "attempts", pool, predicate=mine):
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
    if not gpus or not all(g.isdigit() for g in gpus) or len(set(gpus)) != len(gpus):
        parser.error("Provide distinct numeric GPU indices")
    if args.poll <= 0:
        parser.error("poll must be positive")
    if not args.eval_worker:
        run(args.database, gpus, args.poll)
    elif len(gpus) == 1:
        evaluate_assigned(args.database, gpus[0])
    else:
        parser.error("Evaluation worker requires exactly one GPU")


if __name__ == "__main__":
    main()
