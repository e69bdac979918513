"""Single-node CUDA-suspension controller built on the ``cuda-checkpoint`` utility.

Reference behaviour: ``src/mimir/training/suspension/controller.py:23-297``.  The controller
acts only on the processes a job published in its readiness files (never discovers or
signals other processes) and journals every transition to
``generation_<n>/operations.jsonl`` (intent, then verified or error with the tool's output).

* ``offload``: all ranks must be ready and running; a host-RAM gate (owned GPU MiB x 1.1 +
  1 GiB must fit in ``MemAvailable``) runs first; then every rank is locked, then every rank is
  checkpointed (two passes), and the owned GPU memory must be gone before ``offloaded.json``.
* ``restore``: refuses while a user ``hold`` exists (``RestoreDeferred``), while a new GPU
  occupant appeared on the job's GPUs, or without 512 MiB headroom beyond what still has to
  come back.  Restores checkpointed ranks, unlocks locked ones, and only when every rank runs
  again writes ``restored.json`` and the per-process ``resume.<pid>`` tokens.  Re-running it
  is idempotent; a partially failed restore releases no rank.
* ``cancel_unoffloaded`` releases a readiness handshake that never reached a GPU operation.

``RestoreDeferred`` is a safety gate, not a failure: the CLI exits 75 so supervisors retry
later instead of falling back to disk.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import subprocess
import sys
import tempfile
import time
from collections import defaultdict
from pathlib import Path

from mimir_b200.train.suspension.protocol import (atomic_write, exclusive, matches, process_identity, read_json,
                                                  submit, validate_process)

RESIDUAL_MIB = 64          # per-process GPU memory still counted as "released"
RESTORE_MARGIN_MIB = 512


def _output(argv, timeout=30) -> str:
    return subprocess.run(argv, check=True, text=True, capture_output=True, timeout=timeout).stdout.strip()


def _csv(query: str, fields: str) -> list[list[str]]:
    """Rows of an ``nvidia-smi --query-<query>=<fields>`` listing, values stripped."""
    text = _output(["nvidia-smi", f"--query-{query}={fields}", "--format=csv,noheader,nounits"])
    return [[value.strip() for value in line.split(",")] for line in text.splitlines() if line.strip()]


class CudaBackend:
    """The two external tools the controller drives: ``cuda-checkpoint`` (per-process CUDA state and
    lock / checkpoint / restore / unlock actions) and read-only ``nvidia-smi`` queries."""

    STATES = frozenset({"running", "locked", "checkpointed"})
    LOCK_TIMEOUT_MS = 60000

    def __init__(self, executable: str = "cuda-checkpoint", action_timeout: int = 300):
        self.executable, self.action_timeout = executable, action_timeout

    def state(self, pid: int) -> str:
        reported = _output([self.executable, "--get-state", "--pid", str(pid)]).lower().strip()
        if reported not in self.STATES:
            raise RuntimeError(f"Unsupported CUDA state for {pid}: {reported!r}")
        return reported

    def action(self, pid: int, action: str) -> None:
        argv = [self.executable, "--action", action, "--pid", str(pid)]
        if action == "lock":
            argv += ["--timeout", str(self.LOCK_TIMEOUT_MS)]
        _output(argv, timeout=self.action_timeout)

    def memory(self) -> dict[tuple[int, str], int]:
        """MiB used per (pid, GPU uuid)."""
        return {(int(pid), gpu): int(used) for pid, gpu, used in _csv("compute-apps", "pid,gpu_uuid,used_gpu_memory")}

    def free(self) -> dict[str, int]:
        """Free MiB per GPU uuid."""
        return {gpu: int(free) for gpu, free in _csv("gpu", "uuid,memory.free")}


class RestoreDeferred(RuntimeError):
    """Restoration is unsafe right now (hold, occupant, headroom); retry later, never fall back."""


def _host_available_bytes() -> int:
    for line in Path("/proc/meminfo").read_text().splitlines():
        if line.startswith("MemAvailable:"):
            return int(line.split()[1]) * 1024
    raise RuntimeError("MemAvailable missing from /proc/meminfo")


def _decoded(error, name):
    value = getattr(error, name, None)
    return value.decode(errors="replace") if isinstance(value, bytes) else value


class Journal:
    """Append-only ``operations.jsonl`` of one generation; every entry is fsynced before the
    operation it announces runs."""

    def __init__(self, directory: Path):
        self.path = Path(directory) / "operations.jsonl"

    def add(self, entry: dict) -> None:
        with open(self.path, "a") as handle:
            handle.write(json.dumps(entry | {"time": time.time()}) + "\n")
            handle.flush()
            os.fsync(handle.fileno())


def _owned_mib_by_gpu(allocations: dict, owned: set) -> dict:
    per_gpu: dict[str, int] = defaultdict(int)
    for (pid, gpu), mib in allocations.items():
        if pid in owned:
            per_gpu[gpu] += mib
    return dict(per_gpu)


def _live_pids(identities) -> set:
    alive = set()
    for identity in identities:
        try:
            validate_process(identity)
            alive.add(identity["pid"])
        except (OSError, RuntimeError):
            pass
    return alive


class Controller:
    """Acts on one control directory: the job's published ranks only."""

    def __init__(self, root, backend):
        self.root, self.backend = Path(root), backend

    # ------------------------------------------------------------------ readiness
    def ready(self):
        """(readiness handshake, generation directory) after checking that every published rank
        is the same live process and acknowledged this generation."""
        launch = read_json(self.root / "launch.json")
        ready = read_json(self.root / "suspend_ready.json")
        if (launch["job_id"], launch["ranks"]) != (ready["job_id"], ready["ranks"]):
            raise RuntimeError("Readiness does not match launch")
        resumed = self.root / "resumed.json"
        if resumed.exists() and matches(read_json(resumed), ready):
            raise RuntimeError("This suspension already resumed")
        generation = self.root / f"generation_{ready['generation']:06d}"
        for rank in ready["ranks"]:
            validate_process(rank)
            ack = read_json(generation / f"ready.{rank['pid']}.json")
            if not matches(ack, ready) or any(ack.get(k) != v for k, v in rank.items()):
                raise RuntimeError("Rank readiness mismatch")
        return ready, generation

    def journal(self, directory: Path, entry: dict) -> None:
        Journal(directory).add(entry)

    def transition(self, directory: Path, rank: dict, action: str, expected: str) -> None:
        """One ``cuda-checkpoint`` action on one rank, journaled as intent, then verified or error."""
        log = Journal(directory)
        pid = rank["pid"]
        validate_process(rank)
        log.add({"pid": pid, "action": action, "phase": "intent"})
        try:
            self.backend.action(pid, action)
            reached = self.backend.state(pid)
            if reached != expected:
                raise RuntimeError(f"{action} left {pid} in {reached}")
        except Exception as error:
            log.add({"pid": pid, "action": action, "phase": "error", "error": str(error),
                     "stdout": _decoded(error, "stdout"), "stderr": _decoded(error, "stderr")})
            raise
        log.add({"pid": pid, "action": action, "phase": "verified"})

    def _states(self, ranks) -> dict:
        return {r["pid"]: self.backend.state(r["pid"]) for r in ranks}

    # ------------------------------------------------------------------ offload
    def _admit_offload(self, ready, directory):
        """Checks before any GPU operation; returns (owned MiB per GPU, allocations)."""
        if (directory / "cancelled.json").exists() or (directory / "restored.json").exists():
            raise RuntimeError("This generation has already been released")
        if (directory / "offload.json").exists():
            raise RuntimeError("Offload already attempted; inspect status and use recover")
        if set(self._states(ready["ranks"]).values()) != {"running"}:
            raise RuntimeError("All ranks must be running before initial offload")
        allocations = self.backend.memory()
        needed = _owned_mib_by_gpu(allocations, {r["pid"] for r in ready["ranks"]})
        if not needed:
            raise RuntimeError("No owned GPU allocations detected")
        if _host_available_bytes() < (sum(needed.values()) * 1.1 + 1024) * 1024 ** 2:
            raise RuntimeError("Insufficient host RAM for offload plus safety margin")
        return needed, allocations

    def offload(self, lease_seconds: float = 600) -> None:
        with exclusive(self.root / "controller.lock"):
            ready, directory = self.ready()
            needed, allocations = self._admit_offload(ready, directory)
            owned = {r["pid"] for r in ready["ranks"]}
            others = sorted({pid for pid, gpu in allocations if pid not in owned and gpu in needed})
            atomic_write(directory / "offload.json", ready | {
                "needed_mib": needed, "lease_until": time.time() + lease_seconds,
                "allocations": [{"pid": pid, "gpu": gpu, "mib": mib} for (pid, gpu), mib in allocations.items()
                                if pid in owned],
                "existing_peers": [process_identity(pid) for pid in others]})
            for action, reached in (("lock", "locked"), ("checkpoint", "checkpointed")):
                for rank in ready["ranks"]:  # every rank locked before any is checkpointed
                    self.transition(directory, rank, action, reached)
            leftover = {key: mib for key, mib in self.backend.memory().items() if key[0] in owned}
            if max(leftover.values(), default=0) > RESIDUAL_MIB:
                raise RuntimeError("Owned GPU memory not released; do not admit evaluations")
            atomic_write(directory / "offloaded.json", ready | {"remaining_owned_mib": sum(leftover.values())})

    # ------------------------------------------------------------------ restore
    def _held(self) -> bool:
        if (self.root / "hold").exists():
            return True
        managed = self.root / "managed.json"
        return managed.exists() and (Path(read_json(managed)["supervisor_root"]) / "hold").exists()

    def _check_restore_room(self, ready: dict, receipt: dict, states: dict) -> None:
        """No new occupant on the job's GPUs, and headroom for what still has to come back."""
        pending: dict[str, int] = defaultdict(int)
        for entry in receipt.get("allocations", []):
            if states[entry["pid"]] == "checkpointed":  # after a partial restore only these need room
                pending[entry["gpu"]] += entry["mib"]
        if not pending:
            pending.update(receipt["needed_mib"])
        tolerated = {r["pid"] for r in ready["ranks"]} | _live_pids(receipt.get("existing_peers", []))
        if any(pid not in tolerated and gpu in receipt["needed_mib"] for pid, gpu in self.backend.memory()):
            raise RestoreDeferred("New GPU workload is still present; defer restore")
        free = self.backend.free()
        if any(free.get(gpu, 0) < mib + RESTORE_MARGIN_MIB for gpu, mib in pending.items()):
            raise RestoreDeferred("Not enough GPU headroom to restore safely")

    def _bring_back(self, directory: Path, rank: dict) -> None:
        """checkpointed -> locked -> running, from wherever a previous attempt stopped."""
        state = self.backend.state(rank["pid"])
        if state == "checkpointed":
            self.transition(directory, rank, "restore", "locked")
            state = "locked"
        if state == "locked":
            self.transition(directory, rank, "unlock", "running")

    def restore(self) -> None:
        with exclusive(self.root / "controller.lock"):
            ready, directory = self.ready()
            if self._held():
                raise RestoreDeferred("Explicit user hold exists; remove it before restoration")
            receipt = read_json(directory / "offload.json")
            if not matches(receipt, ready):
                raise RuntimeError("Offload receipt mismatch")
            states = self._states(ready["ranks"])
            if "checkpointed" in states.values():
                self._check_restore_room(ready, receipt, states)
            for rank in ready["ranks"]:
                self._bring_back(directory, rank)
            if set(self._states(ready["ranks"]).values()) != {"running"}:
                raise RuntimeError("Not all ranks restored")  # release nobody after a partial restore
            atomic_write(directory / "restored.json", ready)
            self.release(directory, ready)

    def release(self, directory: Path, ready: dict) -> None:
        """Write each rank's resume token (unless that rank already consumed it)."""
        answer = {key: ready[key] for key in ("job_id", "generation", "step")}
        for rank in ready["ranks"]:
            token = directory / f"resume.{rank['pid']}"
            if not token.with_suffix(token.suffix + ".consumed").exists():
                atomic_write(token, answer | {"start_ticks": rank["start_ticks"]})

    def cancel_unoffloaded(self) -> None:
        """Release a handshake that never reached a GPU operation."""
        with exclusive(self.root / "controller.lock"):
            ready, directory = self.ready()
            if (self.root / "hold").exists() or (directory / "offload.json").exists():
                raise RuntimeError("Cannot cancel: user hold or offload already attempted")
            if set(self._states(ready["ranks"]).values()) != {"running"}:
                raise RuntimeError("Cannot cancel: CUDA state is not running")
            atomic_write(directory / "cancelled.json", ready)
            self.release(directory, ready)

    def status(self) -> dict:
        out = {"launch": read_json(self.root / "launch.json")}
        for name in ("queue", "suspend_ready", "resumed"):
            path = self.root / f"{name}.json"
            if path.exists():
                out[name] = read_json(path)
        return out


def wait_offloaded(proc, backend, controller: Controller, seconds: float, deadline: float, resume_request=None):
    """Hold an offloaded pause for ``seconds``, re-checking liveness, CUDA states and released memory
    (each check journaled as ``pause_health``)."""
    ready, generation = controller.ready()
    pids = {r["pid"] for r in ready["ranks"]}
    log = Journal(generation)
    end = time.monotonic() + seconds
    while True:
        if proc.poll() is not None:
            raise RuntimeError("Worker launcher exited during offloaded pause")
        if resume_request is not None and Path(resume_request).exists():
            log.add({"phase": "early_resume_requested", "request": str(resume_request)})
            return
        controller.ready()
        states = {pid: backend.state(pid) for pid in pids}
        owned = sum(mib for (pid, _), mib in backend.memory().items() if pid in pids)
        if set(states.values()) != {"checkpointed"} or owned > RESIDUAL_MIB * len(pids):
            raise RuntimeError(f"Offloaded state changed: {states}, {owned} MiB")
        left = max(0.0, end - time.monotonic())
        log.add({"phase": "pause_health", "states": states, "owned_gpu_mib": owned, "remaining_seconds": left})
        if left == 0:
            return
        if time.monotonic() >= deadline:
            raise TimeoutError("Deadline exceeded during offloaded pause")
        time.sleep(min(30, left, max(0, deadline - time.monotonic())))


def bootstrap(root: Path, command) -> None:
    """Copy the job handle ``cuda-checkpoint --launch-job`` created, then exec the training command."""
    source = os.environ.get("CUDA_CHECKPOINT_JOB_FILE")
    if not source:
        raise RuntimeError("bootstrap must be invoked through cuda-checkpoint --launch-job")
    handle = Path(tempfile.mkdtemp(prefix="cuda-job-", dir=root)) / "job.bin"
    shutil.copyfile(source, handle)
    handle.chmod(0o600)
    os.environ["CUDA_CHECKPOINT_JOB_FILE"] = str(handle)
    os.execvp(command[0], command)


def _watch(controller: Controller, interval: float, ready_timeout: float) -> None:
    """Recovery watcher for unsupervised jobs: cancel a handshake nobody offloaded in time, restore
    an offload whose lease ran out."""
    while True:
        try:
            ready, directory = controller.ready()
            receipt = directory / "offload.json"
            if not receipt.exists():
                if time.time() >= ready["ready_at"] + ready_timeout:
                    controller.cancel_unoffloaded()
            elif time.time() >= read_json(receipt)["lease_until"]:
                controller.restore()
                print("Restoration released; awaiting resumed acknowledgement", flush=True)
        except (OSError, RuntimeError, subprocess.SubprocessError) as error:
            print(f"[suspend-watch] {error}", flush=True)
        time.sleep(interval)


def _parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(description="CUDA suspension controller")
    parser.add_argument("--cuda-checkpoint", default="cuda-checkpoint")
    sub = parser.add_subparsers(dest="action", required=True)
    for action in ("status", "request", "offload", "restore", "recover", "watch"):
        p = sub.add_parser(action)
        p.add_argument("control_dir", type=Path)
        if action == "request":
            p.add_argument("steps", nargs="+", type=int)
        elif action == "offload":
            p.add_argument("--lease-seconds", type=int, default=600)
        elif action == "watch":
            p.add_argument("--interval", type=float, default=5)
            p.add_argument("--ready-timeout", type=float, default=600)
    for action in ("launch", "_bootstrap"):
        p = sub.add_parser(action)
        p.add_argument("--control-root", required=True, type=Path)
        p.add_argument("command", nargs=argparse.REMAINDER)
    return parser


def _launch(parser, args) -> None:
    command = args.command[1:] if args.command[:1] == ["--"] else args.command
    if not command:
        parser.error("Missing training command")
    args.control_root.mkdir(parents=True, exist_ok=True)
    if args.action == "_bootstrap":
        bootstrap(args.control_root.resolve(), command)
    os.execv(args.cuda_checkpoint, [args.cuda_checkpoint, "--launch-job", sys.executable, "-m",
                                    "mimir_b200.train.suspension.controller", "_bootstrap", "--control-root",
                                    str(args.control_root.resolve()), "--", *command])


def main(argv=None) -> None:
    parser = _parser()
    args = parser.parse_args(argv)
    if args.action in ("launch", "_bootstrap"):
        _launch(parser, args)
        return
    controller = Controller(args.control_dir, CudaBackend(args.cuda_checkpoint))
    if args.action == "request":
        print(submit(args.control_dir, args.steps))
    elif args.action == "status":
        print(json.dumps(controller.status(), indent=2))
    elif args.action == "offload":
        if args.lease_seconds <= 0:
            parser.error("lease-seconds must be positive")
        controller.offload(args.lease_seconds)
    elif args.action in ("restore", "recover"):
        try:
            controller.restore()
        except RestoreDeferred as error:
            print(str(error), file=sys.stderr)
            sys.exit(75)
    else:
        if (controller.root / "managed.json").exists():
            parser.error("This job has a supervisor; do not run a second recovery watcher")
        if args.interval <= 0:
            parser.error("interval must be positive")
        _watch(controller, args.interval, args.ready_timeout)


if __name__ == "__main__":
    main()
