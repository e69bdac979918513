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


def _run(args, timeout=30) -> str:
    return subprocess.run(args, check=True, text=True, capture_output=True, timeout=timeout).stdout.strip()


class CudaBackend:
    """``cuda-checkpoint`` and ``nvidia-smi`` queries (read-only except the checkpoint actions)."""

    STATES = ("running", "locked", "checkpointed")

    def __init__(self, executable: str = "cuda-checkpoint", action_timeout: int = 300):
        self.executable, self.action_timeout = executable, action_timeout

    def state(self, pid: int) -> str:
        out = _run([self.executable, "--get-state", "--pid", str(pid)]).lower().strip()
        if out not in self.STATES:
            raise RuntimeError(f"Unsupported CUDA state for {pid}: {out!r}")
        return out

    def action(self, pid: int, action: str) -> None:
        args = [self.executable, "--action", action, "--pid", str(pid)]
        if action == "lock":
            args += ["--timeout", "60000"]
        _run(args, timeout=self.action_timeout)

    def memory(self) -> dict[tuple[int, str], int]:
        rows = _run(["nvidia-smi", "--query-compute-apps=pid,gpu_uuid,used_gpu_memory",
                     "--format=csv,noheader,nounits"]).splitlines()
        out = {}
        for row in rows:
            pid, gpu, used = (v.strip() for v in row.split(","))
            out[(int(pid), gpu)] = int(used)
        return out

    def free(self) -> dict[str, int]:
        rows = _run(["nvidia-smi", "--query-gpu=uuid,memory.free", "--format=csv,noheader,nounits"]).splitlines()
        return {gpu.strip(): int(free.strip()) for gpu, free in (r.split(",") for r in rows)}


class RestoreDeferred(RuntimeError):
    """Restoration is unsafe right now (hold, occupant, headroom); retry later, never fall back."""


def _host_available_bytes() -> int:
    for line in Path("/proc/meminfo").read_text().splitlines():
        if line.startswith("MemAvailable:"):
            return int(line.split()[1]) * 1024
    raise RuntimeError("MemAvailable missing from /proc/meminfo")


class Controller:
    def __init__(self, root, backend):
        self.root, self.backend = Path(root), backend

    # ------------------------------------------------------------------ readiness
    def ready(self):
        launch = read_json(self.root / "launch.json")
        ready = read_json(self.root / "suspend_ready.json")
        if launch["job_id"] != ready["job_id"] or launch["ranks"] != ready["ranks"]:
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
        with open(directory / "operations.jsonl", "a") as f:
            f.write(json.dumps(entry | {"time": time.time()}) + "\n")
            f.flush()
            os.fsync(f.fileno())

    def transition(self, directory: Path, rank: dict, action: str, expected: str) -> None:
        validate_process(rank)
        self.journal(directory, {"pid": rank["pid"], "action": action, "phase": "intent"})
        try:
            self.backend.action(rank["pid"], action)
            state = self.backend.state(rank["pid"])
            if state != expected:
                raise RuntimeError(f"{action} left {rank['pid']} in {state}")
        except Exception as error:
            def text(name):
                v = getattr(error, name, None)
                return v.decode(errors="replace") if isinstance(v, bytes) else v
            self.journal(directory, {"pid": rank["pid"], "action": action, "phase": "error", "error": str(error),
                                     "stdout": text("stdout"), "stderr": text("stderr")})
            raise
        self.journal(directory, {"pid": rank["pid"], "action": action, "phase": "verified"})

    # ------------------------------------------------------------------ offload / restore
    def offload(self, lease_seconds: float = 600) -> None:
        with exclusive(self.root / "controller.lock"):
            ready, directory = self.ready()
            if (directory / "cancelled.json").exists() or (directory / "restored.json").exists():
                raise RuntimeError("This generation has already been released")
            if (directory / "offload.json").exists():
                raise RuntimeError("Offload already attempted; inspect status and use recover")
            ranks = ready["ranks"]
            if any(self.backend.state(r["pid"]) != "running" for r in ranks):
                raise RuntimeError("All ranks must be running before initial offload")
            owned = {r["pid"] for r in ranks}
            allocations = self.backend.memory()
            needed: dict[str, int] = defaultdict(int)
            for (pid, gpu), mib in allocations.items():
                if pid in owned:
                    needed[gpu] += mib
            if not needed:
                raise RuntimeError("No owned GPU allocations detected")
            if _host_available_bytes() < (sum(needed.values()) * 1.1 + 1024) * 1024 ** 2:
                raise RuntimeError("Insufficient host RAM for offload plus safety margin")
            peers = sorted({pid for pid, gpu in allocations if pid not in owned and gpu in needed})
            atomic_write(directory / "offload.json", ready | {
                "needed_mib": dict(needed), "lease_until": time.time() + lease_seconds,
                "allocations": [{"pid": pid, "gpu": gpu, "mib": mib} for (pid, gpu), mib in allocations.items()
                                if pid in owned],
                "existing_peers": [process_identity(pid) for pid in peers]})
            for rank in ranks:  # every rank locked before any is checkpointed
                self.transition(directory, rank, "lock", "locked")
            for rank in ranks:
                self.transition(directory, rank, "checkpoint", "checkpointed")
            left = {k: v for k, v in self.backend.memory().items() if k[0] in owned}
            if any(mib > RESIDUAL_MIB for mib in left.values()):
                raise RuntimeError("Owned GPU memory not released; do not admit evaluations")
            atomic_write(directory / "offloaded.json", ready | {"remaining_owned_mib": sum(left.values())})

    def _held(self) -> bool:
        managed = self.root / "managed.json"
        supervisor_hold = managed.exists() and (Path(read_json(managed)["supervisor_root"]) / "hold").exists()
        return (self.root / "hold").exists() or supervisor_hold

    def restore(self) -> None:
        with exclusive(self.root / "controller.lock"):
            ready, directory = self.ready()
            if self._held():
                raise RestoreDeferred("Explicit user hold exists; remove it before restoration")
            receipt = read_json(directory / "offload.json")
            if not matches(receipt, ready):
                raise RuntimeError("Offload receipt mismatch")
            states = {r["pid"]: self.backend.state(r["pid"]) for r in ready["ranks"]}
            if "checkpointed" in states.values():
                self._check_restore_room(ready, receipt, states)
            for rank in ready["ranks"]:
                state = self.backend.state(rank["pid"])
                if state == "checkpointed":
                    self.transition(directory, rank, "restore", "locked")
                    state = "locked"
                if state == "locked":
                    self.transition(directory, rank, "unlock", "running")
            if any(self.backend.state(r["pid"]) != "running" for r in ready["ranks"]):
                raise RuntimeError("Not all ranks restored")
            atomic_write(directory / "restored.json", ready)
            self.release(directory, ready)

    def _check_restore_room(self, ready: dict, receipt: dict, states: dict) -> None:
        needed: dict[str, int] = defaultdict(int)
        for a in receipt.get("allocations", []):
            if states[a["pid"]] == "checkpointed":  # after a partial restore only these need room
                needed[a["gpu"]] += a["mib"]
        if not needed:
            needed.update(receipt["needed_mib"])
        allowed = {r["pid"] for r in ready["ranks"]}
        for peer in receipt.get("existing_peers", []):
            try:
                validate_process(peer)
                allowed.add(peer["pid"])
            except (OSError, RuntimeError):
                pass
        if any(pid not in allowed and gpu in receipt["needed_mib"] for pid, gpu in self.backend.memory()):
            raise RestoreDeferred("New GPU workload is still present; defer restore")
        free = self.backend.free()
        if any(free.get(gpu, 0) < mib + RESTORE_MARGIN_MIB for gpu, mib in needed.items()):
            raise RestoreDeferred("Not enough GPU headroom to restore safely")

    def release(self, directory: Path, ready: dict) -> None:
        for rank in ready["ranks"]:
            token = directory / f"resume.{rank['pid']}"
            if not token.with_suffix(token.suffix + ".consumed").exists():
                atomic_write(token, {k: ready[k] for k in ("job_id", "generation", "step")}
                             | {"start_ticks": rank["start_ticks"]})

    def cancel_unoffloaded(self) -> None:
        with exclusive(self.root / "controller.lock"):
            ready, directory = self.ready()
            if (self.root / "hold").exists() or (directory / "offload.json").exists():
                raise RuntimeError("Cannot cancel: user hold or offload already attempted")
            if any(self.backend.state(r["pid"]) != "running" for r in ready["ranks"]):
                raise RuntimeError("Cannot cancel: CUDA state is not running")
            atomic_write(directory / "cancelled.json", ready)
            self.release(directory, ready)

    def status(self) -> dict:
        out = {"launch": read_json(self.root / "launch.json")}
        for name in ("queue", "suspend_ready", "resumed"):
            if (self.root / f"{name}.json").exists():
                out[name] = read_json(self.root / f"{name}.json")
        return out


def wait_offloaded(proc, backend, controller: Controller, seconds: float, deadline: float, resume_request=None):
    """Hold an offloaded pause for ``seconds``, re-checking liveness, states and released memory."""
    ready, generation = controller.ready()
    pids = {r["pid"] for r in ready["ranks"]}
    end = time.monotonic() + seconds
    while True:
        if proc.poll() is not None:
            raise RuntimeError("Worker launcher exited during offloaded pause")
        if resume_request is not None and Path(resume_request).exists():
            controller.journal(generation, {"phase": "early_resume_requested", "request": str(resume_request)})
            return
        controller.ready()
        states = {pid: backend.state(pid) for pid in pids}
        owned = sum(mib for (pid, _), mib in backend.memory().items() if pid in pids)
        if set(states.values()) != {"checkpointed"} or owned > RESIDUAL_MIB * len(pids):
            raise RuntimeError(f"Offloaded state changed: {states}, {owned} MiB")
        remaining = max(0.0, end - time.monotonic())
        controller.journal(generation, {"phase": "pause_health", "states": states, "owned_gpu_mib": owned,
                                        "remaining_seconds": remaining})
        if not remaining:
            return
        if time.monotonic() >= deadline:
            raise TimeoutError("Deadline exceeded during offloaded pause")
        time.sleep(min(30, remaining, max(0, deadline - time.monotonic())))


def bootstrap(root: Path, command) -> None:
    """Copy the job handle ``cuda-checkpoint --launch-job`` created, then exec the training command."""
    source = os.environ.get("CUDA_CHECKPOINT_JOB_FILE")
    if not source:
        raise RuntimeError("bootstrap must be invoked through cuda-checkpoint --launch-job")
    dest = Path(tempfile.mkdtemp(prefix="cuda-job-", dir=root)) / "job.bin"
    shutil.copyfile(source, dest)
    dest.chmod(0o600)
    os.environ["CUDA_CHECKPOINT_JOB_FILE"] = str(dest)
    os.execvp(command[0], command)


def main(argv=None) -> None:
    parser = argparse.ArgumentParser(description="CUDA suspension controller")
    parser.add_argument("--cuda-checkpoint", default="cuda-checkpoint")
    sub = parser.add_subparsers(dest="action", required=True)
    for action in ("status", "request", "offload", "restore", "recover", "watch"):
        p = sub.add_parser(action)
        p.add_argument("control_dir", type=Path)
        if action == "request":
            p.add_argument("steps", nargs="+", type=int)
        if action == "offload":
            p.add_argument("--lease-seconds", type=int, default=600)
        if action == "watch":
            p.add_argument("--interval", type=float, default=5)
            p.add_argument("--ready-timeout", type=float, default=600)
    for action in ("launch", "_bootstrap"):
        p = sub.add_parser(action)
        p.add_argument("--control-root", required=True, type=Path)
        p.add_argument("command", nargs=argparse.REMAINDER)
    args = parser.parse_args(argv)
    if args.action in ("launch", "_bootstrap"):
        command = args.command[1:] if args.command[:1] == ["--"] else args.command
        if not command:
            parser.error("Missing training command")
        args.control_root.mkdir(parents=True, exist_ok=True)
        if args.action == "_bootstrap":
            bootstrap(args.control_root.resolve(), command)
        os.execv(args.cuda_checkpoint, [args.cuda_checkpoint, "--launch-job", sys.executable, "-m",
                                        "mimir_b200.train.suspension.controller", "_bootstrap", "--control-root",
                                        str(args.control_root.resolve()), "--", *command])
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
        while True:
            try:
                ready, directory = controller.ready()
                receipt = directory / "offload.json"
                if not receipt.exists():
                    if time.time() >= ready["ready_at"] + args.ready_timeout:
                        controller.cancel_unoffloaded()
                elif time.time() >= read_json(receipt)["lease_until"]:
                    controller.restore()
                    print("Restoration released; awaiting resumed acknowledgement", flush=True)
            except (OSError, RuntimeError, subprocess.SubprocessError) as error:
                print(f"[suspend-watch] {error}", flush=True)
            time.sleep(args.interval)


if __name__ == "__main__":
    main()
