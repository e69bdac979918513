"""Owner of a CUDA-suspendable single-node launch, with a bounded disk-restart fallback.

Behavioural reference: ``src/mimir/training/suspension/supervisor.py:21-262``.

The supervisor runs attempts.  An attempt:

1. waits until the selected GPUs are free (no foreign process on them, at least
   ``min_free_mib`` free, no ``hold`` file; ``stop.request`` ends the wait);
2. starts training through ``controller launch`` in a new session under ``attempt-<uuid>/`` and
   keeps recording the process tree it owns (pid + start-time identities, so a recycled pid is
   never signalled);
3. while the job is suspended, restores it on ``restore.request`` or when the offload lease runs
   out;
4. when restoring fails, the launcher died while suspended, or ``fallback.request`` appears, stops
   only its own processes and restarts training from the regular checkpoint that the readiness
   handshake named, with the suspend steps still pending (at most ``max_restarts`` per step).

``stop.request`` ends supervision without a restart.  File names are the suspension protocol.
"""
from __future__ import annotations

import argparse
import os
import signal
import subprocess
import sys
import time
import uuid
from pathlib import Path

from mimir_b200.train.suspension.controller import CudaBackend
from mimir_b200.train.suspension.protocol import (atomic_write, exclusive, matches, process_identity, read_json, steps,
                                                  validate_process)

CONTROLLER = "mimir_b200.train.suspension.controller"
STOP_WAIT_S = 20


# ------------------------------------------------------------------ restart command
def overrides(command, values: dict) -> list[str]:
    """``command`` with every ``key=value`` (or ``+key=value``) override of ``values`` replaced."""
    replaced = set(values)

    def key(arg: str) -> str:
        return arg.split("=", 1)[0].lstrip("+")

    return [a for a in command if key(a) not in replaced] + [f"{k}={v}" for k, v in values.items()]


def verified_checkpoint(ready: dict):
    """(published tag directory, tag) of the regular checkpoint a readiness handshake names."""
    from mimir_b200.ckpt.contract import validate
    sidecar = Path(ready["checkpoint"]).resolve()
    tag = f"step_{int(ready['step'])}"
    if sidecar.name != f"checkpoint_state_{tag}.json":
        raise RuntimeError("Suspension did not name its regular checkpoint")
    state = read_json(sidecar)
    if state["step"] != ready["step"] or state.get("carry_policy") != "none":
        raise RuntimeError("Checkpoint step mismatch or unsupported carry policy")
    if not validate(sidecar.parent):
        raise RuntimeError(f"Incomplete recovery checkpoint: {sidecar}")
    return sidecar.parent, tag


def _still_pending(control: Path, ready: dict) -> list[int]:
    """Suspend steps after the handshake's step: the queue plus any unclaimed request."""
    queue = read_json(control / "queue.json")
    if queue["job_id"] != ready["job_id"]:
        raise RuntimeError("Queue identity mismatch")
    pending = list(queue["pending"])
    unclaimed = control / "suspend_after_steps"
    if unclaimed.exists():
        pending += steps(unclaimed.read_text())
    return [s for s in steps(pending) if s > ready["step"]]


def restart_command(command, root: Path, ready: dict) -> list[str]:
    """The training command that resumes from the handshake's checkpoint."""
    directory, tag = verified_checkpoint(ready)
    remaining = _still_pending(root, ready)
    return overrides(command, {"resume_checkpoint_path": str(directory), "resume_checkpoint_tag": tag,
                               "resume_step": "null", "resume_epoch": "null", "resume_batch_in_epoch": "null",
                               "reset_ema_on_resume": "false",
                               "suspend_after_steps": str(remaining).replace(" ", "")})


# ------------------------------------------------------------------ the owned process tree
def _alive(identity: dict) -> bool:
    try:
        validate_process(identity)
        return True
    except (FileNotFoundError, ProcessLookupError, RuntimeError):
        return False


class OwnedTree:
    """The launcher and every descendant seen so far (torchrun workers start their own sessions,
    so the tree is re-scanned while it is alive)."""

    def __init__(self, proc):
        self.proc = proc
        self.launcher = process_identity(proc.pid)
        self.members: dict[int, dict] = {}

    def refresh(self) -> dict:
        import psutil
        try:
            validate_process(self.launcher)
            top = psutil.Process(self.proc.pid)
            for p in (top, *top.children(recursive=True)):
                try:
                    self.members[p.pid] = process_identity(p.pid)
                except (OSError, RuntimeError):
                    pass
        except (OSError, RuntimeError, psutil.NoSuchProcess):
            pass
        return self.members

    def _check_ranks_are_ours(self, ready) -> None:
        for rank in (ready or {}).get("ranks", []):
            if not _alive(rank):
                continue  # gone or recycled: never signal a replacement
            mine = self.members.get(rank["pid"])
            if mine is None or any(rank[k] != v for k, v in mine.items()):
                raise RuntimeError("Refusing to signal a rank outside the recorded process tree")

    def stop(self, ready=None) -> None:
        """SIGTERM, then SIGKILL, only to identity-checked members of the tree."""
        import psutil
        self.refresh()
        self._check_ranks_are_ours(ready)
        members = list(self.members.values())
        for sig in (signal.SIGTERM, signal.SIGKILL):
            for ident in members:
                try:
                    handle = psutil.Process(ident["pid"])
                    validate_process(ident)
                    handle.send_signal(sig)  # psutil re-checks the creation time against pid reuse
                except (FileNotFoundError, ProcessLookupError, RuntimeError, psutil.NoSuchProcess):
                    continue
            deadline = time.monotonic() + STOP_WAIT_S
            while time.monotonic() < deadline:
                self.proc.poll()
                if not any(_alive(ident) for ident in members):
                    return
                time.sleep(0.2)
        raise RuntimeError("Owned workers did not exit; refusing a second training launch")


# ------------------------------------------------------------------ GPU gate
def gpu_uuids() -> set[str]:
    out = subprocess.check_output(["nvidia-smi", "--query-gpu=index,uuid", "--format=csv,noheader"], text=True)
    by_index = dict(line.strip().split(", ") for line in out.splitlines())
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", ",".join(by_index)).split(",")
    return {by_index.get(v, v) for v in visible}


def gpus_available(backend, selected, minimum: int, root: Path, peers=()) -> bool:
    tolerated = {p["pid"] for p in peers if _alive_or_os_error(p)}
    if (root / "hold").exists():
        return False
    if any(gpu in selected and pid not in tolerated for pid, gpu in backend.memory()):
        return False
    free = backend.free()
    return all(free.get(gpu, 0) >= minimum for gpu in selected)


def _alive_or_os_error(identity: dict) -> bool:
    try:
        validate_process(identity)
        return True
    except (OSError, RuntimeError):
        return False


def wait_for_gpus(backend, selected, minimum: int, root: Path, interval: float, peers=()) -> None:
    while not gpus_available(backend, selected, minimum, root, peers):
        if (root / "stop.request").exists():
            raise RuntimeError("Supervisor stop requested while waiting for GPUs")
        time.sleep(interval)
    if (root / "stop.request").exists():
        raise RuntimeError("Supervisor stop requested while waiting for GPUs")


# ------------------------------------------------------------------ restore
def restore_or_fail(root: Path, executable: str, timeout: float, ack_timeout: float) -> bool:
    """The controller's restore: False when it deferred (hold/occupancy), True once the workers
    acknowledged the resume."""
    done = subprocess.run([sys.executable, "-m", CONTROLLER, "--cuda-checkpoint", executable, "restore", str(root)],
                          timeout=timeout)
    if done.returncode == 75:
        return False
    done.check_returncode()
    ready = read_json(root / "suspend_ready.json")
    acknowledged = root / "resumed.json"
    deadline = time.monotonic() + ack_timeout
    while time.monotonic() < deadline:
        if acknowledged.exists() and matches(read_json(acknowledged), ready):
            return True
        time.sleep(1)
    raise TimeoutError("Workers failed to acknowledge resume after CUDA restoration")


def _active_state(attempt_root: Path, root: Path):
    """(worker control directory, unresolved readiness handshake or None)."""
    launches = list(attempt_root.glob("*/launch.json"))
    if len(launches) > 1:
        raise RuntimeError("Ambiguous worker launch")
    if not launches:
        return None, None
    active = launches[0].parent
    if not (active / "managed.json").exists():
        atomic_write(active / "managed.json", {"supervisor_root": str(root)})
    atomic_write(root / "active.json", {"control_dir": str(active)})
    ready_file, resumed_file = active / "suspend_ready.json", active / "resumed.json"
    ready = read_json(ready_file) if ready_file.exists() else None
    if ready and resumed_file.exists() and matches(read_json(resumed_file), ready):
        ready = None  # that suspension already resumed
    return active, ready


class Supervisor:
    def __init__(self, args, command):
        self.args, self.command = args, command
        self.root = args.control_root.resolve()
        self.root.mkdir(parents=True, exist_ok=True)
        self.backend = CudaBackend(args.cuda_checkpoint)
        self.selected = gpu_uuids()
        self.peers = ([process_identity(pid) for pid in {pid for pid, gpu in self.backend.memory()
                                                         if gpu in self.selected}]
                      if args.allow_existing_peers else [])
        self.attempt = 0
        self.restarts: dict[int, int] = {}

    def run(self) -> None:
        with exclusive(self.root / "supervisor.lock"):
            while self._attempt():
                self.attempt += 1

    def _launch(self, attempt_root: Path):
        actual = overrides(self.command, {"suspend_control_dir": str(attempt_root)})
        proc = subprocess.Popen([sys.executable, "-m", CONTROLLER, "--cuda-checkpoint", self.args.cuda_checkpoint,
                                 "launch", "--control-root", str(attempt_root), "--", *actual], start_new_session=True)
        tree = OwnedTree(proc)
        atomic_write(self.root / "supervisor.json", {"owner": process_identity(), "launcher": tree.launcher,
                                                     "attempt": self.attempt, "command": actual,
                                                     "attempt_root": str(attempt_root)})
        return proc, tree

    def _attempt(self) -> bool:
        """One launch; True when it ended in a disk restart (another attempt follows)."""
        args = self.args
        wait_for_gpus(self.backend, self.selected, args.min_free_mib, self.root, args.interval, self.peers)
        attempt_root = self.root / f"attempt-{uuid.uuid4().hex}"
        attempt_root.mkdir()
        proc, tree = self._launch(attempt_root)
        ready = None
        try:
            while True:
                tree.refresh()
                if (self.root / "stop.request").exists():
                    raise RuntimeError("Explicit supervisor stop; no automatic restart")
                active, ready = _active_state(attempt_root, self.root)
                if ready and self._handle_suspended(active, ready, proc, tree):
                    self.command = read_json(self.root / "restart_pending.json")["command"]
                    return True
                if proc.poll() is not None:
                    if proc.returncode:
                        raise RuntimeError(f"Training exited with {proc.returncode}")
                    return False
                time.sleep(args.interval)
        finally:
            tree.stop(ready)

    def _handle_suspended(self, active: Path, ready: dict, proc, tree: OwnedTree) -> bool:
        """Restore a due suspension; on failure prepare a disk restart and return True."""
        generation = active / f"generation_{ready['generation']:06d}"
        lease = generation / "offload.json"
        fallback = generation / "fallback.request"
        if ((self.root / "hold").exists() or (active / "hold").exists()) and not fallback.exists():
            return False
        lease_over = lease.exists() and time.time() >= read_json(lease)["lease_until"]
        due = (generation / "restore.request").exists() or lease_over
        launcher_gone = proc.poll() is not None
        if not (due or fallback.exists() or launcher_gone):
            return False
        try:
            if fallback.exists():
                raise RuntimeError("Controller requested disk fallback")
            if launcher_gone:
                raise RuntimeError("Training launcher exited while suspended")
            restore_or_fail(active, self.args.cuda_checkpoint, self.args.restore_timeout, self.args.ack_timeout)
            return False
        except (RuntimeError, OSError, subprocess.SubprocessError) as error:
            self._prepare_disk_restart(active, generation, ready, tree, error)
            return True

    def _prepare_disk_restart(self, active, generation, ready, tree, error) -> None:
        step = ready["step"]
        if self.restarts.get(step, 0) >= self.args.max_restarts:
            raise RuntimeError("Disk restart budget exhausted") from error
        previous = read_json(self.root / "supervisor.json")["command"]
        with exclusive(active / "controller.lock"), exclusive(active / "requests.lock"):
            command = restart_command(previous, active, ready)
            atomic_write(generation / "disk_fallback.json", {"error": str(error), "checkpoint": ready["checkpoint"],
                                                              "command": command, "time": time.time()})
            tree.stop(ready)
        atomic_write(self.root / "restart_pending.json", {"step": step, "checkpoint": ready["checkpoint"],
                                                          "command": command, "time": time.time()})
        print(f"[suspend] disk fallback from step {step}: {error}", flush=True)
        self.restarts[step] = self.restarts.get(step, 0) + 1


def supervise(args, command) -> None:
    Supervisor(args, command).run()


def main(argv=None) -> None:
    parser = argparse.ArgumentParser(description="CUDA suspension supervisor")
    parser.add_argument("--control-root", type=Path, required=True)
    parser.add_argument("--cuda-checkpoint", default="cuda-checkpoint")
    parser.add_argument("--max-restarts", type=int, default=3)
    parser.add_argument("--restore-timeout", type=float, default=900)
    parser.add_argument("--ack-timeout", type=float, default=120)
    parser.add_argument("--min-free-mib", type=int, default=178000)
    parser.add_argument("--interval", type=float, default=5)
    parser.add_argument("--allow-existing-peers", action="store_true")
    parser.add_argument("command", nargs=argparse.REMAINDER)
    args = parser.parse_args(argv)
    command = args.command[1:] if args.command[:1] == ["--"] else args.command
    if not command or min(args.restore_timeout, args.ack_timeout, args.interval) <= 0 or args.max_restarts < 0:
        parser.error("A command and positive timeouts are required; max-restarts must be nonnegative")
    for sig in (signal.SIGTERM, signal.SIGINT):
        signal.signal(sig, lambda *_, s=sig: sys.exit(128 + s))
    supervise(args, command)


if __name__ == "__main__":
    main()
