"""Owner of a CUDA-suspendable single-node launch, with a bounded disk-restart fallback.

Reference behaviour: ``src/mimir/training/suspension/supervisor.py:21-262``.

Each attempt waits until the selected GPUs are free (no foreign occupant, ``min_free_mib``
free, no ``hold``), launches training through ``controller launch`` in its own session under
``attempt-<uuid>/``, and records the process tree it owns (identity-checked, so a recycled pid
is never signalled).  While the job is suspended it restores on ``restore.request`` or lease
expiry.  If restoration fails, the launcher died while suspended, or a ``fallback.request``
appears, it stops only its own processes and restarts from the regular checkpoint the
readiness handshake named, with the remaining suspend steps; at most ``max_restarts`` times per
step.  ``stop.request`` ends supervision without a restart.
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


def overrides(command, values: dict) -> list[str]:
    """``command`` with ``key=value`` overrides replaced (also ``+key=``) by ``values``."""
    keys = set(values)
    return [a for a in command if a.split("=", 1)[0].lstrip("+") not in keys] + [f"{k}={v}" for k, v in values.items()]


def verified_checkpoint(ready: dict):
    """(published tag directory, tag) of the regular checkpoint named by a readiness handshake."""
    from mimir_b200.ckpt.contract import validate
    path = Path(ready["checkpoint"]).resolve()
    tag = f"step_{int(ready['step'])}"
    if path.name != f"checkpoint_state_{tag}.json":
        raise RuntimeError("Suspension did not name its regular checkpoint")
    state = read_json(path)
    if state["step"] != ready["step"] or state.get("carry_policy") != "none":
        raise RuntimeError("Checkpoint step mismatch or unsupported carry policy")
    if not validate(path.parent):
        raise RuntimeError(f"Incomplete recovery checkpoint: {path}")
    return path.parent, tag


def restart_command(command, root: Path, ready: dict) -> list[str]:
    directory, tag = verified_checkpoint(ready)
    queue = read_json(root / "queue.json")
    if queue["job_id"] != ready["job_id"]:
        raise RuntimeError("Queue identity mismatch")
    pending = list(queue["pending"])
    request = root / "suspend_after_steps"
    if request.exists():
        pending += steps(request.read_text())
    remaining = [s for s in steps(pending) if s > ready["step"]]
    return overrides(command, {"resume_checkpoint_path": str(directory), "resume_checkpoint_tag": tag,
                               "resume_step": "null", "resume_epoch": "null", "resume_batch_in_epoch": "null",
                               "reset_ema_on_resume": "false",
                               "suspend_after_steps": str(remaining).replace(" ", "")})


def remember_owned(proc) -> dict:
    """Record the launcher and its descendants (torchrun workers run in their own sessions)."""
    import psutil
    owned = getattr(proc, "owned_processes", {})
    try:
        validate_process(proc.launch_identity)
        root = psutil.Process(proc.pid)
        for p in [root, *root.children(recursive=True)]:
            try:
                owned[p.pid] = process_identity(p.pid)
            except (OSError, RuntimeError):
                pass
    except (OSError, RuntimeError, psutil.NoSuchProcess):
        pass
    proc.owned_processes = owned
    return owned


def stop_owned(proc, ready=None) -> None:
    """TERM then KILL only identity-checked processes recorded for this launcher."""
    import psutil
    owned = remember_owned(proc)
    identities = list(owned.values())
    for rank in (ready or {}).get("ranks", []):
        try:
            validate_process(rank)
        except (FileNotFoundError, ProcessLookupError, RuntimeError):
            continue  # gone or recycled: never signal a replacement
        if rank["pid"] not in owned or any(rank[k] != v for k, v in owned[rank["pid"]].items()):
            raise RuntimeError("Refusing to signal a rank outside the recorded process tree")
    for sig, wait in ((signal.SIGTERM, 20), (signal.SIGKILL, 20)):
        for ident in identities:
            try:
                p = psutil.Process(ident["pid"])
                validate_process(ident)
                p.send_signal(sig)  # psutil re-checks creation time against pid reuse
            except (FileNotFoundError, ProcessLookupError, RuntimeError, psutil.NoSuchProcess):
                continue
        deadline = time.monotonic() + wait
        while time.monotonic() < deadline:
            proc.poll()
            alive = []
            for ident in identities:
                try:
                    validate_process(ident)
                    alive.append(ident)
                except (FileNotFoundError, ProcessLookupError, RuntimeError):
                    pass
            if not alive:
                return
            time.sleep(0.2)
    raise RuntimeError("Owned workers did not exit; refusing a second training launch")


def gpu_uuids() -> set[str]:
    out = subprocess.check_output(["nvidia-smi", "--query-gpu=index,uuid", "--format=csv,noheader"], text=True)
    mapping = dict(line.strip().split(", ") for line in out.splitlines())
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", ",".join(mapping)).split(",")
    return {mapping.get(v, v) for v in visible}


def gpus_available(backend, selected, minimum: int, root: Path, peers=()) -> bool:
    allowed = set()
    for peer in peers:
        try:
            validate_process(peer)
            allowed.add(peer["pid"])
        except (OSError, RuntimeError):
            pass
    free = backend.free()
    return (not (root / "hold").exists()
            and not any(gpu in selected and pid not in allowed for pid, gpu in backend.memory())
            and all(free.get(gpu, 0) >= minimum for gpu in selected))


def wait_for_gpus(backend, selected, minimum: int, root: Path, interval: float, peers=()) -> None:
    while True:
        if (root / "stop.request").exists():
            raise RuntimeError("Supervisor stop requested while waiting for GPUs")
        if gpus_available(backend, selected, minimum, root, peers):
            return
        time.sleep(interval)


def restore_or_fail(root: Path, executable: str, timeout: float, ack_timeout: float) -> bool:
    """Run the controller's restore; False when deferred (hold/occupancy), True once workers resumed."""
    result = subprocess.run([sys.executable, "-m", "mimir_b200.train.suspension.controller", "--cuda-checkpoint",
                             executable, "restore", str(root)], timeout=timeout)
    if result.returncode == 75:
        return False
    result.check_returncode()
    ready = read_json(root / "suspend_ready.json")
    deadline = time.monotonic() + ack_timeout
    while time.monotonic() < deadline:
        path = root / "resumed.json"
        if path.exists() and matches(read_json(path), ready):
            return True
        time.sleep(1)
    raise TimeoutError("Workers failed to acknowledge resume after CUDA restoration")


def _active_state(attempt_root: Path, root: Path):
    launches = list(attempt_root.glob("*/launch.json"))
    if len(launches) > 1:
        raise RuntimeError("Ambiguous worker launch")
    if not launches:
        return None, None
    active = launches[0].parent
    if not (active / "managed.json").exists():
        atomic_write(active / "managed.json", {"supervisor_root": str(root)})
    atomic_write(root / "active.json", {"control_dir": str(active)})
    path = active / "suspend_ready.json"
    ready = read_json(path) if path.exists() else None
    resumed = active / "resumed.json"
    if ready and resumed.exists() and matches(read_json(resumed), ready):
        ready = None
    return active, ready


def supervise(args, command) -> None:
    root = args.control_root.resolve()
    root.mkdir(parents=True, exist_ok=True)
    backend = CudaBackend(args.cuda_checkpoint)
    selected = gpu_uuids()
    peers = ([process_identity(pid) for pid in {pid for pid, gpu in backend.memory() if gpu in selected}]
             if args.allow_existing_peers else [])
    with exclusive(root / "supervisor.lock"):
        attempt, restarts = 0, {}
        while True:
            wait_for_gpus(backend, selected, args.min_free_mib, root, args.interval, peers)
            attempt_root = root / f"attempt-{uuid.uuid4().hex}"
            attempt_root.mkdir()
            actual = overrides(command, {"suspend_control_dir": str(attempt_root)})
            proc = subprocess.Popen([sys.executable, "-m", "mimir_b200.train.suspension.controller",
                                     "--cuda-checkpoint", args.cuda_checkpoint, "launch", "--control-root",
                                     str(attempt_root), "--", *actual], start_new_session=True)
            proc.launch_identity = process_identity(proc.pid)
            atomic_write(root / "supervisor.json", {"owner": process_identity(), "launcher": proc.launch_identity,
                                                    "attempt": attempt, "command": actual,
                                                    "attempt_root": str(attempt_root)})
            ready = None
            try:
                while True:
                    remember_owned(proc)
                    if (root / "stop.request").exists():
                        raise RuntimeError("Explicit supervisor stop; no automatic restart")
                    active, ready = _active_state(attempt_root, root)
                    if ready and _handle_suspended(args, root, active, ready, proc, restarts):
                        command = read_json(root / "restart_pending.json")["command"]
                        attempt += 1
                        break
                    if proc.poll() is not None:
                        if proc.returncode:
                            raise RuntimeError(f"Training exited with {proc.returncode}")
                        return
                    time.sleep(args.interval)
            finally:
                stop_owned(proc, ready)


def _handle_suspended(args, root: Path, active: Path, ready: dict, proc, restarts: dict) -> bool:
    """Restore a due suspension; on failure prepare a disk restart and return True."""
    generation = active / f"generation_{ready['generation']:06d}"
    receipt = generation / "offload.json"
    fallback = generation / "fallback.request"
    held = (root / "hold").exists() or (active / "hold").exists()
    if held and not fallback.exists():
        return False
    due = (generation / "restore.request").exists() or (receipt.exists() and time.time() >= read_json(receipt)["lease_until"])
    if not (due or fallback.exists() or proc.poll() is not None):
        return False
    try:
        if fallback.exists():
            raise RuntimeError("Controller requested disk fallback")
        if proc.poll() is not None:
            raise RuntimeError("Training launcher exited while suspended")
        restore_or_fail(active, args.cuda_checkpoint, args.restore_timeout, args.ack_timeout)
        return False
    except (RuntimeError, OSError, subprocess.SubprocessError) as error:
        if restarts.get(ready["step"], 0) >= args.max_restarts:
            raise RuntimeError("Disk restart budget exhausted") from error
        previous = read_json(root / "supervisor.json")["command"]
        with exclusive(active / "controller.lock"), exclusive(active / "requests.lock"):
            command = restart_command(previous, active, ready)
            atomic_write(generation / "disk_fallback.json", {"error": str(error), "checkpoint": ready["checkpoint"],
                                                              "command": command, "time": time.time()})
            stop_owned(proc, ready)
        atomic_write(root / "restart_pending.json", {"step": ready["step"], "checkpoint": ready["checkpoint"],
                                                      "command": command, "time": time.time()})
        print(f"[suspend] disk fallback from step {ready['step']}: {error}", flush=True)
        restarts[ready["step"]] = restarts.get(ready["step"], 0) + 1
        return True


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
