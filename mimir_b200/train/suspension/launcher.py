"""Resource-owning launcher for CUDA suspension with the (external) NCCL checkpoint shim.

Reference behaviour: ``src/mimir/training/suspension/launcher.py:14-84``.  Under
``launcher.lock`` it starts a dedicated loopback Redis key-value store (the shim's
rendezvous, address in ``kvs.txt``), waits for ``PING -> +PONG``, then runs the supervisor
with ``LD_PRELOAD=<shim>:<nccl>`` and tears both down when the supervisor exits.  The shim,
NCCL build, Redis and ``cuda-checkpoint`` executables come from a settings JSON; none ships
with this project.
"""
from __future__ import annotations

import argparse
import os
import signal
import socket
import subprocess
import sys
import time
from pathlib import Path

from mimir_b200.train.suspension.protocol import atomic_write, exclusive, read_json


def child_environment(settings: dict, kvs: Path) -> dict:
    shim, nccl = Path(settings["shim_library"]), Path(settings["nccl_library"])
    for lib in (shim, nccl):
        if not lib.is_file():
            raise FileNotFoundError(lib)
    env = os.environ.copy()
    env.update(LD_PRELOAD=f"{shim}:{nccl}", LD_LIBRARY_PATH=":".join([str(nccl.parent), *settings.get("library_dirs", [])]),
               NCCL_CHECKPOINT_KVS_PATH=str(kvs), TRAINING_SUSPEND_NCCL_SHIM="1")
    return env


def _free_loopback_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _wait_redis(proc, port: int, seconds: float = 20) -> None:
    deadline = time.monotonic() + seconds
    while True:
        if proc.poll() is not None:
            raise RuntimeError("Dedicated Redis failed to start; see redis.log")
        try:
            with socket.create_connection(("127.0.0.1", port), timeout=1) as conn:
                conn.sendall(b"*1\r\n$4\r\nPING\r\n")
                if conn.recv(1024).startswith(b"+PONG"):
                    return
        except OSError:
            pass
        if time.monotonic() >= deadline:
            raise TimeoutError("Redis startup deadline")
        time.sleep(0.1)


def supervisor_command(settings: dict, root: Path, command) -> list[str]:
    return [sys.executable, "-m", "mimir_b200.train.suspension.supervisor", "--control-root", str(root),
            "--cuda-checkpoint", settings["cuda_checkpoint"], "--max-restarts", str(settings.get("max_restarts", 3)),
            "--min-free-mib", str(settings.get("min_free_mib", 178000)),
            *(["--allow-existing-peers"] if settings.get("allow_existing_peers") else []), "--", *command]


def main(argv=None) -> None:
    parser = argparse.ArgumentParser(description="CUDA suspension launcher")
    parser.add_argument("--settings", type=Path, required=True)
    parser.add_argument("--control-root", type=Path, required=True)
    parser.add_argument("command", nargs=argparse.REMAINDER)
    args = parser.parse_args(argv)
    command = args.command[1:] if args.command[:1] == ["--"] else args.command
    if not command:
        parser.error("Training command required")
    settings = read_json(args.settings)
    root = args.control_root.resolve()
    root.mkdir(parents=True, exist_ok=True)
    for sig in (signal.SIGTERM, signal.SIGINT):
        signal.signal(sig, lambda *_, s=sig: sys.exit(128 + s))
    with exclusive(root / "launcher.lock"):
        port = _free_loopback_port()
        kvs = root / "kvs.txt"
        atomic_write(kvs, f"127.0.0.1:{port}\n")
        env = child_environment(settings, kvs)
        supervisor = None
        with (root / "redis.log").open("a") as log:
            redis = subprocess.Popen([settings["redis_server"], "--bind", "127.0.0.1", "--port", str(port), "--save",
                                      "", "--appendonly", "no", "--protected-mode", "yes"], stdout=log,
                                     stderr=subprocess.STDOUT)
            try:
                _wait_redis(redis, port)
                supervisor = subprocess.Popen(supervisor_command(settings, root, command), env=env)
                status = supervisor.wait()
                if status:
                    raise SystemExit(status)
            finally:
                try:
                    if supervisor is not None and supervisor.poll() is None:
                        supervisor.terminate()
                        supervisor.wait(timeout=90)
                finally:
                    redis.terminate()
                    redis.wait(timeout=20)


if __name__ == "__main__":
    main()
