"""Host-only file protocol shared by the training hook and its controllers (no torch imports).

Reference behaviour: ``src/mimir/training/suspension/protocol.py:14-116``.  File names and
JSON shapes are part of the protocol between independent processes, so they match:

* ``atomic_write`` — temp file in the same directory, fsync, ``os.replace``, fsync the directory;
* ``exclusive`` — non-blocking ``flock`` (a dead owner releases it; the inode is never unlinked);
* ``process_identity`` — ``pid`` + start time in clock ticks (``/proc/<pid>/stat`` field 22) +
  hostname + boot id, so a recycled pid is never mistaken for the original process;
* requests — ``suspend_after_steps`` (space-separated positive steps) merged under
  ``requests.lock``; the hook claims the file by renaming it to ``request.<uuid>.claimed``,
  invalid claims are quarantined as ``.rejected`` with a ``.rejected.json`` reason;
* ``wait_json`` — poll a JSON record until its ``job_id``/``generation``/``step`` match.
"""
from __future__ import annotations

import fcntl
import json
import os
import socket
import tempfile
import time
import uuid
from contextlib import contextmanager
from pathlib import Path

_TOKEN_KEYS = ("job_id", "generation", "step")
_IDENTITY_KEYS = ("pid", "start_ticks", "host", "boot_id")


def atomic_write(path, value) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, temp = tempfile.mkstemp(prefix=f".{path.name}.", dir=path.parent)
    try:
        with os.fdopen(fd, "w") as f:
            f.write(value if isinstance(value, str) else json.dumps(value, sort_keys=True))
            f.flush()
            os.fsync(f.fileno())
        os.replace(temp, path)
        dfd = os.open(path.parent, os.O_RDONLY | os.O_DIRECTORY)
        try:
            os.fsync(dfd)
        finally:
            os.close(dfd)
    finally:
        if os.path.exists(temp):
            os.unlink(temp)


def read_json(path):
    return json.loads(Path(path).read_text())


@contextmanager
def exclusive(path):
    """Hold a non-blocking exclusive flock on ``path`` (raises ``BlockingIOError`` if held)."""
    with open(path, "a+") as f:
        fcntl.flock(f, fcntl.LOCK_EX | fcntl.LOCK_NB)
        try:
            yield
        finally:
            fcntl.flock(f, fcntl.LOCK_UN)


def process_identity(pid=None) -> dict:
    pid = os.getpid() if pid is None else int(pid)
    fields = Path(f"/proc/{pid}/stat").read_text().rsplit(")", 1)[1].split()
    if fields[0] == "Z":
        raise RuntimeError(f"Process {pid} is a zombie")
    return {"pid": pid, "start_ticks": fields[19], "host": socket.gethostname(),
            "boot_id": Path("/proc/sys/kernel/random/boot_id").read_text().strip()}


def validate_process(identity: dict) -> None:
    if process_identity(identity["pid"]) != {k: identity[k] for k in _IDENTITY_KEYS}:
        raise RuntimeError(f"Process identity changed: {identity}")


def steps(values) -> list[int]:
    """Parse suspend steps (a string or an iterable); every value must be a positive integer."""
    if isinstance(values, str):
        values = values.split()
    out = set()
    for v in values:
        if isinstance(v, bool) or not str(v).isdigit() or int(v) < 1:
            raise ValueError(f"Invalid suspend step: {v!r}")
        out.add(int(v))
    return sorted(out)


def submit(root, values) -> list[int]:
    """Add suspend steps to a running job's request file; returns the merged pending list."""
    root = Path(root)
    read_json(root / "launch.json")  # a typo'd or uninitialised control dir fails here
    with exclusive(root / "requests.lock"):
        path = root / "suspend_after_steps"
        merged = steps((steps(path.read_text()) if path.exists() else []) + steps(values))
        atomic_write(path, " ".join(map(str, merged)) + "\n")
    return merged


def claim(root):
    """Take ownership of pending requests: ``(claimed path, steps)`` or ``(None, [])``."""
    root = Path(root)
    path = root / "suspend_after_steps"
    with exclusive(root / "requests.lock"):
        if not path.exists():
            return None, []
        claimed = root / f"request.{uuid.uuid4().hex}.claimed"
        os.replace(path, claimed)
    try:
        return claimed, steps(claimed.read_text())
    except ValueError as error:
        atomic_write(claimed.with_suffix(".rejected.json"), {"error": str(error)})
        claimed.rename(claimed.with_suffix(".rejected"))
        return None, []


def matches(record: dict, expected: dict) -> bool:
    return all(record.get(k) == expected[k] for k in _TOKEN_KEYS)


def wait_json(path, expected: dict, interval: float, timeout=None) -> dict:
    start = time.monotonic()
    while True:
        try:
            record = read_json(path)
            if matches(record, expected):
                return record
        except FileNotFoundError:
            pass
        if timeout is not None and time.monotonic() - start > timeout:
            raise TimeoutError(f"Waiting for {path}")
        time.sleep(interval)
