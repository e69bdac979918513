"""File protocol shared by the training hook and the processes that suspend it (no torch imports).

Behavioural reference: ``src/mimir/training/suspension/protocol.py:14-116``.  Independent
processes (the training ranks, a controller, a supervisor, a user's ``submit``) talk through a
control directory, so file names and JSON keys are the protocol:

* every record is replaced atomically (temporary file in the same directory, fsync, rename,
  fsync of the directory), so a reader sees the old or the new version, never a torn one;
* single-writer sections hold a non-blocking ``flock`` (released by the kernel if the owner dies;
  the lock file is never unlinked, so its inode stays the one everyone locks);
* a process is identified by pid + start time in clock ticks (``/proc/<pid>/stat`` field 22) +
  host name + boot id, so a recycled pid is never mistaken for the original process;
* suspend requests live in ``suspend_after_steps`` (space-separated positive steps), merged
  under ``requests.lock``; the hook claims them by renaming the file to
  ``request.<uuid>.claimed``; a claim that does not parse is quarantined as ``.rejected`` with a
  ``.rejected.json`` reason;
* records that answer a request carry ``job_id``, ``generation`` and ``step``; a waiter polls
  until all three match.
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
from typing import Iterable, Optional

REQUEST_FILE = "suspend_after_steps"
REQUEST_LOCK = "requests.lock"
ANSWER_KEYS = ("job_id", "generation", "step")
IDENTITY_KEYS = ("pid", "start_ticks", "host", "boot_id")


# ------------------------------------------------------------------ atomic records
def _fsync_directory(directory: Path) -> None:
    fd = os.open(directory, os.O_RDONLY | os.O_DIRECTORY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def atomic_write(path, value) -> None:
    """Replace ``path`` with ``value`` (a string, or JSON with sorted keys) atomically."""
    target = Path(path)
    target.parent.mkdir(parents=True, exist_ok=True)
    text = value if isinstance(value, str) else json.dumps(value, sort_keys=True)
    fd, scratch = tempfile.mkstemp(prefix=f".{target.name}.", dir=target.parent)
    try:
        with os.fdopen(fd, "w") as handle:
            handle.write(text)
            handle.flush()
            os.fsync(handle.fileno())
        os.replace(scratch, target)
        _fsync_directory(target.parent)
    finally:
        if os.path.exists(scratch):
            os.unlink(scratch)


def read_json(path):
    return json.loads(Path(path).read_text())


@contextmanager
def exclusive(path):
    """Hold a non-blocking exclusive flock on ``path``; ``BlockingIOError`` if someone else does."""
    with open(path, "a+") as handle:
        fcntl.flock(handle, fcntl.LOCK_EX | fcntl.LOCK_NB)
        try:
            yield
        finally:
            fcntl.flock(handle, fcntl.LOCK_UN)


# ------------------------------------------------------------------ process identity
def _boot_id() -> str:
    return Path("/proc/sys/kernel/random/boot_id").read_text().strip()


def process_identity(pid=None) -> dict:
    """``{pid, start_ticks, host, boot_id}`` of a live (non-zombie) process."""
    pid = os.getpid() if pid is None else int(pid)
    # Fields after the parenthesised command name: state is the first, start time the 20th.
    after_name = Path(f"/proc/{pid}/stat").read_text().rsplit(")", 1)[1].split()
    state, start_ticks = after_name[0], after_name[19]
    if state == "Z":
        raise RuntimeError(f"Process {pid} is a zombie")
    return {"pid": pid, "start_ticks": start_ticks, "host": socket.gethostname(), "boot_id": _boot_id()}


def validate_process(identity: dict) -> None:
    """Raise unless the process recorded in ``identity`` is still the same running process."""
    recorded = {key: identity[key] for key in IDENTITY_KEYS}
    if process_identity(identity["pid"]) != recorded:
        raise RuntimeError(f"Process identity changed: {identity}")


# ------------------------------------------------------------------ suspend requests
def steps(values) -> list[int]:
    """Sorted distinct suspend steps from a string or an iterable; each must be a positive integer."""
    items: Iterable = values.split() if isinstance(values, str) else values
    parsed = set()
    for item in items:
        text = str(item)
        if isinstance(item, bool) or not text.isdigit() or int(text) < 1:
            raise ValueError(f"Invalid suspend step: {item!r}")
        parsed.add(int(text))
    return sorted(parsed)


def submit(root, values) -> list[int]:
    """Add suspend steps to a running job's pending requests; returns the merged list.  A control
    directory without ``launch.json`` (a typo, or a job not yet launched) is refused."""
    control = Path(root)
    read_json(control / "launch.json")
    requests = control / REQUEST_FILE
    with exclusive(control / REQUEST_LOCK):
        pending = steps(requests.read_text()) if requests.exists() else []
        merged = steps(pending + steps(values))
        atomic_write(requests, " ".join(str(s) for s in merged) + "\n")
    return merged


def _quarantine(claimed: Path, error: ValueError) -> None:
    atomic_write(claimed.with_suffix(".rejected.json"), {"error": str(error)})
    claimed.rename(claimed.with_suffix(".rejected"))


def claim(root) -> tuple[Optional[Path], list[int]]:
    """Take ownership of the pending requests: ``(claimed file, steps)``, or ``(None, [])`` when
    there are none or they do not parse (then they are quarantined)."""
    control = Path(root)
    requests = control / REQUEST_FILE
    with exclusive(control / REQUEST_LOCK):
        if not requests.exists():
            return None, []
        claimed = control / f"request.{uuid.uuid4().hex}.claimed"
        os.replace(requests, claimed)
    try:
        return claimed, steps(claimed.read_text())
    except ValueError as error:
        _quarantine(claimed, error)
        return None, []


# ------------------------------------------------------------------ answers
def matches(record: dict, expected: dict) -> bool:
    return all(record.get(key) == expected[key] for key in ANSWER_KEYS)


def wait_json(path, expected: dict, interval: float, timeout=None) -> dict:
    """Poll ``path`` until it holds a record answering ``expected``; ``TimeoutError`` after
    ``timeout`` seconds (None: wait forever)."""
    deadline = None if timeout is None else time.monotonic() + timeout
    while True:
        try:
            record = read_json(path)
        except FileNotFoundError:
            record = None
        if record is not None and matches(record, expected):
            return record
        if deadline is not None and time.monotonic() > deadline:
            raise TimeoutError(f"Waiting for {path}")
        time.sleep(interval)
