"""Local SQLite (WAL) job queue: immutable attempt snapshots, fenced leases, resources, holds.

Reference behaviour: ``src/mimir/scheduling/store.py:12-158``.  The table layout (``jobs``,
``dependencies``, ``attempts``, ``resources``) is kept so either framework's monitor reads
the other's queue.

* ``add`` validates kind, retry bound and a filename-safe id; dependencies carry a policy:
  ``success`` (parent must succeed) or ``terminal`` (parent must merely finish).  Training
  may not wait on administrative jobs and waits on evaluations only through ``terminal``.
* ``claim`` first marks jobs ``blocked`` whose ``success`` prerequisites failed (to a fixed
  point), then takes the oldest runnable, unheld job whose resources are free, snapshots its
  config into ``attempts`` and fences it with a fresh owner token and a lease.
* ``finish`` only accepts the current owner token; failures marked transient or OOM are
  retried while attempts remain (OOM halves the declared client controls
  ``max_connections`` and ``batch_size``; commands are never rewritten).
* ``recover`` returns expired leases to the queue only when the caller confirms their owner
  process is gone (lease expiry alone never frees a GPU).
"""
from __future__ import annotations

import json
import os
import sqlite3
import string
import time
import uuid
from contextlib import contextmanager
from pathlib import Path

TERMINAL = {"succeeded", "failed", "cancelled", "blocked"}
KINDS = {"train", "checkpoint_wait", "export", "inference", "score", "merge", "publish", "average", "eval"}
_SAFE = set(string.ascii_letters + string.digits + "_.-")

_SCHEMA = """
PRAGMA journal_mode=WAL;
CREATE TABLE IF NOT EXISTS jobs (
  id TEXT PRIMARY KEY, kind TEXT NOT NULL, config TEXT NOT NULL,
  state TEXT NOT NULL DEFAULT 'pending', held INTEGER NOT NULL DEFAULT 0,
  owner TEXT, lease REAL, attempt INTEGER NOT NULL DEFAULT 0,
  max_attempts INTEGER NOT NULL DEFAULT 3, result TEXT, created REAL NOT NULL, worker_identity TEXT);
CREATE TABLE IF NOT EXISTS dependencies (
  job TEXT REFERENCES jobs(id), dependency TEXT REFERENCES jobs(id),
  policy TEXT CHECK(policy IN ('success','terminal')), PRIMARY KEY(job,dependency));
CREATE TABLE IF NOT EXISTS attempts (
  token TEXT PRIMARY KEY, job TEXT REFERENCES jobs(id), number INTEGER,
  config TEXT NOT NULL, started REAL, finished REAL, state TEXT, result TEXT);
CREATE TABLE IF NOT EXISTS resources (
  name TEXT PRIMARY KEY, token TEXT NOT NULL REFERENCES attempts(token));
"""

_BLOCK = """UPDATE jobs SET state='blocked' WHERE state='pending' AND id IN
  (SELECT d.job FROM dependencies d JOIN jobs j ON j.id=d.dependency
   WHERE d.policy='success' AND j.state IN ('failed','cancelled','blocked'))"""

_RUNNABLE = """SELECT * FROM jobs j WHERE state='pending' AND held=0 AND NOT EXISTS
  (SELECT 1 FROM dependencies d JOIN jobs p ON p.id=d.dependency WHERE d.job=j.id AND
   ((d.policy='success' AND p.state!='succeeded') OR
    (d.policy='terminal' AND p.state NOT IN ('succeeded','failed','cancelled','blocked'))))
  ORDER BY created,id"""


def _identity() -> str:
    import psutil
    return json.dumps({"pid": os.getpid(), "created": psutil.Process().create_time()})


class Store:
    def __init__(self, path):
        self.path = Path(path)
        self.path.parent.mkdir(parents=True, exist_ok=True)
        with self.connect() as db:
            db.executescript(_SCHEMA)

    def connect(self) -> sqlite3.Connection:
        db = sqlite3.connect(self.path, timeout=30)
        db.row_factory = sqlite3.Row
        db.execute("PRAGMA foreign_keys=ON")
        db.execute("PRAGMA synchronous=FULL")
        return db

    @contextmanager
    def transaction(self):
        db = self.connect()
        try:
            db.execute("BEGIN IMMEDIATE")
            yield db
            db.commit()
        except BaseException:
            db.rollback()
            raise
        finally:
            db.close()

    def add(self, identity: str, kind: str, config: dict, dependencies=(), max_attempts: int = 3, *,
            held: bool = False) -> None:
        if not isinstance(held, bool):
            raise ValueError("held must be a boolean")
        if kind not in KINDS or max_attempts < 1:
            raise ValueError("Invalid job kind or retry bound")
        if not identity or not set(identity) <= _SAFE:
            raise ValueError("Job ID must be a safe filename")
        with self.transaction() as db:
            db.execute("INSERT INTO jobs(id,kind,config,max_attempts,created,held) VALUES(?,?,?,?,?,?)",
                       (identity, kind, json.dumps(config, allow_nan=False), max_attempts, time.time(), int(held)))
            for parent_id, policy in dependencies:
                if parent_id == identity:
                    raise ValueError("Self-dependency")
                parent = db.execute("SELECT kind FROM jobs WHERE id=?", (parent_id,)).fetchone()
                if kind == "train" and parent:
                    if parent["kind"] in ("merge", "publish", "average"):
                        raise ValueError("Training cannot depend on administrative completion")
                    if parent["kind"] in ("eval", "inference", "score") and policy != "terminal":
                        raise ValueError("Training handoffs require terminal evaluation dependencies")
                db.execute("INSERT INTO dependencies VALUES(?,?,?)", (identity, parent_id, policy))

    def edit(self, identity: str, config: dict) -> None:
        with self.transaction() as db:
            n = db.execute("UPDATE jobs SET config=? WHERE id=? AND state='pending'",
                           (json.dumps(config, allow_nan=False), identity)).rowcount
            if n != 1:
                raise ValueError("Only pending jobs can be edited")

    def hold(self, identity: str, value: bool) -> None:
        with self.transaction() as db:
            db.execute("UPDATE jobs SET held=? WHERE id=?", (int(value), identity))

    def claim(self, ttl: float = 120, predicate=None):
        if ttl <= 0:
            raise ValueError("Positive lease duration required")
        with self.transaction() as db:
            while db.execute(_BLOCK).rowcount:
                pass
            for row in db.execute(_RUNNABLE).fetchall():
                config = json.loads(row["config"])
                if predicate is not None and not predicate(dict(row) | {"config": config}):
                    continue
                resources = sorted(set(config.get("resources", [])))
                if any(db.execute("SELECT 1 FROM resources WHERE name=?", (r,)).fetchone() for r in resources):
                    continue
                token, now, number = uuid.uuid4().hex, time.time(), row["attempt"] + 1
                db.execute("UPDATE jobs SET state='running',owner=?,lease=?,attempt=?,worker_identity=? WHERE id=?",
                           (token, now + ttl, number, _identity(), row["id"]))
                db.execute("INSERT INTO attempts VALUES(?,?,?,?,?,?,?,?)",
                           (token, row["id"], number, row["config"], now, None, "running", None))
                db.executemany("INSERT INTO resources VALUES(?,?)", [(r, token) for r in resources])
                return dict(row) | {"owner": token, "attempt": number, "config": config}
        return None

    def heartbeat(self, token: str, ttl: float = 120) -> None:
        with self.transaction() as db:
            if db.execute("UPDATE jobs SET lease=? WHERE owner=? AND state='running'",
                          (time.time() + ttl, token)).rowcount != 1:
                raise RuntimeError("Lease ownership lost")

    def finish(self, token: str, success: bool, result, *, transient: bool = False, oom: bool = False) -> None:
        with self.transaction() as db:
            job = db.execute("SELECT * FROM jobs WHERE owner=? AND state='running'", (token,)).fetchone()
            if job is None:
                raise RuntimeError("Stale attempt cannot finish")
            config = json.loads(job["config"])
            retry = not success and (transient or oom) and job["attempt"] < job["max_attempts"]
            if oom:
                controls = config.setdefault("controls", {})
                controls["max_connections"] = max(1, controls.get("max_connections", 4) // 2)
                controls["batch_size"] = max(1, controls.get("batch_size", 8) // 2)
            state = "succeeded" if success else "failed"
            db.execute("UPDATE attempts SET finished=?,state=?,result=? WHERE token=?",
                       (time.time(), state, json.dumps(result), token))
            db.execute("UPDATE jobs SET state=?,config=?,owner=NULL,lease=NULL,result=? WHERE id=?",
                       ("pending" if retry else state, json.dumps(config), json.dumps(result), job["id"]))
            db.execute("DELETE FROM resources WHERE token=?", (token,))

    def recover(self, is_running) -> list[str]:
        recovered = []
        with self.transaction() as db:
            for row in db.execute("SELECT * FROM jobs WHERE state='running' AND lease<?", (time.time(),)).fetchall():
                if is_running(dict(row)):
                    continue
                state = "pending" if row["attempt"] < row["max_attempts"] else "failed"
                db.execute("UPDATE attempts SET state=?,finished=?,result=? WHERE token=?",
                           ("abandoned", time.time(), json.dumps({"reason": "owner died"}), row["owner"]))
                db.execute("DELETE FROM resources WHERE token=?", (row["owner"],))
                db.execute("UPDATE jobs SET state=?,owner=NULL,lease=NULL WHERE id=?", (state, row["id"]))
                recovered.append(row["id"])
        return recovered

    def rows(self) -> list[dict]:
        with self.connect() as db:
            return [dict(r) for r in db.execute("SELECT * FROM jobs ORDER BY created")]

    def backup(self, destination) -> None:
        destination = Path(destination)
        if destination.exists():
            raise FileExistsError(destination)
        with self.connect() as source, sqlite3.connect(destination) as target:
            source.backup(target)
            if target.execute("PRAGMA integrity_check").fetchone()[0] != "ok":
                raise RuntimeError("Backup integrity failed")
