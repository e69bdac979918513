"""In-loop suspension hook: checkpoint at a requested step, publish readiness, pause for a token.

Behavioural reference: ``src/mimir/training/suspension/runtime.py:11-135``.

Per job the hook owns ``<root>/<job_id>/`` (the control directory) and speaks the file protocol
of :mod:`.protocol`:

1. Every ``poll_steps`` steps rank 0 claims pending requests and broadcasts them, so every rank
   holds the same queue (persisted as ``queue.json``).
2. At the first due step all ranks save a checkpoint, finish their collectives and device work,
   release cached device memory (and, with the NCCL checkpoint shim, prepare NCCL), then write
   ``generation_<n>/ready.<pid>.json``.  Rank 0 waits for every rank's file and publishes
   ``suspend_ready.json``.
3. An external controller checkpoints the processes (``cuda-checkpoint``) and, after restoring
   them, writes a ``resume.<pid>`` token per process.  From readiness until that token only host
   polling runs: no device call, no collective.
4. Each rank consumes its token, restores NCCL, joins a barrier; rank 0 writes ``resumed.json``.
"""
from __future__ import annotations

import os
import time
import uuid
from pathlib import Path

from mimir_b200.train.suspension.protocol import atomic_write, claim, process_identity, steps, wait_json

READY_TIMEOUT_S = 300


class _Group:
    """The collectives the hook needs, reduced to no-ops in a single process."""

    def __init__(self, torch, dist, device):
        self.torch, self.dist, self.device = torch, dist, device
        self.active = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank() if self.active else 0
        self.size = dist.get_world_size() if self.active else 1

    def from_rank0(self, value):
        if not self.active:
            return value
        box = [value]
        self.dist.broadcast_object_list(box, src=0)
        return box[0]

    def gather(self, value) -> list:
        if not self.active:
            return [value]
        out = [None] * self.size
        self.dist.all_gather_object(out, value)
        return out

    def settle(self) -> None:
        """Every rank here and every launched device operation finished."""
        if self.active:
            self.dist.barrier()
        if self.device.type == "cuda":
            self.torch.cuda.synchronize(self.device)


class _Queue:
    """Pending suspend steps (sorted) and the ones already served."""

    def __init__(self, initial):
        self.pending = steps(initial)
        self.served: set[int] = set()

    def merge(self, values) -> None:
        self.pending = sorted((set(self.pending) | set(values)) - self.served)

    def due(self, step: int) -> list[int]:
        return [s for s in self.pending if s <= step]

    def serve(self, step: int) -> list[int]:
        done = self.due(step)
        self.served.update(done)
        self.pending = [s for s in self.pending if s > step]
        return done

    def record(self, job_id) -> dict:
        return {"pending": self.pending, "consumed": sorted(self.served), "job_id": job_id}


def _nccl_shim_requested() -> bool:
    return os.environ.get("TRAINING_SUSPEND_NCCL_SHIM", os.environ.get("SUSPEND_TEST_NCCL_SHIM")) == "1"


class SuspendHook:
    def __init__(self, root, initial_steps, device, poll_steps: int = 10, wait_seconds: float = 2):
        import torch
        import torch.distributed as dist
        if poll_steps < 1 or wait_seconds <= 0:
            raise ValueError("Suspension poll intervals must be positive")
        self.device, self.torch = device, torch
        self.poll_steps, self.wait_seconds = poll_steps, wait_seconds
        self.nccl_shim = None
        if _nccl_shim_requested():
            if device.type != "cuda":
                raise ValueError("NCCL checkpoint shim requires CUDA")
            from mimir_b200.train.suspension.nccl_shim import NcclCheckpointShim
            self.nccl_shim = NcclCheckpointShim()
        self.group = _Group(torch, dist, device)
        self.rank, self.world = self.group.rank, self.group.size
        if int(os.environ.get("LOCAL_WORLD_SIZE", self.world)) != self.world:
            raise ValueError("Suspension supports one node only")
        self.requests = _Queue(initial_steps)
        self.generation = 0
        self.job_id = self.group.from_rank0(uuid.uuid4().hex if self.rank == 0 else None)
        self.root = Path(root).resolve() / self.job_id
        self.root.mkdir(parents=True, exist_ok=True)
        self.identity = self._identity()
        self.ranks = self.group.gather(self.identity)
        self._check_ranks()
        if self.rank == 0:
            atomic_write(self.root / "launch.json", {"job_id": self.job_id, "ranks": self.ranks,
                                                     "device": device.type, "initial_steps": self.requests.pending})
            self._save_queue()
            print(f"[suspend] control_dir={self.root}", flush=True)
        self.group.settle()

    # ------------------------------------------------------------------ set-up
    def _identity(self) -> dict:
        identity = process_identity() | {"rank": self.rank}
        if self.device.type == "cuda":
            job_file = os.environ.get("CUDA_CHECKPOINT_JOB_FILE")
            if not job_file:
                raise RuntimeError("Start CUDA-suspendable training through the suspension launcher "
                                   "(python -m mimir_b200.train.suspension.launcher) before CUDA initialises")
            info = os.stat(job_file)
            identity["cuda_job"] = [info.st_dev, info.st_ino]
        return identity

    def _check_ranks(self) -> None:
        if len({r["host"] for r in self.ranks}) != 1:
            raise ValueError("Ranks must be on one host")
        if self.device.type == "cuda" and len({tuple(r["cuda_job"]) for r in self.ranks}) != 1:
            raise ValueError("Ranks did not inherit the same CUDA checkpoint job")

    @property
    def queue(self) -> list:
        """Pending suspend steps, sorted."""
        return self.requests.pending

    @property
    def consumed(self) -> set:
        return self.requests.served

    def _save_queue(self) -> None:
        atomic_write(self.root / "queue.json", self.requests.record(self.job_id))

    # ------------------------------------------------------------------ requests
    def _claim_on_rank0(self):
        if self.rank != 0:
            return None, []
        try:
            return claim(self.root)
        except BlockingIOError:  # a writer holds the request lock: pick it up at the next poll
            return None, []
        except OSError as error:  # rank 0 must still reach the broadcast, or its peers wait forever
            print(f"[suspend] request read failed, retrying next poll: {error}", flush=True)
            return None, []

    def _poll_requests(self) -> None:
        claimed, values = self._claim_on_rank0()
        self.requests.merge(self.group.from_rank0(values))
        if self.rank == 0:
            self._save_queue()
            if claimed:
                claimed.rename(claimed.with_suffix(".accepted"))

    # ------------------------------------------------------------------ suspension
    def after_step(self, step: int, save_checkpoint, stopping: bool = False) -> bool:
        """Return True if training paused (and resumed) at this step."""
        if stopping:
            return False
        if step % self.poll_steps == 0:
            self._poll_requests()
        if not self.requests.due(step):
            return False
        checkpoint = save_checkpoint()
        requested = self.requests.serve(step)
        self.generation += 1
        token = {"job_id": self.job_id, "generation": self.generation, "step": step}
        folder = self.root / f"generation_{self.generation:06d}"
        folder.mkdir(exist_ok=True)
        self._quiesce()
        atomic_write(folder / f"ready.{os.getpid()}.json", token | self.identity)
        if self.rank == 0:
            self._announce_ready(folder, token, checkpoint, requested)
        self._await_resume(folder, token)
        if self.nccl_shim:
            self.nccl_shim.restore()
        self.group.settle()
        if self.rank == 0:
            atomic_write(self.root / "resumed.json", token)
            print(f"[suspend] resumed step={step} generation={self.generation}", flush=True)
        return True

    def _quiesce(self) -> None:
        """Finish every collective and every device operation; no device call follows until resume."""
        self.group.settle()
        if self.device.type == "cuda":
            self.torch.cuda.empty_cache()
            self.torch.cuda.synchronize(self.device)
        if self.nccl_shim:
            self.nccl_shim.prepare()

    def _announce_ready(self, folder, token, checkpoint, requested) -> None:
        for r in self.ranks:
            wait_json(folder / f"ready.{r['pid']}.json", token, self.wait_seconds, READY_TIMEOUT_S)
        self._save_queue()
        atomic_write(self.root / "suspend_ready.json", token | {
            "ranks": self.ranks, "checkpoint": str(checkpoint), "requested_steps": requested, "ready_at": time.time()})
        print(f"[suspend] ready step={token['step']} generation={self.generation}", flush=True)

    def _await_resume(self, folder, token) -> None:
        """Host polling only: wait for this process's resume token (written for this very process:
        same start time), then mark it consumed."""
        mine = folder / f"resume.{os.getpid()}"
        while wait_json(mine, token, self.wait_seconds).get("start_ticks") != self.identity["start_ticks"]:
            time.sleep(self.wait_seconds)
        mine.rename(folder / f"resume.{os.getpid()}.consumed")
