"""In-loop suspension hook: checkpoint at a requested step, publish readiness, pause for a token.

Reference behaviour: ``src/mimir/training/suspension/runtime.py:11-135``.

Every ``poll_steps`` steps rank 0 claims pending requests and broadcasts them, so all ranks
agree on the queue.  At the first due step all ranks save a checkpoint, finish their
collectives (barrier + device synchronize), release cached device memory, optionally call the
NCCL checkpoint shim, and write ``generation_<n>/ready.<pid>.json``.  Rank 0 waits for every
rank's ready file and publishes ``suspend_ready.json``; an external controller then
checkpoints the processes (``cuda-checkpoint``) and, after restoring them, writes one
``resume.<pid>`` token per process.  From readiness until the token only host polling runs.
"""
from __future__ import annotations

import os
import time
import uuid
from pathlib import Path

from mimir_b200.train.suspension.protocol import atomic_write, claim, process_identity, steps, wait_json


class SuspendHook:
    def __init__(self, root, initial_steps, device, poll_steps: int = 10, wait_seconds: float = 2):
        import torch
        import torch.distributed as dist
        if poll_steps < 1 or wait_seconds <= 0:
            raise ValueError("Suspension poll intervals must be positive")
        self.torch, self.dist, self.device = torch, dist, device
        self.nccl_shim = None
        if os.environ.get("TRAINING_SUSPEND_NCCL_SHIM", os.environ.get("SUSPEND_TEST_NCCL_SHIM")) == "1":
            if device.type != "cuda":
                raise ValueError("NCCL checkpoint shim requires CUDA")
            from mimir_b200.train.suspension.nccl_shim import NcclCheckpointShim
            self.nccl_shim = NcclCheckpointShim()
        self.distributed = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank() if self.distributed else 0
        self.world = dist.get_world_size() if self.distributed else 1
        if int(os.environ.get("LOCAL_WORLD_SIZE", self.world)) != self.world:
            raise ValueError("Suspension supports one node only")
        self.queue = steps(initial_steps)
        self.consumed: set[int] = set()
        self.poll_steps, self.wait_seconds = poll_steps, wait_seconds
        self.generation = 0
        self.job_id = self._broadcast(uuid.uuid4().hex if self.rank == 0 else None)
        self.root = Path(root).resolve() / self.job_id
        self.root.mkdir(parents=True, exist_ok=True)
        self.identity = process_identity() | {"rank": self.rank}
        if device.type == "cuda":
            job_file = os.environ.get("CUDA_CHECKPOINT_JOB_FILE")
            if not job_file:
                raise RuntimeError("Start CUDA-suspendable training through the suspension launcher "
                                   "(python -m mimir_b200.train.suspension.launcher) before CUDA initialises")
            st = os.stat(job_file)
            self.identity["cuda_job"] = [st.st_dev, st.st_ino]
        ranks = [self.identity]
        if self.distributed:
            ranks = [None] * self.world
            dist.all_gather_object(ranks, self.identity)
        if len({r["host"] for r in ranks}) != 1:
            raise ValueError("Ranks must be on one host")
        if device.type == "cuda" and len({tuple(r["cuda_job"]) for r in ranks}) != 1:
            raise ValueError("Ranks did not inherit the same CUDA checkpoint job")
        self.ranks = ranks
        if self.rank == 0:
            atomic_write(self.root / "launch.json", {"job_id": self.job_id, "ranks": ranks,
                                                     "device": device.type, "initial_steps": self.queue})
            self._save_queue()
            print(f"[suspend] control_dir={self.root}", flush=True)
        self._barrier()

    def _broadcast(self, value):
        if not self.distributed:
            return value
        box = [value]
        self.dist.broadcast_object_list(box, src=0)
        return box[0]

    def _barrier(self) -> None:
        if self.distributed:
            self.dist.barrier()
        if self.device.type == "cuda":
            self.torch.cuda.synchronize(self.device)

    def _save_queue(self) -> None:
        atomic_write(self.root / "queue.json", {"pending": self.queue, "consumed": sorted(self.consumed),
                                                "job_id": self.job_id})

    def _poll_requests(self) -> None:
        claimed, values = None, []
        if self.rank == 0:
            try:
                claimed, values = claim(self.root)
            except BlockingIOError:
                pass  # a writer holds the request lock; pick it up at the next poll
            except OSError as error:
                # rank 0 must still reach the broadcast below or its peers wait forever
                print(f"[suspend] request read failed, retrying next poll: {error}", flush=True)
        values = self._broadcast(values)
        self.queue = sorted((set(self.queue) | set(values)) - self.consumed)
        if self.rank == 0:
            self._save_queue()
            if claimed:
                claimed.rename(claimed.with_suffix(".accepted"))

    def after_step(self, step: int, save_checkpoint, stopping: bool = False) -> bool:
        """Return True if training paused (and resumed) at this step."""
        if stopping:
            return False
        if step % self.poll_steps == 0:
            self._poll_requests()
        if not self.queue or self.queue[0] > step:
            return False
        checkpoint = save_checkpoint()
        due = [s for s in self.queue if s <= step]
        self.consumed.update(due)
        self.queue = [s for s in self.queue if s > step]
        self.generation += 1
        token = {"job_id": self.job_id, "generation": self.generation, "step": step}
        gen_dir = self.root / f"generation_{self.generation:06d}"
        gen_dir.mkdir(exist_ok=True)
        self._barrier()  # every collective done before readiness; no device work after this point
        if self.device.type == "cuda":
            self.torch.cuda.empty_cache()
            self.torch.cuda.synchronize(self.device)
        if self.nccl_shim:
            self.nccl_shim.prepare()
        atomic_write(gen_dir / f"ready.{os.getpid()}.json", token | self.identity)
        if self.rank == 0:
            for r in self.ranks:
                wait_json(gen_dir / f"ready.{r['pid']}.json", token, self.wait_seconds, 300)
            self._save_queue()
            atomic_write(self.root / "suspend_ready.json", token | {
                "ranks": self.ranks, "checkpoint": str(checkpoint), "requested_steps": due, "ready_at": time.time()})
            print(f"[suspend] ready step={step} generation={self.generation}", flush=True)
        resume = gen_dir / f"resume.{os.getpid()}"
        while True:
            receipt = wait_json(resume, token, self.wait_seconds)
            if receipt.get("start_ticks") == self.identity["start_ticks"]:
                break
            time.sleep(self.wait_seconds)
        resume.rename(gen_dir / f"resume.{os.getpid()}.consumed")
        if self.nccl_shim:
            self.nccl_shim.restore()
        self._barrier()
        if self.rank == 0:
            atomic_write(self.root / "resumed.json", token)
            print(f"[suspend] resumed step={step} generation={self.generation}", flush=True)
        return True
