"""Expert parallelism: each rank of an expert-parallel group owns ``num_experts / size`` experts.

The reference has no expert parallelism (every rank holds every expert and runs them on its own
tokens, ``src/mimir/model/expert_mixtures.py:73,92-104``).  Here token-slots travel to the rank
that owns their expert and back, through CUDA-IPC buffers that every rank of the group maps
(``csrc/moe.cu``: the dispatch kernel stores rows into the owner's buffer, the combine kernel
loads them back and applies the routing weights).  One-element collectives order the phases.

Route plan (identical arithmetic on every rank, from the all-gathered per-expert counts
``C[source, expert]``): the rows of a destination rank are grouped by its experts in order,
then by source rank, then by token order, so a buffer holds exactly the routed rows — no
capacity factor and no dropped tokens.  Buffers come from a pool whose growth is decided from
``C`` (known to every rank), so all ranks allocate and exchange IPC handles in lockstep.

Without CUDA the same plan runs with ``all_to_all_single`` (Gloo), which the CPU tests use.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor

_ROW_QUANTUM = 4096  # pool buffers grow in whole multiples of this many rows


@dataclass
class RoutePlan:
    rows: Tensor            # int32 [T, k]: row of each token-slot in its destination rank's buffer
    dst: Tensor             # int32 [T, k]: destination rank of each token-slot
    send_counts: list       # rows this rank sends to each rank
    recv_counts: list       # rows this rank receives from each rank
    expert_rows: list       # rows per local expert (receive side, in buffer order)
    expert_rows_dev: Tensor  # the same, int32 on the device (for kernels that schedule on the device)
    capacity: int           # max rows any rank of the group receives
    order: Tensor           # token-slot indices sorted by (expert, token): the send order
    counts: Tensor          # host int64 [W, E]: rows every source rank routes to every expert


class PeerBuffer:
    """A bf16 buffer of ``capacity x width`` elements every rank of the group can address."""

    def __init__(self, ep: "ExpertParallel", capacity: int, width: int):
        self.capacity, self.width = capacity, width
        nbytes = capacity * width * 2
        if ep.cuda and ep.size > 1:
            from mimir_b200.ops._ext import ext
            C = ext()
            self.storage, handle = C.ipc_alloc(nbytes, ep.device.index)
            self.local = self.storage.view(torch.bfloat16)
            self.ptrs = ep.share(handle, self.local)
        else:
            self.local = torch.zeros(capacity * width, dtype=torch.bfloat16, device=ep.device)
            self.ptrs = [self.local.data_ptr()] if ep.cuda else []

    def view(self, offset_rows: int, rows: int, d: int) -> Tensor:
        return self.local[offset_rows * d:(offset_rows + rows) * d].view(rows, d)

    def peer_ptrs(self, offset_rows: int, d: int) -> list:
        return [p + offset_rows * d * 2 for p in self.ptrs]


class ExpertParallel:
    def __init__(self, num_experts: int, device: torch.device, group: Optional[dist.ProcessGroup] = None):
        self.group = group
        self.size = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % self.size:
            raise ValueError(f"{num_experts} experts cannot be split over {self.size} expert-parallel ranks")
        if self.size > 8:
            raise ValueError("Expert parallelism over peer memory supports one node (<= 8 ranks)")
        self.num_experts = num_experts
        self.local = num_experts // self.size
        self.first = self.rank * self.local
        self.device = device
        self.cuda = device.type == "cuda"
        self._pool: list[PeerBuffer] = []
        self._busy: set[int] = set()
        self._opened: list[int] = []

    def owns(self, expert: int) -> bool:
        return self.first <= expert < self.first + self.local

    # ------------------------------------------------------------------ collectives
    def barrier(self) -> None:
        if self.size > 1:
            flag = torch.zeros(1, device=self.device)
            dist.all_reduce(flag, group=self.group)

    def share(self, handle: Tensor, local: Tensor) -> list:
        from mimir_b200.ops._ext import ext
        C = ext()
        everyone = [bytes(handle.numpy().tobytes())]
        if self.size > 1:
            everyone = [None] * self.size
            dist.all_gather_object(everyone, bytes(handle.numpy().tobytes()), group=self.group)
        out = []
        for k, h in enumerate(everyone):
            if k == self.rank:
                out.append(local.data_ptr())
                continue
            ptr = C.ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8), self.device.index)
            self._opened.append(ptr)
            out.append(ptr)
        return out

    def acquire(self, rows: int, width: int) -> PeerBuffer:
        """A free pool buffer with room for ``rows x width`` (every rank calls this in the same order
        with the same arguments, so allocations happen in lockstep)."""
        for i, buf in enumerate(self._pool):
            if i not in self._busy and buf.capacity * buf.width >= rows * width:
                self._busy.add(i)
                return buf
        capacity = -(-max(rows, 1) * width // (_ROW_QUANTUM * width)) * _ROW_QUANTUM
        self._pool.append(PeerBuffer(self, capacity, width))
        self._busy.add(len(self._pool) - 1)
        return self._pool[-1]

    def release(self, buf: PeerBuffer) -> None:
        self._busy.discard(self._pool.index(buf))

    def close(self) -> None:
        if self.cuda and self._opened:
            from mimir_b200.ops._ext import ext
            for ptr in self._opened:
                ext().ipc_close(ptr, self.device.index)
        self._opened, self._pool, self._busy = [], [], set()

    # ------------------------------------------------------------------ route plan
    def plan(self, topi: Tensor) -> RoutePlan:
        T, k = topi.shape
        E, W, L = self.num_experts, self.size, self.local
        flat = topi.reshape(-1)
        counts = torch.bincount(flat, minlength=E).to(torch.int64)
        if W > 1:
            everyone = torch.empty(W * E, dtype=torch.int64, device=counts.device)
            dist.all_gather_into_tensor(everyone, counts, group=self.group)
            C = everyone.view(W, E)
        else:
            C = counts.view(1, E)
        per_dest = C.sum(0).view(W, L)                            # rows per (destination rank, local expert)
        base = (per_dest.cumsum(1) - per_dest).reshape(E)         # first row of each expert at its destination
        src_off = (C.cumsum(0) - C)[self.rank]                    # rows of lower source ranks within each expert
        order = torch.argsort(flat, stable=True)                  # by expert, token order within an expert
        sorted_e = flat[order]
        start = counts.cumsum(0) - counts
        within = torch.arange(flat.numel(), device=flat.device) - start[sorted_e]
        rows = torch.empty_like(flat)
        rows[order] = base[sorted_e] + src_off[sorted_e] + within
        rows_dev = C.sum(0).view(W, L)[self.rank].to(torch.int32)
        host = C.cpu()
        recv_rows = host.sum(0).view(W, L)
        expert_rows = recv_rows[self.rank].tolist()
        send = host[self.rank].view(W, L).sum(1).tolist()
        recv = host.view(W, W, L)[:, self.rank].sum(1).tolist()
        return RoutePlan(rows=rows.view(T, k).to(torch.int32), dst=(flat // L).view(T, k).to(torch.int32),
                         send_counts=send, recv_counts=recv, expert_rows=expert_rows, expert_rows_dev=rows_dev,
                         capacity=int(recv_rows.sum(1).max()), order=order, counts=host)


_GROUPS: dict = {}


class _LocalGroup(ExpertParallel):
    """One rank holding every expert (the grouped dispatch without expert parallelism)."""

    def __init__(self, num_experts: int, device: torch.device):
        self.group, self.size, self.rank = None, 1, 0
        self.num_experts, self.local, self.first = num_experts, num_experts, 0
        self.device, self.cuda = device, device.type == "cuda"
        self._pool, self._busy, self._opened = [], set(), []


def expert_parallel(num_experts: int, device: torch.device, distributed: bool = True) -> ExpertParallel:
    """The process-wide expert-parallel group for ``num_experts`` on ``device``: all ranks of the
    default group when ``distributed``, else this rank alone."""
    key = (num_experts, str(device), distributed and dist.is_initialized())
    if key not in _GROUPS:
        _GROUPS[key] = ExpertParallel(num_experts, device) if key[2] else _LocalGroup(num_experts, device)
    return _GROUPS[key]
