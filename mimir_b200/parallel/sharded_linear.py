"""Projection weights sharded by rows over the GPUs of one node, gathered inside the forward GEMM.

ZeRO-3 sharding (the reference's FSDP2 units, ``src/mimir/training/distributed.py:14-40``) keeps
``1 / world`` of every weight on each rank and all-gathers the rest before the layer's forward
(NCCL all-gather, then the GEMM).  :class:`ShardedLinear` keeps its rows the same way, in memory
that every rank of the node maps (CUDA IPC), and its forward is ONE kernel
(``gemm_allgather``, ``csrc/gemm.cu``): tcgen05 tiles of ``x @ W^T`` that read this rank's rows
locally while gatherer warps pull the other ranks' rows over NVLink into a local copy of the whole
weight; tiles of a peer's columns read that copy once it is complete (or the peer's memory
directly before then).  The copy is kept, so:

* later forwards with the same weights (gradient accumulation) run the plain GEMM on it, and
* the backward's input gradient ``dy @ W`` reads it locally (no second all-gather);
* the weight gradient ``dy^T x`` is reduce-scattered in fp32 with NCCL onto the owners' rows.

Contract: every rank calls :meth:`ShardedLinear.publish` after its rows change (after
construction and after each optimizer step), and the forward reads peers' rows only between two
publishes.  ``publish`` is a one-element all-reduce on the current stream, so no rank's next
forward runs before every rank's update has finished; the backward's reduce-scatter orders every
rank's reads before any rank's next update.

Without CUDA (Gloo tests) the same module all-gathers with ``all_gather_into_tensor`` and runs
``F.linear``.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import Tensor, nn


def _exchange(handle: Tensor, local_ptr: int, group, world: int, rank: int, device: torch.device, opened: list) -> list:
    """Every rank's pointer to one IPC buffer (this rank's own pointer at ``rank``)."""
    from mimir_b200.ops._ext import ext
    C = ext()
    everyone = [bytes(handle.numpy().tobytes())]
    devices = [device.index]
    if world > 1:
        everyone, devices = [None] * world, [None] * world
        dist.all_gather_object(everyone, bytes(handle.numpy().tobytes()), group=group)
        dist.all_gather_object(devices, device.index, group=group)
    out = []
    for k, h in enumerate(everyone):
        if k == rank:
            out.append(local_ptr)
            continue
        if not C.peer_access_possible(device.index, devices[k]):
            raise RuntimeError(f"GPU {device.index} cannot access peer rank {k}")
        ptr = C.ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8), device.index)
        opened.append(ptr)
        out.append(ptr)
    return out


class _GatheredLinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, shard, module):
        ctx.module = module
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        y = module._forward_matrix(x2)
        ctx.save_for_backward(x2)
        ctx.x_shape = x.shape
        return y.view(*x.shape[:-1], y.shape[-1])

    @staticmethod
    def backward(ctx, dy):
        (x2,) = ctx.saved_tensors
        m = ctx.module
        dy2 = dy.reshape(-1, dy.shape[-1])
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            dx = m._input_grad(dy2).view(ctx.x_shape)
        dshard = m._shard_grad(dy2, x2) if ctx.needs_input_grad[1] else None
        return dx, dshard, None


class ShardedLinear(nn.Module):
    """``y = x W^T`` (no bias) with ``W`` [out_features, in_features] sharded by rows over ``group``.

    ``weight`` is the full initial matrix, identical on every rank; each rank keeps rows
    ``[rank * S, (rank + 1) * S)`` (``S = out_features / world``) as the parameter ``shard``.
    On CUDA the weight is bf16; ``out_features`` must be a multiple of 256 and of 128 x world.
    """

    def __init__(self, weight: Tensor, group: Optional[dist.ProcessGroup] = None, device=None):
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        device = torch.device(device) if device is not None else weight.device
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = device
        self.cuda = device.type == "cuda"
        N, K = weight.shape
        if N % self.world:
            raise ValueError(f"{N} rows cannot be split over {self.world} ranks")
        self.out_features, self.in_features = N, K
        S = N // self.world
        rows = weight.detach()[self.rank * S:(self.rank + 1) * S]
        self._opened: list = []
        if self.cuda:
            if N % 256 or N % (128 * self.world) or K % 8:
                raise ValueError("CUDA sharded projections need out_features % 256 == 0, "
                                 "out_features % (128 x world) == 0 and in_features % 8 == 0")
            if self.world > 8:
                raise ValueError("the fused all-gather reads peers of one node (<= 8 ranks)")
            from mimir_b200.ops._ext import ext
            buf, handle = ext().ipc_alloc(S * K * 2, device.index)
            self._storage = buf
            local = buf.view(torch.bfloat16).view(S, K)
            local.copy_(rows.to(device=device, dtype=torch.bfloat16))
            self.shard = nn.Parameter(local)
            self.shard_ptrs = _exchange(handle, local.data_ptr(), group, self.world, self.rank, device, self._opened)
            self.gathered = torch.empty(N, K, dtype=torch.bfloat16, device=device)
            self.flags = torch.zeros(N // 128, dtype=torch.int32, device=device)
        else:
            self.shard = nn.Parameter(rows.to(device).clone())
            self.gathered = torch.empty(N, K, dtype=weight.dtype, device=device)
        self.calls = 0        # fused-kernel launches (the counters' epoch)
        self.version = 0      # publishes seen
        self.gathered_version = -1
        self.publish()

    # ------------------------------------------------------------------ contract
    def publish(self) -> None:
        """Every rank, after its rows changed: orders all updates before any rank's next read."""
        if self.world > 1:
            flag = torch.zeros(1, device=self.device)
            dist.all_reduce(flag, group=self.group)
        self.version += 1

    def close(self) -> None:
        if self.cuda and self._opened:
            from mimir_b200.ops._ext import ext
            for ptr in self._opened:
                ext().ipc_close(ptr, self.device.index)
        self._opened = []

    # ------------------------------------------------------------------ compute
    def _forward_matrix(self, x2: Tensor) -> Tensor:
        if self.gathered_version == self.version:  # the local copy is current: plain GEMM
            if self.cuda:
                from mimir_b200.ops.gemm import mm_nt
                return mm_nt(x2, self.gathered)
            return F.linear(x2, self.gathered)
        self.gathered_version = self.version
        if self.cuda:
            from mimir_b200.ops._ext import ext
            self.calls += 1
            return ext().gemm_allgather(x2, self.shard_ptrs, self.rank, self.gathered, self.flags, self.calls)
        if self.world > 1:
            dist.all_gather_into_tensor(self.gathered, self.shard.detach().contiguous(), group=self.group)
        else:
            self.gathered.copy_(self.shard.detach())
        return F.linear(x2, self.gathered)

    def _input_grad(self, dy2: Tensor) -> Tensor:
        if self.cuda:
            from mimir_b200.ops.gemm import mm_nn
            return mm_nn(dy2, self.gathered)
        return dy2 @ self.gathered

    def _shard_grad(self, dy2: Tensor, x2: Tensor) -> Tensor:
        if self.cuda:
            from mimir_b200.ops.gemm import mm_tn
            full = torch.empty(self.out_features, self.in_features, dtype=torch.float32, device=self.device)
            mm_tn(dy2, x2, out=full)
        else:
            full = (dy2.t().float() @ x2.float())
        if self.world > 1:
            S = self.out_features // self.world
            mine = torch.empty(S, self.in_features, dtype=torch.float32, device=self.device)
            if self.cuda:
                dist.reduce_scatter_tensor(mine, full, group=self.group)
            else:  # Gloo: sum, then this rank's rows
                dist.all_reduce(full, group=self.group)
                mine = full[self.rank * S:(self.rank + 1) * S]
            full = mine
        return full.to(self.shard.dtype)

    def forward(self, x: Tensor) -> Tensor:
        if self.cuda and x.dtype != torch.bfloat16:
            raise TypeError("the CUDA sharded projection computes in bf16")
        return _GatheredLinearFn.apply(x, self.shard, self)

    # ------------------------------------------------------------------ checkpoints
    def _save_to_state_dict(self, destination, prefix, keep_vars):
        """Checkpoints hold the whole matrix as ``weight`` (every rank calls ``state_dict``: it
        all-gathers), so they load at any world size."""
        destination[prefix + "weight"] = self.full_weight()

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        key = prefix + "weight"
        if key not in state_dict:
            missing_keys.append(key)
            return
        full = state_dict[key]
        if tuple(full.shape) != (self.out_features, self.in_features):
            error_msgs.append(f"{key}: shape {tuple(full.shape)} != {(self.out_features, self.in_features)}")
            return
        S = self.out_features // self.world
        with torch.no_grad():
            self.shard.copy_(full[self.rank * S:(self.rank + 1) * S].to(self.shard.dtype))
        self.publish()

    def full_weight(self) -> Tensor:
        """The whole matrix (an all-gather; for checks and export)."""
        out = torch.empty(self.out_features, self.in_features, dtype=self.shard.dtype, device=self.device)
        if self.world > 1:
            dist.all_gather_into_tensor(out, self.shard.detach().contiguous(), group=self.group)
        else:
            out.copy_(self.shard.detach())
        return out
