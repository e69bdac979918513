"""Replicated-weight data parallelism with a fused reduce-scatter + AdamATan2 + all-gather step.

Design (one process per GPU).  Every rank keeps the whole model in the compute dtype (bf16)
— a 1.3B-parameter model is 2.6 GB, small next to 180 GB of HBM — so forward and backward
run with no collective at all.  The fp32 master weights and the optimizer slots are sharded
exactly like FSDP2 shards a parameter (dim 0 split in ``ceil(rows / world)`` chunks), so a DCP
checkpoint written here has the same keys, shapes, dtypes and shard placement
(``model.<fqn>``, ``optim.state.<fqn>.{step,exp_avg,exp_avg_sq,param_ema}``, ``Shard(0)``) as one
written by FSDP2, and either can resume the other.

The weights and gradients live in two flat buffers allocated with ``cudaMalloc`` and shared
over CUDA IPC, so each rank can address every peer's buffers over NVLink.  One optimizer step
is one kernel per rank (``csrc/dp_fused.cu``): for the rank's own shard it loads the peers'
bf16 gradients, sums them in fp32, applies AdamATan2 (decoupled weight decay, atan2 update,
first/second moments, EMA) to the fp32 master shard and stores the rounded bf16 weights into
every rank's weight buffer.  A one-element NCCL all-reduce before and after the kernel orders
it with the other ranks: before, every rank's backward is complete; after, every rank's
stores have landed.  NVLink traffic per rank and step is ``(world-1)/world`` of the bf16
gradients in and of the bf16 weights out; there is no fp32 gradient traffic at all.

With global-norm clipping the step is two kernels: a reduce pass that writes the fp32 reduced
gradient shard and per-CTA sums of squares, one scalar all-reduce for the norm, then the
update pass reading the reduced shard with the clip coefficient.

Without clipping the AdamATan2 update overlaps the backward.  The trainable parameters form
buckets (one per transformer block, one per other parameter).  The engine counts the gradient
arrivals of every parameter in a step and notes the order in which the buckets received their
last arrival; once two consecutive steps agree on the counts, it knows how many arrivals make a
parameter's gradient final, and the noted order (rank 0's, on every rank) becomes the firing
order.  During the last micro-batch's backward, a bucket whose parameters have all arrived (and
every bucket before it in that order) is updated on a side stream: an event on the backward stream orders the update after every kernel that read those
weights or wrote those gradients, and on several ranks a one-element all-reduce on the side
stream waits until every rank's backward has passed the bucket.  The optimizer step updates
what is left, joins the side stream and closes with the usual barrier.  A gradient that arrives
for a bucket after its update raised an error (the model's graph changed between steps).

On CPU (tests, Gloo) the same algorithm runs with PyTorch collectives (all-reduce of the
gradients, the reference AdamATan2 arithmetic on the shard, all-gather of the weights).
"""
from __future__ import annotations

import math
import os
from contextlib import contextmanager
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist
from torch import Tensor, nn
from torch.optim.optimizer import Optimizer

_ALIGN = 8  # elements: 16 bytes of bf16, 32 bytes of fp32
_LOCAL_FLAG = 256  # segment kind flag: rank-local parameter (csrc/dp_fused.cu kLocalFlag)


def is_local(p: Tensor) -> bool:
    """A rank-local parameter (an expert owned by this expert-parallel rank): its gradient is
    complete on this rank, so it is neither reduced nor gathered."""
    return bool(getattr(p, "_mimir_rank_local", False))


def _align(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


@dataclass
class ParamSlot:
    fqn: str
    param: nn.Parameter
    shape: torch.Size
    flat: int              # element offset in the flat weight/grad buffers
    numel: int
    rows: int              # dim-0 extent (1 for scalars)
    row0: int              # first owned row
    rows_mine: int         # owned rows (may be 0)
    shard: int             # element offset in the shard buffers
    trainable: bool
    local: bool = False    # rank-local (expert-parallel) parameter: never reduced or gathered

    @property
    def shard_numel(self) -> int:
        return self.rows_mine * (self.numel // self.rows)

    @property
    def shard_flat(self) -> int:
        return self.flat + self.row0 * (self.numel // self.rows)

    def local_shape(self) -> tuple:
        return (self.rows_mine, *self.shape[1:]) if len(self.shape) else (self.rows_mine,)


class ReplicatedEngine:
    def __init__(self, model: nn.Module, *, compute_dtype: torch.dtype, device: torch.device,
                 group: Optional[dist.ProcessGroup] = None):
        self.model, self.device, self.compute_dtype = model, device, compute_dtype
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.cuda = device.type == "cuda"
        if self.cuda and compute_dtype != torch.bfloat16:
            raise ValueError("The fused CUDA step keeps bf16 replicated weights")
        if self.world > 8:
            raise ValueError("The fused step supports one node (<= 8 ranks)")
        self._broadcast_initial_state()
        self.slots = self._layout()
        self.total = self.slots[-1].flat + _align(self.slots[-1].numel) if self.slots else 0
        # Replicated parameters come first (same offsets on every rank); rank-local ones follow.
        self.replicated_total = min((s.flat for s in self.slots if s.local), default=self.total)
        self.shard_total = max((s.shard + _align(s.shard_numel) for s in self.slots), default=0)
        self._allocate()
        self.reduced: Optional[Tensor] = None
        # Parameters that received a gradient since the last zero_grad: like the per-parameter
        # optimizer, a parameter without one (e.g. outside the truncated-BPTT window) is not
        # updated at all (no decay, no moment update, no step count).
        self.touched: set[str] = set()
        self._grads_zero = False  # known to be all zero (set by zero_grad, cleared by an arrival)
        self.arrivals: dict[str, int] = {}
        for s in self.slots:
            if s.trainable:
                s.param.register_post_accumulate_grad_hook(lambda _p, fqn=s.fqn: self._arrived(fqn))
                # Ops that accumulate straight into the gradient view report it here instead.
                s.param._mimir_grad_sink = lambda _p, fqn=s.fqn: self._arrived(fqn)
        self.buckets = self._buckets()
        self._bucket_of = {s.fqn: b for b, bucket in enumerate(self.buckets) for s in bucket}
        self.order = list(range(len(self.buckets)))  # firing order (learned)
        self._position = {b: i for i, b in enumerate(self.order)}
        self._last_arrival: dict[int, int] = {}  # bucket -> sequence number of its latest arrival
        self.overlap_enabled = os.environ.get("MIMIR_OVERLAP_UPDATE", "1") != "0"
        self.expected: Optional[dict[str, int]] = None  # arrivals per parameter in one step
        self.overlap_ready: Optional[bool] = None  # decided (the same on every rank) after learning
        self._learn_steps = 0
        self._arrival_seq = 0
        self._armed = None  # the optimizer updating bucket by bucket during this backward
        self._next = 0  # next bucket to update, in bucket order
        self._late: Optional[str] = None
        self._side = None
        self._compute = None

    # ------------------------------------------------------------------ setup
    @torch.no_grad()
    def _broadcast_initial_state(self) -> None:
        if self.world == 1:
            return
        for t in [p for p in self.model.parameters() if not is_local(p)] + list(self.model.buffers()):
            dist.broadcast(t.data, src=dist.get_global_rank(self.group, 0) if self.group else 0, group=self.group)

    def _layout(self) -> list[ParamSlot]:
        slots, flat, shard = [], 0, 0
        named = list(self.model.named_parameters())
        for fqn, p in [x for x in named if not is_local(x[1])] + [x for x in named if is_local(x[1])]:
            rows = p.shape[0] if p.dim() > 0 else 1
            chunk = rows if is_local(p) else math.ceil(rows / self.world)
            row0 = 0 if is_local(p) else min(rows, self.rank * chunk)
            mine = max(0, min(rows, row0 + chunk) - row0)
            slot = ParamSlot(fqn, p, p.shape, flat, p.numel(), rows, row0, mine, shard, p.requires_grad, is_local(p))
            slots.append(slot)
            flat += _align(p.numel())
            shard += _align(slot.shard_numel)
        return slots

    @torch.no_grad()
    def _allocate(self) -> None:
        nbytes = self.total * self.compute_dtype.itemsize
        if self.cuda:
            from mimir_b200.ops._ext import ext
            C = ext()
            wbuf, whandle = C.ipc_alloc(nbytes, self.device.index)
            gbuf, ghandle = C.ipc_alloc(nbytes, self.device.index)
            self._keep = (wbuf, gbuf)
            self.weights = wbuf.view(self.compute_dtype)
            self.grads = gbuf.view(self.compute_dtype)
            self._open_peers(whandle, ghandle)
        else:
            self.weights = torch.zeros(self.total, dtype=self.compute_dtype)
            self.grads = torch.zeros(self.total, dtype=self.compute_dtype)
        f32 = dict(dtype=torch.float32, device=self.device)
        self.master = torch.zeros(self.shard_total, **f32)
        for s in self.slots:
            full = s.param.detach().to(torch.float32).reshape(s.rows, -1)
            self.master[s.shard:s.shard + s.shard_numel] = full[s.row0:s.row0 + s.rows_mine].reshape(-1)
            self.weights[s.flat:s.flat + s.numel] = s.param.detach().reshape(-1).to(self.compute_dtype)
            s.param.data = self.weights[s.flat:s.flat + s.numel].view(s.shape)
            if s.trainable:
                s.param.grad = self.grads[s.flat:s.flat + s.numel].view(s.shape)

    def _open_peers(self, whandle: Tensor, ghandle: Tensor) -> None:
        self._opened = []
        self.peer_weights, self.peer_grads = self._share([whandle, ghandle], [self.weights, self.grads])

    def _share(self, handles: list, locals_: list) -> list:
        """Exchange CUDA IPC handles with every rank; per handle, the list of every rank's pointer."""
        from mimir_b200.ops._ext import ext
        C = ext()
        mine = tuple(bytes(h.numpy().tobytes()) for h in handles)
        everyone = [mine]
        devices = [self.device.index]
        if self.world > 1:
            everyone, devices = [None] * self.world, [None] * self.world
            dist.all_gather_object(everyone, mine, group=self.group)
            dist.all_gather_object(devices, self.device.index, group=self.group)
        out = [[] for _ in handles]
        for k, theirs in enumerate(everyone):
            if k != self.rank and not C.peer_access_possible(self.device.index, devices[k]):
                raise RuntimeError(f"GPU {self.device.index} cannot access peer rank {k} over NVLink/PCIe")
            for j, h in enumerate(theirs):
                if k == self.rank:
                    out[j].append(locals_[j].data_ptr())
                    continue
                ptr = C.ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8), self.device.index)
                self._opened.append(ptr)
                out[j].append(ptr)
        return out

    def shared_buffer(self, nbytes: int) -> tuple[Tensor, list]:
        """A zeroed device buffer every rank can address: (this rank's uint8 tensor, all ranks' pointers)."""
        if not self.cuda:
            return torch.zeros(nbytes, dtype=torch.uint8), []
        from mimir_b200.ops._ext import ext
        buf, handle = ext().ipc_alloc(max(nbytes, 32), self.device.index)
        self._keep = self._keep + (buf,)
        return buf, self._share([handle], [buf])[0]

    def close(self) -> None:
        if self.cuda and getattr(self, "_opened", None):
            from mimir_b200.ops._ext import ext
            for ptr in self._opened:
                ext().ipc_close(ptr, self.device.index)
            self._opened = []

    def _buckets(self) -> list[list[ParamSlot]]:
        """Trainable slots grouped by transformer block (the name up to its first integer
        component, e.g. ``model.layers.3``); every other parameter is a bucket of its own."""
        groups: dict[str, list[ParamSlot]] = {}
        for s in self.slots:
            if not s.trainable:
                continue
            parts = s.fqn.split(".")
            key = next((".".join(parts[:i + 1]) for i, part in enumerate(parts) if part.isdigit()), s.fqn)
            groups.setdefault(key, []).append(s)
        return list(groups.values())[::-1]

    # ------------------------------------------------------------------ update overlapped with the backward
    def _arrived(self, fqn: str) -> None:
        self._grads_zero = False
        self.touched.add(fqn)
        n = self.arrivals.get(fqn, 0)
        self.arrivals[fqn] = n + 1
        b = self._bucket_of[fqn]
        if self.expected is not None:  # slots of the bucket whose count equals the expectation
            e = self.expected.get(fqn, 0)
            if n == e:
                self._done[b] -= 1
            elif n + 1 == e:
                self._done[b] += 1
        self._arrival_seq += 1
        self._last_arrival[b] = self._arrival_seq
        if self._armed is None:
            return
        if self._position[b] < self._next:
            self._late = self._late or fqn
            return
        while self._next < len(self.order) and self._bucket_final(self.order[self._next]):
            self._fire(self.order[self._next])
            self._next += 1

    def _bucket_final(self, b: int) -> bool:
        # every slot's arrival count equals the learned one (kept per arrival: O(1) here, where a
        # scan of the bucket per arrival cost O(slots^2) per MoE block)
        return self._done[b] == len(self.buckets[b])

    def _fire(self, b: int) -> None:
        slots = [s for s in self.buckets[b] if s.fqn in self.touched]
        if not slots and self.world == 1:
            return  # (on several ranks every rank still takes the bucket's barrier)
        if not self.cuda:
            self._armed.update_slots(slots)
            return
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(self.device))
        self._side.wait_event(ready)
        with torch.cuda.stream(self._side):
            self._armed.update_slots(slots, lean=True)

    @contextmanager
    def compute_stream(self):
        """Run the forward and backward on a high-priority stream (when the overlap is enabled):
        the block scheduler then hands a freed SM to a waiting backward CTA before a pending CTA of
        the update, which runs on a default-priority side stream.  The caller's stream waits for
        the compute stream on exit."""
        if not (self.cuda and self.overlap_enabled):
            yield
            return
        if self._compute is None:
            self._compute = torch.cuda.Stream(self.device, priority=-100)  # clamped to the highest
        outer = torch.cuda.current_stream(self.device)
        self._compute.wait_stream(outer)
        try:
            with torch.cuda.stream(self._compute):
                yield
        finally:
            outer.wait_stream(self._compute)

    def arm_overlap(self, optimizer) -> bool:
        """Before the last micro-batch's backward: update buckets as their gradients become final.
        Needs an optimizer whose ``update_slots`` works per bucket and arrival counts that two
        steps agreed on."""
        if not (self.overlap_enabled and self.overlap_ready and getattr(optimizer, "bucket_updates", False)
                and self.reduced is None):
            return False
        if self.cuda and self._side is None:
            self._side = torch.cuda.Stream(self.device)
        self._armed, self._next, self._late = optimizer, 0, None
        return True

    def disarm_overlap(self) -> None:
        self._armed = None

    def overlap_armed(self) -> bool:
        return self._armed is not None

    def finish_overlap(self) -> None:
        """Optimizer step after an armed backward: update the remaining buckets, join the side
        stream, then the closing barrier (every rank's weight stores have landed)."""
        try:
            while self._next < len(self.order):
                self._fire(self.order[self._next])
                self._next += 1
        finally:
            self._armed = None
        if self.cuda:
            torch.cuda.current_stream(self.device).wait_stream(self._side)
        self.barrier()
        if self._late is not None:
            raise RuntimeError(f"A gradient of {self._late} arrived after its bucket was updated: the model's "
                               "backward changed between steps (set MIMIR_OVERLAP_UPDATE=0 for such models)")

    def learn_arrivals(self) -> None:
        """After an optimizer step: this step's arrival counts become the expectation.  Until the
        overlap is decided, the order in which the buckets received their last arrival becomes
        the firing order (rank 0's on every rank, so all ranks take their per-bucket barriers in
        the same order), and the overlap is switched on once two consecutive steps agree on
        counts and order on every rank (off for good after 8 steps without agreement).  The
        decision takes two collectives per learning step and none afterwards."""
        same_counts = self.arrivals == self.expected
        self.expected = dict(self.arrivals)
        self._done_start = [sum(1 for s in bucket if self.expected.get(s.fqn, 0) == 0) for bucket in self.buckets]
        self._done = [len(bucket) for bucket in self.buckets]  # now every count equals the expectation
        if self.overlap_ready is not None or not self.overlap_enabled:
            return
        self._learn_steps += 1
        last = self._last_arrival
        order = sorted(range(len(self.buckets)), key=lambda b: (b not in last, last.get(b, 0), b))
        if self.world > 1:
            box = [order]
            dist.broadcast_object_list(box, src=dist.get_global_rank(self.group, 0) if self.group else 0,
                                       group=self.group)
            order = box[0]
            flag = torch.tensor([float(same_counts)], device=self.device)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
            same_counts = bool(flag.item())
        agreed = same_counts and order == self.order
        self.order = order
        self._position = {b: i for i, b in enumerate(order)}
        if agreed:
            self.overlap_ready = True
        elif self._learn_steps >= 8:
            self.overlap_ready = False

    # ------------------------------------------------------------------ step plumbing
    def zero_grad(self) -> None:
        # Gradients reach the buffer only through arrivals (accumulation hooks and sinks), so a
        # buffer that saw none since it was last zeroed is still zero (training zeroes it both
        # after a step and before the next one; the second is free).
        if not self._grads_zero:
            if self.cuda:
                from mimir_b200.ops._ext import ext
                ext().zero_bytes(self.grads)
            else:
                self.grads.zero_()
            self._grads_zero = True
        self.touched.clear()
        self.arrivals.clear()
        if self.expected is not None:
            self._done = list(self._done_start)
        self._last_arrival.clear()
        self._arrival_seq = 0

    def barrier(self) -> None:
        if self.world == 1:
            return
        flag = torch.zeros(1, device=self.device)
        dist.all_reduce(flag, group=self.group)

    def segments(self, lrs: dict, wds: dict, bc1: dict, bc2_sqrt: dict, extra: Optional[dict] = None
                 ) -> tuple[Tensor, int]:
        """Packed device segment table: one entry per owned, non-empty shard of every parameter
        named in ``lrs`` (per-parameter learning rate, weight decay and bias corrections).
        ``extra`` maps a name to ``(kind, dst, dst_rank, has_m)`` for the non-AdamATan2 kinds
        (1 Adam with eps, 2 Muon gather to the owner's workspace offset ``dst``, 3 Muon apply)."""
        from mimir_b200.ops._ext import ext
        C = ext()
        chunk = C.dp_chunk_elements()
        rows, block = [], 0
        for s in self.slots:
            if s.fqn not in lrs or s.shard_numel == 0:
                continue
            n = s.shard_numel
            kind, dst, dst_rank, has_m = (extra or {}).get(s.fqn, (0, 0, 0, 1))
            kind |= _LOCAL_FLAG if s.local else 0
            vec = int(s.shard_flat % 8 == 0 and s.shard % 8 == 0 and n % 8 == 0 and dst % 8 == 0)
            rows.append((s.shard_flat, s.shard, n, block, lrs[s.fqn], wds[s.fqn], bc1[s.fqn], bc2_sqrt[s.fqn], vec,
                         kind, dst, dst_rank, has_m))
            block += (n + chunk - 1) // chunk
        dt = np.dtype([("flat", "<i8"), ("shard", "<i8"), ("n", "<i8"), ("block", "<i8"), ("lr", "<f4"),
                       ("wd", "<f4"), ("bc1", "<f4"), ("bc2", "<f4"), ("vec", "<i4"), ("kind", "<i4"),
                       ("dst", "<i8"), ("dst_rank", "<i4"), ("has_m", "<i4")])
        assert dt.itemsize == C.dp_segment_bytes()
        table = np.array(rows, dtype=dt)
        host = torch.from_numpy(table.view(np.uint8).copy())
        return host.pin_memory().to(self.device, non_blocking=True), block

    @torch.no_grad()
    def reduce_for_clipping(self) -> Tensor:
        """Reduce the gradients of this rank's shards into ``self.reduced``; return the global sum of squares."""
        if self.cuda:
            from mimir_b200.ops._ext import ext
            self.barrier()
            zero = {s.fqn: 0.0 for s in self.slots if s.trainable}
            table, blocks = self.segments(zero, zero, zero, zero)
            self.reduced = torch.empty(self.shard_total, dtype=torch.float32, device=self.device)
            partial = torch.empty(max(blocks, 1), dtype=torch.float32, device=self.device)
            ext().dp_reduce(self.peer_grads, table, blocks, self.reduced, partial, self.rank)
            total = partial[:blocks].double().sum().reshape(1)
        else:
            full = self.summed_grads()
            self.reduced = torch.zeros(self.shard_total, dtype=torch.float32)
            for s in self.slots:
                if s.trainable and s.shard_numel:
                    self.reduced[s.shard:s.shard + s.shard_numel] = full[s.shard_flat:s.shard_flat + s.shard_numel]
            total = self.reduced.double().square().sum().reshape(1)
        if self.world > 1:
            dist.all_reduce(total, group=self.group)
        return total

    def summed_grads(self, slots: Optional[list] = None) -> Tensor:
        """fp32 gradients summed over the ranks (rank-local parameters keep their own); with
        ``slots``, only their ranges are reduced."""
        full = self.grads.to(torch.float32)
        if self.world > 1:
            if slots is None:
                dist.all_reduce(full[:self.replicated_total], group=self.group)
            else:
                for s in slots:
                    if not s.local:
                        dist.all_reduce(full[s.flat:s.flat + s.numel], group=self.group)
        return full

    @torch.no_grad()
    def gather_weights(self, slots: Optional[list] = None) -> None:
        """Rebuild every rank's replicated weights from the master shards (after a load)."""
        for s in self.slots if slots is None else slots:
            local = self.master[s.shard:s.shard + s.shard_numel].to(self.compute_dtype)
            if self.world == 1 or s.local:
                self.weights[s.shard_flat:s.shard_flat + s.shard_numel] = local
                continue
            chunk = math.ceil(s.rows / self.world) * (s.numel // s.rows)
            padded = torch.zeros(chunk, dtype=self.compute_dtype, device=self.device)
            padded[:local.numel()] = local
            out = torch.empty(chunk * self.world, dtype=self.compute_dtype, device=self.device)
            dist.all_gather_into_tensor(out, padded, group=self.group)
            self.weights[s.flat:s.flat + s.numel] = out[:s.numel]

    # ------------------------------------------------------------------ checkpoint views
    def mesh(self):
        from torch.distributed.device_mesh import init_device_mesh
        if getattr(self, "_mesh", None) is None:
            if not dist.is_initialized():  # single process: DTensor views need a 1-rank group
                dist.init_process_group("nccl" if self.cuda else "gloo", store=dist.HashStore(), rank=0, world_size=1)
            self._mesh = init_device_mesh(self.device.type, (self.world,))
        return self._mesh

    def shard_dtensor(self, s: ParamSlot, buffer: Tensor):
        """The shard of ``s`` in ``buffer`` as a ``Shard(0)`` DTensor (a rank-local parameter: the plain
        full tensor, which only its owner rank saves and loads)."""
        from torch.distributed.tensor import DTensor, Shard
        local = buffer[s.shard:s.shard + s.shard_numel].view(s.local_shape())
        if s.local:
            return local
        full_stride = torch.empty(s.shape, device="meta").stride()
        return DTensor.from_local(local, self.mesh(), [Shard(0)], run_check=False, shape=s.shape, stride=full_stride)


class ReplicatedAdamATan2(Optimizer):
    """AdamATan2 over a :class:`ReplicatedEngine` (same slots and group keys as ``AdamATan2``)."""

    def __init__(self, engine: ReplicatedEngine, lr: float = 1e-3, betas=(0.9, 0.95), weight_decay: float = 0.1,
                 ema: Optional[float] = None, ema_dtype=None, parameter_lr_scales: Optional[dict] = None):
        params = [s.param for s in engine.slots if s.trainable]
        defaults = dict(lr=lr, betas=betas, weight_decay=weight_decay, ema=ema,
                        ema_dtype=None if ema_dtype is None else str(ema_dtype).removeprefix("torch."))
        super().__init__(params, defaults)
        self.engine = engine
        self.parameter_lr_scales = parameter_lr_scales
        self.grad_scale: Optional[Tensor] = None
        f32 = dict(dtype=torch.float32, device=engine.device)
        n = engine.shard_total
        self.exp_avg = torch.zeros(n, **f32) if betas[0] > 0 else None
        self.exp_avg_sq = torch.zeros(n, **f32)
        self.ema = engine.master.clone() if ema is not None else None
        for s in engine.slots:
            if s.trainable:
                self.state[s.param]["step"] = torch.tensor(0.0)

    def zero_grad(self, set_to_none: bool = True) -> None:  # noqa: ARG002 - gradients are views
        self.engine.zero_grad()

    def _lr(self, group, p) -> float:
        lr = group["lr"]
        return float(lr * self.parameter_lr_scales[p]) if self.parameter_lr_scales is not None else float(lr)

    bucket_updates = True  # the update of one set of parameters does not depend on the others

    @torch.no_grad()
    def step(self, closure=None):
        if closure is not None:
            raise ValueError("Closures are not supported")
        if getattr(self, "shared_parameter_updates", None):
            raise ValueError("Shared gate-donor updates are not supported by the replicated engine")
        eng = self.engine
        try:
            if eng.overlap_armed():
                eng.finish_overlap()
            else:
                self.update_slots([s for s in eng.slots if s.trainable and s.fqn in eng.touched], closing=True)
        finally:
            eng.reduced = None
            self.grad_scale = None
        eng.learn_arrivals()

    @torch.no_grad()
    def update_slots(self, slots: list, closing: bool = False, lean: bool = False) -> None:
        """AdamATan2 for the touched trainable ``slots``: one fused kernel on the current stream,
        after a barrier on several ranks (their gradients for these slots are final); ``closing``
        adds the barrier after it (every rank's weight stores have landed); ``lean`` selects the
        kernel variant that runs beside the backward's kernels."""
        eng = self.engine
        (group,) = self.param_groups
        b1, b2 = group["betas"]
        lrs, wds, bc1, bc2_sqrt = {}, {}, {}, {}
        corrections: dict = {}  # step value -> (bc1, sqrt(bc2)); parameters almost always share one
        for s in slots:
            st = self.state[s.param]
            st["step"] += 1
            lrs[s.fqn] = self._lr(group, s.param)
            wds[s.fqn] = float(group["weight_decay"])
            key = float(st["step"])
            if key not in corrections:
                # bias corrections exactly as the per-parameter optimizer forms them (fp32 tensors)
                corrections[key] = ((1 - b1 ** st["step"]) if self.exp_avg is not None else torch.tensor(1.0),
                                    (1 - b2 ** st["step"]).sqrt())
            bc1[s.fqn], bc2_sqrt[s.fqn] = corrections[key]
        ema = group["ema"]
        if eng.cuda:
            from mimir_b200.ops._ext import ext
            table, blocks = eng.segments(lrs, wds, {k: float(v) for k, v in bc1.items()},
                                         {k: float(v) for k, v in bc2_sqrt.items()})
            if eng.reduced is None:
                eng.barrier()  # every rank's backward has finished writing these gradients
            ext().dp_step(eng.peer_grads, eng.peer_weights, table, blocks, eng.master, self.exp_avg, self.exp_avg_sq,
                          self.ema, eng.reduced, self.grad_scale, b1, b2, ema if ema is not None else 0.0, [], eng.rank,
                          lean)
            if closing:
                eng.barrier()  # every rank's weight stores have landed
        else:
            self._step_cpu(lrs, wds, bc1, bc2_sqrt, b1, b2, ema, None if closing else slots)

    def _step_cpu(self, lrs: dict, wds: dict, bc1: dict, bc2_sqrt: dict, b1, b2, ema, slots=None) -> None:
        eng = self.engine
        if eng.reduced is None:
            full = eng.summed_grads(slots)
        scale = self.grad_scale if self.grad_scale is not None else None
        for s in eng.slots:
            if s.fqn not in lrs or s.shard_numel == 0:
                continue
            sl = slice(s.shard, s.shard + s.shard_numel)
            g = (eng.reduced[sl] if eng.reduced is not None
                 else full[s.shard_flat:s.shard_flat + s.shard_numel]).clone()
            if scale is not None:
                g = g * scale
            w, v = eng.master[sl], self.exp_avg_sq[sl]
            lr = lrs[s.fqn]
            if wds[s.fqn] != 0:
                w.mul_(1 - lr * wds[s.fqn])
            v.mul_(b2).addcmul_(g, g, value=1 - b2)
            denom = v.sqrt() / bc2_sqrt[s.fqn]
            if self.exp_avg is not None:
                m = self.exp_avg[sl]
                m.lerp_(g, 1 - b1)
                w.add_(torch.atan2(m, denom), alpha=-(lr / bc1[s.fqn]))
            else:
                w.add_(torch.atan2(g, denom), alpha=-lr)
            if self.ema is not None:
                self.ema[sl].lerp_(w, 1 - ema)
        eng.gather_weights(slots)

    # ------------------------------------------------------------------ checkpoint views
    def slot_buffers(self, s: ParamSlot) -> dict:
        """Optimizer slot name -> the shard buffer holding it, for parameter slot ``s``."""
        out = {"exp_avg": self.exp_avg} if self.exp_avg is not None else {}
        out["exp_avg_sq"] = self.exp_avg_sq
        return out | ({"param_ema": self.ema} if self.ema is not None else {})

    def dcp_state(self) -> dict:
        """``get_optimizer_state_dict``-shaped optimizer state with ``Shard(0)`` DTensor slots."""
        eng = self.engine
        state = {}
        for s in eng.slots:
            if not s.trainable:
                continue
            entry = {"step": self.state[s.param]["step"]}
            if self.exp_avg is not None:
                entry["exp_avg"] = eng.shard_dtensor(s, self.exp_avg)
            entry["exp_avg_sq"] = eng.shard_dtensor(s, self.exp_avg_sq)
            if self.ema is not None:
                entry["param_ema"] = eng.shard_dtensor(s, self.ema)
            state[s.fqn] = entry
        groups = [{k: v for k, v in g.items() if k != "params"} | {"params": [s.fqn for s in eng.slots if s.trainable]}
                  for g in self.param_groups]
        return {"state": state, "param_groups": groups}

    def load_dcp_state(self, loaded: dict) -> None:
        """Adopt ``param_groups`` hyper-parameters and the ``step`` counters after a DCP load
        (the slot tensors were loaded in place into the shard buffers)."""
        for s in self.engine.slots:
            if s.trainable and s.fqn in loaded["state"]:
                step = loaded["state"][s.fqn]["step"]
                self.state[s.param]["step"] = step.detach().clone() if torch.is_tensor(step) else torch.tensor(float(step))
        for group, saved in zip(self.param_groups, loaded.get("param_groups", [])):
            for key, value in saved.items():
                if key != "params":
                    group[key] = value


class ReplicatedMuonAdamW(ReplicatedAdamATan2):
    """MuonAdamW over a :class:`ReplicatedEngine`: Muon (Newton-Schulz orthogonalised momentum)
    for the hidden matrices, Adam (eps 1e-8) for everything else, with the state slots
    (``momentum_buffer`` / ``exp_avg`` / ``exp_avg_sq`` / ``param_ema``) and group keys of
    :class:`mimir_b200.optim.muon.MuonAdamW`, so checkpoints interchange with the FSDP2 path.

    Reference behaviour: ``src/mimir/model/muon.py:62-108``, where every rank all-gathers every
    matrix and runs the same Newton-Schulz chain.  Here each matrix has one owner rank (greedy
    balance of the Newton-Schulz FLOPs) holding an fp32 workspace that every rank can address,
    and one step is:

    1. fused kernel, every rank over its ``Shard(0)`` rows: peer-load and sum the bf16 gradients;
       Adam for the non-matrix parameters (new bf16 weights stored to every rank); for each Muon
       matrix the momentum update on the fp32 shard, with the Nesterov input stored straight into
       the owner's workspace (the gather);
    2. every owner orthogonalises its matrices in place, batched over equal-shape logical pieces,
       so each matrix is orthogonalised once per job instead of once per rank;
    3. fused kernel: every rank peer-loads its rows of the orthogonalised matrices from their
       owners, applies decoupled decay, the update and the EMA to its fp32 master shard and stores
       the bf16 weights to every rank (the scatter and the all-gather).

    One-element all-reduces order the phases.  Without CUDA the same algorithm runs with
    PyTorch collectives.
    """

    bucket_updates = False  # a Muon matrix needs every rank's rows before its owner orthogonalises it

    def __init__(self, engine: ReplicatedEngine, *, momentum: float = 0.95, ns_steps: int = 5,
                 muon_lr_scale: float = 1.0, **kwargs):
        from mimir_b200.optim.muon import matrix_splits
        if not 0 <= momentum < 1 or ns_steps < 1 or muon_lr_scale <= 0:
            raise ValueError("Invalid Muon momentum, iterations or LR scale")
        if any(s.local for s in engine.slots):
            raise ValueError("MuonAdamW on the replicated engine does not support expert-parallel parameters")
        super().__init__(engine, **kwargs)
        for group in self.param_groups:
            group.update(optimizer_kind="muon_adamw", muon_momentum=momentum, muon_ns_steps=ns_steps,
                         muon_lr_scale=muon_lr_scale)
        self.has_m = self.exp_avg is not None
        if self.exp_avg is None:  # the Muon momentum lives in the first-moment buffer
            self.exp_avg = torch.zeros(engine.shard_total, dtype=torch.float32, device=engine.device)
        self.splits = {s.fqn: matrix_splits(s.fqn, s.param) for s in engine.slots if s.trainable}
        self.owner, self.work_offset, sizes = self._assign_owners()
        self.work_buf, self.peer_work = engine.shared_buffer(4 * max(sizes, default=0))
        self.work = self.work_buf.view(torch.float32)

    def _assign_owners(self):
        def cost(s):
            rows, cols = s.rows // self.splits[s.fqn], s.numel // s.rows
            m, n = min(rows, cols), max(rows, cols)
            return self.splits[s.fqn] * (2 * m * m * n + m ** 3)
        world = self.engine.world
        matrices = [s for s in self.engine.slots if self.splits.get(s.fqn)]
        load, owner, offset, sizes = [0] * world, {}, {}, [0] * world
        for s in sorted(matrices, key=cost, reverse=True):  # stable: ties keep model order
            k = min(range(world), key=lambda r: (load[r], r))
            load[k] += cost(s)
            owner[s.fqn], offset[s.fqn] = k, sizes[k]
            sizes[k] += _align(s.numel)
        return owner, offset, sizes

    def slot_buffers(self, s: ParamSlot) -> dict:
        if self.splits.get(s.fqn):
            out = {"momentum_buffer": self.exp_avg}
        else:
            out = ({"exp_avg": self.exp_avg} if self.has_m else {}) | {"exp_avg_sq": self.exp_avg_sq}
        return out | ({"param_ema": self.ema} if self.ema is not None else {})

    @torch.no_grad()
    def step(self, closure=None):
        if closure is not None:
            raise ValueError("Closures are not supported")
        if getattr(self, "shared_parameter_updates", None):
            raise ValueError("Shared gate-donor updates are not supported by the replicated engine")
        eng = self.engine
        (group,) = self.param_groups
        b1, b2 = group["betas"]
        beta, wd = float(group["muon_momentum"]), float(group["weight_decay"])
        first = {"lr": {}, "wd": {}, "bc1": {}, "bc2": {}, "extra": {}}
        second = {"lr": {}, "wd": {}, "bc1": {}, "bc2": {}, "extra": {}}
        owned, corrections = [], {}
        for s in eng.slots:
            if not s.trainable or s.fqn not in eng.touched:
                continue
            st = self.state[s.param]
            st["step"] += 1
            lr = self._lr(group, s.param)
            if self.splits.get(s.fqn):
                dst = self.work_offset[s.fqn] + s.row0 * (s.numel // s.rows)
                k = self.owner[s.fqn]
                for table, entry in ((first, (0.0, 0.0, beta, 1.0, (2, dst, k, 0))),
                                     (second, (lr * group["muon_lr_scale"], wd, 1.0, 1.0, (3, dst, k, 0)))):
                    for key, value in zip(("lr", "wd", "bc1", "bc2", "extra"), entry):
                        table[key][s.fqn] = value
                if k == eng.rank:
                    owned.append(s)
            else:
                first["lr"][s.fqn], first["wd"][s.fqn] = lr, wd
                key = float(st["step"])
                if key not in corrections:
                    corrections[key] = (float(1 - b1 ** st["step"]) if self.has_m else 1.0,
                                        float(1 - b2 ** st["step"]))
                first["bc1"][s.fqn], first["bc2"][s.fqn] = corrections[key]
                first["extra"][s.fqn] = (1, 0, 0, int(self.has_m))
        ema = group["ema"]
        if not eng.cuda:
            self._step_cpu_muon(first, second, owned, group)
        else:
            from mimir_b200.ops._ext import ext
            C = ext()
            ema_decay = ema if ema is not None else 0.0
            if eng.reduced is None:
                eng.barrier()  # every rank's backward has finished writing its gradients
            table, blocks = eng.segments(first["lr"], first["wd"], first["bc1"], first["bc2"], first["extra"])
            C.dp_step(eng.peer_grads, eng.peer_weights, table, blocks, eng.master, self.exp_avg, self.exp_avg_sq,
                      self.ema, eng.reduced, self.grad_scale, b1, b2, ema_decay, self.peer_work, eng.rank, False)
            eng.barrier()  # every shard of every matrix has reached its owner
            self._orthogonalise(owned, group["muon_ns_steps"])
            eng.barrier()  # every owner has finished
            table, blocks = eng.segments(second["lr"], second["wd"], second["bc1"], second["bc2"], second["extra"])
            C.dp_step(eng.peer_grads, eng.peer_weights, table, blocks, eng.master, self.exp_avg, self.exp_avg_sq,
                      self.ema, None, None, b1, b2, ema_decay, self.peer_work, eng.rank, False)
            eng.barrier()  # every rank's weight stores have landed
        eng.reduced = None
        self.grad_scale = None

    def _matrix(self, s: ParamSlot) -> Tensor:
        off = self.work_offset[s.fqn]
        return self.work[off:off + s.numel].view(s.rows, -1)

    def _orthogonalise(self, owned: list, steps: int) -> None:
        """Newton-Schulz in place on this rank's matrices, batched over equal-shape logical pieces."""
        from mimir_b200.optim.muon import orthogonalize
        from mimir_b200.optim.newton_schulz import orthogonalize_pieces_, tensor_core_ns_enabled
        by_shape: dict = {}
        for s in owned:
            for piece in self._matrix(s).chunk(self.splits[s.fqn], dim=0):
                by_shape.setdefault(tuple(piece.shape), []).append(piece)
        for (rows, cols), pieces in by_shape.items():
            scale = math.sqrt(max(1, rows / cols))
            if tensor_core_ns_enabled(pieces[0]):
                orthogonalize_pieces_(pieces, steps, scale)  # batched bf16 tcgen05 chain
                continue
            out = orthogonalize(torch.stack(pieces), steps) * scale
            for piece, o in zip(pieces, out):
                piece.copy_(o)

    def _step_cpu_muon(self, first: dict, second: dict, owned: list, group) -> None:
        eng = self.engine
        b1, b2 = group["betas"]
        ema = group["ema"]
        if eng.reduced is None:
            full = eng.summed_grads()
        for s in eng.slots:
            if s.fqn not in first["lr"]:
                continue
            sl = slice(s.shard, s.shard + s.shard_numel)
            g = (eng.reduced[sl] if eng.reduced is not None else full[s.shard_flat:s.shard_flat + s.shard_numel]).clone()
            if self.grad_scale is not None:
                g = g * self.grad_scale
            w = eng.master[sl]
            if self.splits.get(s.fqn):
                mom = self.exp_avg[sl]
                mom.lerp_(g, 1 - group["muon_momentum"])
                matrix = torch.zeros(s.rows, s.numel // s.rows)
                matrix[s.row0:s.row0 + s.rows_mine] = g.lerp(mom, group["muon_momentum"]).view(s.local_shape())
                if eng.world > 1:
                    dist.all_reduce(matrix, group=eng.group)  # disjoint rows: the gather
                if self.owner[s.fqn] == eng.rank:  # the workspace holds only the owner's matrices
                    self._matrix(s).copy_(matrix)
                continue
            lr, wd = first["lr"][s.fqn], first["wd"][s.fqn]
            if self.has_m:
                self.exp_avg[sl].lerp_(g, 1 - b1)
                num = self.exp_avg[sl] / first["bc1"][s.fqn]
            else:
                num = g
            self.exp_avg_sq[sl].lerp_(g.square(), 1 - b2)
            upd = num / ((self.exp_avg_sq[sl] / first["bc2"][s.fqn]).sqrt() + 1e-8)
            w.mul_(1 - lr * wd).add_(upd, alpha=-lr)
            if self.ema is not None:
                self.ema[sl].lerp_(w, 1 - ema)
        self._orthogonalise(owned, group["muon_ns_steps"])
        for s in eng.slots:
            if s.fqn not in second["lr"]:
                continue
            mine = self.owner[s.fqn] == eng.rank
            matrix = self._matrix(s).clone() if mine else torch.empty(s.rows, s.numel // s.rows)
            if eng.world > 1:
                dist.broadcast(matrix, src=dist.get_global_rank(eng.group, self.owner[s.fqn]) if eng.group
                               else self.owner[s.fqn], group=eng.group)
            sl = slice(s.shard, s.shard + s.shard_numel)
            lr, w = second["lr"][s.fqn], eng.master[sl]
            w.mul_(1 - lr * second["wd"][s.fqn]).add_(matrix[s.row0:s.row0 + s.rows_mine].reshape(-1), alpha=-lr)
            if self.ema is not None:
                self.ema[sl].lerp_(w, 1 - ema)
        eng.gather_weights()

    def dcp_state(self) -> dict:
        out = super().dcp_state()
        for s in self.engine.slots:
            if s.trainable:
                out["state"][s.fqn] = {"step": self.state[s.param]["step"]} | {
                    name: self.engine.shard_dtensor(s, buf) for name, buf in self.slot_buffers(s).items()}
        return out


def model_dcp_state(engine: ReplicatedEngine) -> dict:
    """``model.state_dict()``-shaped dict: fp32 master shards as ``Shard(0)`` DTensors + buffers."""
    out = {s.fqn: engine.shard_dtensor(s, engine.master) for s in engine.slots}
    for name, buf in engine.model.named_buffers():
        if name in engine.model.state_dict():
            out[name] = buf
    return out


def wrap_replicated(model: nn.Module, device: torch.device, compute_dtype: torch.dtype) -> ReplicatedEngine:
    engine = ReplicatedEngine(model, compute_dtype=compute_dtype, device=device)
    model.replicated_engine = engine
    return engine


def engine_of(model: nn.Module) -> Optional[ReplicatedEngine]:
    return getattr(model, "replicated_engine", None)
