"""Token -> expert dispatch plans for sparse MoE.

Reference: ``src/mimir/model/expert_mixtures.py:92-104`` builds each expert's token list
with ``nonzero`` per expert.  Here one stable sort of the (expert, token) selections
yields every expert's list (ascending token order, as the reference's ``nonzero``) and the
per-expert counts in a single host transfer.
"""
from __future__ import annotations

import os

import torch


class MoEPlan:
    def __init__(self, weights: torch.Tensor):
        n_experts = weights.shape[-1]
        selected = (weights != 0)
        token_ids = torch.arange(weights.shape[0], device=weights.device)
        pairs_e = torch.nonzero(selected.t(), as_tuple=False)  # [(expert, token)] sorted by expert then token
        self.tokens = pairs_e[:, 1].contiguous()
        counts = torch.bincount(pairs_e[:, 0], minlength=n_experts)
        self.offsets = [0] + torch.cumsum(counts, 0).tolist()
        del token_ids

    def indices(self, expert: int) -> torch.Tensor:
        return self.tokens[self.offsets[expert]:self.offsets[expert + 1]]


def moe_plan(weights: torch.Tensor) -> MoEPlan:
    return MoEPlan(weights)


# ----------------------------------------------------------------------------------------
# Grouped experts with an expert-parallel token exchange
# ----------------------------------------------------------------------------------------
def _swiglu_fwd(gu: torch.Tensor) -> torch.Tensor:
    from mimir_b200.ops._ext import ext, kernels_enabled
    if kernels_enabled(gu) and gu.shape[-1] % 16 == 0:
        return ext().swiglu_fwd(gu)
    gate, up = gu.chunk(2, dim=-1)
    return torch.nn.functional.silu(gate) * up


def _swiglu_bwd(gu: torch.Tensor, dp: torch.Tensor) -> torch.Tensor:
    from mimir_b200.ops._ext import ext, kernels_enabled
    if kernels_enabled(gu) and gu.shape[-1] % 16 == 0:
        return ext().swiglu_bwd(dp.contiguous(), gu)
    gate, up = gu.float().chunk(2, dim=-1)
    sig = torch.sigmoid(gate)
    dgate = dp.float() * up * sig * (1 + gate * (1 - sig))
    dup = dp.float() * gate * sig
    return torch.cat([dgate, dup], dim=-1).to(gu.dtype)


def _split_rows(t, expert_rows):
    out, s = [], 0
    for n in expert_rows:
        out.append(t[s:s + n])
        s += n
    return out


class _Exchange:
    """Moves token-slot rows between the source ranks and the expert owners for one plan.

    CUDA: peer-memory kernels (``csrc/moe.cu``) into/out of ``PeerBuffer`` regions.
    CPU: ``all_to_all_single`` plus the (source, expert) -> (expert, source) row permutation.
    """

    def __init__(self, ep, plan, T: int, k: int, d: int):
        self.ep, self.plan, self.T, self.k, self.d = ep, plan, T, k, d
        self.rows_in = sum(plan.expert_rows)
        if not ep.cuda:
            W, L = ep.size, ep.local
            C = plan.counts.view(W, W, L)[:, ep.rank]            # [source, local expert]
            src_start = torch.cumsum(C.sum(1), 0) - C.sum(1)     # where each source's rows land in the recv order
            within = torch.cumsum(C, 1) - C                      # offset of each expert inside a source's chunk
            pieces = [torch.arange(int(src_start[s] + within[s, e]), int(src_start[s] + within[s, e] + C[s, e]))
                      for e in range(L) for s in range(W)]
            self.perm = torch.cat(pieces) if pieces else torch.zeros(0, dtype=torch.long)  # buffer row -> recv row

    # ---------------------------------------------------------------- CPU helpers
    def _a2a(self, rows: torch.Tensor, send_counts, recv_counts) -> torch.Tensor:
        if self.ep.size == 1:
            return rows
        import torch.distributed as dist
        out = rows.new_empty((sum(recv_counts), rows.shape[1]))
        dist.all_to_all_single(out, rows.contiguous(), recv_counts, send_counts, group=self.ep.group)
        return out

    def to_owner_cpu(self, slot_rows: torch.Tensor) -> torch.Tensor:
        """[T*k, d] rows in slot order -> [rows_in, d] rows in this rank's buffer order."""
        sent = slot_rows[self.plan.order]
        recv = self._a2a(sent, self.plan.send_counts, self.plan.recv_counts)
        return recv[self.perm]

    def from_owner_cpu(self, buffer_rows: torch.Tensor) -> torch.Tensor:
        """[rows_in, d] rows in buffer order -> [T*k, d] rows in slot order."""
        recv = torch.empty_like(buffer_rows)
        recv[self.perm] = buffer_rows
        back = self._a2a(recv, self.plan.recv_counts, self.plan.send_counts)
        out = torch.empty_like(back)
        out[self.plan.order] = back
        return out


def _grouped_kernel_ok(xp, weights) -> bool:
    from mimir_b200.ops._ext import kernels_enabled
    if not (kernels_enabled(xp) and xp.dtype == torch.bfloat16 and os.environ.get("MIMIR_MOE_CUBLAS") != "1"):
        return False
    gu, dn = weights[0], weights[1]
    d, f2 = xp.shape[1], gu.shape[0]
    return (d % 128 == 0 and f2 % 128 == 0 and (f2 // 2) % 64 == 0 and len(weights) // 2 <= 256
            and all(w.is_contiguous() for w in weights))


def _expert_forward(xp, expert_rows, weights, y=None, rows_dev=None):
    """Per local expert: ``y = down(swiglu(x @ gate_up^T))`` on its contiguous rows.

    CUDA: two launches of the tcgen05 grouped GEMM (``csrc/grouped_gemm.cu``) for all experts,
    with the SwiGLU kernel in between; returns the packed ``[gate | up]`` projections of all rows
    (one tensor).  Otherwise one GEMM pair per expert; returns the per-expert projections."""
    y = torch.empty_like(xp) if y is None else y
    if rows_dev is not None and _grouped_kernel_ok(xp, weights):
        from mimir_b200.ops._ext import ext
        C = ext()
        gu = torch.empty(xp.shape[0], weights[0].shape[0], dtype=xp.dtype, device=xp.device)
        C.grouped_gemm(xp, list(weights[0::2]), rows_dev, gu, False)
        C.grouped_gemm(ext().swiglu_fwd(gu), list(weights[1::2]), rows_dev, y, False)
        return y, gu
    gus, s = [], 0
    for i, n in enumerate(expert_rows):
        gu_w, dn_w = weights[2 * i], weights[2 * i + 1]
        if n:
            gu = xp[s:s + n] @ gu_w.t()
            torch.matmul(_swiglu_fwd(gu), dn_w.t(), out=y[s:s + n])
        else:
            gu = xp.new_empty((0, gu_w.shape[0]))
        gus.append(gu)
        s += n
    return y, gus


def _weight_grad(w, a, b):
    """Gradient ``a @ b`` of weight ``w``.  When the replicated engine owns ``w.grad`` (a view into
    its flat buffer, with a ``_mimir_grad_sink`` callback), the GEMM accumulates into it in place
    (one read of the old gradient instead of a temporary plus an add) and autograd gets None;
    ``a is None`` means a zero gradient."""
    sink = getattr(w, "_mimir_grad_sink", None)
    if sink is not None and w.grad is not None:
        if a is not None:
            w.grad.addmm_(a, b)
        sink(w)
        return None
    return torch.zeros_like(w) if a is None else (a @ b).to(w.dtype)


def _expert_backward(dy, xp, gus, expert_rows, weights, dxp, rows_dev=None):
    if torch.is_tensor(gus):  # forward ran the grouped kernel: input gradients grouped too
        return _expert_backward_grouped(dy, xp, gus, expert_rows, weights, dxp, rows_dev)
    grads, s = [], 0
    for i, n in enumerate(expert_rows):
        gu_w, dn_w = weights[2 * i], weights[2 * i + 1]
        if n:
            gu = gus[i]
            # reads of the expert's weights first, then its gradients (announced to the engine)
            dgu = _swiglu_bwd(gu, dy[s:s + n] @ dn_w)
            torch.matmul(dgu, gu_w, out=dxp[s:s + n])
            d_dn = _weight_grad(dn_w, dy[s:s + n].t(), _swiglu_fwd(gu))
            d_gu = _weight_grad(gu_w, dgu.t(), xp[s:s + n])
        else:  # every expert gets a gradient (zero) so all ranks update the same parameters
            d_gu, d_dn = _weight_grad(gu_w, None, None), _weight_grad(dn_w, None, None)
        grads += [d_gu, d_dn]
        s += n
    return grads


def _expert_backward_grouped(dy, xp, gu, expert_rows, weights, dxp, rows_dev):
    """Input gradients with the grouped kernel ("nn": ``dact = dy @ W_down``, ``dx = dgu @ W_gate_up``),
    one SwiGLU-backward launch for all rows, and the weight gradients with the grouped
    weight-gradient kernel (reduction over each expert's rows)."""
    from mimir_b200.ops._ext import ext
    C = ext()
    rows = dy.shape[0]
    dact = torch.empty(rows, gu.shape[1] // 2, dtype=dy.dtype, device=dy.device)
    C.grouped_gemm(dy, list(weights[1::2]), rows_dev, dact, True)
    dgu = C.swiglu_bwd(dact, gu)
    C.grouped_gemm(dgu, list(weights[0::2]), rows_dev, dxp, True)
    act = C.swiglu_fwd(gu)
    # Weight gradients, one grouped launch per projection, accumulated in place: into the
    # engine's gradient views when it owns them, else into fresh zero tensors handed to autograd.
    targets, out, sunk = [], [], []
    for w in weights:
        sink = getattr(w, "_mimir_grad_sink", None)
        if sink is not None and w.grad is not None:
            sunk.append((sink, w))
            targets.append(w.grad)
            out.append(None)
        else:
            z = torch.zeros_like(w)
            targets.append(z)
            out.append(z)
    C.grouped_wgrad(dy, act, list(expert_rows), targets[1::2])
    C.grouped_wgrad(dgu, xp, list(expert_rows), targets[0::2])
    for sink, w in sunk:  # announced only once the kernels that write them are enqueued
        sink(w)
    return out


class _GroupedExpertsFn(torch.autograd.Function):
    """Saved for backward (through ``save_for_backward``, so activation checkpointing can drop and
    recompute them): the owner-side input rows ``xp``, the gate/up projections, and ``ys``, the
    expert outputs of this rank's token-slots as the forward combine loaded them.  No peer buffer
    is held from the forward to the backward: each exchange's buffer goes back to the pool as soon
    as its last kernel is issued (the next exchange's collective orders any reuse)."""

    @staticmethod
    def forward(ctx, x, topw, ep, plan, keep, *weights):
        T, d = x.shape
        k = topw.shape[1]
        ex = _Exchange(ep, plan, T, k, d)
        ctx.ex, ctx.n_weights = ex, len(weights)
        w32 = topw.float().contiguous()
        if ep.cuda:
            from mimir_b200.ops._ext import ext
            C = ext()
            buf = ep.acquire(2 * plan.capacity, d)
            C.moe_dispatch(x.contiguous(), plan.rows, plan.dst, buf.peer_ptrs(0, d), k, plan.capacity)
            ep.barrier()  # every rank's rows have landed in their owners' buffers
            xp = buf.view(0, ex.rows_in, d)
            _, gus = _expert_forward(xp, plan.expert_rows, weights, buf.view(plan.capacity, ex.rows_in, d),
                                     plan.expert_rows_dev)
            ep.barrier()  # every owner's outputs are in place
            ys = torch.empty(T * k, d, dtype=x.dtype, device=x.device) if keep else None
            out = C.moe_combine(buf.peer_ptrs(plan.capacity, d), plan.rows, plan.dst, w32, T, k, d, ys, plan.capacity)
            if keep:
                xp = xp.clone()
            ep.release(buf)
        else:
            slots = x.repeat_interleave(k, dim=0) if k > 1 else x
            xp = ex.to_owner_cpu(slots)
            y, gus = _expert_forward(xp, plan.expert_rows, weights)
            ys = ex.from_owner_cpu(y)
            out = (ys.view(T, k, d).float() * w32.unsqueeze(-1)).sum(1).to(x.dtype)
        if keep:
            ctx.gus_is_tensor = torch.is_tensor(gus)
            gus = [gus] if ctx.gus_is_tensor else list(gus)
            ctx.n_gus = len(gus)
            ctx.save_for_backward(w32, xp, ys, *gus, *weights)
        return out

    @staticmethod
    def backward(ctx, dout):
        ex, plan, ep = ctx.ex, ctx.ex.plan, ctx.ex.ep
        saved = ctx.saved_tensors
        w32, xp, ys = saved[:3]
        gus = saved[3:3 + ctx.n_gus]
        weights = saved[3 + ctx.n_gus:]
        gus = gus[0] if ctx.gus_is_tensor else list(gus)
        T, k, d = ex.T, ex.k, ex.d
        dout = dout.contiguous()
        if ep.cuda:
            from mimir_b200.ops._ext import ext
            C = ext()
            gbuf = ep.acquire(2 * plan.capacity, d)
            ep.barrier()  # every owner is done with the previous use of this buffer
            dw = C.moe_combine_bwd(dout, w32, plan.rows, plan.dst, ys, gbuf.peer_ptrs(0, d), k, plan.capacity)
            ep.barrier()  # the scaled output gradients have reached their owners
            dy = gbuf.view(0, ex.rows_in, d)
            dxp = gbuf.view(plan.capacity, ex.rows_in, d)
            grads = _expert_backward(dy, xp, gus, plan.expert_rows, weights, dxp, plan.expert_rows_dev)
            ep.barrier()  # every owner's input gradients are in place
            dx = C.moe_combine(gbuf.peer_ptrs(plan.capacity, d), plan.rows, plan.dst, None, T, k, d, None,
                               plan.capacity)
            ep.release(gbuf)
        else:
            dys = (dout.float().unsqueeze(1) * w32.unsqueeze(-1)).to(dout.dtype).reshape(T * k, d)
            dw = (dout.float().unsqueeze(1) * ys.view(T, k, d).float()).sum(-1)
            dy = ex.to_owner_cpu(dys)
            dxp = torch.empty_like(xp)
            grads = _expert_backward(dy, xp, gus, plan.expert_rows, weights, dxp)
            dx = ex.from_owner_cpu(dxp).view(T, k, d).float().sum(1).to(dout.dtype)
        return (dx, dw, None, None, None, *grads)


def grouped_experts(x: torch.Tensor, topw: torch.Tensor, topi: torch.Tensor, ep, weights: list) -> torch.Tensor:
    """``sum_j topw[t, j] * expert_{topi[t, j]}(x[t])`` with this rank's experts' weights
    ``[gate_up_0, down_0, gate_up_1, down_1, ...]`` (experts ``ep.first ... ep.first + ep.local - 1``).

    The rows of every expert are exchanged with its owner rank (``ep``); within an expert the
    rows are in token order, as the reference's per-expert ``nonzero`` lists
    (``src/mimir/model/expert_mixtures.py:92-104``)."""
    plan = ep.plan(topi)
    keep = torch.is_grad_enabled() and (x.requires_grad or topw.requires_grad or any(w.requires_grad for w in weights))
    return _GroupedExpertsFn.apply(x, topw, ep, plan, keep, *weights)
