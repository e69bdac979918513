"""MuonAdamW: Muon (Newton-Schulz orthogonalised momentum) for hidden matrices, Adam for the rest.

Reference behaviour: ``src/mimir/model/muon.py:15-108``.

* Newton-Schulz: 5 iterations of ``X <- a X + (b G + c G^2) X`` with ``G = X X^T`` and
  (a, b, c) = (3.4445, -4.7750, 2.0315) on the Frobenius-normalised fp32 matrix, transposed
  first when it has more rows than columns (the published Muon quintic iteration).
* Packed projections are orthogonalised per logical matrix: gqkv -> 4 (gate, Q, K, V),
  gate_up -> 2, o/down -> 1; each piece is scaled by ``sqrt(max(1, rows/cols))``.
* Nesterov-style update ``grad.lerp(momentum, beta)`` after ``momentum.lerp_(grad, 1-beta)``.
* Non-matrix parameters use plain Adam (eps 1e-8) with decoupled weight decay.

Distributed (FSDP2 / DTensor) parameters: the reference all-gathers every matrix on every
rank and runs the same Newton-Schulz chain redundantly everywhere.  Here each matrix has an
owner rank (round-robin); shards are gathered to the owner only, the owner orthogonalises,
and the result is scattered back as shards, so the NS FLOPs are split across ranks.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from mimir_b200.optim.adam_atan2 import AdamATan2

NS_COEFFS = (3.4445, -4.7750, 2.0315)


def orthogonalize(matrix, steps=5):
    x = matrix.float()
    tall = x.shape[-2] > x.shape[-1]
    if tall:
        x = x.mT
    x = x / (x.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    a, b, c = NS_COEFFS
    for _ in range(steps):
        gram = x @ x.mT
        x = a * x + (b * gram + c * gram @ gram) @ x
    return x.mT if tall else x


def matrix_splits(name, parameter):
    if name.endswith("attn.gqkv_proj.weight"):
        count = 4
    elif name.endswith("gate_up_proj.weight"):
        count = 2
    elif name.endswith(("o_proj.weight", "down_proj.weight")):
        count = 1
    else:
        return None
    if parameter.ndim != 2 or parameter.shape[0] % count:
        raise ValueError(f"Unsupported Muon logical matrix layout: {name}: {parameter.shape}")
    return count


def muon_update(full, count, steps):
    """Orthogonalised update of a packed matrix: each of its ``count`` logical pieces separately,
    scaled by sqrt(max(1, rows/cols)).  On CUDA the pieces go through the batched tcgen05 chain."""
    from mimir_b200.optim.newton_schulz import orthogonalize_batch, tensor_core_ns_enabled
    pieces = full.chunk(count, dim=0)
    scale = math.sqrt(max(1, pieces[0].shape[0] / pieces[0].shape[1]))
    if tensor_core_ns_enabled(full):
        return (orthogonalize_batch(torch.stack(pieces), steps) * scale).reshape(full.shape).to(full.dtype)
    return torch.cat([orthogonalize(p, steps) * math.sqrt(max(1, p.shape[0] / p.shape[1])) for p in pieces])


class MuonAdamW(AdamATan2):
    def __init__(self, named_parameters, *, momentum=0.95, ns_steps=5, muon_lr_scale=1.0,
                 distributed_mode: str = "owner", **kwargs):
        if not 0 <= momentum < 1 or ns_steps < 1 or muon_lr_scale <= 0:
            raise ValueError("Invalid Muon momentum, iterations or LR scale")
        if distributed_mode not in ("owner", "replicated"):
            raise ValueError("distributed_mode must be 'owner' or 'replicated'")
        named = list(named_parameters)
        self.matrix_layout = {p: matrix_splits(n, p) for n, p in named}
        self.distributed_mode = distributed_mode
        super().__init__([p for _, p in named], **kwargs)
        for group in self.param_groups:
            group.update(optimizer_kind="muon_adamw", muon_momentum=momentum, muon_ns_steps=ns_steps,
                         muon_lr_scale=muon_lr_scale)
        for p, count in self.matrix_layout.items():
            if count is not None:
                st = self.state[p]
                st.pop("exp_avg", None)
                st.pop("exp_avg_sq")
                st["momentum_buffer"] = torch.zeros_like(p)

    @torch.no_grad()
    def step(self, closure=None):
        if closure is not None:
            raise ValueError("Closures are not supported")
        from mimir_b200.optim.gate_updates import donor_updates
        with donor_updates(self) as passive:
            self._step_groups(passive)

    def _step_groups(self, passive):
        pending = []  # (group, param, lr, momentum update) for distributed owner mode
        for group in self.param_groups:
            for p in group["params"]:
                if not p.requires_grad or p in passive or p.grad is None:
                    continue
                count = self.matrix_layout[p]
                st = self.state[p]
                st["step"] += 1
                lr = group["lr"] * (self.parameter_lr_scales[p] if self.parameter_lr_scales is not None else 1)
                g = p.grad
                if count is not None:
                    beta = group["muon_momentum"]
                    st["momentum_buffer"].lerp_(g, 1 - beta)
                    upd = g.lerp(st["momentum_buffer"], beta)
                    lr = lr * group["muon_lr_scale"]
                    if _is_dtensor(p) and self.distributed_mode == "owner":
                        pending.append((group, p, lr, upd))
                        continue
                    upd = self._replicated_update(p, upd, count, group["muon_ns_steps"])
                else:
                    b1, b2 = group["betas"]
                    if "exp_avg" in st:
                        st["exp_avg"].lerp_(g, 1 - b1)
                        num = st["exp_avg"] / (1 - b1 ** st["step"])
                    else:
                        num = g
                    st["exp_avg_sq"].lerp_(g.square(), 1 - b2)
                    upd = num / ((st["exp_avg_sq"] / (1 - b2 ** st["step"])).sqrt() + 1e-8)
                self._apply(group, p, lr, upd)
        if pending:
            self._owner_updates(pending)

    def _apply(self, group, p, lr, upd):
        p.mul_(1 - lr * group["weight_decay"]).add_(upd, alpha=-lr)
        st = self.state[p]
        if "param_ema" in st:
            st["param_ema"].lerp_(p.to(st["param_ema"].dtype), 1 - group["ema"])

    def _replicated_update(self, p, upd, count, steps):
        if _is_dtensor(upd):
            from torch.distributed.tensor import distribute_tensor
            full = muon_update(upd.full_tensor(), count, steps)
            return distribute_tensor(full.to(p.dtype), p.device_mesh, p.placements)
        return muon_update(upd, count, steps).to(p.dtype)

    def _owner_updates(self, pending):
        """Gather each matrix to a round-robin owner, orthogonalise there, scatter shards back."""
        from torch.distributed.tensor import DTensor
        mesh = pending[0][1].device_mesh
        group = mesh.get_group()
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        for index, (g, p, lr, upd) in enumerate(pending):
            owner = index % world
            local = upd.to_local().contiguous()
            # Shard(0) with possibly uneven shards: gather row counts first.
            rows = torch.tensor([local.shape[0]], device=local.device)
            all_rows = [torch.zeros_like(rows) for _ in range(world)]
            dist.all_gather(all_rows, rows, group=group)
            all_rows = [int(r.item()) for r in all_rows]
            width = local.shape[1]
            max_rows = max(all_rows)
            padded = torch.zeros((max_rows, width), dtype=local.dtype, device=local.device)
            padded[:local.shape[0]] = local
            bucket = [torch.empty_like(padded) for _ in range(world)] if rank == owner else None
            dist.gather(padded, bucket, dst=dist.get_global_rank(group, owner), group=group)
            out = torch.empty_like(padded)
            scatter_list = None
            if rank == owner:
                full = torch.cat([b[:r] for b, r in zip(bucket, all_rows)])
                result = muon_update(full, self.matrix_layout[p], g["muon_ns_steps"]).to(local.dtype)
                scatter_list, offset = [], 0
                for r in all_rows:
                    piece = torch.zeros_like(padded)
                    piece[:r] = result[offset:offset + r]
                    scatter_list.append(piece)
                    offset += r
            dist.scatter(out, scatter_list, src=dist.get_global_rank(group, owner), group=group)
            shard = out[:local.shape[0]].to(p.dtype)
            upd_d = DTensor.from_local(shard, p.device_mesh, p.placements, run_check=False,
                                       shape=p.shape, stride=p.stride())
            self._apply(g, p, lr, upd_d)


def _is_dtensor(t) -> bool:
    try:
        from torch.distributed.tensor import DTensor
    except ImportError:  # pragma: no cover
        return False
    return isinstance(t, DTensor)
