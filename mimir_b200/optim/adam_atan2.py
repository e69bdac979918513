"""AdamATan2 (the framework's default "AdamW") with decoupled weight decay and an EMA slot.

Reference behaviour: ``src/mimir/model/adam_atan2.py:25-166``.  State slots and
``param_groups`` keys are identical (``step``, ``exp_avg``, ``exp_avg_sq``, ``param_ema``;
``lr``, ``betas``, ``weight_decay``, ``ema``, ``ema_dtype``) so optimizer checkpoints are
interchangeable.

On CUDA the whole step is one fused multi-tensor kernel per (dtype, device) bucket
(:func:`mimir_b200.ops.optim.adam_atan2_multi`); on CPU the reference's exact sequence of
PyTorch ops runs, which keeps CPU results bit-identical.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor
from torch.optim.optimizer import Optimizer

from mimir_b200.ops._ext import kernels_enabled


def _dtype_name(dtype) -> Optional[str]:
    if dtype is None:
        return None
    return (dtype if isinstance(dtype, str) else str(dtype)).removeprefix("torch.")


def _resolve_dtype(name: Optional[str]) -> Optional[torch.dtype]:
    if name is None:
        return None
    dtype = getattr(torch, name, None)
    if not isinstance(dtype, torch.dtype):
        raise ValueError(f"Unsupported dtype name: {name}")
    return dtype


def _local(t: Tensor) -> Tensor:
    to_local = getattr(t, "to_local", None)
    return to_local() if callable(to_local) else t


class AdamATan2(Optimizer):
    def __init__(self, params, lr: float | Tensor = 1e-3, betas: Tuple[float, float] = (0.9, 0.95),
                 weight_decay: float = 0.1, ema: Optional[float] = None, ema_dtype=None,
                 parameter_lr_scales: Optional[dict] = None, fused: Optional[bool] = None):
        if isinstance(lr, Tensor) and lr.numel() != 1:
            raise ValueError("Tensor lr must be 1-element")
        if not 0.0 <= lr:
            raise ValueError(f"Invalid learning rate: {lr}")
        if not 0.0 <= betas[0] < 1.0:
            raise ValueError(f"Invalid beta parameter at index 0: {betas[0]}")
        if not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"Invalid beta parameter at index 1: {betas[1]}")
        if not 0.0 <= weight_decay:
            raise ValueError(f"Invalid weight_decay value: {weight_decay}")
        defaults = dict(lr=lr, betas=betas, weight_decay=weight_decay, ema=ema, ema_dtype=_dtype_name(ema_dtype))
        super().__init__(params, defaults)
        self.parameter_lr_scales = parameter_lr_scales
        self.fused = fused
        self._init_state()

    @torch.no_grad()
    def _init_state(self):
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state[p]
                st["step"] = torch.tensor(0.0, dtype=torch.get_default_dtype())
                if group["betas"][0] > 0:
                    st["exp_avg"] = torch.zeros_like(p)
                st["exp_avg_sq"] = torch.zeros_like(p)
                if group["ema"] is not None:
                    st["param_ema"] = torch.empty_like(p, dtype=_resolve_dtype(group["ema_dtype"])).copy_(p)

    def _lr(self, group, p):
        lr = group["lr"]
        if self.parameter_lr_scales is not None:
            lr = lr * self.parameter_lr_scales[p]
        return lr

    @torch.no_grad()
    def step(self, closure=None):
        assert closure is None, "Closure is not supported"
        from mimir_b200.optim.gate_updates import donor_updates
        with donor_updates(self) as passive:
            for group in self.param_groups:
                fused_items = []
                for p in group["params"]:
                    if p in passive or p.grad is None:
                        continue
                    if self._use_fused(p):
                        fused_items.append(p)
                    else:
                        self._step_reference(group, p)
                if fused_items:
                    self._step_fused(group, fused_items)

    def _use_fused(self, p) -> bool:
        if self.fused is False:
            return False
        return kernels_enabled(_local(p)) and _local(p).dtype in (torch.float32, torch.bfloat16)

    def _step_reference(self, group, p):
        st, g, lr = self.state[p], p.grad, self._lr(group, p)
        b1, b2 = group["betas"]
        if group["weight_decay"] != 0:
            p.mul_(1 - lr * group["weight_decay"])
        if "exp_avg" in st:
            st["exp_avg"].lerp_(g, 1 - b1)
        st["exp_avg_sq"].mul_(b2).addcmul_(g, g, value=1 - b2)
        st["step"] += 1
        bc1 = 1 - b1 ** st["step"]
        bc2_sqrt = (1 - b2 ** st["step"]).sqrt()
        denom = st["exp_avg_sq"].sqrt() / bc2_sqrt
        if "exp_avg" in st:
            p.add_(torch.atan2(st["exp_avg"], denom), alpha=-(lr / bc1))
        else:
            p.add_(torch.atan2(g, denom), alpha=-lr)
        if "param_ema" in st:
            src = p if p.dtype == st["param_ema"].dtype else p.to(st["param_ema"].dtype)
            st["param_ema"].lerp_(src, 1 - group["ema"])

    def _step_fused(self, group, params):
        from mimir_b200.ops.optim import adam_atan2_multi
        b1, b2 = group["betas"]
        buckets: dict = {}
        for p in params:
            st = self.state[p]
            st["step"] += 1
            # Bias corrections as the reference computes them (fp32 tensors), folded to scalars.
            step = st["step"]
            bc1 = (1 - b1 ** step) if "exp_avg" in st else torch.tensor(1.0)
            bc2_sqrt = (1 - b2 ** step).sqrt()
            lr = self._lr(group, p)
            key = (_local(p).dtype, _local(p).device, "exp_avg" in st, "param_ema" in st)
            buckets.setdefault(key, []).append((p, float(lr), float(bc1), float(bc2_sqrt)))
        for (_, _, has_m, has_ema), items in buckets.items():
            ps = [_local(p) for p, *_ in items]
            gs = [_local(p.grad) for p, *_ in items]
            ms = [_local(self.state[p]["exp_avg"]) for p, *_ in items] if has_m else None
            vs = [_local(self.state[p]["exp_avg_sq"]) for p, *_ in items]
            es = [_local(self.state[p]["param_ema"]) for p, *_ in items] if has_ema else None
            adam_atan2_multi(ps, gs, ms, vs, es, [lr for _, lr, _, _ in items], [bc1 for *_, bc1, _ in items],
                             [bc2 for *_, bc2 in items], b1, b2, group["weight_decay"],
                             group["ema"] if has_ema else None)

    @torch.no_grad()
    def swap_ema(self):
        """Swap parameters and their EMA copies (call again to swap back)."""
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state[p]
                if "param_ema" in st:
                    tmp = torch.empty_like(p).copy_(p)
                    p.copy_(st["param_ema"])
                    st["param_ema"].copy_(tmp)

    def load_state_dict(self, state_dict):
        # Optimizer.load_state_dict casts floating slots to the parameter dtype; an fp32 EMA of
        # bf16 parameters must keep its dtype, so restore it after the base-class load.
        keep = []
        dtypes = [g.get("ema_dtype") for g in self.param_groups]
        for group, incoming, dtype in zip(self.param_groups, state_dict["param_groups"], dtypes, strict=True):
            for p, ident in zip(group["params"], incoming["params"], strict=True):
                ema = state_dict["state"].get(ident, {}).get("param_ema")
                if ema is not None:
                    keep.append((p, ema.detach().clone(), _resolve_dtype(dtype)))
        out = super().load_state_dict(state_dict)
        for group, dtype in zip(self.param_groups, dtypes, strict=True):
            if dtype is not None:
                group["ema_dtype"] = dtype
        for p, ema, dtype in keep:
            self.state[p]["param_ema"] = ema.to(device=p.device, dtype=dtype or ema.dtype)
        return out
