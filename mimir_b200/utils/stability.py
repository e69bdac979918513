"""Opt-in stability diagnostics: scalar moments of activations, gradients, parameters and slots.

Reference behaviour: ``src/mimir/model/stability_diagnostics.py:53-477``.  The object is only
built on selected steps (a shadow replay of a bounded prefix of the step's batch, no optimizer
step), so ordinary steps carry no hooks or extra kernels.

* Each recorded tensor is reduced to ``[sum, sum of squares, finite count, non-finite count]``
  plus ``max|x|`` over a deterministic strided sample of at most 2^20 elements (the sample is
  taken before any dtype conversion, so huge tensors never get copied).
* Pairs (e.g. a block's input and its residual update) reduce to ``[dot, |a|^2, |b|^2, n]``
  and report a cosine.
* ``finalize`` checks that all ranks recorded the same keys, reduces with two all-reduces
  (SUM for moments, MAX for maxima), derives per-block gradient gains and residual ratios,
  writes one JSONL record under an ``flock`` (rank 0) and exposes tracker-ready summaries.
"""
from __future__ import annotations

import fcntl
import json
import math
import os
from collections import defaultdict
from pathlib import Path
from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor, nn

from mimir_b200.models.common import unwrap_tensor, wrap_tensor

MAX_SAMPLE = 1 << 20


def _local(t: Tensor) -> Tensor:
    return t.to_local() if callable(getattr(t, "to_local", None)) else t


def parameter_group(name: str) -> str:
    """``a.b.layers.3.attn.w`` -> ``a/b/layers/3``; otherwise the owning module path."""
    parts = name.split(".")
    if "layers" in parts:
        i = parts.index("layers")
        if i + 1 < len(parts):
            return "/".join(parts[:i + 2])
    return "/".join(parts[:-1] or parts)


def strided_sample(t: Tensor) -> Tensor:
    """Deterministic view of at most ``MAX_SAMPLE`` elements (strides chosen dim by dim)."""
    t = _local(t.detach())
    for dim in range(t.ndim):
        if t.numel() <= MAX_SAMPLE:
            return t
        rest = t.numel() // t.shape[dim]
        keep = max(1, MAX_SAMPLE // max(rest, 1))
        index = [slice(None)] * t.ndim
        index[dim] = slice(None, None, max(1, math.ceil(t.shape[dim] / keep)))
        t = t[tuple(index)]
    return t if t.numel() <= MAX_SAMPLE else t.reshape(-1)[:MAX_SAMPLE]


def diagnostic_prefixlm_batch(batch: dict, *, max_tokens: int) -> dict:
    """The leading whole packed sequences of ``batch`` that fit ``max_tokens`` (at least one)."""
    if max_tokens < 1:
        raise ValueError("Diagnostic token budget must be positive")
    n = int(unwrap_tensor(batch["numseqs"]).item())
    cu = unwrap_tensor(batch["cu_seqlens"])
    ends = cu[1:n + 1]
    keep = max(1, int((ends <= max_tokens).sum().item()))
    tokens = int(ends[keep - 1].item())
    prefix = unwrap_tensor(batch["prefix_lens"])[:keep]
    causal = unwrap_tensor(batch["causal_lens"])[:keep]
    out = dict(batch)
    for key in ("inputs", "labels", "position_ids"):
        out[key] = unwrap_tensor(batch[key])[:tokens]
    if "routing_category" in batch and unwrap_tensor(batch["routing_category"]).ndim == 1:
        out["routing_category"] = unwrap_tensor(batch["routing_category"])[:tokens]
    out["prefix_lens"] = torch.nn.functional.pad(prefix, (0, 1))
    out["causal_lens"] = causal
    out["cu_seqlens"] = cu[:keep + 1]
    totals = prefix + causal
    out.update(total_seqlen=wrap_tensor(torch.tensor(tokens)), numseqs=wrap_tensor(torch.tensor(keep)),
               max_seqlen_prefix=wrap_tensor(prefix.max().detach().cpu()),
               max_seqlen_causal=wrap_tensor(causal.max().detach().cpu()),
               max_seqlen_all=wrap_tensor(totals.max().detach().cpu()))
    return out


# (summary key, metric-key predicate, reducer); evaluated over the detailed metrics.
def _ends(prefixes, suffix):
    return lambda k: k.startswith(prefixes) and k.endswith(suffix)


_SUMMARY = (
    ("activation_max_abs", _ends(("activation/", "recurrent/"), "max_abs"), max),
    ("activation_nonfinite_fraction_max", _ends(("activation/", "recurrent/"), "nonfinite_fraction"), max),
    ("gradient_max_abs", _ends(("gradient/",), "max_abs"), max),
    ("gradient_nonfinite_fraction_max", _ends(("gradient/",), "nonfinite_fraction"), max),
    ("block_gradient_gain_max", _ends(("derived/H/", "derived/L/"), "gradient_gain"), max),
    ("h_block_gradient_gain_max", _ends(("derived/H/",), "gradient_gain"), max),
    ("l_block_gradient_gain_max", _ends(("derived/L/",), "gradient_gain"), max),
    ("recurrent_gradient_gain_max", _ends(("derived/recurrent/",), "gradient_gain"), max),
    ("residual_ratio_max", lambda k: k.endswith("residual_ratio"), max),
    ("recurrent_injection_ratio_max", lambda k: "injection_ratio" in k, max),
    ("residual_alignment_min", _ends(("pair/",), "_input_residual/cosine"), min),
    ("residual_alignment_max", _ends(("pair/",), "_input_residual/cosine"), max),
    ("attention_gate_near_zero_fraction_max", lambda k: k.endswith("attention/gate_near_zero/mean"), max),
    ("attention_gate_near_one_fraction_max", lambda k: k.endswith("attention/gate_near_one/mean"), max),
    ("parameter_grad_max_abs", lambda k: k.startswith("parameter/") and "/grad/max_abs" in k, max),
)

# derived name -> (numerator, denominator) patterns over a block base ``H/layer_3`` etc.
_BLOCK_RATIOS = {
    "gradient_gain": ("gradient/activation/{}/input/rms", "gradient/activation/{}/output/rms"),
    "attn_residual_ratio": ("activation/{}/attn_residual/rms", "activation/{}/input/rms"),
    "mlp_residual_ratio": ("activation/{}/mlp_residual/rms", "activation/{}/post_attn/rms"),
}


class StabilityDiagnostics:
    def __init__(self, *, step: int, rank: int, output_path: str, context: Optional[dict] = None):
        self.step, self.rank, self.output_path = step, rank, output_path
        self.context = context or {}
        self._moments: dict[str, list[Tensor]] = defaultdict(list)  # each [sum, sumsq, n, nonfinite, max]
        self._pairs: dict[str, list[Tensor]] = defaultdict(list)    # each [dot, l2, r2, n]
        self.wandb_summary: dict[str, float] = {}
        self.wandb_detailed: dict[str, float] = {}

    # -------------------------------------------------------------- recording
    def record_tensor(self, name: str, value: Tensor, *, record_gradient: bool = False) -> None:
        with torch.no_grad():
            x = strided_sample(value).float()
            finite = torch.isfinite(x)
            safe = torch.where(finite, x, torch.zeros_like(x))
            peak = safe.abs().amax() if safe.numel() else safe.new_zeros(())
            self._moments[name].append(torch.stack([safe.sum(), (safe * safe).sum(), finite.sum().float(),
                                                    (~finite).sum().float(), peak]))
        if record_gradient and value.requires_grad:
            value.register_hook(lambda g, key=f"gradient/{name}": self._on_grad(key, g))

    def _on_grad(self, name: str, grad: Tensor) -> Tensor:
        self.record_tensor(name, grad)
        return grad

    def record_pair(self, name: str, left: Tensor, right: Tensor) -> None:
        with torch.no_grad():
            a, b = torch.broadcast_tensors(_local(left.detach()), _local(right.detach()))
            a, b = strided_sample(a).float(), strided_sample(b).float()
            ok = torch.isfinite(a) & torch.isfinite(b)
            a, b = torch.where(ok, a, torch.zeros_like(a)), torch.where(ok, b, torch.zeros_like(b))
            self._pairs[name].append(torch.stack([(a * b).sum(), (a * a).sum(), (b * b).sum(), ok.sum().float()]))

    def record_last_dim_rms(self, name: str, value: Tensor) -> None:
        with torch.no_grad():
            v = _local(value.detach()).float()
            self.record_tensor(name, torch.linalg.vector_norm(v, dim=-1) / math.sqrt(v.shape[-1]))

    def record_fraction(self, name: str, condition: Tensor) -> None:
        self.record_tensor(name, condition.detach().float())

    def record_model_state(self, model: nn.Module, optimizer) -> None:
        names = {}
        for name, p in model.named_parameters():
            names[id(p)] = name
            group = parameter_group(name)
            self.record_tensor(f"parameter/{group}/value", p)
            if p.grad is not None:
                self.record_tensor(f"parameter/{group}/grad", p.grad)
        for p, slots in optimizer.state.items():
            name = names.get(id(p))
            if name is None:
                continue
            for slot in ("exp_avg", "exp_avg_sq", "param_ema"):
                v = slots.get(slot)
                if torch.is_tensor(v) and v.is_floating_point():
                    self.record_tensor(f"optimizer/{parameter_group(name)}/{slot}", v)

    # -------------------------------------------------------------- reduction
    @staticmethod
    def _same_keys_everywhere(keys: list[str]) -> None:
        if not (dist.is_available() and dist.is_initialized()):
            return
        everyone = [None] * dist.get_world_size()
        dist.all_gather_object(everyone, keys)
        if any(k != keys for k in everyone):
            raise RuntimeError("Stability diagnostic keys differ across distributed ranks")

    def finalize(self, *, detailed_wandb: bool = False) -> dict:
        mkeys, pkeys = sorted(self._moments), sorted(self._pairs)
        self._same_keys_everywhere(mkeys + [f"pair:{k}" for k in pkeys])
        distributed = dist.is_available() and dist.is_initialized()
        detail: dict[str, float] = {}
        if mkeys:
            per_key = [torch.stack(self._moments[k]) for k in mkeys]
            sums = torch.stack([m[:, :4].sum(0) for m in per_key])
            peaks = torch.stack([m[:, 4].amax() for m in per_key])
            if distributed:
                dist.all_reduce(sums)
                dist.all_reduce(peaks, op=dist.ReduceOp.MAX)
            for k, (s, s2, n, bad), peak in zip(mkeys, sums.cpu().tolist(), peaks.cpu().tolist()):
                d = max(n, 1.0)
                mean = s / d
                detail[f"{k}/mean"] = mean
                detail[f"{k}/rms"] = math.sqrt(max(s2 / d, 0.0))
                detail[f"{k}/std"] = math.sqrt(max(s2 / d - mean * mean, 0.0))
                detail[f"{k}/max_abs"] = peak
                detail[f"{k}/nonfinite_fraction"] = bad / max(n + bad, 1.0)
        if pkeys:
            pairs = torch.stack([torch.stack(self._pairs[k]).sum(0) for k in pkeys])
            if distributed:
                dist.all_reduce(pairs)
            for k, (dot, l2, r2, _n) in zip(pkeys, pairs.cpu().tolist()):
                detail[f"pair/{k}/cosine"] = dot / max(math.sqrt(l2 * r2), 1e-30)
        self._derive(detail)
        summary = {key: reduce((v for k, v in detail.items() if pred(k)), default=0.0)
                   for key, pred, reduce in _SUMMARY}
        record = {"schema_version": 1, "step": self.step,
                  "world_size": dist.get_world_size() if distributed else 1, "context": self.context,
                  "summary": summary, "metrics": detail}
        if self.rank == 0:
            self._append(record)
        self.wandb_summary = {f"stability/{k}": v for k, v in summary.items()}
        if detailed_wandb:
            self.wandb_detailed = {f"stability_detail/{k}": v for k, v in detail.items()}
        self._moments.clear()
        self._pairs.clear()
        return record

    @staticmethod
    def _derive(m: dict[str, float]) -> None:
        bases = {k[len("activation/"):-len("/input/rms")] for k in m
                 if k.startswith("activation/") and k.endswith("/input/rms") and "/layer_" in k}
        for base in bases:
            for name, (num, den) in _BLOCK_RATIOS.items():
                a, b = m.get(num.format(base)), m.get(den.format(base))
                if a is not None and b is not None:
                    m[f"derived/{base}/{name}"] = a / max(b, 1e-30)
        for base in {k[len("recurrent/"):-len("/hidden/rms")] for k in m
                     if k.startswith("recurrent/") and k.endswith("/hidden/rms")}:
            hidden = m[f"recurrent/{base}/hidden/rms"]
            if (inj := m.get(f"recurrent/{base}/injection/rms")) is not None:
                m[f"derived/recurrent/{base}/injection_ratio"] = inj / max(hidden, 1e-30)
            gi, go = m.get(f"gradient/recurrent/{base}/combined/rms"), m.get(f"gradient/recurrent/{base}/output/rms")
            if gi is not None and go is not None:
                m[f"derived/recurrent/{base}/gradient_gain"] = gi / max(go, 1e-30)

    def _append(self, record: dict) -> None:
        path = Path(self.output_path)
        path.parent.mkdir(parents=True, exist_ok=True)
        line = json.dumps(record, sort_keys=True, separators=(",", ":")) + "\n"
        with path.open("a", encoding="utf-8") as f:
            fcntl.flock(f.fileno(), fcntl.LOCK_EX)
            try:
                f.write(line)
                f.flush()
                os.fsync(f.fileno())
            finally:
                fcntl.flock(f.fileno(), fcntl.LOCK_UN)
