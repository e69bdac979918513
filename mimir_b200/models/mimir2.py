"""Mimir2: the HRM backbone with every opt-in v2 feature.

Reference behaviour: ``src/mimir/model/mimir2.py`` — config and cross-field validation
(``:23-127``), invocation gates (``:130-141``), feature installation (``:144-208``),
forward over hierarchical/looped recurrence with MoS (dense and sparse), persistent H
streams, branch mixing and recurrent memories (``:258-362``), step-scheduled alphas
(``:364-387``) and inactive-gate donor mapping (``:389-403``).

Module names and buffer names are identical to the reference so DCP checkpoints load
unchanged; construction consumes the RNG in the same order (H stack, L stack, zL_init),
so a seed gives the same initial weights.
"""
from __future__ import annotations

import copy
import math
from dataclasses import dataclass
from typing import Optional, Literal

import torch
import torch.nn.functional as F
from pydantic import Field, model_validator
from torch import nn

from mimir_b200.models.branches import BranchedTransformer, BranchExpertMixer, RecurrentMemory
from mimir_b200.models.experts import RoutedBlock, TopKRouter, install_mlp_mixtures
from mimir_b200.models.ngram import NGramMemory
from mimir_b200.models.recurrence import RecurrentBackbone, RecurrentConfig
from mimir_b200.models.transformer import TransformerBlock
from mimir_b200.optim.module_lr import backward_call_counts


class Mimir2Config(RecurrentConfig):
    recurrence_mode: Literal["hierarchical", "looped"] = "hierarchical"
    gates_enabled: bool = False
    gate_alpha_max: float = Field(default=1.0, ge=0, le=1)
    gate_warmup_start_step: int = Field(default=0, ge=0)
    gate_warmup_steps: int = Field(default=2000, ge=0)
    gate_initialize_from_v1: bool = False
    moe_num_experts: int = Field(default=1, ge=1)
    moe_top_k: int = Field(default=1, ge=1)
    moe_levels: Literal["L", "H", "both"] = "L"
    mos_num_experts: int = Field(default=1, ge=1)
    mos_top_k: int = Field(default=1, ge=1)
    mos_state_mode: Literal["shared", "separate"] = "shared"
    expert_freeze_base: bool = False
    router_top1_straight_through: bool = True
    moe_aux_loss_free: bool = False
    mos_aux_loss_free: bool = False
    routing_bias_update_rate: float = Field(default=0.001, ge=0, allow_inf_nan=False)
    residual_branches: int = Field(default=1, ge=1)
    residual_levels: Literal["L", "H", "both"] = "both"
    residual_alpha_max: float = Field(default=1.0, ge=0, le=1)
    residual_warmup_start_step: int = Field(default=0, ge=0)
    residual_warmup_steps: int = Field(default=0, ge=0)
    residual_write_init_scale: float = Field(default=0.1, ge=0)
    residual_input_dependent: bool = False
    h_residual_persistence: bool = False
    h_branch_l_mixing: bool = False
    upcycle_from_dense: bool = False
    moe_sparse: bool = False
    # Additions beyond the reference (defaults keep its behaviour and checkpoint keys):
    # expert FFN width (None: the dense MLP width, experts start as copies of the dense MLP),
    # always-on shared experts of the expert width, the grouped token-exchange implementation of
    # the sparse path, and expert parallelism (experts split over the ranks, tokens exchanged
    # over NVLink peer memory).
    moe_expert_intermediate_size: Optional[int] = Field(default=None, ge=8)
    moe_shared_experts: int = Field(default=0, ge=0)
    moe_dispatch: Literal["index", "grouped"] = "index"
    moe_router_init_std: Optional[float] = Field(default=None, gt=0)  # None: zero rows (reference init)
    moe_expert_parallel: bool = False
    mos_sparse: bool = False
    mos_sparse_routing: Literal["first_token", "prefix_mean"] = "first_token"
    h_memory_branches: int = Field(default=1, ge=1)
    l_memory_branches: int = Field(default=1, ge=1)
    memory_warmup_steps: int = Field(default=2000, ge=0)
    memory_warmup_start_step: int = Field(default=0, ge=0)
    ngram_orders: list[int] = Field(default_factory=list)
    ngram_buckets: int = Field(default=4096, ge=2)
    ngram_heads: int = Field(default=1, ge=1)
    ngram_contextual_gate: bool = False
    ngram_warmup_steps: int = Field(default=2000, ge=0)
    ngram_warmup_start_step: int = Field(default=0, ge=0)
    moe_metadata_bias: list[list[float]] = Field(default_factory=list)
    mos_metadata_bias: list[list[float]] = Field(default_factory=list)
    routing_bias_decay_start: int = Field(default=0, ge=0)
    routing_bias_decay_end: int = Field(default=0, ge=0)
    specialist_training: bool = False
    specialist_router_calibration: bool = False

    @model_validator(mode="after")
    def _validate(self):
        derived = _Derived(self)
        for broken, message in _CONFIG_RULES:
            if broken(self, derived):
                raise ValueError(message)
        return self


class _Derived:
    """Quantities several configuration rules share."""

    def __init__(self, cfg):
        self.h_layers = cfg.H_override.get("n_layers", cfg.n_layers)
        self.looped = cfg.recurrence_mode == "looped"
        self.h_stream_options = cfg.h_residual_persistence or cfg.h_branch_l_mixing
        self.norms = {"L": cfg.norm_type, "H": cfg.H_override.get("norm_type", cfg.norm_type)}


def _bad_metadata_rows(cfg) -> bool:
    tables = ((cfg.moe_metadata_bias, cfg.moe_num_experts), (cfg.mos_metadata_bias, cfg.mos_num_experts))
    return any(len(row) != count or not all(math.isfinite(v) for v in row) for rows, count in tables for row in rows)


def _non_prenorm_branches(cfg, d: _Derived) -> bool:
    return cfg.residual_branches > 1 and any(
        cfg.residual_levels in (level, "both") and d.norms[level] != "pre" for level in ("L", "H"))


# (rule violated?, message) in the order they are checked; the messages are the user interface.
_CONFIG_RULES = (
    (lambda c, d: c.moe_aux_loss_free and c.moe_num_experts < 2, "MoE balancing requires multiple MoE experts"),
    (lambda c, d: c.mos_aux_loss_free and c.mos_num_experts < 2, "MoS balancing requires multiple MoS experts"),
    (lambda c, d: c.n_layers < 1 or d.h_layers < 0, "L requires positive layers and H requires nonnegative layers"),
    (lambda c, d: d.h_layers == 0 and not d.looped, "Zero-layer H requires looped recurrence"),
    (lambda c, d: d.h_stream_options and (d.looped or d.h_layers == 0 or c.residual_branches < 2
                                          or c.residual_levels not in ("H", "both")),
     "H stream options require hierarchical recurrence and multiple H residual branches"),
    (lambda c, d: d.h_stream_options and c.h_memory_branches > 1,
     "H stream options cannot be combined with H recurrent memory"),
    (lambda c, d: d.h_stream_options and c.gate_initialize_from_v1,
     "H stream options require explicit upcycling, not gate-only migration"),
    (lambda c, d: c.h_branch_l_mixing and (c.mos_num_experts < 2 or c.l_memory_branches > 1),
     "Branch-specific L mixing requires MoS and no L recurrent memory"),
    (lambda c, d: d.looped and (c.gates_enabled or c.h_memory_branches > 1 or c.l_memory_branches > 1
                                or c.mos_state_mode != "shared"),
     "Looped recurrence requires shared MoS state, no invocation gates, and no recurrent memory branches; "
     "residual branches are supported"),
    (lambda c, d: c.mos_sparse and c.mos_sparse_routing == "prefix_mean" and c.attn_type != "prefixlm",
     "Prefix-mean routing requires PrefixLM prompt visibility"),
    (lambda c, d: _bad_metadata_rows(c), "Metadata bias rows must contain one finite logit per expert"),
    (lambda c, d: bool(c.routing_bias_decay_end) and c.routing_bias_decay_end <= c.routing_bias_decay_start,
     "Routing bias decay end must follow start"),
    (lambda c, d: c.specialist_training and not c.expert_freeze_base,
     "Specialist training requires a frozen reference expert"),
    (lambda c, d: c.mos_state_mode == "separate" and c.l_memory_branches > 1,
     "Choose expert-specific L states or general L memory branches, not both"),
    (lambda c, d: c.upcycle_from_dense and c.gate_initialize_from_v1, "Use only one migration mode"),
    (lambda c, d: c.gate_initialize_from_v1 and not c.gates_enabled,
     "gate_initialize_from_v1 requires gates_enabled=true"),
    (lambda c, d: (c.moe_dispatch == "grouped" or c.moe_expert_parallel)
     and not (c.moe_sparse and c.moe_num_experts > 1),
     "The grouped MoE dispatch and expert parallelism need moe_sparse with several experts"),
    (lambda c, d: c.moe_expert_parallel and c.moe_dispatch != "grouped",
     "moe_expert_parallel requires moe_dispatch=grouped"),
    (lambda c, d: c.upcycle_from_dense and (c.moe_expert_intermediate_size is not None or c.moe_shared_experts),
     "Upcycling copies the dense MLP: it needs the dense expert width and no shared experts"),
    (lambda c, d: c.moe_expert_parallel and (c.specialist_training or c.expert_freeze_base),
     "Expert parallelism does not support specialist training or a frozen base expert"),
    (lambda c, d: c.moe_top_k > c.moe_num_experts or c.mos_top_k > c.mos_num_experts,
     "Expert top_k must not exceed num_experts"),
    (lambda c, d: c.gate_initialize_from_v1 and (c.moe_num_experts > 1 or c.mos_num_experts > 1
                                                 or c.residual_branches > 1),
     "Expert/branch upcycling requires upcycle_from_dense; gate_initialize_from_v1 only migrates gates"),
    (lambda c, d: _non_prenorm_branches(c, d), "Multiple residual branches currently require pre-norm"),
    (lambda c, d: c.expert_freeze_base and c.moe_num_experts == c.mos_num_experts == 1,
     "expert_freeze_base requires an expert mixture"),
)


@dataclass(frozen=True)
class _Call:
    level: str   # "L" or "H"
    slot: int    # invocation index within the level (gate and cache slot)
    grad: bool   # inside the truncated-BPTT window


def _schedule(h_cycles: int, l_cycles: int, h_window: int, l_window: int) -> list[_Call]:
    """Per H cycle: its L invocations, then its H invocation.  The last ``l_window`` L calls and
    the last ``h_window`` H calls record autograd state."""
    l_total = h_cycles * l_cycles
    calls = []
    for i in range(h_cycles):
        calls.extend(_Call("L", k, k >= l_total - l_window) for k in range(i * l_cycles, (i + 1) * l_cycles))
        calls.append(_Call("H", i, i >= h_cycles - h_window))
    return calls


class _Pass:
    """State of one v2 forward: the two stack states, recurrent memories, MoS expert states and
    routes, per-level extra inputs (routing biases) and the current cycle's L context."""

    def __init__(self, model, x, cache, diagnostics, seq_info, category):
        cfg = model.gate_config
        self.model, self.cache, self.diagnostics = model, cache, diagnostics
        self.looped = cfg.recurrence_mode == "looped"
        self.mixture = cfg.mos_num_experts > 1
        self.z_H, self.z_L = x, model.zL_init
        self.h_streams = model.H_level.core.initialize_streams(x) if cfg.h_residual_persistence else None
        self.memory_modules, self.memories = {}, {}
        for name, start in (("H", self.z_H), ("L", self.z_L)):
            memory = getattr(getattr(model, f"{name}_level"), "memory", None)
            if memory is not None:
                self.memory_modules[name] = memory
                self.memories[name] = memory.initialize(start.expand_as(x))
        moe_bias = model._metadata_bias(category, "moe")
        self.mos_bias = model._metadata_bias(category, "mos")
        self.info = {}
        for name in ("L", "H"):
            self.info[name] = dict(seq_info)
            if moe_bias is not None and cfg.moe_levels in (name, "both"):
                self.info[name]["routing_bias"] = moe_bias
        self.routes = None
        if self.mixture and cfg.mos_sparse:
            from mimir_b200.models.sparse_stacks import cached_sequence_routes, sequence_routes
            self.routes = (sequence_routes(model.L_level.stack_router, x, seq_info, self.mos_bias,
                                           cfg.mos_sparse_routing) if cache is None
                           else cached_sequence_routes(model, x, cache, seq_info, self.mos_bias))
        separate = self.mixture and cfg.mos_state_mode == "separate"
        self.states = [model.zL_init] * cfg.mos_num_experts if separate else None
        self.context = None
        self.collect = None

    def begin_cycle(self) -> None:
        """Start of an H cycle: looped recurrence restarts L from H and gives it no H context
        (None stands for a zero context)."""
        if self.looped:
            self.z_L = self.z_H
        self.context = None if self.looped else self.z_H

    def _attr(self, level: str) -> str:
        return "z_H" if level == "H" else "z_L"

    def read_memory(self, level: str) -> None:
        if level in self.memories:
            setattr(self, self._attr(level), self.memory_modules[level].read_state(self.memories[level]))

    def write_memory(self, level: str) -> None:
        if level in self.memories:
            memory = self.memory_modules[level]
            self.memories[level] = memory.update(self.memories[level], getattr(self, self._attr(level)))
            setattr(self, self._attr(level), memory.read_state(self.memories[level]))


class InvocationGate(nn.Module):
    """``injection * (1 + alpha * tanh(W [hidden; injection] + b))``, zero-initialised (no RNG)."""

    def __init__(self, hidden_size):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(hidden_size, 2 * hidden_size))
        self.bias = nn.Parameter(torch.zeros(hidden_size))

    def forward(self, hidden, injection, alpha):
        from mimir_b200.ops import gate as fused
        if fused.supported(hidden, injection, alpha):  # tcgen05 GEMM + fused bias/tanh/gate kernel
            return fused.invocation_gate(hidden, injection, self.weight, self.bias, alpha)
        hidden, injection = torch.broadcast_tensors(hidden, injection)
        x = torch.cat((hidden, injection), dim=-1)
        gate = F.linear(x, self.weight.to(x.dtype), self.bias.to(x.dtype))
        return injection * (1 + alpha.to(x.dtype) * torch.tanh(gate))


class Mimir2(RecurrentBackbone):
    """The v1 backbone plus the opt-in v2 features.  Features are installed in a fixed order (per
    level L then H: MLP mixtures, routed blocks, residual branches; then the H branch mixer, MoS
    stacks, invocation gates, recurrent memories, routing-bias scale, n-gram memory): the order
    fixes RNG consumption and parameter names, which checkpoints depend on."""

    def __init__(self, config_dict):
        config = Mimir2Config(**config_dict)
        if config.H_cycles < 1 or config.L_cycles < 1:
            raise ValueError("HRM v2 requires positive H/L cycles")
        super().__init__(config_dict)
        self.gate_config = config
        self.has_h_stack = config.H_override.get("n_layers", config.n_layers) > 0
        self._router_options = dict(freeze_base=config.expert_freeze_base,
                                    top1_straight_through=config.router_top1_straight_through)
        for name in ("L", "H"):
            if name == "L" or self.has_h_stack:
                self._install_level(name, getattr(self, f"{name}_level"))
        if config.h_branch_l_mixing:
            self.H_level.l_branch_mixer = BranchExpertMixer(config.residual_branches, config.mos_num_experts)
        if config.mos_num_experts > 1:
            self._install_stack_mixture()
        if config.gates_enabled:
            self.H_level.invocation_gates = nn.ModuleList(InvocationGate(self.hidden_size) for _ in range(self.H_cycles))
            self.L_level.invocation_gates = nn.ModuleList(InvocationGate(self.hidden_size)
                                                          for _ in range(self.H_cycles * self.L_cycles))
            self.register_buffer("gate_alpha", torch.tensor(0.0))
        for name, branches in (("H", config.h_memory_branches), ("L", config.l_memory_branches)):
            if branches > 1:
                getattr(self, f"{name}_level").memory = RecurrentMemory(branches, self.hidden_size)
        if config.moe_metadata_bias or config.mos_metadata_bias:
            self.register_buffer("routing_bias_scale", torch.tensor(1.0))
        self.ngram_enabled = bool(config.ngram_orders)
        if self.ngram_enabled:
            self.ngram = NGramMemory(self.hidden_size, config.ngram_orders, config.ngram_buckets, config.ngram_heads,
                                     config.ngram_contextual_gate)
        if self._needs_explicit_checkpoint(config):
            for m in self.modules():
                if isinstance(m, TransformerBlock):
                    m._v2_explicit_checkpoint = True

    def _install_level(self, name, level):
        """MLP mixtures (and routed blocks), then residual branches, on one level's stack."""
        cfg = self.gate_config
        if cfg.moe_levels in (name, "both"):
            install_mlp_mixtures(level.core, self.hidden_size, cfg.moe_num_experts, cfg.moe_top_k,
                                 sparse=cfg.moe_sparse, balance_enabled=cfg.moe_aux_loss_free,
                                 balance_update_rate=cfg.routing_bias_update_rate,
                                 expert_intermediate_size=cfg.moe_expert_intermediate_size,
                                 shared_experts=cfg.moe_shared_experts, grouped=cfg.moe_dispatch == "grouped",
                                 expert_parallel=cfg.moe_expert_parallel, router_init_std=cfg.moe_router_init_std,
                                 **self._router_options)
            if cfg.moe_num_experts > 1:
                norm = cfg.H_override.get("norm_type", cfg.norm_type) if name == "H" else cfg.norm_type
                level.core.layers = nn.ModuleList(RoutedBlock(block, norm) for block in level.core.layers)
        if cfg.residual_branches > 1 and cfg.residual_levels in (name, "both"):
            level.core = BranchedTransformer(level.core, cfg.residual_branches, cfg.residual_write_init_scale,
                                             cfg.residual_input_dependent)

    def _install_stack_mixture(self):
        """MoS: copies of the L stack as extra experts and a stack router."""
        cfg = self.gate_config
        self.L_level.stack_experts = nn.ModuleList(copy.deepcopy(self.L_level.core)
                                                   for _ in range(cfg.mos_num_experts - 1))
        self.L_level.stack_router = TopKRouter(self.hidden_size, cfg.mos_num_experts, cfg.mos_top_k,
                                               balance_enabled=cfg.mos_aux_loss_free,
                                               balance_update_rate=cfg.routing_bias_update_rate,
                                               **self._router_options)
        if cfg.expert_freeze_base:
            self.L_level.core.requires_grad_(False)

    @staticmethod
    def _needs_explicit_checkpoint(cfg) -> bool:
        """Features whose blocks must be checkpointed explicitly (their state is not a plain
        sequential function of the block input)."""
        return bool(cfg.ngram_orders or cfg.h_memory_branches > 1 or cfg.l_memory_branches > 1 or cfg.moe_sparse
                    or cfg.mos_sparse or cfg.residual_input_dependent or cfg.h_residual_persistence
                    or cfg.h_branch_l_mixing)

    # ---------------------------------------------------------------- caches
    def create_cache(self, **kwargs):
        cfg = self.gate_config
        if cfg.mos_num_experts > 1:
            cores = [self.L_level.core, *self.L_level.stack_experts]
            cache = dict(H=[self.H_level.create_cache(**kwargs) for _ in range(self.H_cycles)],
                         L=[[c.create_cache(**kwargs) for c in cores] for _ in range(self.H_cycles * self.L_cycles)])
            if cfg.mos_sparse:
                cache["mos_routes"] = torch.zeros(kwargs["max_batch_size"], len(cores), device=kwargs.get("device"),
                                                  dtype=torch.float32)
        else:
            cache = super().create_cache(**kwargs)
        if self.ngram_enabled:
            cache = cache | {"ngram_history": {}}
        return cache

    # ---------------------------------------------------------------- helpers
    def _metadata_bias(self, category, kind):
        """Per-token routing logit bias from the batch's routing category (training only)."""
        rows = getattr(self.gate_config, f"{kind}_metadata_bias")
        if category is None or not rows or not self.training or self.gate_config.specialist_router_calibration:
            return None
        return torch.tensor(rows, device=category.device, dtype=torch.float32)[category.long()] * self.routing_bias_scale

    def _inject(self, level, invocation, hidden, other):
        """The injection a stack receives: gated by that invocation's gate when gates are on."""
        if self.gate_config.gates_enabled:
            return level.invocation_gates[invocation](hidden, other, self.gate_alpha)
        return other

    def _stack_step(self, z_L, z_H, states, invocation, cache, diagnostics, seq_info, bias=None, expert_outputs=None):
        """Dense MoS: every L stack expert runs on all tokens; outputs are mixed token-locally."""
        weights = self.L_level.stack_router(z_L + z_H, bias)
        mixed = torch.zeros_like(z_H)
        updated = [] if states is not None else None
        for e, core in enumerate((self.L_level.core, *self.L_level.stack_experts)):
            start = z_L if states is None else states[e]
            scope = None if diagnostics is None else f"L/cycle_{invocation:03d}/expert_{e}"
            y = core(start + self._inject(self.L_level, invocation, start, z_H), **seq_info,
                     cache=None if cache is None else cache[e], stability_diagnostics=diagnostics,
                     stability_scope=scope)
            w = weights[..., e:e + 1]
            mixed = mixed + w.to(y.dtype) * y
            if expert_outputs is not None:
                expert_outputs.append((y, w))
            if updated is not None:
                updated.append(torch.where(w > 0, y, start))
        return mixed, updated

    def _is_v1(self):
        """No v2 feature is on: the plain HRM v1 backbone forward applies."""
        c = self.gate_config
        return (c.recurrence_mode == "hierarchical" and not c.gates_enabled and c.residual_branches == 1
                and c.moe_num_experts == c.mos_num_experts == c.h_memory_branches == c.l_memory_branches == 1)

    # ---------------------------------------------------------------- forward
    def forward(self, carry, x, cache=None, bp_steps=2, stability_diagnostics=None, **seq_info):
        category = seq_info.pop("routing_category", None)
        if self.ngram_enabled:
            x = self.ngram(x, seq_info.pop("token_ids"), seq_info.get("position_ids"),
                           None if cache is None else cache["ngram_history"])
        if self._is_v1():
            return super().forward(carry, x, cache=cache, bp_steps=bp_steps,
                                   stability_diagnostics=stability_diagnostics, **seq_info)
        run = _Pass(self, x, cache, stability_diagnostics, seq_info, category)
        h_window, l_window = backward_call_counts(self.H_cycles, self.L_cycles, bp_steps,
                                                  has_h_stack=self.has_h_stack)
        record = torch.is_grad_enabled()
        last_l = self.L_cycles - 1
        for call in _schedule(self.H_cycles, self.L_cycles, h_window, l_window):
            if call.level == "L":
                if call.slot % self.L_cycles == 0:
                    run.begin_cycle()
                run.collect = [] if self.gate_config.h_branch_l_mixing and call.slot % self.L_cycles == last_l else None
                with torch.set_grad_enabled(record and call.grad):
                    self._run_l(run, call.slot)
            elif not self.has_h_stack:
                run.z_H = run.z_L
            else:
                with torch.set_grad_enabled(record and call.grad):
                    self._run_h(run, call.slot)
        return None, run.z_H

    def _run_l(self, run, k):
        """One L-stack invocation (dense or MoS; optional L memory)."""
        run.read_memory("L")
        context = run.context
        if context is None and (run.mixture or self.gate_config.gates_enabled):
            context = torch.zeros_like(run.z_H)
        if run.mixture:
            run.z_L, run.states = self._mos_step(run.z_L, context, run.states, k, run.cache, run.diagnostics,
                                                 run.info["L"], run.routes, run.mos_bias, run.collect)
        else:
            run.z_L = self._l_invocation(run.z_L, context, k, run.cache, run.diagnostics, run.info["L"])
        run.write_memory("L")

    def _run_h(self, run, i):
        """One H-stack invocation: persistent residual streams, looped (no injection), or gated."""
        cfg = self.gate_config
        run.read_memory("H")
        if run.looped:
            run.z_H = run.z_L
        h_cache = None if run.cache is None else run.cache["H"][i]
        scope = None if run.diagnostics is None else f"H/cycle_{i:03d}"
        if cfg.h_residual_persistence or cfg.h_branch_l_mixing:
            if not cfg.h_residual_persistence:
                run.h_streams = self.H_level.core.initialize_streams(run.z_H)
            l_side = self.H_level.l_branch_mixer(run.collect) if cfg.h_branch_l_mixing else run.z_L.unsqueeze(-2)
            run.h_streams, run.z_H = self.H_level(run.h_streams, self._inject(self.H_level, i, run.h_streams, l_side),
                                                  **run.info["H"], stream_input=True, return_streams=True,
                                                  cache=h_cache, stability_diagnostics=run.diagnostics,
                                                  stability_scope=scope)
            return  # the stream options exclude an H memory (validated)
        if run.looped and run.diagnostics is None:
            run.z_H = self.H_level.core(run.z_H, **run.info["H"], cache=h_cache)  # z + 0: no injection add
        else:
            injection = torch.zeros_like(run.z_L) if run.looped else self._inject(self.H_level, i, run.z_H, run.z_L)
            run.z_H = self.H_level(run.z_H, injection, **run.info["H"], cache=h_cache,
                                   stability_diagnostics=run.diagnostics, stability_scope=scope)
        run.write_memory("H")

    def _l_invocation(self, z_L, context, k, cache, diagnostics, info):
        layer_cache = None if cache is None else cache["L"][k]
        if context is None:
            # Looped mode without gates or mixture: the L stack input is z_L itself (z_L + 0).
            if diagnostics is None:
                return self.L_level.core(z_L, **info, cache=layer_cache)
            context = torch.zeros_like(z_L)
        return self.L_level(z_L, self._inject(self.L_level, k, z_L, context), **info, cache=layer_cache,
                            stability_diagnostics=diagnostics,
                            stability_scope=None if diagnostics is None else f"L/cycle_{k:03d}")

    def _mos_step(self, z_L, context, states, k, cache, diagnostics, info, routes, mos_bias, expert_outputs):
        layer_cache = None if cache is None else cache["L"][k]
        if not self.gate_config.mos_sparse:
            return self._stack_step(z_L, context, states, k, layer_cache, diagnostics, info, mos_bias,
                                    expert_outputs=expert_outputs)
        from mimir_b200.models.sparse_stacks import batched_sparse_stack_step, sparse_stack_step
        if cache is None and z_L.ndim < 3 and context.ndim < 3:
            return sparse_stack_step(self, z_L, context, states, k, diagnostics, info, routes,
                                     expert_outputs=expert_outputs)
        return batched_sparse_stack_step(self, z_L, context, states, k, diagnostics, info, routes, layer_cache,
                                         expert_outputs=expert_outputs)

    # ---------------------------------------------------------------- schedules
    def compute_train_extra_args(self, train_state):
        cfg = self.gate_config
        step = train_state.step
        if hasattr(self, "routing_bias_scale"):
            start, end = cfg.routing_bias_decay_start, cfg.routing_bias_decay_end
            self.routing_bias_scale.fill_(max(0.0, min(1.0, (end - step) / (end - start))) if end else 1.0)

        def ramp(start, steps):
            return min(1.0, max(0, step - start) / steps) if steps else 1.0

        for name in ("H", "L"):
            memory = getattr(getattr(self, f"{name}_level"), "memory", None)
            if memory is not None:
                memory.alpha.fill_(ramp(cfg.memory_warmup_start_step, cfg.memory_warmup_steps))
        if self.ngram_enabled:
            self.ngram.alpha.fill_(ramp(cfg.ngram_warmup_start_step, cfg.ngram_warmup_steps))
        if cfg.gates_enabled:
            self.gate_alpha.fill_(cfg.gate_alpha_max * ramp(cfg.gate_warmup_start_step, cfg.gate_warmup_steps))
        if cfg.residual_branches > 1:
            alpha = cfg.residual_alpha_max * ramp(cfg.residual_warmup_start_step, cfg.residual_warmup_steps)
            for m in self.modules():
                if isinstance(m, BranchedTransformer):
                    m.residual_alpha.fill_(alpha)
        return super().compute_train_extra_args(train_state)

    def configure_gate_updates(self, optimizer, bp_steps):
        """Passive invocation gates (outside this step's backward window) follow the first active
        gate of their level: ``optimizer.shared_parameter_updates`` maps each passive gate
        parameter to its donor (empty without gates or when the donor is frozen)."""
        windows = dict(zip(("H", "L"), backward_call_counts(self.H_cycles, self.L_cycles, bp_steps,
                                                             has_h_stack=self.has_h_stack)))
        mapping = {}
        if self.gate_config.gates_enabled:
            for name in ("H", "L"):
                gates = getattr(self, f"{name}_level").invocation_gates
                first_active = len(gates) - windows[name]
                donor = gates[first_active]
                if any(p.requires_grad for p in donor.parameters()):
                    for passive in gates[:first_active]:
                        mapping.update(zip(passive.parameters(), donor.parameters()))
        optimizer.shared_parameter_updates = mapping
