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
        h_layers = self.H_override.get("n_layers", self.n_layers)
        looped = self.recurrence_mode == "looped"
        if self.moe_aux_loss_free and self.moe_num_experts < 2:
            raise ValueError("MoE balancing requires multiple MoE experts")
        if self.mos_aux_loss_free and self.mos_num_experts < 2:
            raise ValueError("MoS balancing requires multiple MoS experts")
        if self.n_layers < 1 or h_layers < 0:
            raise ValueError("L requires positive layers and H requires nonnegative layers")
        if h_layers == 0 and not looped:
            raise ValueError("Zero-layer H requires looped recurrence")
        if self.h_residual_persistence or self.h_branch_l_mixing:
            if (looped or h_layers == 0 or self.residual_branches < 2 or self.residual_levels not in ("H", "both")):
                raise ValueError("H stream options require hierarchical recurrence and multiple H residual branches")
            if self.h_memory_branches > 1:
                raise ValueError("H stream options cannot be combined with H recurrent memory")
            if self.gate_initialize_from_v1:
                raise ValueError("H stream options require explicit upcycling, not gate-only migration")
        if self.h_branch_l_mixing and (self.mos_num_experts < 2 or self.l_memory_branches > 1):
            raise ValueError("Branch-specific L mixing requires MoS and no L recurrent memory")
        if looped and (self.gates_enabled or self.h_memory_branches > 1 or self.l_memory_branches > 1
                       or self.mos_state_mode != "shared"):
            raise ValueError("Looped recurrence requires shared MoS state, no invocation gates, "
                             "and no recurrent memory branches; residual branches are supported")
        if self.mos_sparse and self.mos_sparse_routing == "prefix_mean" and self.attn_type != "prefixlm":
            raise ValueError("Prefix-mean routing requires PrefixLM prompt visibility")
        for rows, count in ((self.moe_metadata_bias, self.moe_num_experts), (self.mos_metadata_bias, self.mos_num_experts)):
            if any(len(r) != count or not all(math.isfinite(v) for v in r) for r in rows):
                raise ValueError("Metadata bias rows must contain one finite logit per expert")
        if self.routing_bias_decay_end and self.routing_bias_decay_end <= self.routing_bias_decay_start:
            raise ValueError("Routing bias decay end must follow start")
        if self.specialist_training and not self.expert_freeze_base:
            raise ValueError("Specialist training requires a frozen reference expert")
        if self.mos_state_mode == "separate" and self.l_memory_branches > 1:
            raise ValueError("Choose expert-specific L states or general L memory branches, not both")
        if self.upcycle_from_dense and self.gate_initialize_from_v1:
            raise ValueError("Use only one migration mode")
        if self.gate_initialize_from_v1 and not self.gates_enabled:
            raise ValueError("gate_initialize_from_v1 requires gates_enabled=true")
        if (self.moe_dispatch == "grouped" or self.moe_expert_parallel) and not (self.moe_sparse
                                                                               and self.moe_num_experts > 1):
            raise ValueError("The grouped MoE dispatch and expert parallelism need moe_sparse with several experts")
        if self.moe_expert_parallel and self.moe_dispatch != "grouped":
            raise ValueError("moe_expert_parallel requires moe_dispatch=grouped")
        if self.upcycle_from_dense and (self.moe_expert_intermediate_size is not None or self.moe_shared_experts):
            raise ValueError("Upcycling copies the dense MLP: it needs the dense expert width and no shared experts")
        if self.moe_expert_parallel and (self.specialist_training or self.expert_freeze_base):
            raise ValueError("Expert parallelism does not support specialist training or a frozen base expert")
        if self.moe_top_k > self.moe_num_experts or self.mos_top_k > self.mos_num_experts:
            raise ValueError("Expert top_k must not exceed num_experts")
        if self.gate_initialize_from_v1 and (self.moe_num_experts > 1 or self.mos_num_experts > 1
                                             or self.residual_branches > 1):
            raise ValueError("Expert/branch upcycling requires upcycle_from_dense; "
                             "gate_initialize_from_v1 only migrates gates")
        if self.residual_branches > 1:
            for level in ("L", "H"):
                norm = self.H_override.get("norm_type", self.norm_type) if level == "H" else self.norm_type
                if self.residual_levels in (level, "both") and norm != "pre":
                    raise ValueError("Multiple residual branches currently require pre-norm")
        if self.expert_freeze_base and self.moe_num_experts == self.mos_num_experts == 1:
            raise ValueError("expert_freeze_base requires an expert mixture")
        return self


class InvocationGate(nn.Module):
    """``injection * (1 + alpha * tanh(W [hidden; injection] + b))``, zero-initialised (no RNG)."""

    def __init__(self, hidden_size):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(hidden_size, 2 * hidden_size))
        self.bias = nn.Parameter(torch.zeros(hidden_size))

    def forward(self, hidden, injection, alpha):
        hidden, injection = torch.broadcast_tensors(hidden, injection)
        x = torch.cat((hidden, injection), dim=-1)
        gate = F.linear(x, self.weight.to(x.dtype), self.bias.to(x.dtype))
        return injection * (1 + alpha.to(x.dtype) * torch.tanh(gate))


class Mimir2(RecurrentBackbone):
    def __init__(self, config_dict):
        config = Mimir2Config(**config_dict)
        if config.H_cycles < 1 or config.L_cycles < 1:
            raise ValueError("HRM v2 requires positive H/L cycles")
        super().__init__(config_dict)
        self.gate_config = config
        self.has_h_stack = config.H_override.get("n_layers", config.n_layers) > 0
        router_opts = dict(freeze_base=config.expert_freeze_base,
                           top1_straight_through=config.router_top1_straight_through)
        for name in ("L", "H"):
            level = getattr(self, f"{name}_level")
            if name == "H" and not self.has_h_stack:
                continue
            if config.moe_levels in (name, "both"):
                install_mlp_mixtures(level.core, self.hidden_size, config.moe_num_experts, config.moe_top_k,
                                     sparse=config.moe_sparse, balance_enabled=config.moe_aux_loss_free,
                                     balance_update_rate=config.routing_bias_update_rate,
                                     expert_intermediate_size=config.moe_expert_intermediate_size,
                                     shared_experts=config.moe_shared_experts, grouped=config.moe_dispatch == "grouped",
                                     expert_parallel=config.moe_expert_parallel,
                                     router_init_std=config.moe_router_init_std, **router_opts)
                if config.moe_num_experts > 1:
                    norm = config.H_override.get("norm_type", config.norm_type) if name == "H" else config.norm_type
                    level.core.layers = nn.ModuleList(RoutedBlock(b, norm) for b in level.core.layers)
            if config.residual_branches > 1 and config.residual_levels in (name, "both"):
                level.core = BranchedTransformer(level.core, config.residual_branches, config.residual_write_init_scale,
                                                 config.residual_input_dependent)
        if config.h_branch_l_mixing:
            self.H_level.l_branch_mixer = BranchExpertMixer(config.residual_branches, config.mos_num_experts)
        if config.mos_num_experts > 1:
            self.L_level.stack_experts = nn.ModuleList(copy.deepcopy(self.L_level.core)
                                                       for _ in range(config.mos_num_experts - 1))
            self.L_level.stack_router = TopKRouter(self.hidden_size, config.mos_num_experts, config.mos_top_k,
                                                   balance_enabled=config.mos_aux_loss_free,
                                                   balance_update_rate=config.routing_bias_update_rate, **router_opts)
            if config.expert_freeze_base:
                self.L_level.core.requires_grad_(False)
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
        if (config.ngram_orders or config.h_memory_branches > 1 or config.l_memory_branches > 1 or config.moe_sparse
                or config.mos_sparse or config.residual_input_dependent or config.h_residual_persistence
                or config.h_branch_l_mixing):
            for m in self.modules():
                if isinstance(m, TransformerBlock):
                    m._v2_explicit_checkpoint = True

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
        values = getattr(self.gate_config, f"{kind}_metadata_bias")
        if not self.training or self.gate_config.specialist_router_calibration or category is None or not values:
            return None
        table = torch.tensor(values, device=category.device, dtype=torch.float32)
        return table[category.long()] * self.routing_bias_scale

    def _inject(self, level, invocation, hidden, other):
        if not self.gate_config.gates_enabled:
            return other
        return level.invocation_gates[invocation](hidden, other, self.gate_alpha)

    def _stack_step(self, z_L, z_H, states, invocation, cache, diagnostics, seq_info, bias=None, expert_outputs=None):
        """Dense MoS: every L stack expert runs on all tokens; outputs are mixed token-locally."""
        weights = self.L_level.stack_router(z_L + z_H, bias)
        output = torch.zeros_like(z_H)
        next_states = []
        for e, core in enumerate([self.L_level.core, *self.L_level.stack_experts]):
            prev = states[e] if states is not None else z_L
            inj = self._inject(self.L_level, invocation, prev, z_H)
            y = core(prev + inj, **seq_info, cache=cache[e] if cache is not None else None,
                     stability_diagnostics=diagnostics,
                     stability_scope=f"L/cycle_{invocation:03d}/expert_{e}" if diagnostics is not None else None)
            w = weights[..., e:e + 1]
            output = output + w.to(y.dtype) * y
            if expert_outputs is not None:
                expert_outputs.append((y, w))
            if states is not None:
                next_states.append(torch.where(w > 0, y, prev))
        return output, (next_states if states is not None else None)

    def _is_v1(self):
        c = self.gate_config
        return (c.recurrence_mode == "hierarchical" and not c.gates_enabled and c.moe_num_experts == 1
                and c.mos_num_experts == 1 and c.residual_branches == 1
                and c.h_memory_branches == c.l_memory_branches == 1)

    # ---------------------------------------------------------------- forward
    def forward(self, carry, x, cache=None, bp_steps=2, stability_diagnostics=None, **seq_info):
        cfg = self.gate_config
        category = seq_info.pop("routing_category", None)
        if self.ngram_enabled:
            x = self.ngram(x, seq_info.pop("token_ids"), seq_info.get("position_ids"),
                           cache["ngram_history"] if cache is not None else None)
        if self._is_v1():
            return super().forward(carry, x, cache=cache, bp_steps=bp_steps,
                                   stability_diagnostics=stability_diagnostics, **seq_info)
        looped = cfg.recurrence_mode == "looped"
        z_H, z_L = x, self.zL_init
        h_streams = self.H_level.core.initialize_streams(x) if cfg.h_residual_persistence else None
        memories = {}
        for name, value in (("H", z_H), ("L", z_L)):
            memory = getattr(getattr(self, f"{name}_level"), "memory", None)
            if memory is not None:
                memories[name] = memory.initialize(value.expand_as(x))
        moe_bias, mos_bias = self._metadata_bias(category, "moe"), self._metadata_bias(category, "mos")
        level_info = {name: dict(seq_info) for name in ("L", "H")}
        for name in ("L", "H"):
            if moe_bias is not None and cfg.moe_levels in (name, "both"):
                level_info[name]["routing_bias"] = moe_bias
        mixture = cfg.mos_num_experts > 1
        routes = None
        if mixture and cfg.mos_sparse:
            from mimir_b200.models.sparse_stacks import cached_sequence_routes, sequence_routes
            routes = (cached_sequence_routes(self, x, cache, seq_info, mos_bias) if cache is not None else
                      sequence_routes(self.L_level.stack_router, x, seq_info, mos_bias, cfg.mos_sparse_routing))
        states = [self.zL_init] * cfg.mos_num_experts if mixture and cfg.mos_state_mode == "separate" else None
        h_bp, l_bp = backward_call_counts(self.H_cycles, self.L_cycles, bp_steps, has_h_stack=self.has_h_stack)
        grad = torch.is_grad_enabled()
        total_l = self.H_cycles * self.L_cycles
        for i in range(self.H_cycles):
            if looped:
                z_L = z_H
            l_context = None if looped else z_H  # looped: L sees no H injection (a zero tensor in the reference)
            expert_outputs = None
            for k in range(i * self.L_cycles, (i + 1) * self.L_cycles):
                expert_outputs = [] if cfg.h_branch_l_mixing and k == (i + 1) * self.L_cycles - 1 else None
                with torch.set_grad_enabled(grad and k >= total_l - l_bp):
                    if "L" in memories:
                        z_L = self.L_level.memory.read_state(memories["L"])
                    ctx = torch.zeros_like(z_H) if l_context is None and (mixture or cfg.gates_enabled) else l_context
                    if mixture:
                        z_L, states = self._mos_step(z_L, ctx, states, k, cache, stability_diagnostics,
                                                     level_info["L"], routes, mos_bias, expert_outputs)
                    else:
                        z_L = self._l_invocation(z_L, ctx, k, cache, stability_diagnostics, level_info["L"])
                    if "L" in memories:
                        memories["L"] = self.L_level.memory.update(memories["L"], z_L)
                        z_L = self.L_level.memory.read_state(memories["L"])
            if not self.has_h_stack:
                z_H = z_L
                continue
            with torch.set_grad_enabled(grad and i >= self.H_cycles - h_bp):
                if "H" in memories:
                    z_H = self.H_level.memory.read_state(memories["H"])
                if looped:
                    z_H = z_L
                if cfg.h_residual_persistence or cfg.h_branch_l_mixing:
                    if not cfg.h_residual_persistence:
                        h_streams = self.H_level.core.initialize_streams(z_H)
                    l_inj = (self.H_level.l_branch_mixer(expert_outputs) if cfg.h_branch_l_mixing
                             else z_L.unsqueeze(-2))
                    inj = self._inject(self.H_level, i, h_streams, l_inj)
                    h_streams, z_H = self.H_level(h_streams, inj, **level_info["H"], stream_input=True,
                                                  return_streams=True,
                                                  cache=cache["H"][i] if cache is not None else None,
                                                  stability_diagnostics=stability_diagnostics,
                                                  stability_scope=f"H/cycle_{i:03d}" if stability_diagnostics is not None else None)
                    continue
                h_cache = cache["H"][i] if cache is not None else None
                if looped and stability_diagnostics is None:
                    # The reference adds a zero injection here; x + 0 == x, so skip the add.
                    z_H = self.H_level.core(z_H, **level_info["H"], cache=h_cache)
                elif looped:
                    z_H = self.H_level(z_H, torch.zeros_like(z_L), **level_info["H"], cache=h_cache,
                                       stability_diagnostics=stability_diagnostics, stability_scope=f"H/cycle_{i:03d}")
                else:
                    inj = self._inject(self.H_level, i, z_H, z_L)
                    z_H = self.H_level(z_H, inj, **level_info["H"], cache=cache["H"][i] if cache is not None else None,
                                       stability_diagnostics=stability_diagnostics,
                                       stability_scope=f"H/cycle_{i:03d}" if stability_diagnostics is not None else None)
                if "H" in memories:
                    memories["H"] = self.H_level.memory.update(memories["H"], z_H)
                    z_H = self.H_level.memory.read_state(memories["H"])
        return None, z_H

    def _l_invocation(self, z_L, context, k, cache, diagnostics, info):
        scope = f"L/cycle_{k:03d}" if diagnostics is not None else None
        layer_cache = cache["L"][k] if cache is not None else None
        if context is None:
            # Looped mode without gates: the stack input is z_L itself (z_L + 0 in the reference).
            if diagnostics is None:
                return self.L_level.core(z_L, **info, cache=layer_cache)
            context = torch.zeros_like(z_L)
        inj = self._inject(self.L_level, k, z_L, context)
        return self.L_level(z_L, inj, **info, cache=layer_cache, stability_diagnostics=diagnostics,
                            stability_scope=scope)

    def _mos_step(self, z_L, context, states, k, cache, diagnostics, info, routes, mos_bias, expert_outputs):
        cfg = self.gate_config
        layer_cache = cache["L"][k] if cache is not None else None
        if cfg.mos_sparse:
            from mimir_b200.models.sparse_stacks import batched_sparse_stack_step, sparse_stack_step
            if cache is not None or z_L.ndim == 3 or context.ndim == 3:
                return batched_sparse_stack_step(self, z_L, context, states, k, diagnostics, info, routes, layer_cache,
                                                 expert_outputs=expert_outputs)
            return sparse_stack_step(self, z_L, context, states, k, diagnostics, info, routes,
                                     expert_outputs=expert_outputs)
        return self._stack_step(z_L, context, states, k, layer_cache, diagnostics, info, mos_bias,
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
        """Map every gate that gets no gradient this step to the first active gate of its level."""
        h_bp, l_bp = backward_call_counts(self.H_cycles, self.L_cycles, bp_steps, has_h_stack=self.has_h_stack)
        pairs = {}
        if self.gate_config.gates_enabled:
            for level, active in ((self.H_level, h_bp), (self.L_level, l_bp)):
                first = len(level.invocation_gates) - active
                donor = level.invocation_gates[first]
                if not any(p.requires_grad for p in donor.parameters()):
                    continue
                for gate in level.invocation_gates[:first]:
                    pairs.update(zip(gate.parameters(), donor.parameters()))
        optimizer.shared_parameter_updates = pairs
