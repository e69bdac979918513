"""Token-level MLP expert mixtures (MoE), their router, and dense->MoE upcycling.

Reference behaviour: ``src/mimir/model/expert_mixtures.py`` (router ``:11-66``, dense
and sparse mixture ``:69-104``, upcycling ``:107-165``) and
``src/mimir/model/routed_block.py:7-22``.

* The router keeps one parameter row and one bias per expert (so freezing expert 0 is
  real), computes fp32 scores, breaks ties by a stable descending sort, and returns
  softmax-over-top-k weights, or sigmoid affinities renormalised over the top-k when
  aux-loss-free balancing is on (the per-expert ``selection_bias`` only steers selection).
* For top-1 with several experts a straight-through surrogate gives the router a gradient.
* The sparse path runs each expert only on its tokens and still calls every expert (even
  with zero tokens) so all ranks issue identical collectives.  The token lists of all experts
  come from one stable (expert, token) ordering (:mod:`mimir_b200.ops.moe`) with a single
  host transfer of the per-expert counts.
"""
from __future__ import annotations

import copy
import re

import torch
from torch import nn

from mimir_b200 import ops
from mimir_b200.models.transformer import TransformerBlock


class TopKRouter(nn.Module):
    def __init__(self, hidden_size, n, k, *, freeze_base=False, top1_straight_through=True,
                 balance_enabled=False, balance_update_rate=0.001, init_std=None):
        super().__init__()
        if not 1 <= k <= n:
            raise ValueError("Routing requires 1 <= k <= n")
        self.n, self.k = n, k
        self.balance_enabled = balance_enabled
        self.balance_update_rate = balance_update_rate
        if balance_enabled:
            self.register_buffer("selection_bias", torch.zeros(n, dtype=torch.float32))
        self.top1_straight_through = top1_straight_through
        self.rows = nn.ParameterList([nn.Parameter(torch.zeros(hidden_size), requires_grad=not (freeze_base and i == 0))
                                      for i in range(n)])
        self.biases = nn.ParameterList([nn.Parameter(torch.zeros(1), requires_grad=not (freeze_base and i == 0))
                                        for i in range(n)])
        if init_std is not None:  # from-scratch MoE: random rows (zeros route every token to experts 0..k-1)
            with torch.no_grad():
                for row in self.rows:
                    row.normal_(0.0, init_std)
        self.register_buffer("logit_bias", torch.zeros(n))

    def _apply(self, fn, recurse=True):
        # The balancing bias is a counter-driven fp32 quantity: keep it fp32 through .to(dtype).
        before = getattr(self, "selection_bias", None)
        out = super()._apply(fn, recurse=recurse)
        if self.balance_enabled:
            self.selection_bias = (self.selection_bias.float() if before.is_meta
                                   else before.to(device=self.selection_bias.device, dtype=torch.float32))
        return out

    def scores(self, x, logit_bias=None):
        from mimir_b200.ops.router import router_logits
        from mimir_b200.ops.stacked import stacked  # one gradient kernel for all rows under the replicated engine
        s = router_logits(x, stacked(self.rows), stacked(self.biases).reshape(-1)) + self.logit_bias.float()
        if logit_bias is not None:
            s = s + logit_bias.float()
        return s

    def _select(self, selection):
        """Top-k experts per token (stable: ties go to the lower index).  CUDA: one kernel that also
        adds this forward's selections to the routing-balance counts (``csrc/router.cu``)."""
        from mimir_b200.ops._ext import kernels_enabled
        if kernels_enabled(selection) and self.n <= 256:
            from mimir_b200.ops._ext import ext
            from mimir_b200.optim.routing_balance import load_counter
            load = load_counter(self) if self.balance_enabled else None
            flat = selection.detach().reshape(-1, self.n).float().contiguous()
            return ext().router_topk(flat, self.k, load).view(*selection.shape[:-1], self.k), True
        return selection.argsort(dim=-1, descending=True, stable=True)[..., :self.k], False

    def forward(self, x, logit_bias=None, return_indices=False):
        scores = self.scores(x, logit_bias)
        tiny = torch.finfo(torch.float32).tiny
        if self.balance_enabled:
            affinity = scores.sigmoid()
            selection = affinity + self.selection_bias.float()
        else:
            affinity = selection = scores
        chosen, counted = self._select(selection)
        mask = torch.zeros_like(scores, dtype=torch.bool).scatter(-1, chosen, True)
        if self.balance_enabled and not counted:
            from mimir_b200.optim.routing_balance import record_load
            record_load(self, mask)
            weights = affinity * mask
            weights = weights / weights.sum(-1, keepdim=True).clamp_min(tiny)
        else:
            weights = scores.masked_fill(~mask, -torch.inf).softmax(-1)
        if self.k == 1 and self.n > 1 and self.top1_straight_through:
            probs = (affinity / affinity.sum(-1, keepdim=True).clamp_min(tiny)) if self.balance_enabled \
                else scores.softmax(-1)
            surrogate = probs * mask
            weights = weights + (surrogate - surrogate.detach())
        return (weights, chosen) if return_indices else weights


class MLPMixture(nn.Module):
    """Router + experts (+ optional always-on shared experts).

    ``expert_intermediate_size`` gives the experts their own SwiGLU width (otherwise they are
    copies of the dense MLP, as in the reference).  ``grouped`` runs the sparse path as one
    token exchange: the top-k slots are permuted into per-expert row blocks, each expert runs
    one GEMM pair on its block and the outputs are combined with the routing weights
    (:func:`mimir_b200.ops.moe.grouped_experts`).  ``expert_parallel`` additionally splits the
    experts over the ranks: this rank keeps experts ``first .. first + local - 1`` (still named
    ``experts.<global index>``) and exchanges token rows with the other ranks over NVLink.
    """

    def __init__(self, mlp, hidden_size, n, k, *, freeze_base=False, top1_straight_through=True, sparse=False,
                 balance_enabled=False, balance_update_rate=0.001, expert_intermediate_size=None, shared_experts=0,
                 grouped=False, expert_parallel=False, router_init_std=None):
        super().__init__()
        if expert_intermediate_size is None:
            make = lambda i: mlp if i == 0 else copy.deepcopy(mlp)  # noqa: E731
        else:
            from mimir_b200.models.layers import SwiGLU
            make = lambda i: SwiGLU(hidden_size, expert_intermediate_size)  # noqa: E731
        self.sparse, self.grouped, self.k, self.n = sparse, grouped or expert_parallel, k, n
        self.expert_parallel = expert_parallel
        if expert_parallel:
            import torch.distributed as dist
            world = dist.get_world_size() if dist.is_initialized() else 1
            rank = dist.get_rank() if dist.is_initialized() else 0
            if n % world:
                raise ValueError(f"{n} experts cannot be split over {world} expert-parallel ranks")
            local = n // world
            experts = [make(i) for i in range(n)]  # every rank draws every expert's init: EP-independent weights
            self.experts = nn.ModuleDict({str(i): experts[i] for i in range(rank * local, (rank + 1) * local)})
            del experts
            for p in self.experts.parameters():
                p._mimir_rank_local = True
            self.expert_ids = list(range(rank * local, (rank + 1) * local))
        else:
            self.experts = nn.ModuleList([make(i) for i in range(n)])
            self.expert_ids = list(range(n))
        # registered after the experts: the reference's parameter (and state_dict) order
        self.router = TopKRouter(hidden_size, n, k, freeze_base=freeze_base,
                                 top1_straight_through=top1_straight_through, balance_enabled=balance_enabled,
                                 balance_update_rate=balance_update_rate, init_std=router_init_std)
        width = expert_intermediate_size if expert_intermediate_size is not None else None
        if shared_experts:
            from mimir_b200.models.layers import SwiGLU
            self.shared_experts = nn.ModuleList(
                SwiGLU(hidden_size, width) if width is not None else copy.deepcopy(mlp) for _ in range(shared_experts))
        if freeze_base:
            self.experts[0].requires_grad_(False)

    def _expert(self, i):
        return self.experts[str(i)] if self.expert_parallel else self.experts[i]

    def _shared(self, x, stability_diagnostics=None, stability_scope=None):
        out = None
        for i, expert in enumerate(getattr(self, "shared_experts", [])):
            y = expert(x, stability_diagnostics=stability_diagnostics,
                       stability_scope=f"{stability_scope}/shared_{i}" if stability_scope else None)
            out = y if out is None else out + y
        return out

    def forward(self, x, stability_diagnostics=None, stability_scope=None, routing_bias=None):
        weights, chosen = self.router(x, routing_bias, return_indices=True)
        shared = self._shared(x, stability_diagnostics, stability_scope)
        if self.grouped and (stability_diagnostics is None or self.expert_parallel):
            out = self._grouped(x, weights, chosen)
        elif self.sparse:
            out = self._dispatch(x, weights, stability_diagnostics, stability_scope)
        else:
            out = torch.zeros_like(x)
            for i, expert in enumerate(self.experts):
                y = expert(x, stability_diagnostics=stability_diagnostics,
                           stability_scope=f"{stability_scope}/expert_{i}" if stability_scope else None)
                out = out + weights[..., i:i + 1].to(y.dtype) * y
        return out if shared is None else out + shared

    @torch.compiler.disable
    def _grouped(self, x, weights, chosen):
        from mimir_b200.ops.moe import grouped_experts
        from mimir_b200.parallel.expert import expert_parallel
        flat = x.reshape(-1, x.shape[-1])
        topi = chosen.reshape(-1, self.k)
        topw = weights.reshape(-1, self.n).gather(-1, topi)
        ep = expert_parallel(self.n if self.expert_parallel else self.n, flat.device,
                             distributed=self.expert_parallel)
        params = []
        for i in self.expert_ids:
            e = self._expert(i)
            params += [e.gate_up_proj.weight, e.down_proj.weight]
        return grouped_experts(flat, topw, topi, ep, params).reshape_as(x)

    @torch.compiler.disable
    def _dispatch(self, x, weights, diagnostics, scope):
        flat = x.reshape(-1, x.shape[-1])
        w = weights.reshape(-1, len(self.experts))
        plan = ops.moe_plan(w)  # per-expert token lists (one device sort; no per-expert nonzero)
        out = torch.zeros_like(flat)
        for i, expert in enumerate(self.experts):
            idx = plan.indices(i)
            y = expert(flat.index_select(0, idx), stability_diagnostics=diagnostics if idx.numel() else None,
                       stability_scope=f"{scope}/expert_{i}" if scope else None)
            out = out.index_add(0, idx, (y * w[idx, i, None].to(y.dtype)).to(out.dtype))  # autocast: y may be bf16
        return out.reshape_as(x)


def install_mlp_mixtures(core, hidden_size, n, k, **kwargs):
    if n > 1:
        for layer in core.layers:
            layer.mlp = MLPMixture(layer.mlp, hidden_size, n, k, **kwargs)


class RoutedBlock(TransformerBlock):
    """A block whose MLP mixture also receives a per-token routing (metadata) bias."""

    def __init__(self, original, norm_type):
        nn.Module.__init__(self)
        self.attn, self.mlp, self.norm = original.attn, original.mlp, original.norm
        self.norm_type = norm_type

    def forward(self, x, routing_bias=None, stability_diagnostics=None, stability_scope=None, **seq_info):
        attn_kw = dict(stability_diagnostics=stability_diagnostics,
                       stability_scope=f"{stability_scope}/attention" if stability_scope else None)
        mlp_kw = dict(routing_bias=routing_bias, stability_diagnostics=stability_diagnostics,
                      stability_scope=f"{stability_scope}/mlp" if stability_scope else None)
        if self.norm_type == "pre":
            x = x + self.attn(self.norm(x), **seq_info, **attn_kw)
            return x + self.mlp(self.norm(x), **mlp_kw)
        x = self.norm(x + self.attn(x, **seq_info, **attn_kw))
        return self.norm(x + self.mlp(x, **mlp_kw))


# ----------------------------------------------------------------------------------------
# Dense -> MoE/MoS upcycling
# ----------------------------------------------------------------------------------------
NEW_V2_COMPONENTS = {
    "router", "stack_router", "invocation_gates", "gate_alpha", "attn_residual", "mlp_residual", "residual_alpha",
    "residual_readout", "memory", "ngram", "routing_bias_scale", "l_branch_mixer", "shared_experts",
}


def dense_source_key(key: str) -> str:
    """Map an expert key (``...mlp.experts.3.x`` / ``...stack_experts.1.x``) to its dense origin."""
    key = re.sub(r"\.stack_experts\.\d+\.", ".core.", key)
    return re.sub(r"\.mlp\.experts\.\d+\.", ".mlp.", key)


def is_new_v2_key(key: str) -> bool:
    return bool(set(key.split(".")) & NEW_V2_COMPONENTS)


def upcycle_dense_weights(destination, source_state):
    """Copy a dense state dict into an expert model; every expert starts as the dense MLP/stack.

    Missing backbone keys, shape mismatches and unused source keys are errors.
    """
    state = destination.state_dict()
    used = set()
    for key, value in state.items():
        src = dense_source_key(key)
        if src not in source_state:
            if is_new_v2_key(key):
                continue
            raise ValueError(f"Missing dense backbone key: {src}")
        if source_state[src].shape != value.shape:
            raise ValueError(f"Shape mismatch for {key}: {source_state[src].shape} != {value.shape}")
        state[key] = source_state[src].detach().clone()
        used.add(src)
    if set(source_state) != used:
        raise ValueError(f"Unexpected dense source keys: {set(source_state) - used}")
    destination.load_state_dict(state, strict=True)


def upcycle_training_state(destination, optimizer, source_model, source_optimizer):
    """Upcycle weights and clone every optimizer slot (moments, EMA) of the dense source."""
    if type(optimizer) is not type(source_optimizer):
        raise ValueError("Upcycling must retain the optimizer type")
    upcycle_dense_weights(destination, source_model.state_dict())
    src_params = dict(source_model.named_parameters())
    for name, p in destination.named_parameters():
        src = dense_source_key(name)
        if src in src_params:
            state = source_optimizer.state[src_params[src]]
            if set(state) != set(optimizer.state[p]):
                raise ValueError(f"Optimizer slot mismatch for {name}")
            optimizer.state[p] = copy.deepcopy(state)
        elif not is_new_v2_key(name):
            raise ValueError(f"Missing optimizer source for {name}")
