"""Multi-stream residual branches, branch-specific MoS mixing and recurrent memory branches.

Behavioural reference: ``src/mimir/model/residual_branches.py:13-155`` and
``src/mimir/model/recurrent_memory.py:7-23``.

A branched stack carries ``B`` residual streams per token (shape ``[..., B, d]``).  Around every
sublayer (attention, MLP) a :class:`ResidualConnection` does two per-channel softmax mixes over
the branch axis:

* read:  ``x = sum_b softmax_b(alpha * read_logits)[b] * stream[b]``  -> the sublayer input,
* write: ``stream[b] += B * softmax_b(alpha * write_logits)[b] * update``.

``residual_alpha`` scales every logit, so at alpha = 0 all mixes are uniform and the branched
stack computes exactly what a single stream would.  With ``input_dependent`` the logits also get
``tanh(stream) * gain`` (zero-initialised gains).  Write logits start slightly asymmetric (each
sublayer prefers one branch) without consuming the RNG, so seeds keep their meaning.

Parameter and buffer names (``read_logits``, ``write_logits``, ``read_gain``, ``write_gain``,
``attn_residual``, ``mlp_residual``, ``residual_readout``, ``residual_alpha``, ``logits``,
``alpha``) are the checkpoint interface.
"""
from __future__ import annotations

import torch
from torch import nn

from mimir_b200.models.transformer import Transformer, TransformerBlock
from mimir_b200.ops import branches as fused


def _fanout(x: torch.Tensor, branches: int) -> torch.Tensor:
    """``[..., d]`` -> ``[..., branches, d]`` (a broadcast view: every branch starts equal)."""
    return x.unsqueeze(-2).expand(*x.shape[:-1], branches, x.shape[-1])


def _asymmetric_logits(branches: int, width: int, preferred: int, scale: float) -> torch.Tensor:
    """Zero-mean logits over the branch axis with ``scale`` extra on the preferred branch."""
    logits = torch.full((branches, width), -scale / branches)
    logits[preferred % branches] += scale
    return logits


class ResidualConnection(nn.Module):
    def __init__(self, branches, hidden_size, preferred_branch, init_scale, input_dependent=False):
        super().__init__()
        self.branches = branches
        self.read_logits = nn.Parameter(torch.zeros(branches, hidden_size))
        self.write_logits = nn.Parameter(_asymmetric_logits(branches, hidden_size, preferred_branch, init_scale))
        if input_dependent:
            self.read_gain = nn.Parameter(torch.zeros(branches, hidden_size))
            self.write_gain = nn.Parameter(torch.zeros(branches, hidden_size))

    def weights(self, streams, alpha, kind):
        """Softmax over the branch axis of ``alpha * (logits [+ tanh(streams) * gain])``, fp32."""
        logits = (self.read_logits if kind == "read" else self.write_logits).float()
        gain = getattr(self, f"{kind}_gain", None)
        if gain is not None:
            logits = logits + streams.float().tanh() * gain.float()
        return (alpha.float() * logits).softmax(dim=-2)

    def read(self, streams, alpha):
        if fused.fused_supported(streams, alpha):  # one CUDA kernel (ops/branches.py)
            return fused.branch_read(streams, self.read_logits, getattr(self, "read_gain", None), alpha)
        mixed = (streams.float() * self.weights(streams, alpha, "read")).sum(dim=-2)
        return mixed.to(streams.dtype)

    def write(self, streams, update, alpha):
        if fused.fused_supported(streams, alpha):
            return fused.branch_write(streams, update, self.write_logits, getattr(self, "write_gain", None), alpha)
        share = self.branches * self.weights(streams, alpha, "write")
        return (streams.float() + share * update.float().unsqueeze(-2)).to(streams.dtype)


class BranchedTransformerBlock(TransformerBlock):
    """A pre-norm block whose two sublayers read from and write to the residual streams."""

    def __init__(self, original, branches, hidden_size, layer_index, init_scale, input_dependent=False):
        nn.Module.__init__(self)
        self.attn, self.mlp, self.norm = original.attn, original.mlp, original.norm
        self.norm_type = "pre"
        self.attn_residual = ResidualConnection(branches, hidden_size, 2 * layer_index, init_scale, input_dependent)
        self.mlp_residual = ResidualConnection(branches, hidden_size, 2 * layer_index + 1, init_scale,
                                               input_dependent)

    def _around(self, streams, connection, alpha, sublayer):
        return connection.write(streams, sublayer(self.norm(connection.read(streams, alpha))), alpha)

    def forward(self, streams, residual_alpha, stability_diagnostics=None, stability_scope=None, **seq_info):
        if stability_diagnostics is not None and stability_scope is None:
            raise ValueError("stability_scope is required when diagnostics are enabled")
        routing_bias = seq_info.pop("routing_bias", None)

        def scope(name):
            return f"{stability_scope}/{name}" if stability_scope else None

        def attention(x):
            return self.attn(x, **seq_info, stability_diagnostics=stability_diagnostics,
                             stability_scope=scope("attention"))

        def mlp(x):
            extra = {"routing_bias": routing_bias} if hasattr(self.mlp, "router") else {}
            return self.mlp(x, **extra, stability_diagnostics=stability_diagnostics, stability_scope=scope("mlp"))

        streams = self._around(streams, self.attn_residual, residual_alpha, attention)
        streams = self._around(streams, self.mlp_residual, residual_alpha, mlp)
        if stability_diagnostics is not None:
            stability_diagnostics.record_tensor(f"activation/{stability_scope}/residual_streams", streams,
                                                record_gradient=True)
        return streams


class BranchedTransformer(Transformer):
    """Wraps an existing stack (sharing its modules) and runs it over ``B`` residual streams; the
    output is a softmax readout of the streams followed by the stack's final norm."""

    def __init__(self, original: Transformer, branches, init_scale=0.1, input_dependent=False):
        nn.Module.__init__(self)
        if branches < 2:
            raise ValueError("Use the original Transformer for a single residual branch")
        self.branches = branches
        self.head_hint = original.head_hint
        self.norm_f = original.norm_f
        self._cache_heads, self._cache_head_dim = original._cache_heads, original._cache_head_dim
        self._cache_layers = original._cache_layers
        if hasattr(original, "rotary_emb"):
            self.rotary_emb = original.rotary_emb
        hidden = original.head_hint["in"]["dim"]
        self.layers = nn.ModuleList(BranchedTransformerBlock(block, branches, hidden, i, init_scale, input_dependent)
                                    for i, block in enumerate(original.layers))
        self.residual_readout = nn.Parameter(torch.zeros(branches, hidden))
        self.register_buffer("residual_alpha", torch.tensor(0.0))

    def initialize_streams(self, x):
        return _fanout(x, self.branches)

    def process_streams(self, streams, cache=None, stability_diagnostics=None, stability_scope=None, **seq_info):
        if stability_diagnostics is not None and stability_scope is None:
            raise ValueError("stability_scope is required when diagnostics are enabled")
        seq_info = self.rope_info(dict(seq_info))
        for i, block in enumerate(self.layers):
            streams = block(streams, residual_alpha=self.residual_alpha, **seq_info,
                            cache=None if cache is None else cache[i], stability_diagnostics=stability_diagnostics,
                            stability_scope=f"{stability_scope}/layer_{i:03d}" if stability_scope else None)
        return streams

    def readout(self, streams, stability_diagnostics=None, stability_scope=None):
        if fused.fused_supported(streams, self.residual_alpha):
            out = self.norm_f(fused.branch_read(streams, self.residual_readout, None, self.residual_alpha))
        else:
            weights = (self.residual_alpha.float() * self.residual_readout.float()).softmax(dim=0)
            out = self.norm_f((streams.float() * weights).sum(dim=-2).to(streams.dtype))
        if stability_diagnostics is not None:
            stability_diagnostics.record_tensor(f"activation/{stability_scope}/final_norm", out, record_gradient=True)
        return out

    def forward(self, x, cache=None, stability_diagnostics=None, stability_scope=None, stream_input=False,
                return_streams=False, **seq_info):
        streams = self.process_streams(x if stream_input else self.initialize_streams(x), cache=cache,
                                       stability_diagnostics=stability_diagnostics, stability_scope=stability_scope,
                                       **seq_info)
        out = self.readout(streams, stability_diagnostics, stability_scope)
        return (streams, out) if return_streams else out


class BranchExpertMixer(nn.Module):
    """Per-H-branch reweighting of the MoS experts selected for a token.

    Each H branch ``b`` takes the router weights ``w_e`` of the active experts, multiplies them by
    ``exp(logits[b, e])`` (normalised over the active experts), and rescales the result to the
    router's total mass, so zero logits reproduce the router weighting and the top-1
    straight-through derivative survives.  Logits start with each branch preferring one expert.
    """

    def __init__(self, branches, experts, init_scale=0.1):
        super().__init__()
        logits = torch.full((branches, experts), -init_scale / experts)
        logits[torch.arange(branches), torch.arange(branches) % experts] += init_scale
        self.logits = nn.Parameter(logits)

    def forward(self, expert_outputs):
        values = torch.stack([value for value, _ in expert_outputs], dim=-2)            # [..., E, d]
        router = torch.cat([w.expand(*values.shape[:-2], 1) for _, w in expert_outputs], dim=-1).float()  # [..., E]
        off = ~(router > 0).unsqueeze(-2)                                               # [..., 1, E]
        logits = self.logits.float().expand(*router.shape[:-1], *self.logits.shape)     # [..., B, E]
        peak = logits.masked_fill(off, -torch.inf).amax(-1, keepdim=True)
        preference = (logits - peak).masked_fill(off, -torch.inf).exp()
        mix = router.unsqueeze(-2) * preference
        mix = mix / mix.sum(-1, keepdim=True).clamp_min(torch.finfo(torch.float32).tiny)
        mix = mix * router.sum(-1)[..., None, None]
        return torch.einsum("...be,...ed->...bd", mix, values.float()).to(values.dtype)


class RecurrentMemory(ResidualConnection):
    """Depth-recurrent memory branches.  Reading mixes the branches like a residual read; an update
    keeps ``alpha * (1 - write weight)`` of each branch and takes the rest from the new state, so
    at alpha = 0 every branch is simply replaced by it."""

    def __init__(self, branches, hidden_size):
        super().__init__(branches, hidden_size, 0, 0.1, input_dependent=True)
        self.register_buffer("alpha", torch.tensor(0.0))

    def initialize(self, x):
        return _fanout(x, self.branches)

    def read_state(self, states):
        return self.read(states, self.alpha)

    def update(self, states, candidate):
        keep = self.alpha * (1 - self.weights(states, self.alpha, "write"))
        return (keep * states.float() + (1 - keep) * candidate.float().unsqueeze(-2)).to(candidate.dtype)
