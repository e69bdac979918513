"""Multi-stream residual branches, branch-specific MoS mixing, and recurrent memory.

Reference behaviour: ``src/mimir/model/residual_branches.py:13-155`` and
``src/mimir/model/recurrent_memory.py:7-23``.

A branched stack keeps ``B`` residual streams per token.  Each sublayer reads a softmax
mixture of the streams (weights per channel), runs once, and writes its update back to
all streams with ``B * softmax(write_logits)`` weights.  ``residual_alpha`` scales the
logits, so alpha = 0 reproduces a single stream exactly.  Writes are initialised slightly
asymmetrically (a preferred branch per sublayer) without consuming RNG.
"""
from __future__ import annotations

import torch
from torch import nn

from mimir_b200.models.transformer import Transformer, TransformerBlock


class ResidualConnection(nn.Module):
    def __init__(self, branches, hidden_size, preferred_branch, init_scale, input_dependent=False):
        super().__init__()
        self.read_logits = nn.Parameter(torch.zeros(branches, hidden_size))
        write = torch.full((branches, hidden_size), -init_scale / branches)
        write[preferred_branch % branches] += init_scale
        self.write_logits = nn.Parameter(write)
        self.branches = branches
        if input_dependent:
            self.read_gain = nn.Parameter(torch.zeros(branches, hidden_size))
            self.write_gain = nn.Parameter(torch.zeros(branches, hidden_size))

    def weights(self, streams, alpha, kind):
        logits = getattr(self, f"{kind}_logits").float()
        gain = getattr(self, f"{kind}_gain", None)
        if gain is not None:
            logits = logits + streams.float().tanh() * gain.float()
        return (alpha.float() * logits).softmax(dim=-2)

    def read(self, streams, alpha):
        w = self.weights(streams, alpha, "read")
        return (streams.float() * w).sum(dim=-2).to(streams.dtype)

    def write(self, streams, update, alpha):
        w = self.branches * self.weights(streams, alpha, "write")
        return (streams.float() + w * update.float().unsqueeze(-2)).to(streams.dtype)


class BranchedTransformerBlock(TransformerBlock):
    def __init__(self, original, branches, hidden_size, layer_index, init_scale, input_dependent=False):
        nn.Module.__init__(self)
        self.attn, self.mlp, self.norm = original.attn, original.mlp, original.norm
        self.norm_type = "pre"
        self.attn_residual = ResidualConnection(branches, hidden_size, 2 * layer_index, init_scale, input_dependent)
        self.mlp_residual = ResidualConnection(branches, hidden_size, 2 * layer_index + 1, init_scale,
                                               input_dependent)

    def forward(self, streams, residual_alpha, stability_diagnostics=None, stability_scope=None, **seq_info):
        routing_bias = seq_info.pop("routing_bias", None)
        if stability_diagnostics is not None and stability_scope is None:
            raise ValueError("stability_scope is required when diagnostics are enabled")
        x = self.norm(self.attn_residual.read(streams, residual_alpha))
        upd = self.attn(x, **seq_info, stability_diagnostics=stability_diagnostics,
                        stability_scope=f"{stability_scope}/attention" if stability_scope else None)
        streams = self.attn_residual.write(streams, upd, residual_alpha)
        x = self.norm(self.mlp_residual.read(streams, residual_alpha))
        extra = {"routing_bias": routing_bias} if hasattr(self.mlp, "router") else {}
        upd = self.mlp(x, **extra, stability_diagnostics=stability_diagnostics,
                       stability_scope=f"{stability_scope}/mlp" if stability_scope else None)
        streams = self.mlp_residual.write(streams, upd, residual_alpha)
        if stability_diagnostics is not None:
            stability_diagnostics.record_tensor(f"activation/{stability_scope}/residual_streams", streams,
                                                record_gradient=True)
        return streams


class BranchedTransformer(Transformer):
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
        return x.unsqueeze(-2).expand(*x.shape[:-1], self.branches, x.shape[-1])

    def process_streams(self, streams, cache=None, stability_diagnostics=None, stability_scope=None, **seq_info):
        if stability_diagnostics is not None and stability_scope is None:
            raise ValueError("stability_scope is required when diagnostics are enabled")
        seq_info = self.rope_info(dict(seq_info))
        for i, layer in enumerate(self.layers):
            streams = layer(streams, residual_alpha=self.residual_alpha, **seq_info,
                            cache=cache[i] if cache is not None else None,
                            stability_diagnostics=stability_diagnostics,
                            stability_scope=f"{stability_scope}/layer_{i:03d}" if stability_scope else None)
        return streams

    def readout(self, streams, stability_diagnostics=None, stability_scope=None):
        w = (self.residual_alpha.float() * self.residual_readout.float()).softmax(dim=0)
        out = self.norm_f((streams.float() * w).sum(dim=-2).to(streams.dtype))
        if stability_diagnostics is not None:
            stability_diagnostics.record_tensor(f"activation/{stability_scope}/final_norm", out, record_gradient=True)
        return out

    def forward(self, x, cache=None, stability_diagnostics=None, stability_scope=None, stream_input=False,
                return_streams=False, **seq_info):
        streams = x if stream_input else self.initialize_streams(x)
        streams = self.process_streams(streams, cache=cache, stability_diagnostics=stability_diagnostics,
                                       stability_scope=stability_scope, **seq_info)
        out = self.readout(streams, stability_diagnostics, stability_scope)
        return (streams, out) if return_streams else out


class BranchExpertMixer(nn.Module):
    """Per-H-branch reweighting of the selected MoS experts' outputs.

    Zero logits reproduce the router weights; the mixture is rescaled by the total router
    mass so the top-1 straight-through derivative survives.
    """

    def __init__(self, branches, experts, init_scale=0.1):
        super().__init__()
        logits = torch.full((branches, experts), -init_scale / experts)
        logits[torch.arange(branches), torch.arange(branches) % experts] += init_scale
        self.logits = nn.Parameter(logits)

    def forward(self, expert_outputs):
        values = torch.stack([v for v, _ in expert_outputs], dim=-2)
        weights = torch.cat([w.expand(*values.shape[:-2], 1) for _, w in expert_outputs], dim=-1).float()
        active = weights > 0
        logits = self.logits.float().expand(*weights.shape[:-1], *self.logits.shape)
        inactive = ~active.unsqueeze(-2)
        shift = logits.masked_fill(inactive, -torch.inf).amax(-1, keepdim=True)
        pref = (logits - shift).masked_fill(inactive, -torch.inf).exp()
        mix = weights.unsqueeze(-2) * pref
        mix = mix / mix.sum(-1, keepdim=True).clamp_min(torch.finfo(torch.float32).tiny)
        mix = mix * weights.sum(-1)[..., None, None]
        return torch.einsum("...be,...ed->...bd", mix, values.float()).to(values.dtype)


class RecurrentMemory(ResidualConnection):
    """Depth-recurrent memory branches: at alpha = 0 every branch is replaced by the new state."""

    def __init__(self, branches, hidden_size):
        super().__init__(branches, hidden_size, 0, 0.1, input_dependent=True)
        self.register_buffer("alpha", torch.tensor(0.0))

    def initialize(self, x):
        return x.unsqueeze(-2).expand(*x.shape[:-1], self.branches, x.shape[-1])

    def read_state(self, states):
        return self.read(states, self.alpha)

    def update(self, states, candidate):
        retain = self.alpha * (1 - self.weights(states, self.alpha, "write"))
        return (retain * states.float() + (1 - retain) * candidate.float().unsqueeze(-2)).to(candidate.dtype)
