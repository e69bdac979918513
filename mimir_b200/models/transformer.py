"""Transformer stack used by both HRM levels.

Reference behaviour: ``src/mimir/model/transformer.py`` — config and intermediate size
rule (``:22-68``), pre/post-norm block with weightless RMSNorm (``:71-129``), stack with a
RoPE table and final norm for pre-norm (``:208-261``).

Additions: ``num_key_value_heads`` (GQA; ``None`` keeps the reference's KV = Q heads) and
an explicit ``rope`` hand-off so the fused attention kernel gathers RoPE tables itself.
"""
from __future__ import annotations

import math
from typing import Literal, Optional

from pydantic import BaseModel
from torch import Tensor, nn

from mimir_b200 import ops
from mimir_b200.models.common import find_multiple
from mimir_b200.models.layers import Attention, AttnType, Cache, RotaryEmbedding, SwiGLU


class InitConfig(BaseModel):
    in_std: float
    attn_out_std: float
    ff_out_std: float


class TransformerConfig(BaseModel):
    max_seq_len: int
    n_layers: int
    hidden_size: int
    num_heads: int
    num_key_value_heads: Optional[int] = None
    expansion: float
    attn_type: AttnType = "prefixlm"
    # Accepted for config compatibility; the single-pass kernel has no FA4 variants.
    prefixlm_fa4_impl: Literal["gather", "seqused"] = "seqused"
    prefixlm_fa4_grad_mask_impl: Literal["eager", "triton"] = "triton"
    prefixlm_fa4_output_combine_impl: Literal["eager", "triton"] = "triton"
    init_type: Literal["fixed_normal", "lecun_normal", "megatron"]
    init_std: Optional[float] = None
    norm_type: Literal["pre", "post"]
    norm_eps: float
    pos_emb_type: Literal["rope", "none"]
    rope_theta: Optional[float] = None

    @property
    def kv_heads(self) -> int:
        return self.num_key_value_heads or self.num_heads

    @property
    def intermediate_size(self) -> int:
        # GLU width chosen so a SwiGLU has the parameter count of a plain MLP of `expansion`.
        return find_multiple(round(self.expansion * self.hidden_size * 2 / 3), 256)

    @property
    def init_config(self) -> InitConfig:
        if self.init_type == "fixed_normal":
            std = self.init_std if self.init_std is not None else 0.02
            return InitConfig(in_std=std, attn_out_std=std, ff_out_std=std)
        if self.init_type == "lecun_normal":
            return InitConfig(in_std=1.0 / math.sqrt(self.hidden_size), attn_out_std=1.0 / math.sqrt(self.hidden_size),
                              ff_out_std=1.0 / math.sqrt(self.intermediate_size))
        if self.init_type == "megatron":
            std_in = self.init_std if self.init_std is not None else 1.0 / math.sqrt(self.hidden_size)
            std_out = std_in / math.sqrt(2.0 * max(1, self.n_layers))
            return InitConfig(in_std=std_in, attn_out_std=std_out, ff_out_std=std_out)
        raise NotImplementedError(self.init_type)


class RMSNormNoWeight:
    """Weightless RMSNorm callable (a plain object so deep copies of a stack share nothing)."""

    def __init__(self, eps: float):
        self.eps = eps

    def __call__(self, x: Tensor) -> Tensor:
        return ops.rms_norm(x, self.eps)


def _identity(x):
    return x


class TransformerBlock(nn.Module):
    def __init__(self, config: TransformerConfig) -> None:
        super().__init__()
        init = config.init_config
        self.attn = Attention(hidden_size=config.hidden_size, head_dim=config.hidden_size // config.num_heads,
                              num_heads=config.num_heads, num_key_value_heads=config.kv_heads,
                              attn_type=config.attn_type, init_std_in=init.in_std, init_std_out=init.attn_out_std)
        self.mlp = SwiGLU(hidden_size=config.hidden_size, intermediate_size=config.intermediate_size,
                          init_std_in=init.in_std, init_std_out=init.ff_out_std)
        self.norm_type = config.norm_type
        self.norm = RMSNormNoWeight(config.norm_eps)

    def forward(self, x: Tensor, stability_diagnostics=None, stability_scope=None, **seq_info) -> Tensor:
        if stability_diagnostics is not None:
            if stability_scope is None:
                raise ValueError("stability_scope is required when diagnostics are enabled")
            return self._forward_with_diagnostics(x, stability_diagnostics, stability_scope, **seq_info)
        if self.norm_type == "pre":
            h, n = ops.add_rms_norm(x, self.attn(self.norm(x), **seq_info), self.norm.eps)
            return h + self.mlp(n)
        x = self.norm(x + self.attn(x, **seq_info))
        return self.norm(x + self.mlp(x))

    def _forward_with_diagnostics(self, x, diag, scope, **seq_info):
        pre = self.norm_type == "pre"
        diag.record_tensor(f"activation/{scope}/input", x, record_gradient=True)
        if pre:
            attn_in = self.norm(x)
            diag.record_tensor(f"activation/{scope}/attn_norm", attn_in)
        else:
            attn_in = x
        attn_res = self.attn(attn_in, stability_diagnostics=diag, stability_scope=f"{scope}/attention", **seq_info)
        diag.record_tensor(f"activation/{scope}/attn_residual", attn_res, record_gradient=True)
        diag.record_pair(f"{scope}/attn_input_residual", x, attn_res)
        post_attn = x + attn_res if pre else self.norm(x + attn_res)
        diag.record_tensor(f"activation/{scope}/post_attn", post_attn, record_gradient=True)
        if pre:
            mlp_in = self.norm(post_attn)
            diag.record_tensor(f"activation/{scope}/mlp_norm", mlp_in)
        else:
            mlp_in = post_attn
        mlp_res = self.mlp(mlp_in, stability_diagnostics=diag, stability_scope=f"{scope}/mlp")
        diag.record_tensor(f"activation/{scope}/mlp_residual", mlp_res, record_gradient=True)
        diag.record_pair(f"{scope}/mlp_input_residual", post_attn, mlp_res)
        out = post_attn + mlp_res if pre else self.norm(post_attn + mlp_res)
        diag.record_tensor(f"activation/{scope}/output", out, record_gradient=True)
        return out


class Transformer(nn.Module):
    def __init__(self, config: TransformerConfig) -> None:
        super().__init__()
        in_std = config.init_config.in_std
        # Hint for LMHead init: embedding/unembedding width and std.
        self.head_hint = {"in": {"dim": config.hidden_size, "init_std": in_std},
                          "out": {"dim": config.hidden_size, "init_std": in_std}}
        if config.pos_emb_type == "rope":
            assert config.rope_theta is not None
            self.rotary_emb = RotaryEmbedding(config.hidden_size // config.num_heads, config.max_seq_len,
                                              base=config.rope_theta)
        self.layers = nn.ModuleList([TransformerBlock(config) for _ in range(config.n_layers)])
        self.norm_f = RMSNormNoWeight(config.norm_eps) if (config.norm_type == "pre" and config.n_layers > 0) else _identity
        self._cache_heads = config.kv_heads
        self._cache_head_dim = config.hidden_size // config.num_heads
        self._cache_layers = config.n_layers

    def create_cache(self, **kwargs) -> list[Cache]:
        return [Cache.create(**kwargs, num_heads=self._cache_heads, head_dim=self._cache_head_dim)
                for _ in range(self._cache_layers)]

    def rope_info(self, seq_info: dict) -> dict:
        """Replace ``position_ids`` with the ``rope`` hand-off understood by :class:`Attention`."""
        positions = seq_info.pop("position_ids", None)
        seq_info.pop("cos_sin", None)
        if hasattr(self, "rotary_emb"):
            seq_info["rope"] = ((self.rotary_emb.cos_cached, self.rotary_emb.sin_cached), positions)
        return seq_info

    def forward(self, x: Tensor, cache: Optional[list[Cache]] = None, stability_diagnostics=None,
                stability_scope=None, **seq_info) -> Tensor:
        seq_info = self.rope_info(dict(seq_info))
        for index, layer in enumerate(self.layers):
            kwargs = {}
            if stability_diagnostics is not None:
                if stability_scope is None:
                    raise ValueError("stability_scope is required when diagnostics are enabled")
                kwargs = dict(stability_diagnostics=stability_diagnostics,
                              stability_scope=f"{stability_scope}/layer_{index:03d}")
            x = layer(x, **seq_info, **kwargs, cache=cache[index] if cache is not None else None)
        out = self.norm_f(x)
        if stability_diagnostics is not None:
            stability_diagnostics.record_tensor(f"activation/{stability_scope}/final_norm", out, record_gradient=True)
        return out
