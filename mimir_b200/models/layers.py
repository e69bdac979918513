"""Mimir2 building blocks: RoPE, initialised linears, scaled embedding, gated attention, SwiGLU.

Behavioural reference: ``src/mimir/model/layers.py`` (RoPE ``:25-60``, ``LinearInit``
``:63-87``, ``ScaledEmbeddingInit`` ``:90-104``, static ``Cache`` ``:107-115``, gated
attention ``:118-253``, ``SwiGLU`` ``:256-287``).  Parameter names and shapes are kept
identical so DCP checkpoints are interchangeable.

On CUDA the training path of :class:`Attention` and :class:`SwiGLU` runs through the
hand-written sm_100a kernels in :mod:`mimir_b200.ops`: every projection is the tcgen05
CTA-pair GEMM (``ops.linear``), the SwiGLU MLP is two fused GEMMs per direction
(``ops.swiglu_mlp``), and attention is the single-pass prefix-LM kernel with RoPE and the
``sigmoid(gate)`` epilogue fused.  On CPU, and for cached
decode or stability diagnostics, the plain PyTorch formulation below is used; it is also
the numerical oracle for the kernels.
"""
from __future__ import annotations

import math
from typing import Literal, NamedTuple, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from mimir_b200.models.common import find_multiple, trunc_normal_init_, unwrap_tensor  # noqa: F401
from mimir_b200 import ops

CosSin = Tuple[Tensor, Tensor]
AttnType = Literal["causal", "prefixlm"]


def rotate_half(x: Tensor) -> Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_rotary_pos_emb(x: Tensor, cos_sin: CosSin) -> Tensor:
    """fp32 rotary embedding over ``[..., seq, heads, head_dim]`` with tables ``[..., seq, head_dim]``."""
    cos, sin = cos_sin
    return ((x * cos.unsqueeze(-2)) + (rotate_half(x) * sin.unsqueeze(-2))).to(x.dtype)


class RotaryEmbedding(nn.Module):
    """Precomputed fp32 cos/sin tables of shape ``[max_seq_len, head_dim]`` (halves duplicated)."""

    def __init__(self, dim: int, max_seq_len: int, base: float, **kwargs):
        super().__init__()
        inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32, **kwargs) / dim))
        angles = torch.outer(torch.arange(max_seq_len, dtype=torch.float32, **kwargs), inv_freq)
        table = torch.cat((angles, angles), dim=-1)
        self.cos_cached = nn.Buffer(table.cos(), persistent=False)
        self.sin_cached = nn.Buffer(table.sin(), persistent=False)

    def forward(self, position_ids: Optional[Tensor]) -> CosSin:
        if position_ids is None:
            return self.cos_cached, self.sin_cached
        return self.cos_cached[position_ids], self.sin_cached[position_ids]


class LinearInit(nn.Module):
    """Bias-optional linear with truncated LeCun init; ``batch_out_features`` packs several
    projections row-wise into one weight (e.g. gate|Q|K|V)."""

    def __init__(self, in_features: int, out_features: int, bias: bool,
                 batch_out_features: Sequence[int] = (), init_std: Optional[float] = None, **kwargs):
        super().__init__()
        self.in_features = in_features
        std = init_std if init_std is not None else in_features ** -0.5
        rows = math.prod(batch_out_features) * out_features
        self.weight = nn.Parameter(trunc_normal_init_(torch.empty((rows, in_features), **kwargs), std=std))
        self.bias = nn.Parameter(torch.zeros((rows,), **kwargs)) if bias else None

    def forward(self, x: Tensor) -> Tensor:
        return ops.linear(x, self.weight, self.bias)


class ScaledEmbeddingInit(nn.Module):
    """Embedding initialised with std ``init_std`` and multiplied by ``1/init_std`` on lookup."""

    def __init__(self, num_embeddings: int, embedding_dim: int, init_std: float, **kwargs):
        super().__init__()
        self.scale = 1.0 / init_std
        self.embedding_weight = nn.Parameter(
            trunc_normal_init_(torch.empty((num_embeddings, embedding_dim), **kwargs), std=init_std))

    def forward(self, ids: Tensor) -> Tensor:
        return ops.scaled_embedding(ids, self.embedding_weight, self.scale)


class Cache(NamedTuple):
    """Static per-layer KV cache ``[batch, max_seq, kv_heads, head_dim]`` for decode."""
    keys: Tensor
    values: Tensor

    @classmethod
    def create(cls, max_batch_size: int, max_seq_len: int, num_heads: int, head_dim: int, **kwargs):
        shape = (max_batch_size, max_seq_len, num_heads, head_dim)
        return cls(keys=torch.zeros(shape, **kwargs), values=torch.zeros(shape, **kwargs))


class Attention(nn.Module):
    """Gated (G, Q, K, V packed) attention with RoPE and a prefix-LM or causal mask.

    Output is ``o_proj(sigmoid(gate) * attention(q, k, v))`` where ``gate`` has one value
    per query element.  GQA is supported when ``num_key_value_heads`` divides ``num_heads``.
    """

    def __init__(self, hidden_size, head_dim, num_heads, num_key_value_heads, attn_type,
                 init_std_in=None, init_std_out=None, **kwargs):
        super().__init__()
        kwargs = {k: v for k, v in kwargs.items() if not k.startswith("prefixlm_fa4")}
        self.head_dim = head_dim
        self.num_heads = num_heads
        self.num_key_value_heads = num_key_value_heads
        self.attn_type = attn_type
        self.gqkv_proj = LinearInit(hidden_size, head_dim, batch_out_features=(2 * num_heads + 2 * num_key_value_heads,),
                                    bias=False, init_std=init_std_in, **kwargs)
        self.o_proj = LinearInit(head_dim * num_heads, hidden_size, bias=False, init_std=init_std_out, **kwargs)

    # -- decode path (static cache) ---------------------------------------------------
    def _attention_with_cache(self, q, k, v, cache: Cache, cache_lengths, causal, cache_batch_indices=None):
        batch, seqlen = q.shape[:2]
        positions = cache_lengths[:, None] + torch.arange(seqlen, device=q.device, dtype=cache_lengths.dtype)
        rows = torch.arange(batch, device=q.device) if cache_batch_indices is None else cache_batch_indices
        cache.keys[rows[:, None], positions] = k
        cache.values[rows[:, None], positions] = v
        kv_len = cache_lengths + seqlen
        max_kv = int(kv_len.max().item())
        if cache_batch_indices is None:
            keys, values = cache.keys[:batch, :max_kv], cache.values[:batch, :max_kv]
        else:
            keys, values = cache.keys[rows, :max_kv], cache.values[rows, :max_kv]
        if self.num_heads != self.num_key_value_heads:
            rep = self.num_heads // self.num_key_value_heads
            keys, values = keys.repeat_interleave(rep, dim=2), values.repeat_interleave(rep, dim=2)
        key_pos = torch.arange(max_kv, device=q.device)
        allowed = key_pos[None, :] < kv_len[:, None]
        if causal:
            allowed = allowed[:, None, :] & (key_pos[None, None, :] <= positions[:, :, None])
        else:
            allowed = allowed[:, None, :]
        bias = torch.zeros((batch, seqlen, max_kv), dtype=q.dtype, device=q.device)
        bias = bias.masked_fill(~allowed, torch.finfo(q.dtype).min)
        out = F.scaled_dot_product_attention(q.transpose(1, 2), keys.transpose(1, 2), values.transpose(1, 2),
                                             attn_mask=bias[:, None])
        return out.transpose(1, 2)

    def forward(self, hidden_states: Tensor, cos_sin: Optional[CosSin] = None, cache: Optional[Cache] = None,
                cache_lengths: Optional[Tensor] = None, stability_diagnostics=None, stability_scope=None,
                rope=None, **seq_info) -> Tensor:
        """``rope`` is ``((cos_table, sin_table), position_ids)`` from the owning stack; the
        fused kernel path gathers the tables itself, the fallback materialises ``cos_sin``."""
        gqkv = self.gqkv_proj(hidden_states)
        H, KV, hd = self.num_heads, self.num_key_value_heads, self.head_dim
        is_causal = self.attn_type == "causal"
        if (cache is None and stability_diagnostics is None and rope is not None and rope[1] is not None
                and gqkv.ndim == 2 and ops.kernels_enabled(gqkv)):
            gated = ops.gated_prefixlm_attention(gqkv, rope[0], rope[1], H, KV, hd, is_causal,
                                                 {n: unwrap_tensor(t) for n, t in seq_info.items()})
            return self.o_proj(gated)
        if cos_sin is None and rope is not None:
            (cos_t, sin_t), positions = rope
            cos_sin = (cos_t, sin_t) if positions is None else (cos_t[positions], sin_t[positions])

        shaped = gqkv.unflatten(-1, (2 * H + 2 * KV, hd))
        gate, query, key, value = shaped.split((H, H, KV, KV), dim=-2)
        if cos_sin is not None:
            query = apply_rotary_pos_emb(query, cos_sin)
            key = apply_rotary_pos_emb(key, cos_sin)
        if stability_diagnostics is not None:
            _record_attention_diagnostics(stability_diagnostics, stability_scope, gate, query, key, value, hd)
        if cache is None:
            attn = ops.prefixlm_attention(query, key, value, is_causal,
                                          **{n: unwrap_tensor(t) for n, t in seq_info.items()})
        else:
            attn = self._attention_with_cache(query, key, value, cache, cache_lengths, is_causal,
                                              seq_info.get("cache_batch_indices"))
        gated = (torch.sigmoid(gate) * attn).flatten(-2)
        if stability_diagnostics is not None:
            stability_diagnostics.record_tensor(f"activation/{stability_scope}/gated_attention_output", gated,
                                                record_gradient=True)
        out = self.o_proj(gated)
        if stability_diagnostics is not None:
            stability_diagnostics.record_tensor(f"activation/{stability_scope}/projected_output", out,
                                                record_gradient=True)
        return out


def _record_attention_diagnostics(diag, scope, gate, query, key, value, head_dim):
    if scope is None:
        raise ValueError("stability_scope is required when diagnostics are enabled")
    gate_values = torch.sigmoid(gate)
    for name, t in (("gate_logits", gate), ("gate_values", gate_values), ("query", query), ("key", key),
                    ("value", value)):
        diag.record_tensor(f"activation/{scope}/{name}", t, record_gradient=True)
        diag.record_last_dim_rms(f"activation/{scope}/{name}_head_rms", t)
    diag.record_fraction(f"activation/{scope}/gate_near_zero", gate_values < 0.01)
    diag.record_fraction(f"activation/{scope}/gate_near_one", gate_values > 0.99)
    if query.shape[-2] == key.shape[-2]:
        diag.record_tensor(f"activation/{scope}/aligned_qk_score", (query * key).sum(-1) / math.sqrt(head_dim))


class SwiGLU(nn.Module):
    """``down(silu(gate) * up)`` with gate|up packed in one projection."""

    def __init__(self, hidden_size: int, intermediate_size: int, init_std_in=None, init_std_out=None, **kwargs):
        super().__init__()
        self.gate_up_proj = LinearInit(hidden_size, intermediate_size, batch_out_features=(2,), bias=False,
                                       init_std=init_std_in, **kwargs)
        self.down_proj = LinearInit(intermediate_size, hidden_size, bias=False, init_std=init_std_out, **kwargs)

    def forward(self, x, stability_diagnostics=None, stability_scope=None):
        if stability_diagnostics is None and ops.swiglu_mlp_supported(x, self.gate_up_proj.weight,
                                                                      self.down_proj.weight):
            return ops.swiglu_mlp(x, self.gate_up_proj.weight, self.down_proj.weight)
        gu = self.gate_up_proj(x)
        if stability_diagnostics is None:
            return self.down_proj(ops.swiglu(gu))
        if stability_scope is None:
            raise ValueError("stability_scope is required when diagnostics are enabled")
        gate, up = gu.chunk(2, dim=-1)
        product = F.silu(gate) * up
        for name, t in (("gate", gate), ("up", up), ("product", product)):
            stability_diagnostics.record_tensor(f"activation/{stability_scope}/{name}", t, record_gradient=True)
            stability_diagnostics.record_last_dim_rms(f"activation/{stability_scope}/{name}_token_rms", t)
        out = self.down_proj(product)
        stability_diagnostics.record_tensor(f"activation/{stability_scope}/down_output", out, record_gradient=True)
        return out
