"""Prefix-LM attention over packed variable-length sequences.

Mask rule (reference ``src/mimir/model/flash_attention_prefixlm_dense.py:61-69``): inside
sequence ``s`` with prompt length ``P``, a query row ``r < P`` sees keys ``[0, P)``
(bidirectional prompt) and a row ``r >= P`` sees keys ``[0, r]`` (causal answer).  Rows
never see another sequence.  ``is_causal=True`` makes every row causal.

The reference runs this as two FlashAttention-4 launches (prompt rows, then answer rows
with shifted ``cu_seqlens``) plus Triton kernels that mask undefined gradient rows and
combine the two outputs (``src/mimir/model/flash_attention_prefixlm_fa4.py:353-406``).
Here one sm_100a kernel covers every row of a 128-row query tile in a single pass, with
per-row key limits and whole-tile skipping, and (in :func:`gated_prefixlm_attention`)
also applies RoPE to Q/K beforehand and the ``sigmoid(gate)`` output gate in its epilogue.

:func:`dense_prefixlm_attention` is the fp32-capable PyTorch oracle.
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from mimir_b200.ops._ext import ext, kernels_enabled
from mimir_b200.data.prefixlm import prefixlm_mask


def _int(v) -> int:
    return int(v.item()) if isinstance(v, torch.Tensor) else int(v)


def dense_prefixlm_attention(q, k, v, is_causal, prefix_lens, causal_lens, cu_seqlens, total_seqlen, numseqs,
                             max_seqlen_prefix=None, max_seqlen_causal=None, max_seqlen_all=None, **_unused):
    """Per-sequence SDPA with the explicit prefix-LM mask; q ``[T,H,d]``, k/v ``[T,KV,d]``."""
    n = _int(numseqs)
    total = _int(total_seqlen)
    bounds = cu_seqlens[:n + 1].tolist()
    prefix = prefix_lens[:n].tolist()
    causal = causal_lens[:n].tolist()
    out = torch.zeros_like(q)
    rep = q.shape[-2] // k.shape[-2]
    if q.shape[-2] % k.shape[-2]:
        raise ValueError(f"Query heads {q.shape[-2]} must be divisible by key/value heads {k.shape[-2]}.")
    for s in range(n):
        start, end = bounds[s], bounds[s + 1]
        length = end - start
        if length == 0:
            continue
        if prefix[s] + causal[s] != length:
            raise ValueError(f"Bad PrefixLM lengths for sequence {s}: {prefix[s]} + {causal[s]} != {length}")
        ks, vs = k[start:end], v[start:end]
        if rep > 1:
            ks, vs = ks.repeat_interleave(rep, dim=-2), vs.repeat_interleave(rep, dim=-2)
        mask = prefixlm_mask(prefix[s], length, is_causal, device=q.device)
        o = F.scaled_dot_product_attention(q[start:end].transpose(0, 1)[None], ks.transpose(0, 1)[None],
                                           vs.transpose(0, 1)[None], attn_mask=mask[None, None])
        out[start:end] = o[0].transpose(0, 1)
    if total < q.shape[0]:
        out[total:] = 0
    return out


def prefixlm_attention(q, k, v, is_causal, prefix_lens, causal_lens, cu_seqlens, total_seqlen, numseqs,
                       max_seqlen_prefix=None, max_seqlen_causal=None, max_seqlen_all=None, **_unused):
    """Public op with the reference signature (``flash_attn_varlen_prefixlm``)."""
    if kernels_enabled(q) and q.dtype == torch.bfloat16 and q.shape[-1] == 128 and _fmha_ready():
        return _PrefixLMAttentionFn.apply(q, k, v, bool(is_causal), prefix_lens, cu_seqlens, _int(numseqs))
    return dense_prefixlm_attention(q, k, v, is_causal, prefix_lens, causal_lens, cu_seqlens, total_seqlen,
                                    numseqs)


def _fmha_ready() -> bool:
    return hasattr(ext(), "fmha_fwd")


def _fmha_bwd_ready() -> bool:
    return hasattr(ext(), "fmha_bwd")


def forward_kernel():
    """``(kernel, plan kind)`` of the attention forward: the two-query-tile kernel
    (``fmha_fwd2``, default) or the one-tile kernel (``MIMIR_FMHA_FWD=1``)."""
    C = ext()
    if os.environ.get("MIMIR_FMHA_FWD", "2") == "2" and hasattr(C, "fmha_fwd2"):
        return C.fmha_fwd2, "fwd2"
    return C.fmha_fwd, "fwd"


def attention_plan(cu_seqlens: torch.Tensor, prefix_lens: torch.Tensor, numseqs: int, total_tokens: int,
                   is_causal: bool, backward: bool = False, kind: str | None = None):
    """Device tile schedule ``(tiles, ntiles)`` for a packed batch, cached on the metadata tensor.

    ``kind`` is ``"bwd"`` (key blocks), ``"fwd"`` (128-row query tiles) or ``"fwd2"`` (256-row
    query tiles); by default the backward schedule or the active forward kernel's.  Every
    attention layer of a forward (and its backward) sees the same packed layout, so the
    schedule is built once per batch; the cache is invalidated if ``cu_seqlens`` is modified.
    """
    kind = kind or ("bwd" if backward else forward_kernel()[1])
    key = (kind, bool(is_causal), int(numseqs), int(total_tokens), prefix_lens.data_ptr(),
           prefix_lens._version)
    cache = getattr(cu_seqlens, "_mimir_fmha_plans", None)
    if cache is None or cache[0] != cu_seqlens._version:
        cache = (cu_seqlens._version, {})
        try:
            cu_seqlens._mimir_fmha_plans = cache
        except (AttributeError, RuntimeError):  # pragma: no cover - tensor subclasses without __dict__
            pass
    plan = cache[1].get(key)
    if plan is None:
        build = {"bwd": ext().fmha_bwd_plan, "fwd": ext().fmha_plan, "fwd2": getattr(ext(), "fmha_plan2", None)}[kind]
        plan = build(cu_seqlens, prefix_lens, int(numseqs), int(total_tokens), bool(is_causal))
        cache[1][key] = plan
    return plan


class _PrefixLMAttentionFn(torch.autograd.Function):
    """Plain (ungated, no RoPE) attention through the FMHA kernels: q/k/v are ``[T, heads, 128]``."""

    @staticmethod
    def forward(ctx, q, k, v, is_causal, prefix_lens, cu_seqlens, numseqs):
        T, H, D = q.shape
        KV = k.shape[1]
        q2, k2, v2 = q.reshape(T, H * D).contiguous(), k.reshape(T, KV * D).contiguous(), v.reshape(T, KV * D).contiguous()
        cu, pl = cu_seqlens.to(torch.int32).contiguous(), prefix_lens.to(torch.int32).contiguous()
        fwd, kind = forward_kernel()
        tiles, ntiles = attention_plan(cu, pl, numseqs, T, is_causal, kind=kind)
        out, lse = fwd(q2, 0, k2, 0, v2, 0, None, 0, H, KV, is_causal, cu, pl, numseqs, tiles, ntiles)
        ctx.save_for_backward(q2, k2, v2, out, lse, cu, pl, tiles, ntiles)
        ctx.info = (H, KV, is_causal, numseqs)
        return out.view(T, H, D)

    @staticmethod
    def backward(ctx, dout):
        q2, k2, v2, out, lse, cu, pl, tiles, ntiles = ctx.saved_tensors
        H, KV, is_causal, numseqs = ctx.info
        T = q2.shape[0]
        do = dout.reshape(T, -1).contiguous()
        if not _fmha_bwd_ready():
            raise RuntimeError("fmha_bwd kernel missing from mimir_b200._C")
        delta = ext().attn_delta(do, out, H)
        kv_tiles, kv_ntiles = attention_plan(cu, pl, numseqs, T, is_causal, backward=True)
        dq, dk, dv = ext().fmha_bwd(q2, 0, k2, 0, v2, 0, do, lse, delta, H, KV, is_causal, cu, pl, numseqs,
                                    kv_tiles, kv_ntiles)
        return dq.view(T, H, -1).to(q2.dtype), dk.view(T, KV, -1).to(q2.dtype), dv.view(T, KV, -1).to(q2.dtype), \
            None, None, None, None


# ----------------------------------------------------------------------------------------
# Fused gated attention block: RoPE(q,k) -> prefix-LM FMHA -> sigmoid(gate) * O
# ----------------------------------------------------------------------------------------
def _rope_torch(x, cos, sin):
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return ((x * cos.unsqueeze(-2)) + rot * sin.unsqueeze(-2)).to(x.dtype)


def gated_attention_composite(gqkv, tables, positions, H, KV, hd, is_causal, seq_info):
    """PyTorch formulation of the fused block (RoPE, attention, gate); used where no kernel applies."""
    shaped = gqkv.unflatten(-1, (2 * H + 2 * KV, hd))
    gate, q, k, v = shaped.split((H, H, KV, KV), dim=-2)
    cos, sin = tables[0][positions], tables[1][positions]
    q, k = _rope_torch(q, cos, sin), _rope_torch(k, cos, sin)
    attn = dense_prefixlm_attention(q, k, v, is_causal, **seq_info)
    return (torch.sigmoid(gate) * attn).flatten(-2)


class _GatedAttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gqkv, cos, sin, positions, H, KV, hd, is_causal, cu_seqlens, prefix_lens, numseqs):
        C = ext()
        T = gqkv.shape[0]
        qk = C.rope_qk(gqkv, cos, sin, positions, H, KV)  # rotated [T, (H+KV)*hd]
        fwd, kind = forward_kernel()
        tiles, ntiles = attention_plan(cu_seqlens, prefix_lens, numseqs, T, is_causal, kind=kind)
        # q at column 0 of qk, k at H*hd; v at (2H+KV)*hd of gqkv; gate at column 0 of gqkv.
        y, lse, o = fwd(qk, 0, qk, H * hd, gqkv, (2 * H + KV) * hd, gqkv, 0, H, KV, is_causal,
                               cu_seqlens, prefix_lens, numseqs, tiles, ntiles)
        ctx.save_for_backward(gqkv, qk, o, lse, cos, sin, positions, cu_seqlens, prefix_lens, tiles, ntiles)
        ctx.info = (H, KV, hd, is_causal, numseqs)
        return y

    @staticmethod
    def backward(ctx, dy):
        gqkv, qk, o, lse, cos, sin, positions, cu, pl, tiles, ntiles = ctx.saved_tensors
        H, KV, hd, is_causal, numseqs = ctx.info
        if not _fmha_bwd_ready():
            return (_recompute_backward(gqkv, dy, (cos, sin), positions, H, KV, hd, is_causal, cu, pl, numseqs),
                    None, None, None, None, None, None, None, None, None, None)
        C = ext()
        dgqkv = torch.empty_like(gqkv)
        # dO = dy * sigmoid(g); dgate -> dgqkv[:, :H*hd]; delta = rowsum(dO * O) per (head, token).
        do, delta = C.attn_gate_bwd(dy.contiguous(), o, gqkv, dgqkv, H)
        kv_tiles, kv_ntiles = attention_plan(cu, pl, numseqs, gqkv.shape[0], is_causal, backward=True)
        dq, dk, dv = C.fmha_bwd(qk, 0, qk, H * hd, gqkv, (2 * H + KV) * hd, do, lse, delta, H, KV, is_causal,
                                cu, pl, numseqs, kv_tiles, kv_ntiles)
        C.rope_qk_bwd(dq, dk, dv, cos, sin, positions, dgqkv, H, KV)  # un-rotate into the packed gradient
        return dgqkv, None, None, None, None, None, None, None, None, None, None


def _recompute_backward(gqkv, dy, tables, positions, H, KV, hd, is_causal, cu, pl, numseqs):
    """Backward through the PyTorch formulation (used only if the extension lacks fmha_bwd)."""
    with torch.enable_grad():
        g = gqkv.detach().requires_grad_(True)
        T = g.shape[0]
        info = dict(cu_seqlens=cu, prefix_lens=pl, causal_lens=torch.zeros_like(pl), total_seqlen=int(cu[numseqs]),
                    numseqs=numseqs)
        # causal_lens are only used for a consistency check in the dense oracle; derive them.
        lengths = (cu[1:numseqs + 1] - cu[:numseqs])
        info["causal_lens"] = torch.cat([lengths - pl[:numseqs], torch.zeros(pl.numel() - numseqs, dtype=pl.dtype,
                                                                                device=pl.device)])
        if is_causal:
            info["causal_lens"][:numseqs] = lengths
            info["prefix_lens"] = torch.zeros_like(pl)
        out = gated_attention_composite(g, tables, positions.long(), H, KV, hd, is_causal, info)
        out.backward(dy)
    del T
    return g.grad


def gated_prefixlm_attention(gqkv, tables, positions, H, KV, hd, is_causal, seq_info):
    """``sigmoid(gate) * attention(rope(q), rope(k), v)`` from the packed ``[T, (2H+2KV)*hd]`` projection."""
    if gqkv.dtype == torch.bfloat16 and hd == 128 and _fmha_ready():
        cu = seq_info["cu_seqlens"]
        pl = seq_info["prefix_lens"]
        cu = (cu if cu.dtype == torch.int32 else cu.to(torch.int32)).contiguous()
        pl = (pl if pl.dtype == torch.int32 else pl.to(torch.int32)).contiguous()
        return _GatedAttentionFn.apply(gqkv.contiguous(), tables[0], tables[1], positions.to(torch.int32).contiguous(),
                                       H, KV, hd, bool(is_causal), cu, pl, _int(seq_info["numseqs"]))
    return gated_attention_composite(gqkv, tables, positions, H, KV, hd, is_causal, seq_info)
