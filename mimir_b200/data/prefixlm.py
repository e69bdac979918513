"""Packed prefix-LM batch metadata.

A packed batch holds ``numseqs`` sequences back to back; sequence ``s`` has
``prefix_lens[s]`` bidirectional prompt tokens followed by ``causal_lens[s]`` causal
tokens.  The per-sequence arrays are padded to ``batch_max_tokens`` entries and
``cu_seqlens`` has ``numseqs + 1`` meaningful entries, matching the reference's batch
format (``src/mimir/model/flash_attention_prefixlm_v2.py:21-35``) so corpora and
collated batches are interchangeable.
"""
from __future__ import annotations

import numpy as np
import torch

PREFIXLM_TENSOR_KEYS = ("prefix_lens", "causal_lens", "cu_seqlens")
PREFIXLM_SCALAR_KEYS = ("total_seqlen", "numseqs", "max_seqlen_prefix", "max_seqlen_causal", "max_seqlen_all")


def compute_aux_seq_tensors_scalars(prefix_lens: np.ndarray, causal_lens: np.ndarray, batch_max_tokens: int):
    prefix_lens = np.asarray(prefix_lens, dtype=np.int32)
    causal_lens = np.asarray(causal_lens, dtype=np.int32)
    totals = prefix_lens + causal_lens
    n = totals.shape[0]
    tensors = {
        "prefix_lens": np.pad(prefix_lens, (0, batch_max_tokens - n)),
        "causal_lens": np.pad(causal_lens, (0, batch_max_tokens - n)),
        "cu_seqlens": np.pad(np.cumsum(totals, dtype=np.int32), (1, batch_max_tokens - n - 1)),
    }
    scalars = {"total_seqlen": int(totals.sum()), "numseqs": n,
               "max_seqlen_prefix": int(prefix_lens.max()), "max_seqlen_causal": int(causal_lens.max()),
               "max_seqlen_all": int(totals.max())}
    return tensors, scalars


def prefixlm_mask(prefix_len: int, seq_len: int, is_causal: bool, device=None) -> torch.Tensor:
    """Boolean ``[seq, seq]`` visibility: prefix rows see the prefix; causal rows see keys <= row."""
    pos = torch.arange(seq_len, device=device)
    causal = pos[None, :] <= pos[:, None]
    if is_causal:
        return causal
    in_prefix = pos < prefix_len
    return (in_prefix[:, None] & in_prefix[None, :]) | (~in_prefix[:, None] & causal)
