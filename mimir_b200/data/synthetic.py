"""Synthetic corpus generator in the packed prefix-LM format (no network needed).

Writes ``tokens.npy``, ``epoch_{e}/{inst_start,inst_len,resp_start,resp_len}.npy`` (and optional
``category_id.npy``) and ``metadata.json``.  Token ids are uniform or Zipf(s)-distributed over
the vocabulary; prompt lengths are uniform in ``[min_prefix, max_prefix]`` (at least 1: labels
use ``len(prompt) - 1``) and answer lengths fill each example to ``seq_len`` tokens (or are
uniform in a range).  Each epoch row order is an independent permutation.
"""
from __future__ import annotations

import json
import os
from typing import Optional

import numpy as np


def zipf_tokens(rng: np.random.Generator, n: int, vocab: int, s: float) -> np.ndarray:
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    p = ranks ** (-s)
    p /= p.sum()
    return rng.choice(vocab, size=n, p=p).astype(np.int32)


def write_corpus(path: str, *, rows: int = 64, seq_len: int = 512, vocab: int = 1024, min_prefix: int = 1,
                 max_prefix: Optional[int] = None, epochs: int = 1, seed: int = 0, zipf: Optional[float] = None,
                 categories: int = 0, answer_len_range: Optional[tuple[int, int]] = None) -> str:
    """Create a synthetic corpus at ``path``; returns ``path``.

    Every example has ``seq_len + 1`` tokens (prompt + answer) unless ``answer_len_range`` is
    given, so a packed example occupies exactly ``seq_len`` input positions.
    """
    rng = np.random.default_rng(seed)
    max_prefix = max_prefix if max_prefix is not None else seq_len // 2
    if not 1 <= min_prefix <= max_prefix < seq_len:
        raise ValueError("need 1 <= min_prefix <= max_prefix < seq_len")
    prefix = rng.integers(min_prefix, max_prefix + 1, size=rows)
    if answer_len_range is None:
        answer = seq_len + 1 - prefix
    else:
        answer = rng.integers(answer_len_range[0], answer_len_range[1] + 1, size=rows)
    lengths = prefix + answer
    total = int(lengths.sum())
    tokens = zipf_tokens(rng, total, vocab, zipf) if zipf else rng.integers(0, vocab, size=total).astype(np.int32)
    starts = np.concatenate([[0], np.cumsum(lengths)[:-1]])
    os.makedirs(path, exist_ok=True)
    np.save(os.path.join(path, "tokens.npy"), tokens)
    cats = rng.integers(0, categories, size=rows) if categories else None
    for e in range(epochs):
        order = rng.permutation(rows) if e > 0 else np.arange(rows)
        d = os.path.join(path, f"epoch_{e}")
        os.makedirs(d, exist_ok=True)
        np.save(os.path.join(d, "inst_start.npy"), starts[order].astype(np.int64))
        np.save(os.path.join(d, "inst_len.npy"), prefix[order].astype(np.int64))
        np.save(os.path.join(d, "resp_start.npy"), (starts + prefix)[order].astype(np.int64))
        np.save(os.path.join(d, "resp_len.npy"), answer[order].astype(np.int64))
        if cats is not None:
            np.save(os.path.join(d, "category_id.npy"), cats[order].astype(np.int64))
    meta = {"tokenizer_info": {"vocab_size": vocab, "name": "synthetic"}, "max_seq_len": int(lengths.max()),
            "total_length": total}
    with open(os.path.join(path, "metadata.json"), "w") as f:
        json.dump(meta, f)
    return path


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("path")
    ap.add_argument("--rows", type=int, default=64)
    ap.add_argument("--seq-len", type=int, default=512)
    ap.add_argument("--vocab", type=int, default=1024)
    ap.add_argument("--max-prefix", type=int, default=None)
    ap.add_argument("--epochs", type=int, default=1)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--zipf", type=float, default=None)
    ap.add_argument("--categories", type=int, default=0)
    a = ap.parse_args()
    write_corpus(a.path, rows=a.rows, seq_len=a.seq_len, vocab=a.vocab, max_prefix=a.max_prefix, epochs=a.epochs,
                 seed=a.seed, zipf=a.zipf, categories=a.categories)
