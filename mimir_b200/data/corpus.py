"""Packed prefix-LM corpus: memory-mapped token stream, LPT multipack sampling, resumable iteration.

Format (reference ``src/mimir/corpus/sampled.py:18-216``), directory ``dataset_path``:

* ``tokens.npy`` — one integer token stream;
* ``epoch_{e}/{inst_start,inst_len,resp_start,resp_len}.npy`` — aligned row indices, one row
  per example (prompt = ``inst``, answer = ``resp``); optional ``epoch_{e}/category_id.npy``;
* ``metadata.json`` — ``{"tokenizer_info": {"vocab_size": V, ...}, "max_seq_len": S, "total_length": N}``.

A batch packs whole examples into ``batch_max_length`` tokens: inputs are the prompt followed
by the answer without its last token; labels are the answer (and, unless ``target_only``, the
shifted prompt); the prompt is the bidirectional prefix.  Resume either skips whole batches of
an epoch or restarts at a global row cursor.

The LPT bin packing runs in native code (``mimir_b200._host``); a pure-Python fallback with the
same semantics is kept for environments without the compiled module.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, fields
from typing import Any, Optional

import numpy as np
import pydantic
import torch
import torch.distributed as dist
from torch.utils.data import IterableDataset, get_worker_info

from mimir_b200.data.prefixlm import compute_aux_seq_tensors_scalars
from mimir_b200.models.common import IGNORE_LABEL_ID, find_multiple


# ----------------------------------------------------------------------------------------
# LPT allocation
# ----------------------------------------------------------------------------------------
def _sift(heap, ids, n):
    u = 1
    while (u << 1) <= n:
        v = u << 1
        if (v | 1) <= n and heap[v | 1] < heap[v]:
            v |= 1
        if heap[u] <= heap[v]:
            break
        heap[u], heap[v] = heap[v], heap[u]
        if ids is not None:
            ids[u], ids[v] = ids[v], ids[u]
        u = v


def _lpt_fits(a, c, n):
    heap = [0] * (n + 1)
    for size in sorted(a.tolist(), reverse=True):
        heap[1] += size
        if heap[1] > c:
            return False
        _sift(heap, None, n)
    return True


def _lpt_assign(a, n, rank):
    order = np.argsort(a, kind="mergesort")[::-1]
    heap = [0] * (n + 1)
    ids = list(range(-1, n))
    mine = []
    for idx in order.tolist():
        heap[1] += int(a[idx])
        if ids[1] == rank:
            mine.append(idx)
        _sift(heap, ids, n)
    return np.array(mine, dtype=np.int64)


def allocate_python(lengths: np.ndarray, start: int, rank: int, c: int, n: int):
    total, end = 0, start
    while end < lengths.size:
        total += int(lengths[end])
        end += 1
        if total >= c * n:
            break
    a = lengths[start:end]
    lo, hi = 1, 1 + a.size
    while hi - lo > 1:
        mid = (lo + hi) // 2
        if _lpt_fits(a[:mid], c, n):
            lo = mid
        else:
            hi = mid
    return lo >= n, lo, start + _lpt_assign(a[:lo], n, rank), int(np.sum(a[:lo]))


def allocate(lengths: np.ndarray, start: int, rank: int, c: int, n: int):
    """(is_full, rows_used, this rank's row indices, tokens_used) for the batch starting at ``start``."""
    try:
        from mimir_b200 import _host
    except ImportError:
        return allocate_python(np.asarray(lengths, dtype=np.int64), start, rank, c, n)
    full, used, batch, tokens = _host.multipack_allocate(np.ascontiguousarray(lengths, dtype=np.int64), int(start),
                                                         int(rank), int(c), int(n))
    return bool(full), int(used), batch, int(tokens)


class MultipackDistributedBatchSampler:
    """Unpadded length-aware sampler: LPT-balanced packing of consecutive rows over ranks."""

    def __init__(self, batch_max_length: int, lengths: np.ndarray, num_replicas: Optional[int] = None,
                 rank: Optional[int] = None, drop_last_batch: bool = False):
        if num_replicas is None:
            num_replicas = dist.get_world_size()
        if rank is None:
            rank = dist.get_rank()
        self.num_replicas, self.rank, self.drop_last_batch = num_replicas, rank, drop_last_batch
        self.batch_max_length = batch_max_length
        self.lengths = np.asarray(lengths)
        self.eff_total_used = 0
        self.eff_total_slots = 0

    def iter_with_info(self, start_index: int = 0):
        if start_index < 0:
            raise ValueError(f"start_index must be non-negative, got {start_index}")
        while start_index < self.lengths.size:
            first = start_index
            full, used, batch, tokens = allocate(self.lengths, start_index, self.rank, self.batch_max_length,
                                                 self.num_replicas)
            start_index += used
            if not full:
                break
            if self.drop_last_batch and start_index >= self.lengths.size:
                break
            self.eff_total_used += tokens
            self.eff_total_slots += self.num_replicas * self.batch_max_length
            yield batch, {"global_row_start": int(first), "global_row_end": int(start_index),
                          "global_numseq": int(used), "global_batch_totlen": int(tokens)}

    def __iter__(self):
        for batch, _ in self.iter_with_info():
            yield batch

    def estimate_num_batches(self):
        return round(np.sum(self.lengths) / (self.num_replicas * self.batch_max_length))

    def efficiency(self):
        return self.eff_total_used / self.eff_total_slots


class HomogeneousSampler(MultipackDistributedBatchSampler):
    """Category-homogeneous global microbatches, round-robin over categories (in a seeded order).

    Reference: ``src/mimir/corpus/homogeneous.py:7-54``.  The row cursor is virtual: resume replays
    the deterministic allocation and refuses cursors that fall inside a batch.
    """

    def __init__(self, *, categories, seed=0, **kwargs):
        super().__init__(**kwargs)
        if categories.shape != self.lengths.shape or categories.dtype.kind not in "iu":
            raise ValueError("category_id.npy must be an integer vector aligned with epoch rows")
        if np.any(categories < 0) or np.any(self.lengths > self.batch_max_length):
            raise ValueError("Invalid category or overlength example")
        keys = np.unique(categories)
        np.random.default_rng(seed).shuffle(keys)
        order = np.argsort(categories, kind="stable")
        sorted_cat = categories[order]
        self.groups = [order[np.searchsorted(sorted_cat, k, "left"):np.searchsorted(sorted_cat, k, "right")]
                       for k in keys]
        self.group_lengths = [self.lengths[g] for g in self.groups]

    def iter_with_info(self, start_index=0):
        if start_index < 0:
            raise ValueError("Negative row cursor")
        pos = [0] * len(self.groups)
        cursor = 0
        active = True
        while active:
            active = False
            for gid, rows in enumerate(self.groups):
                if pos[gid] >= len(rows):
                    continue
                active = True
                full, used, selected, tokens = allocate(self.group_lengths[gid], pos[gid], self.rank,
                                                        self.batch_max_length, self.num_replicas)
                pos[gid] += used
                before, cursor = cursor, cursor + used
                if not full:
                    pos[gid] = len(rows)
                    continue
                if before < start_index < cursor:
                    raise ValueError("Resume cursor falls inside a homogeneous batch")
                if before < start_index:
                    continue
                self.eff_total_used += tokens
                self.eff_total_slots += self.num_replicas * self.batch_max_length
                yield rows[selected], dict(global_row_start=before, global_row_end=cursor, global_numseq=int(used),
                                           global_batch_totlen=int(tokens))


# ----------------------------------------------------------------------------------------
# Dataset
# ----------------------------------------------------------------------------------------
class V1DatasetConfig(pydantic.BaseModel):
    seed: int
    dataset_path: str
    batch_max_length: int
    drop_last_batch: bool
    target_only: bool
    rank: int
    num_replicas: int
    homogeneous_categories: bool = False
    routing_categories: bool = False


class V1DatasetMeta(pydantic.BaseModel):
    tokenizer_info: dict[str, Any] = {}
    vocab_size: Optional[int] = None
    max_seq_len: int
    total_length: int


@dataclass
class V1DatasetIndices:
    inst_start: np.ndarray
    inst_len: np.ndarray
    resp_start: np.ndarray
    resp_len: np.ndarray


def validate_arrays(tokens, idx: V1DatasetIndices):
    """Bounded integer/shape/range checks of the token stream and row indices."""
    arrays = [idx.inst_start, idx.inst_len, idx.resp_start, idx.resp_len]
    if tokens.ndim != 1 or tokens.dtype.kind not in "iu":
        raise ValueError("tokens.npy must be an integer vector")
    if any(a.ndim != 1 or a.dtype.kind not in "iu" or len(a) != len(arrays[0]) for a in arrays):
        raise ValueError("Index arrays must be aligned integer vectors")
    for off in range(0, len(arrays[0]), 1_000_000):
        s, pl, r, rl = [a[off:off + 1_000_000] for a in arrays]
        if any(np.any(a < 0) for a in (s, pl, r, rl)) or np.any(rl < 1):
            raise ValueError("Negative offsets or empty responses")
        if np.any(s > len(tokens)) or np.any(r > len(tokens)):
            raise ValueError("Index starts outside token stream")
        if np.any(pl > len(tokens) - s) or np.any(rl > len(tokens) - r):
            raise ValueError("Index ends outside token stream")


class V1Dataset(IterableDataset):
    def __init__(self, config: V1DatasetConfig):
        super().__init__()
        self.config = config
        self.metadata = self._load_metadata()
        self._data = None
        self._indices: Optional[V1DatasetIndices] = None
        self._sampler = None
        self._epoch = 0
        self._start_batch = 0
        self._start_row_cursor: Optional[int] = None

    def _load_metadata(self) -> V1DatasetMeta:
        with open(os.path.join(self.config.dataset_path, "metadata.json")) as f:
            meta = V1DatasetMeta(**json.load(f))
        meta.max_seq_len -= 1  # autoregressive shift
        assert meta.vocab_size is None
        meta.vocab_size = find_multiple(meta.tokenizer_info.pop("vocab_size"), 256)
        return meta

    def set_epoch(self, epoch: int):
        if epoch < 0:
            raise ValueError(f"Dataset epoch must be non-negative, got {epoch}")
        if self._sampler is not None:
            raise RuntimeError("Cannot change dataset epoch after iteration has started")
        self._epoch = epoch

    def set_start_batch(self, start_batch: int):
        if start_batch < 0:
            raise ValueError(f"Dataset start batch must be non-negative, got {start_batch}")
        if self._sampler is not None:
            raise RuntimeError("Cannot change dataset start batch after iteration has started")
        self._start_batch = start_batch

    def set_start_row_cursor(self, cursor: int):
        if cursor < 0:
            raise ValueError(f"Dataset start row cursor must be non-negative, got {cursor}")
        if self._sampler is not None:
            raise RuntimeError("Cannot change dataset start row cursor after iteration has started")
        self._start_row_cursor = cursor

    def _begin_epoch(self):
        root = self.config.dataset_path
        if self._data is None:
            self._data = np.load(os.path.join(root, "tokens.npy"), mmap_mode="r")
        self._indices = V1DatasetIndices(**{f.name: np.load(os.path.join(root, f"epoch_{self._epoch}", f"{f.name}.npy"),
                                                             mmap_mode="r") for f in fields(V1DatasetIndices)})
        validate_arrays(self._data, self._indices)
        if self.config.homogeneous_categories or self.config.routing_categories:
            self._categories = np.load(os.path.join(root, f"epoch_{self._epoch}", "category_id.npy"), mmap_mode="r")
            if (self._categories.ndim != 1 or self._categories.dtype.kind not in "iu"
                    or len(self._categories) != len(self._indices.inst_len)):
                raise ValueError("category_id.npy must be an integer vector aligned with epoch rows")
        self._epoch += 1
        lengths = self._indices.inst_len + self._indices.resp_len - 1
        kwargs = dict(lengths=lengths, batch_max_length=self.config.batch_max_length,
                      drop_last_batch=self.config.drop_last_batch, rank=self.config.rank,
                      num_replicas=self.config.num_replicas)
        if self.config.homogeneous_categories:
            self._sampler = HomogeneousSampler(categories=self._categories, seed=self.config.seed + self._epoch - 1,
                                               **kwargs)
        else:
            self._sampler = MultipackDistributedBatchSampler(**kwargs)

    def _load_batch(self, rows: np.ndarray):
        assert self._data is not None and self._indices is not None
        idx = self._indices
        inputs, labels, positions, plens, clens = [], [], [], [], []
        for row in rows.tolist():
            i = np.asarray(self._data[idx.inst_start[row]: idx.inst_start[row] + idx.inst_len[row]], dtype=np.int32)
            o = np.asarray(self._data[idx.resp_start[row]: idx.resp_start[row] + idx.resp_len[row]], dtype=np.int32)
            inputs += [i, o[:-1]]
            labels += [np.full(len(i) - 1, IGNORE_LABEL_ID, np.int32) if self.config.target_only else i[1:], o]
            positions += [np.arange(len(i), dtype=np.int32), np.arange(len(i), len(i) + len(o) - 1, dtype=np.int32)]
            plens.append(len(i))
            clens.append(len(o) - 1)
        batch = {k: np.concatenate(v).astype(np.int32) if v else np.zeros(0, np.int32)
                 for k, v in (("inputs", inputs), ("labels", labels), ("position_ids", positions))}
        pad = self.config.batch_max_length - batch["inputs"].shape[0]
        if pad > 0:
            for k, fill in (("inputs", 0), ("labels", IGNORE_LABEL_ID), ("position_ids", 0)):
                batch[k] = np.pad(batch[k], (0, pad), constant_values=fill)
        tensors, scalars = compute_aux_seq_tensors_scalars(np.array(plens, np.int32), np.array(clens, np.int32),
                                                           self.config.batch_max_length)
        out = {k: torch.from_numpy(v) for k, v in (batch | tensors).items()}
        if self.config.homogeneous_categories:
            cats = self._categories[rows]
            if len(cats) == 0 or np.any(cats != cats[0]):
                raise ValueError("Expected a nonempty homogeneous microbatch")
            out["routing_category"] = torch.tensor(int(cats[0]))
        elif self.config.routing_categories:
            cats = self._categories[rows]
            if np.any(cats < 0):
                raise ValueError("Routing categories must be nonnegative")
            lengths = idx.inst_len[rows] + idx.resp_len[rows] - 1
            routed = np.repeat(cats.astype(np.int64), lengths.astype(np.int64))
            if pad > 0:
                routed = np.pad(routed, (0, pad))
            out["routing_category"] = torch.from_numpy(routed)
        return out, scalars

    def __iter__(self):
        info = get_worker_info()
        assert info is None or info.num_workers == 1
        self._begin_epoch()
        start_batch, self._start_batch = self._start_batch, 0
        cursor, self._start_row_cursor = self._start_row_cursor, None
        it = self._sampler.iter_with_info(start_index=cursor) if cursor is not None else self._sampler.iter_with_info()
        for number, (rows, resume) in enumerate(it, start=1):
            if cursor is None and number <= start_batch:
                continue
            batch, scalars = self._load_batch(rows)
            yield batch, scalars | {"resume_info": resume}
