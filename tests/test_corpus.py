"""Corpus sampling/batching parity with the reference sampler (when installed) and resume semantics."""
import os
import sys

import numpy as np
import pytest
import torch

from mimir_b200.data.corpus import V1Dataset, V1DatasetConfig, allocate, allocate_python
from mimir_b200.data.synthetic import write_corpus

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


def test_native_allocator_matches_python():
    rng = np.random.default_rng(0)
    lengths = rng.integers(1, 300, size=500).astype(np.int64)
    lengths[10:20] = 100  # ties
    for n in (1, 2, 3, 8):
        start = 0
        while start < lengths.size:
            a = allocate(lengths, start, n - 1, 1024, n)
            b = allocate_python(lengths, start, n - 1, 1024, n)
            assert a[0] == b[0] and a[1] == b[1] and a[3] == b[3] and np.array_equal(a[2], b[2])
            start += a[1]


def _cfg(path, rank=0, world=1, **kw):
    return V1DatasetConfig(seed=0, dataset_path=path, batch_max_length=1024, drop_last_batch=False, target_only=True,
                           rank=rank, num_replicas=world, **kw)


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "mimir")), reason="reference not installed")
@pytest.mark.parametrize("world", [1, 2])
def test_batches_match_reference(tmp_path, world):
    if REF not in sys.path:
        sys.path.append(REF)
    from mimir.corpus.sampled import V1Dataset as RefDataset, V1DatasetConfig as RefConfig
    path = write_corpus(str(tmp_path / "c"), rows=60, seq_len=200, vocab=500, answer_len_range=(5, 150), epochs=2)
    for rank in range(world):
        ours = V1Dataset(_cfg(path, rank, world))
        ref = RefDataset(RefConfig(**_cfg(path, rank, world).model_dump()))
        assert ours.metadata.model_dump() == ref.metadata.model_dump()
        for epoch in range(2):
            ours.set_epoch(epoch) if epoch == 0 else None
            a, b = list(ours), list(ref)
            assert len(a) == len(b) > 0
            for (ba, sa), (bb, sb) in zip(a, b):
                assert sa == sb
                assert set(ba) == set(bb)
                for k in ba:
                    assert torch.equal(ba[k], bb[k]), k
            ours._sampler = ref._sampler = None


def test_resume_by_batch_and_cursor(tmp_path):
    path = write_corpus(str(tmp_path / "c"), rows=50, seq_len=100, vocab=300, answer_len_range=(5, 80))
    full = list(V1Dataset(_cfg(path)))
    ds = V1Dataset(_cfg(path))
    ds.set_start_batch(3)
    skipped = list(ds)
    assert len(skipped) == len(full) - 3
    for (a, _), (b, _) in zip(skipped, full[3:]):
        assert torch.equal(a["inputs"], b["inputs"])
    cursor = full[2][1]["resume_info"]["global_row_end"]
    ds = V1Dataset(_cfg(path))
    ds.set_start_row_cursor(cursor)
    resumed = list(ds)
    assert torch.equal(resumed[0][0]["inputs"], full[3][0]["inputs"])
