# SPDX-License-Identifier: Apache-2.0
"""Indexer pool top-k oracle (no GPU): the expansion against golden vectors
made by the reference's own `expand_row` (tests/golden/make_indexer_golden.py),
and the selection against torch.topk."""
import numpy as np
import torch

from oracle import oracle as O
from tests.golden import cases as C

GOLDEN = C.__file__.rsplit("/", 1)[0]


def test_expand_row_matches_reference_goldens():
    g = np.load(f"{GOLDEN}/indexer_golden.npz")
    assert len(g["cases"]) == 40
    for c in g["cases"]:
        seq_len, pool_size, tail = (int(v) for v in g[f"c{c}__meta"])
        row = O.expand_row([int(p) for p in g[f"c{c}__pools"]], seq_len, pool_size, bool(tail))
        assert row == g[f"c{c}__row"].tolist(), c


def test_selection_matches_torch_topk_and_width():
    gen = torch.Generator().manual_seed(3)
    logits = torch.randn(6, 3000, generator=gen)
    seq_lens = torch.tensor([4 * 3000, 4 * 3000 + 3, 1000, 4 * 512 + 1, 7, 0], dtype=torch.int32)
    out = O.pool_topk_expand(logits, seq_lens, 512, 4, 2176)
    assert out.shape == (6, 2176)
    for t in range(6):
        n = min(int(seq_lens[t]) // 4, 3000)
        k = min(512, n)
        if k:
            want = torch.topk(logits[t, :n], k).indices.tolist()
            assert out[t, 0:4 * k:4].tolist() == [4 * p for p in want]
        assert (out[t, 4 * k:2048] == -1).all()
        tl = int(seq_lens[t]) % 4
        assert out[t, 2048:2051].tolist() == [int(seq_lens[t]) // 4 * 4 + o if o < tl else -1 for o in range(3)]
        assert (out[t, 2051:] == -1).all()


def test_ties_signed_zero_and_nan_order():
    logits = torch.tensor([[1.0, 5.0, 5.0, float("nan"), 5.0, -2.0, -float("nan"), 0.0, -0.0, 0.0]])
    out = O.pool_topk_expand(logits, torch.tensor([40], dtype=torch.int32), 10, 1, 12)
    # NaN of either sign first (pool order), ties in pool order, +0.0 above -0.0
    assert out[0, :10].tolist() == [3, 6, 1, 2, 4, 0, 7, 9, 8, 5]
