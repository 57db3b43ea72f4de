# SPDX-License-Identifier: Apache-2.0
"""Indexer pool top-k + expansion on the GPU (csrc/titan_indexer.cu) against
the oracle (whose expansion is pinned to the reference's expand_row): exact
int32 rows, including ties, NaN, short contexts, every tail phase and the
decode shape (65,536 pools of 4 = 262,144 tokens, 2176-wide rows)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _check(logits, seq_lens, k, pool, width, device):
    from kernels.titan_indexer import pool_topk_expand
    got = pool_topk_expand(logits.to(device), seq_lens.to(device), k, pool, width).cpu().numpy()
    want = O.pool_topk_expand(logits, seq_lens, k, pool, width)
    bad = np.nonzero((got != want).any(1))[0]
    assert bad.size == 0, (bad[:5], got[bad[0]][:12] if bad.size else None, want[bad[0]][:12] if bad.size else None)


def test_decode_shape(native_lib, cuda_device):
    g = torch.Generator().manual_seed(1)
    P = 65536
    logits = torch.randn(8, P, generator=g)
    seq_lens = torch.tensor([262144, 262143, 262142, 262141, 200001, 131072, 2049, 5], dtype=torch.int32)
    _check(logits, seq_lens, 512, 4, 2176, cuda_device)


def test_prefill_rows_all_lengths(native_lib, cuda_device):
    """Query rows at every context length from 1 to 2200 tokens (all valid
    pools taken below 2048 tokens) and a few long ones."""
    g = torch.Generator().manual_seed(2)
    lens = list(range(1, 2201, 7)) + [65536, 65537, 99999]
    logits = torch.randn(len(lens), 40000, generator=g)
    _check(logits, torch.tensor(lens, dtype=torch.int32), 512, 4, 2176, cuda_device)


# Up to 9 rows take the cluster form on a 148-SM B200 (5 rows: clusters of
# 16 CTAs, the slice-sum reduction; 8 rows: clusters of 8, every CTA summing
# the whole histogram), 40 rows the one-CTA-per-row form.
@pytest.mark.parametrize("rows", [5, 8, 40])
@pytest.mark.parametrize("levels", [3, 40])
def test_heavy_ties(native_lib, cuda_device, levels, rows):
    """Logits on a few levels: the k-th largest value is shared by many pools,
    taken in pool order (3 levels: more than 4096 candidates, the multi-pass
    selection; 40 levels: the candidate path with ~500 ties)."""
    g = torch.Generator().manual_seed(levels)
    logits = torch.randint(0, levels, (rows, 20000), generator=g).float()
    _check(logits, torch.full((rows,), 80000, dtype=torch.int32), 512, 4, 2176, cuda_device)


def test_decode_shape_one_cta_per_row(native_lib, cuda_device):
    """The decode shape with enough rows for the one-CTA-per-row form."""
    g = torch.Generator().manual_seed(6)
    logits = torch.randn(24, 65536, generator=g)
    seq_lens = torch.randint(262000, 262145, (24,), generator=g, dtype=torch.int32)
    seq_lens[3] = 5
    _check(logits, seq_lens, 512, 4, 2176, cuda_device)


def test_nan_inf_and_small_k(native_lib, cuda_device):
    g = torch.Generator().manual_seed(4)
    logits = torch.randn(4, 5000, generator=g)
    logits[0, ::97] = float("nan")
    logits[1, ::13] = float("inf")
    logits[2, ::7] = float("-inf")
    logits[3, 100:4000] = 0.0
    logits[3, 5] = -0.0
    seq = torch.tensor([20000, 19999, 18000, 20003], dtype=torch.int32)
    for k, pool, width in ((512, 4, 2176), (1, 4, 8), (37, 1, 40), (1024, 2, 2049), (300, 16, 4815)):
        _check(logits, seq, k, pool, width, cuda_device)
    # the same rows repeated (8 rows: clusters of 8; 40 rows: one CTA per row)
    _check(logits.repeat(2, 1), seq.repeat(2), 512, 4, 2176, cuda_device)
    _check(logits.repeat(10, 1), seq.repeat(10), 512, 4, 2176, cuda_device)


def test_strided_rows_and_empty(native_lib, cuda_device):
    from kernels.titan_indexer import pool_topk_expand
    g = torch.Generator().manual_seed(5)
    big = torch.randn(3, 9000, generator=g)
    view = big[:, :7000]                       # row stride 9000 > 7000 pools
    _check(view, torch.tensor([28000, 100, 0], dtype=torch.int32), 512, 4, 2176, cuda_device)
    empty = pool_topk_expand(torch.zeros(0, 16, device=cuda_device), torch.zeros(0, dtype=torch.int32,
                                                                               device=cuda_device))
    assert empty.shape == (0, 2176)
