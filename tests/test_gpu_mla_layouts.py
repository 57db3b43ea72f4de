# SPDX-License-Identifier: Apache-2.0
"""Cache layouts and index edge cases of the TMA row gather.

The reader describes the cache to the tensor memory accelerator as `seq_kv`
rows of 528 bytes, `kv.stride(0)` bytes apart: rows outside [0, seq_kv) read
as zeros and are masked, padding between rows is never read, a four-row
gather group whose rows are all masked is skipped.  Results must not depend on
any of that: a padded cache gives the contiguous cache's bits, masked rows
behave like index -1 (kernels/titan_mla.py:126-133), and an empty cache gives
zeros.  Tolerance against the FP32 oracle: |out - ref| <= 2e-2 + 1e-2 |ref|.
"""
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def _cache(rows, seed, device):
    from kernels.titan_kv import store_int8
    g = torch.Generator().manual_seed(seed)
    cache = torch.empty(rows, 1, 528, dtype=torch.int8, device=device)
    store_int8(torch.randn(rows, 512, generator=g).to(torch.bfloat16).to(device), cache.view(rows, 1, 528),
               torch.arange(rows, device=device))
    return cache


def _bits(t):
    return t.view(torch.int16)


@pytest.mark.parametrize("pitch", [544, 1056, 528 + 16 * 7])
@pytest.mark.parametrize("splits", [0, 1, 4])
def test_padded_row_stride_matches_contiguous(pitch, splits, native_lib, cuda_device):
    from kernels.titan_mla import triton_mla_sparse_attention as attn
    rows, tokens, topk = 3000, 3, 512
    dense = _cache(rows, 11, cuda_device)
    padded = torch.randint(-128, 128, (rows, pitch), dtype=torch.int8, device=cuda_device)  # garbage padding
    padded[:, :528] = dense.view(rows, 528)
    kv_pad = padded[:, :528].view(rows, 1, 528)
    assert kv_pad.stride(0) == pitch
    g = torch.Generator().manual_seed(pitch + splits)
    q = torch.randn(tokens, 16, 512, generator=g).to(torch.bfloat16).to(cuda_device)
    idx = torch.randint(-8, rows + 8, (tokens, 1, topk), generator=g, dtype=torch.int32).to(cuda_device)
    ref = attn(q, dense, idx, 0.05, num_kv_splits=splits)
    out = attn(q, kv_pad, idx, 0.05, num_kv_splits=splits)
    assert torch.equal(_bits(out), _bits(ref))


def test_last_row_and_tiny_cache(native_lib, cuda_device):
    """Indices at seq_kv - 1 (the last row of an exactly sized cache) are read;
    seq_kv and beyond, negative and extreme int32 values are masked."""
    from kernels.titan_mla import triton_mla_sparse_attention as attn
    for rows in (1, 5, 97):
        kv = _cache(rows, rows, cuda_device)
        idx = torch.full((2, 1, 64), -1, dtype=torch.int32)
        idx[0, 0, :8] = rows - 1
        idx[0, 0, 8:16] = torch.arange(8) % rows
        idx[0, 0, 16:20] = torch.tensor([rows, rows + 1, 2 ** 31 - 1, -(2 ** 31)], dtype=torch.int32)
        idx[1, 0, 40] = rows - 1                           # one valid row in an otherwise masked tile
        g = torch.Generator().manual_seed(rows)
        q = torch.randn(2, 16, 512, generator=g).to(torch.bfloat16)
        ref = O.mla_sparse_attention(q, kv.view(rows, 528).cpu(), idx, 0.07)
        for splits in (0, 1, 2):
            out = attn(q.to(cuda_device), kv, idx.to(cuda_device), 0.07, num_kv_splits=splits).float().cpu()
            assert bool(((out - ref).abs() <= ATOL + RTOL * ref.abs()).all()), (rows, splits)


def test_masked_groups_between_valid_ones(native_lib, cuda_device):
    """Tiles where whole four-row gather groups are masked (not issued) next to
    valid ones: masking by -1, by >= seq_kv and valid rows interleave."""
    from kernels.titan_mla import triton_mla_sparse_attention as attn
    rows = 4096
    kv = _cache(rows, 5, cuda_device)
    g = torch.Generator().manual_seed(9)
    idx = torch.randint(0, rows, (4, 1, 256), generator=g, dtype=torch.int32)
    pos = torch.arange(256)
    idx[0, 0, (pos // 4) % 2 == 0] = -1                   # every other group of 4 positions
    idx[1, 0, pos % 32 >= 4] = rows + 5                   # only 4 valid positions per tile
    idx[2, 0, :] = -1
    idx[2, 0, 255] = 7                                    # a single valid row, the last position
    q = torch.randn(4, 16, 512, generator=g).to(torch.bfloat16)
    ref = O.mla_sparse_attention(q, kv.view(rows, 528).cpu(), idx, 0.06)
    for splits in (0, 1, 3, 8):
        out = attn(q.to(cuda_device), kv, idx.to(cuda_device), 0.06, num_kv_splits=splits).float().cpu()
        assert bool(((out - ref).abs() <= ATOL + RTOL * ref.abs()).all()), splits


def test_empty_cache_gives_zeros(native_lib, cuda_device):
    from kernels.titan_mla import triton_mla_sparse_attention as attn
    kv = torch.empty(0, 1, 528, dtype=torch.int8, device=cuda_device)
    q = torch.randn(2, 16, 512, device=cuda_device).to(torch.bfloat16)
    idx = torch.randint(-4, 100, (2, 1, 96), dtype=torch.int32, device=cuda_device)
    for splits in (0, 1, 2):
        out = attn(q, kv, idx, 0.1, num_kv_splits=splits)
        torch.cuda.synchronize()
        assert not out.any()
