# SPDX-License-Identifier: Apache-2.0
"""Host side of the W4A16 MoE GEMM (no GPU): the packed weight layout the
kernel reads, checked by unpacking it the way the kernel does (per step of
128 k, per quarter, per row, nibble pairs at positions (i, i + 4))."""
import numpy as np
import pytest
import torch

from kernels.titan_moe_gemm import pack_weights


def _unpack_like_kernel(packed, E, N, K):
    """Read the packed bytes at the kernel's offsets: tile t of pair np at
    step kc is at ((e ntn + 2 np) nk + kc nts + t) x 8 KB."""
    ntn, nk = N // 128, K // 128
    flat = packed.numpy()
    out = np.zeros((E, N, K), np.uint8)
    for e in range(E):
        for np_ in range((ntn + 1) // 2):
            nts = min(2, ntn - 2 * np_)
            for kc in range(nk):
                for t in range(nts):
                    off = ((e * ntn + 2 * np_) * nk + kc * nts + t) * 8192
                    blk = flat[off:off + 8192].reshape(4, 128, 16)
                    tile = 2 * np_ + t
                    for c in range(4):
                        words = blk[c].copy().view(np.uint32)                  # [128, 4]
                        for w4 in range(4):
                            w = words[:, w4].astype(np.uint64)
                            for i in range(4):
                                lo = (w >> (4 * i)) & 15                       # position i      -> k 2i
                                hi = (w >> (16 + 4 * i)) & 15                  # position i + 4  -> k 2i + 1
                                k0 = kc * 128 + 32 * c + 8 * w4 + 2 * i
                                out[e, tile * 128:(tile + 1) * 128, k0] = lo
                                out[e, tile * 128:(tile + 1) * 128, k0 + 1] = hi
    return out


@pytest.mark.parametrize("E,N,K", [(1, 128, 128), (3, 256, 384), (2, 384, 128)])
def test_pack_roundtrip(E, N, K):
    g = torch.Generator().manual_seed(E * N + K)
    q = torch.randint(0, 16, (E, N, K), generator=g, dtype=torch.uint8)
    packed = pack_weights(q)
    assert packed.dtype == torch.uint8 and packed.numel() == E * N * K // 2
    assert np.array_equal(_unpack_like_kernel(packed, E, N, K), q.numpy())


def test_pack_rejects_bad_shapes():
    with pytest.raises(ValueError):
        pack_weights(torch.zeros(1, 100, 128, dtype=torch.uint8))
    with pytest.raises(ValueError):
        pack_weights(torch.zeros(1, 128, 100, dtype=torch.uint8))
    with pytest.raises(ValueError):
        pack_weights(torch.zeros(1, 128, 128, dtype=torch.int32))


def test_oracle_dequant_rounding():
    """bf16((q - 8) * s): exact products of a 4-bit code and a bf16 scale,
    rounded once to bf16."""
    from oracle import oracle as O
    q = torch.tensor([[[0, 8, 15] + [8] * 125]], dtype=torch.uint8)
    s = torch.tensor([[[0.1]]], dtype=torch.float32).to(torch.bfloat16)
    w = O.moe_w4a16_dequant(q, s)
    sv = float(s.float())
    assert w[0, 0, 0].item() == torch.tensor(-8 * sv).to(torch.bfloat16).item()
    assert w[0, 0, 1].item() == 0.0
    assert w[0, 0, 2].item() == torch.tensor(7 * sv).to(torch.bfloat16).item()
