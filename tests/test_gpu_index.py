# SPDX-License-Identifier: Apache-2.0
"""Paged index conversion and the fused paged sparse MLA on the GPU.

The conversion (titan_convert_req_index_to_global) must equal vLLM's kernel
(golden vectors) and the oracle bit for bit; the fused reader
(triton_mla_sparse_attention_paged) must equal conversion + reader bit for
bit, and the FP32 oracle within the MLA tolerance.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.golden import cases as C

pytestmark = pytest.mark.gpu
GOLDEN = C.__file__.rsplit("/", 1)[0]
ATOL, RTOL = 2e-2, 1e-2


def test_conversion_matches_vllm_goldens(native_lib, cuda_device):
    from kernels.titan_index import triton_convert_req_index_to_global_index as conv
    gold = np.load(f"{GOLDEN}/index_golden.npz")
    for case in C.INDEX_CASES:
        inp = {k: v.to(cuda_device) for k, v in C.index_inputs(case).items()}
        out = conv(inp["req_id"], inp["block_table"], inp["token_indices"], BLOCK_SIZE=case.block_size,
                   NUM_TOPK_TOKENS=case.topk)
        assert np.array_equal(out.cpu().numpy(), gold[f"{case.name}__out"]), case.name


@pytest.mark.parametrize("block_size,stride_rows", [(64, 64), (64, 80), (48, 48), (16, 24)])
def test_conversion_layouts(native_lib, cuda_device, block_size, stride_rows):
    """Padded block strides, non-power-of-two blocks, a strided and unaligned
    index view (scalar path), a transposed block table, and token requests
    that are not rows of the table (-1)."""
    from kernels.titan_index import triton_convert_req_index_to_global_index as conv
    g = torch.Generator().manual_seed(block_size + stride_rows)
    T, R, NB, topk = 7, 3, 11, 256
    req = torch.randint(0, R, (T,), generator=g, dtype=torch.int32)
    req[3], req[5] = R, -1
    bt_t = torch.randint(0, 1000, (NB, R), generator=g, dtype=torch.int32)
    wide = torch.randint(-5, NB * block_size + 30, (T, topk + 9), generator=g, dtype=torch.int32)
    want = O.convert_req_index_to_global(req.numpy(), bt_t.t().numpy(), wide[:, 3:3 + topk].numpy(), block_size,
                                         stride_rows)
    dev = cuda_device
    out = conv(req.to(dev), bt_t.to(dev).t(), wide.to(dev)[:, 3:3 + topk], BLOCK_SIZE=block_size,
               NUM_TOPK_TOKENS=topk, BLOCK_STRIDE_ROWS=stride_rows)
    assert np.array_equal(out.cpu().numpy(), want)
    assert (want[3] == -1).all() and (want[5] == -1).all()


def _paged_setup(device, block_size, stride_rows, tokens, seed, topk=2176, reqs=2, blocks_per_req=40):
    from kernels.titan_kv import store_int8
    g = torch.Generator().manual_seed(seed)
    n_blocks = reqs * blocks_per_req + 8
    rows = n_blocks * stride_rows
    latent = torch.randn(rows, 512, generator=g).to(torch.bfloat16)
    cache = torch.zeros((rows + 255) // 256, 256, 528, dtype=torch.int8, device=device)
    store_int8(latent.to(device), cache, torch.arange(rows, device=device))
    perm = torch.randperm(n_blocks, generator=g)[:reqs * blocks_per_req].to(torch.int32)
    bt = perm.view(reqs, blocks_per_req)
    req = torch.randint(0, reqs, (tokens,), generator=g, dtype=torch.int32)
    tok = torch.randint(-2, blocks_per_req * block_size + 50, (tokens, topk), generator=g, dtype=torch.int32)
    q = torch.randn(tokens, 16, 512, generator=g).to(torch.bfloat16)
    return cache.view(-1, 528)[:rows], q, tok, req, bt


@pytest.mark.parametrize("block_size,stride_rows,tokens", [(64, 64, 1), (64, 80, 3), (48, 48, 2)])
def test_fused_paged_attention_equals_conversion_then_reader(native_lib, cuda_device, block_size, stride_rows,
                                                             tokens):
    from kernels.titan_index import triton_convert_req_index_to_global_index as conv
    from kernels.titan_mla import triton_mla_sparse_attention as attn
    from kernels.titan_mla import triton_mla_sparse_attention_paged as attn_paged
    rows, q, tok, req, bt = _paged_setup(cuda_device, block_size, stride_rows, tokens, 40 + tokens)
    dev = cuda_device
    kv = rows.view(-1, 1, 528)
    qd, tokd, reqd, btd = q.to(dev), tok.to(dev), req.to(dev), bt.to(dev)
    glob = conv(reqd, btd, tokd, BLOCK_SIZE=block_size, NUM_TOPK_TOKENS=tok.shape[1], BLOCK_STRIDE_ROWS=stride_rows)
    ref = O.mla_sparse_attention(q, rows.cpu(), glob.cpu().view(tokens, 1, -1), 512 ** -0.5)
    for splits in (None, 1, 4, 17, 32, 80):
        two = attn(qd, kv, glob.view(tokens, 1, -1), 512 ** -0.5, num_kv_splits=splits)
        one = attn_paged(qd, kv, tokd, reqd, btd, block_size, 512 ** -0.5, block_stride_rows=stride_rows,
                         num_kv_splits=splits)
        assert torch.equal(one, two), splits
        d = (one.float().cpu() - ref).abs()
        assert bool((d <= ATOL + RTOL * ref.abs()).all()), (splits, d.max().item())
    from kernels import titan_native
    assert titan_native.device_error(qd) == 0
