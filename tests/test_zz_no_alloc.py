# SPDX-License-Identifier: Apache-2.0
"""The allocation-free MLA entry point, titan_mla_sparse_attention_noalloc.

Some callers cannot allocate device memory: a plugin inside a host engine that
owns the whole device pool, or code that issues work while another thread
captures a stream in global mode (cudaMalloc is refused then).  For them the
library keeps the split-KV scratch in a static 8 MiB device array.  This test
calls that entry point directly through the C ABI, twice in a row on different
inputs, and checks each output against the regular entry point (which takes a
caller-allocated workspace) and against the FP32 oracle, with the MLA
tolerance used by the other tests.
It is collected last so a failure here cannot hide another test's result, and
it sets up everything it needs so it also passes alone in a fresh process.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def _inputs(device, tokens, seed, rows=8192):
    from kernels.titan_kv import store_int8
    g = torch.Generator().manual_seed(seed)
    latent = torch.randn(rows, 512, generator=g).to(torch.bfloat16)
    cache = torch.zeros(rows // 256, 256, 528, dtype=torch.int8, device=device)
    store_int8(latent.to(device), cache, torch.arange(rows, device=device))
    q = torch.randn(tokens, 16, 512, generator=g).to(torch.bfloat16).to(device)
    idx = torch.randint(-20, rows + 20, (tokens, 2176), generator=g, dtype=torch.int32).to(device)
    return cache.view(rows, 528), q, idx


def _call(lib, q, rows, idx, out, splits, workspace=None, noalloc=False):
    stream = torch.cuda.current_stream(q.device).cuda_stream
    args = [q.data_ptr(), q.stride(0), q.stride(1), rows.data_ptr(), rows.stride(0), rows.shape[0],
            idx.data_ptr(), idx.stride(0), idx.shape[1], out.data_ptr(), out.stride(0), out.stride(1),
            q.shape[0], q.shape[1], ctypes.c_float(512 ** -0.5), splits]
    if noalloc:
        return lib.titan_mla_sparse_attention_noalloc(*args, stream)
    return lib.titan_mla_sparse_attention(*args, workspace.data_ptr(), workspace.numel(), stream)


@pytest.mark.parametrize("tokens,splits", [(2, 64), (1, 3), (8, 16)])
def test_noalloc_matches_workspace_entry_point(native_lib, cuda_device, tokens, splits):
    lib = native_lib
    assert lib.titan_mla_noalloc_scratch_bytes() == 8 << 20
    need = lib.titan_mla_workspace_bytes(tokens, 16, splits)
    assert 0 < need <= lib.titan_mla_noalloc_scratch_bytes()
    for call, seed in enumerate((101, 202)):          # two calls in a row share the static scratch
        rows, q, idx = _inputs(cuda_device, tokens, seed + tokens)
        ref = torch.empty(tokens, 16, 512, dtype=torch.bfloat16, device=cuda_device)
        ws = torch.empty(need, dtype=torch.uint8, device=cuda_device)
        assert _call(lib, q, rows, idx, ref, splits, workspace=ws) == 0, lib.titan_last_error()
        out = torch.full_like(ref, float("nan"))
        torch.cuda.synchronize()
        before = torch.cuda.memory_stats(cuda_device).get("allocation.all.allocated", 0)
        assert _call(lib, q, rows, idx, out, splits, noalloc=True) == 0, lib.titan_last_error()
        after = torch.cuda.memory_stats(cuda_device).get("allocation.all.allocated", 0)
        torch.cuda.synchronize()
        assert after == before, "the allocation-free entry point allocated through torch"
        o, r = out.float(), ref.float()
        assert torch.isfinite(o).all()
        assert bool(((o - r).abs() <= ATOL + RTOL * r.abs()).all()), (call, (o - r).abs().max().item())
        # and on its own against the oracle
        from oracle import oracle as O
        want = O.mla_sparse_attention(q.cpu(), rows.cpu(), idx.cpu(), 512 ** -0.5)
        oc = o.cpu()
        assert bool(((oc - want).abs() <= ATOL + RTOL * want.abs()).all()), (call, (oc - want).abs().max().item())


def test_noalloc_rejects_calls_beyond_the_scratch(native_lib, cuda_device):
    lib = native_lib
    tokens, splits = 64, 64                            # needs 128 MiB of partials
    assert lib.titan_mla_workspace_bytes(tokens, 16, splits) > lib.titan_mla_noalloc_scratch_bytes()
    rows, q, idx = _inputs(cuda_device, tokens, 7, rows=1024)
    out = torch.empty(tokens, 16, 512, dtype=torch.bfloat16, device=cuda_device)
    rc = _call(lib, q, rows, idx, out, splits, noalloc=True)
    assert rc == 1
    assert b"static scratch" in lib.titan_last_error()
