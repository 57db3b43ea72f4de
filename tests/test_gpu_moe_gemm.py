# SPDX-License-Identifier: Apache-2.0
"""W4A16 MoE GEMM on the GPU (csrc/titan_moe_gemm.cu, tcgen05) against the
oracle: every list of a split_align over seeded routes, gate/up form (A =
tokens, top_k = 8) and down form (A = routed rows, top_k = 1, router
weights applied), all four block sizes, Zipf-skewed and invalid routes.

Tolerance: both sides round to bf16 at the end from sums of the same
bf16-rounded weights and activations (fp32 on the GPU, float64 in the
oracle), so they differ by at most about one bf16 step: |out - ref| <=
1e-2 |ref| + 1e-3 max|ref|.  Rows that no list holds keep their marker."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
MARK = 7.0


def _close(out, ref):
    out, ref = out.float().cpu(), ref.float()
    tol = 1e-2 * ref.abs() + 1e-3 * ref.abs().max()
    return bool(((out - ref).abs() <= tol).all()), (out - ref).abs().max().item()


def _routes(M, top_k, E, dist, g):
    if dist == "zipf":
        w = torch.arange(1, E + 1, dtype=torch.float64) ** -1.1
        return torch.stack([torch.multinomial(w, top_k, replacement=top_k > E, generator=g) for _ in range(M)])
    r = torch.randint(0, E, (M, top_k), generator=g)
    if dist == "invalid":
        r[::3, 1] = -1
        r[::5, 2] = E + 3
    return r


@pytest.mark.parametrize("E,N,K,M,dist", [
    (4, 128, 128, 5, "uniform"),
    (16, 256, 512, 64, "uniform"),
    (16, 128, 256, 200, "zipf"),
    (24, 128, 256, 33, "invalid"),
    (288, 256, 1024, 96, "zipf"),
])
def test_gate_up_and_down_against_oracle(native_lib, cuda_device, E, N, K, M, dist):
    from kernels import titan_moe_split_align as split_mod
    from kernels.titan_moe_gemm import moe_w4a16_gemm, pack_weights
    top_k = 8
    g = torch.Generator().manual_seed(E * 1000 + N + K + M)
    q = torch.randint(0, 16, (E, N, K), generator=g, dtype=torch.uint8)
    scales = (torch.rand(E, K // 128, N, generator=g) * 0.02 + 0.002).to(torch.bfloat16)
    w_deq = O.moe_w4a16_dequant(q, scales)
    packed = pack_weights(q).to(cuda_device)
    sc = scales.to(cuda_device)
    routes = _routes(M, top_k, E, dist, g).to(torch.int32)
    rows = M * top_k
    buf = split_mod.buffers(rows, E, cuda_device)
    lists = split_mod.split_align(routes.to(cuda_device), E, buf)
    sizes_used = [int(n.item()) for _, _, _, n in lists]
    # gate/up: A = tokens, C rows = routed rows
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    c = torch.full((rows, N), MARK, dtype=torch.bfloat16, device=cuda_device)
    ref = torch.full((rows, N), MARK, dtype=torch.bfloat16)
    ad = a.to(cuda_device)
    for bs, s, e, n in lists:
        moe_w4a16_gemm(ad, c, packed, sc, s, e, n, None, bs, top_k, False, M, N, K)
        O.moe_w4a16_gemm(a, w_deq, s, e, n, None, bs, top_k, False, M, ref)
    ok, err = _close(c, ref)
    assert ok, ("gate/up", err, sizes_used)
    # down: A = routed rows, top_k = 1, router weights on the output
    a2 = torch.randn(rows, K, generator=g).to(torch.bfloat16)
    tw = torch.rand(rows, generator=g, dtype=torch.float32)
    c2 = torch.full((rows, N), MARK, dtype=torch.bfloat16, device=cuda_device)
    ref2 = torch.full((rows, N), MARK, dtype=torch.bfloat16)
    for bs, s, e, n in lists:
        moe_w4a16_gemm(a2.to(cuda_device), c2, packed, sc, s, e, n, tw.to(cuda_device), bs, 1, True, rows, N, K)
        O.moe_w4a16_gemm(a2, w_deq, s, e, n, tw, bs, 1, True, rows, ref2)
    ok, err = _close(c2, ref2)
    assert ok, ("down", err, sizes_used)
    from kernels import titan_native
    assert titan_native.device_error(c) == 0


def test_every_block_size_and_graph_replay(native_lib, cuda_device):
    """One expert per block size (rows 64 + 48 + 32 + 16 = 160 for expert 0,
    48 for expert 1, ...), the GEMMs captured in a CUDA graph and replayed on
    new activations."""
    from kernels import titan_moe_split_align as split_mod
    from kernels.titan_moe_gemm import moe_w4a16_gemm, pack_weights
    E, N, K = 4, 256, 256
    g = torch.Generator().manual_seed(77)
    counts = [160, 48, 32, 16]
    flat = torch.cat([torch.full((n,), e, dtype=torch.int32) for e, n in enumerate(counts)])
    flat = flat[torch.randperm(flat.numel(), generator=g)]
    routes = flat.view(-1, 8)
    M = routes.shape[0]
    rows = M * 8
    q = torch.randint(0, 16, (E, N, K), generator=g, dtype=torch.uint8)
    scales = (torch.rand(E, K // 128, N, generator=g) * 0.05 + 0.01).to(torch.bfloat16)
    w_deq = O.moe_w4a16_dequant(q, scales)
    packed, sc = pack_weights(q).to(cuda_device), scales.to(cuda_device)
    buf = split_mod.buffers(rows, E, cuda_device)
    lists = split_mod.split_align(routes.to(cuda_device), E, buf)
    assert all(int(n.item()) > 0 for _, _, _, n in lists)
    a = torch.zeros(M, K, dtype=torch.bfloat16, device=cuda_device)
    c = torch.zeros(rows, N, dtype=torch.bfloat16, device=cuda_device)

    def step():
        for bs, s, e, n in lists:
            moe_w4a16_gemm(a, c, packed, sc, s, e, n, None, bs, 8, False, M, N, K)
    step()
    graph = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        with torch.cuda.graph(graph, stream=st):
            step()
    torch.cuda.current_stream().wait_stream(st)
    for seed in (1, 2):
        ah = torch.randn(M, K, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)
        a.copy_(ah)
        graph.replay()
        torch.cuda.synchronize()
        ref = torch.zeros(rows, N, dtype=torch.bfloat16)
        for bs, s, e, n in lists:
            O.moe_w4a16_gemm(ah, w_deq, s, e, n, None, bs, 8, False, M, ref)
        ok, err = _close(c, ref)
        assert ok, (seed, err)
    graph.reset()


def test_rejects_bad_arguments(native_lib, cuda_device):
    from kernels.titan_moe_gemm import moe_w4a16_gemm
    d = cuda_device
    a = torch.zeros(4, 128, dtype=torch.bfloat16, device=d)
    c = torch.zeros(32, 128, dtype=torch.bfloat16, device=d)
    packed = torch.zeros(128 * 128 // 2, dtype=torch.uint8, device=d)
    sc = torch.zeros(1, 1, 128, dtype=torch.bfloat16, device=d)
    ids = torch.zeros(64, dtype=torch.int32, device=d)
    n = torch.zeros(1, dtype=torch.int32, device=d)
    from kernels.titan_native import TitanError
    with pytest.raises(TitanError):
        moe_w4a16_gemm(a, c, packed, sc, ids, ids, n, None, 24, 8, False, 4, 128, 128)   # block size
    with pytest.raises(ValueError):
        moe_w4a16_gemm(a, c, packed[:-1], sc, ids, ids, n, None, 16, 8, False, 4, 128, 128)
    with pytest.raises(ValueError):
        moe_w4a16_gemm(a, c, packed, sc, ids, ids, n, None, 16, 8, True, 4, 128, 128)  # weights missing


def _vllm_marlin():
    try:
        from vllm import _custom_ops as ops
        torch.ops._C.gptq_marlin_repack  # noqa: B018  (the compiled extension loaded)
        return ops
    except Exception as exc:  # vLLM absent or its extension does not load here
        pytest.skip(f"vLLM Marlin unavailable: {type(exc).__name__}: {exc}")


@pytest.mark.parametrize("E,N,K,M", [(8, 256, 512, 96), (32, 512, 1024, 300)])
def test_matches_vllm_marlin(native_lib, cuda_device, E, N, K, M):
    """The same codes, scales, activations and split_align lists through
    vLLM's moe_wna16_marlin_gemm (the kernel the reference runs for this
    step, called as profiles/sm74/titan_prefill/marlin.py:427-437 does) and
    through ours: both round fp32 sums of the same bf16 products to bf16, so
    each element agrees to one bf16 step of itself or 2^-8 of the largest."""
    _vllm_marlin()
    from vllm import _custom_ops as ops
    from vllm.model_executor.layers.quantization.utils.marlin_utils import marlin_make_workspace_new
    from vllm.scalar_type import scalar_types

    import bench
    from kernels import titan_moe_split_align as split_mod
    from kernels.titan_moe_gemm import moe_w4a16_gemm, pack_weights
    top_k, d = 8, cuda_device
    g = torch.Generator().manual_seed(E + N + K + M)
    q = torch.randint(0, 16, (E, N, K), generator=g, dtype=torch.uint8).to(d)
    scales = (torch.rand(E, K // 128, N, generator=g) * 0.02 + 0.002).to(torch.bfloat16).to(d)
    routes = _routes(M, top_k, E, "zipf", g).to(torch.int32).to(d)
    lists = split_mod.split_align(routes, E, split_mod.buffers(M * top_k, E, d))
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).to(d)
    ours = torch.zeros(M * top_k, N, dtype=torch.bfloat16, device=d)
    packed = pack_weights(q)
    for bs, s, e, n in lists:
        moe_w4a16_gemm(a, ours, packed, scales, s, e, n, None, bs, top_k, False, M, N, K)
    w, sm = bench.marlin_weights(q, scales)
    ref = torch.zeros_like(ours)
    ws = marlin_make_workspace_new(d, 4)
    tw = torch.ones(M, top_k, dtype=torch.float32, device=d)
    for bs, s, e, n in lists:
        tk, tn, bps = bench.MARLIN_THREAD_CFG.get(bs, (-1, -1, -1))
        ops.moe_wna16_marlin_gemm(a, ref, w, None, sm, None, None, None, None, None, ws, s, e, n, tw,
                                  moe_block_size=bs, top_k=top_k, mul_topk_weights=False,
                                  b_q_type=scalar_types.uint4b8, size_m=M, size_n=N, size_k=K, is_k_full=True,
                                  use_atomic_add=False, use_fp32_reduce=True, is_zp_float=False,
                                  thread_k=tk, thread_n=tn, blocks_per_sm=bps)
    torch.cuda.synchronize()
    o, r = ours.float(), ref.float()
    tol = torch.maximum(r.abs() * 2 ** -7, torch.full_like(r, 2 ** -8) * r.abs().max())
    assert r.abs().max() > 0
    assert bool(((o - r).abs() <= tol).all()), (o - r).abs().max().item()
