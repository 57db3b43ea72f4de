# SPDX-License-Identifier: Apache-2.0
"""W4A16 MoE GEMM over the split-align block lists, for B200 (sm_100a).

The consumer of `titan_moe_split_align.split_align`'s lists: the reference
runs one vLLM `moe_wna16_marlin_gemm` per list for the gate/up projection
(A = the tokens, top_k = 8) and one per list for the down projection (A = the
activated routed rows, top_k = 1, outputs scaled by the router weights)
(profiles/sm74/titan_prefill/marlin.py:417-444).  For each of the
ntpp / block_size blocks b with expert e = expert_ids[b] and routed rows
s = sorted_ids[b * block_size : (b + 1) * block_size]:

    C[s, :] = A[s // top_k, :] @ W_e^T          (ids >= size_m * top_k are padding)
    W_e[n, k] = bf16((q[e, n, k] - 8) * scales[e, k // 128, n])    (uint4b8, group 128)
    C[s, :] *= topk_weights[s]                   (mul_topk_weights)

The kernel (`titan_moe_w4a16_gemm`, csrc/titan_moe_gemm.cu) runs on the
5th-generation tensor cores: tcgen05.mma with the accumulator in tensor
memory, activation rows gathered by TMA (tile::gather4), weights
dequantised into tensor memory as the MMA's A operand.  Weights use this
build's own packing (`pack_weights`), not Marlin's tile permutation; the
scales keep the [E, K / 128, N] layout.
"""
import ctypes

import torch

try:
    from . import titan_native as _native
except ImportError:
    import titan_native as _native

GROUP = 128
TILE_N = 128
STEP_K = 128
_NIBBLE_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)


def pack_weights(q: torch.Tensor) -> torch.Tensor:
    """uint4b8 codes q (uint8 [E, N, K], values 0..15) -> the kernel's packed
    layout, uint8 [E * N * K / 2].  Per expert, the 128-feature tiles go in
    pairs (a last odd tile alone); per pair and 128-wide k step (one scale
    group), the pair's tiles back to back, 8 KB each as
    [quarter c][128 rows][16 B] (quarter c: the row's k 32c .. 32c + 31).  A
    32-bit word holds eight consecutive k, its nibble positions 0..7 holding
    k offsets 0, 2, 4, 6, 1, 3, 5, 7, so that positions (i, i + 4) are the
    consecutive pair (2i, 2i + 1)."""
    if q.dtype != torch.uint8 or q.dim() != 3:
        raise ValueError("pack_weights: q must be uint8 [E, N, K]")
    E, N, K = q.shape
    if N % TILE_N or K % GROUP:
        raise ValueError("pack_weights: N must be a multiple of 128 and K of 128")
    ntn, nk = N // TILE_N, K // STEP_K
    x = q.reshape(E, ntn, TILE_N, nk, 4, 4, 8)[..., list(_NIBBLE_ORDER)]  # [E, tile, r, kc, c, w, 8]
    b = (x[..., 0::2] & 15) | ((x[..., 1::2] & 15) << 4)                 # [E, tile, r, kc, c, w, 4]
    blocks = b.permute(0, 1, 3, 4, 2, 5, 6).reshape(E, ntn, nk, 8192)
    parts = []
    if ntn >= 2:
        full = blocks[:, :ntn // 2 * 2].reshape(E, ntn // 2, 2, nk, 8192).permute(0, 1, 3, 2, 4)
        parts.append(full.reshape(E, -1))
    if ntn % 2:
        parts.append(blocks[:, ntn - 1].reshape(E, -1))
    return torch.cat(parts, dim=1).contiguous().view(-1)


def moe_w4a16_gemm(a: torch.Tensor, c: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor,
                   sorted_ids: torch.Tensor, expert_ids: torch.Tensor, ntpp: torch.Tensor,
                   topk_weights: torch.Tensor | None, moe_block_size: int, top_k: int,
                   mul_topk_weights: bool, size_m: int, size_n: int, size_k: int) -> torch.Tensor:
    """One list GEMM (argument meaning of vLLM's moe_wna16_marlin_gemm as the
    reference calls it): writes the listed rows of c [size_m * top_k, size_n]
    bf16 and returns c.  a: bf16 [size_m, size_k] (row stride a multiple of 8
    elements); packed: pack_weights(q); scales: bf16 [E, size_k / 128, size_n];
    sorted_ids / expert_ids / ntpp: one list of split_align (int32, CUDA)."""
    if a.dtype != torch.bfloat16 or c.dtype != torch.bfloat16 or scales.dtype != torch.bfloat16:
        raise ValueError("moe_w4a16_gemm: a, c and scales must be bf16")
    if a.dim() != 2 or a.shape[1] != size_k or a.stride(1) != 1 or a.shape[0] < size_m:
        raise ValueError("moe_w4a16_gemm: a must be [size_m, size_k] with a contiguous last dim")
    if c.dim() != 2 or c.shape[0] < size_m * top_k or c.shape[1] != size_n or c.stride(1) != 1:
        raise ValueError("moe_w4a16_gemm: c must be [size_m * top_k, size_n] with a contiguous last dim")
    E = scales.shape[0]
    if scales.shape != (E, size_k // GROUP, size_n) or not scales.is_contiguous():
        raise ValueError("moe_w4a16_gemm: scales must be contiguous [E, size_k / 128, size_n]")
    if packed.dtype != torch.uint8 or packed.numel() != E * size_n * size_k // 2 or not packed.is_contiguous():
        raise ValueError("moe_w4a16_gemm: packed must come from pack_weights for [E, size_n, size_k]")
    for t in (sorted_ids, expert_ids, ntpp):
        if t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("moe_w4a16_gemm: sorted_ids, expert_ids and ntpp must be contiguous int32 CUDA tensors")
    if mul_topk_weights and (topk_weights is None or topk_weights.dtype != torch.float32
                             or not topk_weights.is_contiguous()):
        raise ValueError("moe_w4a16_gemm: mul_topk_weights needs contiguous float32 topk_weights")
    dev = a.device
    if any(t.device != dev for t in (c, packed, scales, sorted_ids, expert_ids, ntpp)):
        raise ValueError("moe_w4a16_gemm: all tensors must be on one CUDA device")
    lib = _native.load()
    with _native.on_device(dev):
        rc = lib.titan_moe_w4a16_gemm(
            a.data_ptr(), a.stride(0), size_m, c.data_ptr(), c.stride(0), packed.data_ptr(), scales.data_ptr(),
            sorted_ids.data_ptr(), expert_ids.data_ptr(),
            min(expert_ids.numel(), sorted_ids.numel() // int(moe_block_size)), ntpp.data_ptr(),
            topk_weights.data_ptr() if mul_topk_weights else None, int(moe_block_size), int(top_k),
            1 if mul_topk_weights else 0, E, size_n, size_k, _native.stream_of(a))
    _native.check(rc, "moe_w4a16_gemm")
    return c
