# SPDX-License-Identifier: Apache-2.0
"""Pool top-k of the sparse indexer and its expansion to token positions, for
B200 (sm_100a): the step that writes the MLA reader's 2176 indices per query.

The reference's indexer scores pools of `pool_size` tokens, takes the
top-`topk` pools per query with a CUDA top-k, and expands them to token
positions with the fork's `expand_pools_and_append_tail`
(integration/patch_decode_indexer.py:49-104,
integration/patch_indexer_sharding.py:58-104); the expansion is defined by the
reference test's own model `expand_row` (tests/verify_indexer_sharding.py:
68-76) and lands in an index buffer 2176 columns wide (:239-241).  Here one
kernel (`titan_pool_topk_expand`, csrc/titan_indexer.cu) does both:

    valid pools p < seq_len // pool_size (complete pools);
    pools = the `topk` valid pools of largest logit, by logit descending
            (equal logits: smaller pool first), -1 where fewer are valid;
    out[t] = [p * pool_size + o for p in pools for o in range(pool_size)]
             (-1 for a -1 pool) + the tail of the partial last pool
             (pool_size - 1 entries) + -1 up to `width`.
"""
import torch

try:
    from . import titan_native as _native
except ImportError:
    import titan_native as _native

TOPK = 512
POOL = 4
WIDTH = 2176


def pool_topk_expand(logits: torch.Tensor, seq_lens: torch.Tensor, topk: int = TOPK, pool_size: int = POOL,
                     width: int = WIDTH, out: torch.Tensor | None = None) -> torch.Tensor:
    """logits: float32 [T, P] pool scores (row stride any, last dim contiguous);
    seq_lens: int32 [T] tokens of each query's context (position + 1).
    Returns (or fills) int32 [T, width] token indices."""
    if logits.dtype != torch.float32 or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("pool_topk_expand: logits must be float32 [T, P] with a contiguous last dim")
    T = logits.shape[0]
    if seq_lens.dtype != torch.int32 or seq_lens.numel() < T or not seq_lens.is_contiguous():
        raise ValueError("pool_topk_expand: seq_lens must be contiguous int32 [T]")
    if not logits.is_cuda or seq_lens.device != logits.device:
        raise ValueError("pool_topk_expand: logits and seq_lens must be CUDA tensors on one device")
    if width < topk * pool_size + pool_size - 1:
        raise ValueError("pool_topk_expand: width below topk * pool_size + pool_size - 1")
    if out is None:
        out = torch.empty(T, width, dtype=torch.int32, device=logits.device)
    elif out.dtype != torch.int32 or out.shape != (T, width) or out.stride(1) != 1 or out.device != logits.device:
        raise ValueError("pool_topk_expand: out must be int32 [T, width] on the logits' device")
    lib = _native.load()
    with _native.on_device(logits.device):
        rc = lib.titan_pool_topk_expand(logits.data_ptr(), logits.stride(0), seq_lens.data_ptr(), T, int(topk),
                                        int(pool_size), out.data_ptr(), out.stride(0), int(width),
                                        _native.stream_of(logits))
    _native.check(rc, "pool_topk_expand")
    return out
