# SPDX-License-Identifier: Apache-2.0
"""Single-CTA deterministic MoE alignment for Titan decode B=1..8 on B200.

Drop-in for the reference `titan_moe_align_small`
(kernels/titan_moe_align.py:49-81): 288 experts, top-k 8, block M 8, no
expert-parallel map; invalid routes are ignored.  The kernel is
`titan_moe_align_small` in libtitan_b200.so (csrc/titan_moe_align.cu): one warp
does the layout with match-any / popcount ranks and a warp prefix scan.
"""
import torch

try:
    from . import titan_native as _native
except ImportError:
    import titan_native as _native


def titan_moe_align_small(
    topk_ids,
    block_size=8,
    num_experts=288,
    expert_map=None,
    pad_sorted_ids=False,
    ignore_invalid_experts=True,
    *,
    num_warps=None,
):
    """Return exactly the stable baseline's three tensors, including padding.

    (sorted_ids int32 [8R], expert_ids int32 [R], postpad int32 [1]) for the
    R = 8B routes of topk_ids [B, 8].  num_warps and pad_sorted_ids do not
    change the outputs.  Raises ValueError like kernels/titan_moe_align.py:60-77.
    """
    if (topk_ids.ndim != 2 or not 1 <= topk_ids.shape[0] <= 8
            or topk_ids.shape[1] != 8 or block_size != 8 or num_experts != 288
            or expert_map is not None or not ignore_invalid_experts):
        raise ValueError('Titan small alignment requires B1..8/top8/E288/block8/EPoff/ignore-invalid')
    if not topk_ids.is_cuda or not topk_ids.is_contiguous():
        raise ValueError('Titan small alignment requires contiguous CUDA route IDs')
    if topk_ids.dtype not in (torch.int32, torch.int64):
        raise ValueError('Route IDs must be int32 or int64')
    routes = topk_ids.numel()
    # R < 288 routes: the padded storage is capped at R * block_size, already a
    # multiple of eight, so pad_sorted_ids cannot change the layout.
    sorted_ids = torch.empty(routes * 8, dtype=torch.int32, device=topk_ids.device)
    expert_ids = torch.empty(routes, dtype=torch.int32, device=topk_ids.device)
    postpad = torch.empty(1, dtype=torch.int32, device=topk_ids.device)
    if num_warps is None:
        num_warps = 1 if routes <= 16 else 4
    if num_warps not in (1, 2, 4):
        raise ValueError('Candidate warp counts are 1, 2, or 4')
    lib = _native.entry()
    with _native.on_device(topk_ids.device):
        rc = lib.moe_align(
            topk_ids.data_ptr(), 1 if topk_ids.dtype == torch.int64 else 0, routes,
            sorted_ids.data_ptr(), expert_ids.data_ptr(), postpad.data_ptr(), num_warps,
            _native.stream_of(topk_ids))
    _native.check(rc, "titan_moe_align_small")
    return sorted_ids, expert_ids, postpad
