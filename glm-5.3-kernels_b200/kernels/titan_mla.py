# SPDX-License-Identifier: Apache-2.0
"""Sparse NoPE MLA over a per-token INT8 KV cache, for B200 (sm_100a).

Drop-in for the reference `triton_mla_sparse_attention`
(kernels/titan_mla.py:452-581) with the same argument order, defaults,
assertions and split heuristic (`_choose_num_kv_splits`, :432-449).  The
compute runs in libtitan_b200.so (csrc/titan_mla.cu): a bulk-copy (TMA) row
gather into shared memory, bf16 tensor-core MMAs with fp32 online softmax, and
a combine kernel for split-KV launches.

528 bytes/token: 512 signed INT8 values followed by 1 FP32 scale + 12 zero bytes.
"""

import functools

import torch

try:
    from . import titan_native as _native
except ImportError:
    import titan_native as _native

LOG2E = 1.4426950408889634
LOGE2 = 0.6931471805599453

# GLM-5.3 sparse MLA shape constants (kernels/titan_mla.py:23-29).
_BLOCK_DMODEL = 512
_BLOCK_DPE = 64
_BLOCK_DV = 512
_DIM_QK = _BLOCK_DMODEL + _BLOCK_DPE  # 576
_BLOCK_H = 16
_ROW_BYTES = 528

# Smallest top-k granule the API accepts (the reference's smallest BLOCK_N,
# kernels/titan_mla.py:45-49); kept so the same inputs are accepted/rejected.
_MIN_BLOCK_N = 32

# Split-count candidates and heuristic constants (kernels/titan_mla.py:53-56).
KV_SPLITS_CANDIDATES = (1, 2, 4, 8, 16)
_MIN_TOPK_PER_SPLIT = 128
_SPLIT_MAX_OCCUPANCY = 4


@functools.lru_cache(maxsize=64)
def num_compute_units(device_index):
    return torch.cuda.get_device_properties(device_index).multi_processor_count


def _cdiv(a, b):
    return -(-a // b)


def _next_power_of_2(n):
    return 1 if n <= 1 else 1 << (int(n) - 1).bit_length()


@functools.lru_cache(maxsize=256)
def _choose_num_kv_splits(num_tokens: int, num_head_groups: int, index_topk: int, sm_count: int) -> int:
    """Pick a power-of-2 split count that fills the device without dropping
    per-split work below _MIN_TOPK_PER_SPLIT; 1 when the single-pass grid
    already reaches ~1/_SPLIT_MAX_OCCUPANCY of the SMs.  Same policy and
    results as kernels/titan_mla.py:432-449.
    """
    baseline = num_tokens * num_head_groups
    if baseline == 0 or baseline * _SPLIT_MAX_OCCUPANCY >= sm_count:
        return 1
    ideal = _next_power_of_2(max(1, index_topk // _MIN_TOPK_PER_SPLIT))
    max_splits = max(1, sm_count // baseline)
    max_splits = 1 << (max_splits.bit_length() - 1)  # floor to a power of 2
    num_kv_splits = min(ideal, max_splits)
    while num_kv_splits > 1 and index_topk % num_kv_splits != 0:
        num_kv_splits //= 2
    return max(1, num_kv_splits)


# Cost model of the B200 kernel, fitted to back-to-back B=1 / B=4 / B=8
# sweeps on B200 (microseconds): one 32-row tile per CTA, the cluster merge,
# and the combine launch (plus a per-partial term) when a token has more than
# one cluster.  Decode grids are kept to one CTA per SM: two co-resident CTAs
# slow each other's tiles more than the extra parallelism returns.
_TILE_ROWS = 32
_COST_TILE_US = 1.25
_COST_CLUSTER_MERGE_US = 1.2
_COST_COMBINE_US = 1.4
_COST_COMBINE_PER_PARTIAL_US = 0.05
_MAX_CLUSTER = 16
_max_clusters_cache = {}


def _max_active_clusters(device_index):
    """{cluster size: co-resident clusters} of the MLA kernel on this device."""
    if device_index not in _max_clusters_cache:
        lib = _native.load()
        with torch.cuda.device(device_index):
            table = {c: lib.titan_mla_max_active_clusters(c) for c in (1, 2, 4, 8, 16)}
        _max_clusters_cache[device_index] = table
    return _max_clusters_cache[device_index]


def _choose_kv_splits_b200(num_tokens, num_head_groups, index_topk, sm_count, max_clusters):
    return _choose_kv_splits_b200_cached(num_tokens, num_head_groups, index_topk, sm_count,
                                         tuple(sorted(max_clusters.items())))


@functools.lru_cache(maxsize=1024)
def _choose_kv_splits_b200_cached(num_tokens, num_head_groups, index_topk, sm_count, max_clusters_items):
    """Auto split count for the B200 kernel.

    Candidates are split counts S whose whole grid (tokens x groups x S CTAs)
    fits one CTA per SM and whose clusters (C = largest power of two <= 16 dividing S
    that the device can co-schedule in one wave) fit at once; the cheapest
    under the cost model above wins (ties: fewer splits).  The reference's
    `_choose_num_kv_splits` targets its own SM80 kernel and stays available.
    """
    max_clusters = dict(max_clusters_items)
    units = num_tokens * num_head_groups
    if units == 0 or units >= sm_count:
        return 1
    best, best_cost = 1, None
    for S in range(1, sm_count // units + 1):
        C = 1  # same rule as the launcher: largest power of two dividing S whose clusters all fit
        cs = 2
        while cs <= _MAX_CLUSTER and S % cs == 0:
            if units * (S // cs) <= max(0, max_clusters.get(cs, 0)):
                C = cs
            cs *= 2
        nc = S // C
        rows = -(-index_topk // S)
        cost = max(1, -(-rows // _TILE_ROWS)) * _COST_TILE_US
        cost += _COST_CLUSTER_MERGE_US if C > 1 else 0.0
        cost += (_COST_COMBINE_US + _COST_COMBINE_PER_PARTIAL_US * nc) if nc > 1 else 0.0
        if best_cost is None or cost < best_cost - 1e-9:
            best, best_cost = S, cost
    return best


def _aligned16(t):
    return t.data_ptr() % 16 == 0 and all((s * t.element_size()) % 16 == 0 for s in t.stride()[:-1])


def triton_mla_sparse_attention(
    q: torch.Tensor,
    kv: torch.Tensor,
    indices: torch.Tensor,
    sm_scale: float,
    num_kv_splits: int | None = None,
    sm_count: int | None = None,
) -> torch.Tensor:
    """Sparse MLA attention over top-k indices.

    Args:
        q:         [num_tokens, num_heads_q, 512] bf16
        kv:        [seq_kv, 1, 528] int8 packed cache (528-byte rows)
        indices:   [num_tokens, 1, topk] int32; entries outside [0, seq_kv) are masked
        sm_scale:  softmax scale
        num_kv_splits: override the auto-heuristic; None/0 = auto (the B200 policy,
                   `_choose_kv_splits_b200`), 1 = single pass.
        sm_count:  cached device SM count for the split heuristic.

    Returns:
        out:   [num_tokens, num_heads_q, 512] bf16 (a new tensor)
    """
    num_tokens, num_heads_q, dim_qk = q.shape
    # Shape contract of kernels/titan_mla.py:478-488.
    assert dim_qk in (_BLOCK_DMODEL, _DIM_QK), (
        f"sparse MLA kernel requires dim_qk={_BLOCK_DMODEL} (NoPE) or "
        f"{_DIM_QK} (RoPE), got {dim_qk}"
    )
    block_dpe = dim_qk - _BLOCK_DMODEL
    assert kv.shape[1] == 1 and kv.shape[2] == (_ROW_BYTES if kv.dtype == torch.int8 else dim_qk)
    index_topk = indices.shape[2]
    assert index_topk % _MIN_BLOCK_N == 0, (
        f"topk ({index_topk}) must be a multiple of the smallest autotune "
        f"BLOCK_N ({_MIN_BLOCK_N})"
    )
    # This build carries the INT8 NoPE path (GLM-5.3, qk_rope_head_dim = 0).
    assert block_dpe == 0 and kv.dtype == torch.int8, (
        "the B200 kernel implements the INT8 NoPE path: dim_qk=512 with a [seq_kv, 1, 528] int8 cache")
    assert q.dtype == torch.bfloat16, "q must be bf16"
    assert q.is_cuda and kv.is_cuda and indices.is_cuda, "sparse MLA runs on CUDA tensors only"
    assert q.device == kv.device == indices.device, "q, kv and indices must share a device"

    kv_group_num = num_heads_q
    num_head_groups = _cdiv(num_heads_q, min(_BLOCK_H, kv_group_num))

    if num_kv_splits is None or num_kv_splits == 0:
        if sm_count is None:
            sm_count = num_compute_units(q.device.index)
        num_kv_splits = _choose_kv_splits_b200(num_tokens, num_head_groups, index_topk, sm_count,
                                               _max_active_clusters(q.device.index))

    out = torch.empty((num_tokens, num_heads_q, _BLOCK_DV), dtype=torch.bfloat16, device=q.device)
    if num_tokens == 0:
        return out

    seq_kv = kv.shape[0]
    if q.stride(-1) != 1 or not _aligned16(q):
        q = q.contiguous()
    idx = indices[:, 0, :]
    if idx.dtype != torch.int32:
        # Out-of-range wide indices must stay masked after narrowing.
        idx = torch.where((idx >= 0) & (idx < seq_kv), idx, -1).to(torch.int32)
    if idx.stride(-1) != 1:
        idx = idx.contiguous()
    kv_row_stride = kv.stride(0)  # bytes (int8)

    lib = _native.load()
    ws_bytes = lib.titan_mla_workspace_bytes(num_tokens, num_heads_q, num_kv_splits)
    # Split partials live in a caching-allocator buffer, like the reference's
    # `mid_out` (kernels/titan_mla.py:533-537): graph-capture safe, no sync.
    workspace = torch.empty(max(ws_bytes, 0), dtype=torch.uint8, device=q.device) if ws_bytes > 0 else None
    with _native.on_device(q.device):
        rc = lib.titan_mla_sparse_attention(
            q.data_ptr(), q.stride(0), q.stride(1),
            kv.data_ptr(), kv_row_stride, seq_kv,
            idx.data_ptr(), idx.stride(0), index_topk,
            out.data_ptr(), out.stride(0), out.stride(1),
            num_tokens, num_heads_q, float(sm_scale), int(num_kv_splits),
            workspace.data_ptr() if workspace is not None else None, ws_bytes,
            _native.stream_of(q))
    _native.check(rc, "triton_mla_sparse_attention")
    return out
