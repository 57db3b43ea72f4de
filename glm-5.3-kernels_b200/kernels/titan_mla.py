# SPDX-License-Identifier: Apache-2.0
"""Sparse NoPE MLA over a per-token INT8 KV cache, for B200 (sm_100a).

Drop-in for the reference `triton_mla_sparse_attention`
(kernels/titan_mla.py:452-581) with the same argument order, defaults and
assertions; the automatic split count is this kernel's own policy
(`_choose_kv_splits_b200`), an explicit `num_kv_splits` is honoured.  The
compute runs in libtitan_b200.so (csrc/titan_mla.cu): rows gathered by the
tensor memory accelerator (`tile::gather4`, four rows per load) into a
shared-memory ring laid out as the lanes' tensor-core fragments, bf16 MMAs
with fp32 online softmax, and split
partials merged in the same launch: by the split CTAs of a token after a
counter barrier (flat merge, decode batches up to 16), or inside
thread-block clusters and, across clusters, by the last CTA to finish
(arrival counters).

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


@functools.lru_cache(maxsize=64)
def num_compute_units(device_index):
    return torch.cuda.get_device_properties(device_index).multi_processor_count


def _cdiv(a, b):
    return -(-a // b)


# Cost model of the B200 kernel (microseconds): 32-row tiles per CTA, the
# merge inside a thread-block cluster (cheaper for larger clusters: each CTA
# reduces 512 / C dims), the merge across clusters (done by the last CTA to
# finish when NC <= C, else by the combine kernel; both plus a per-partial
# term), and a penalty when more clusters are launched than fit with one CTA
# per SM (they then share SMs and slow each other's gathers).  Fitted to a
# B200 sweep of every split count with at most one CTA per SM for B = 1..8
# (calls back to back in CUDA graphs, cold L2, the current reader): the
# median of the parameter sets whose picks match the best measured split
# count at every batch size.  Split counts whose partials would otherwise
# need the combine kernel (8 <= S <= 160, grid resident at once) are merged
# by the split CTAs themselves without clusters (flat merge: a counter
# barrier per token, then each CTA merges a share of the columns); its terms
# reproduce the measured best split count of every batch size 1..8 (68, 68,
# 34, 34, 23, 23, 17, 17).
_TILE_ROWS = 32
_COST_TILE_US = 0.5
_COST_CLUSTER_MERGE_US = {2: 1.0, 4: 1.0, 8: 0.8, 16: 0.6}
_COST_SPLIT_MERGE_US = 0.8
_COST_SPLIT_MERGE_PER_PARTIAL_US = 0.05
_COST_COMBINE_US = 1.0
_COST_COMBINE_PER_PARTIAL_US = 0.05
_COST_SHARED_SM_US = 1.5
_COST_FLAT_MERGE_US = 0.8
_COST_FLAT_MERGE_PER_PARTIAL_US = 0.005
_FLAT_MIN_SPLITS, _FLAT_MAX_SPLITS = 8, 160
_MAX_CLUSTER = 16
_CLUSTER_SIZES = (1, 2, 4, 8, 16)
_cluster_tables_cache = {}


def _cluster_tables(device_index):
    """((C, co-resident clusters, clusters with an SM per CTA), ...) for C in
    1, 2, 4, 8, 16: the MLA kernel's cluster capacity on this device."""
    tables = _cluster_tables_cache.get(device_index)
    if tables is None:
        lib = _native.load()
        with torch.cuda.device(device_index):
            tables = tuple((c, lib.titan_mla_max_active_clusters(c), lib.titan_mla_max_exclusive_clusters(c))
                           for c in _CLUSTER_SIZES)
        _cluster_tables_cache[device_index] = tables
    return tables


def _launch_layout(units, S, tables):
    """(C, NC, flat) as the launcher picks them when given arrival counters:
    C = the largest power of two <= 16 dividing S whose units * S / C
    clusters are all co-resident; when the NC = S / C cluster partials would
    need the combine kernel (NC > C) and the flat merge applies (16 <= S <=
    160, all units * S CTAs co-resident), C = 1, NC = S, flat."""
    C = 1
    for c, capacity, _ in tables:
        if c == 1:
            continue
        if S % c:
            break
        if units * (S // c) <= max(0, capacity):
            C = c
    nc = S // C
    resident = dict((c, cap) for c, cap, _ in tables).get(1, 0)
    if (nc > 1 and not (C >= 2 and nc <= C) and _FLAT_MIN_SPLITS <= S <= _FLAT_MAX_SPLITS
            and units * S <= resident):
        return 1, S, True
    return C, nc, False


@functools.lru_cache(maxsize=1024)
def _choose_kv_splits_b200(num_tokens, num_head_groups, index_topk, sm_count, tables):
    """Auto split count for the B200 kernel.

    Candidates keep the whole grid (tokens x groups x S CTAs) within one CTA
    per SM; the cheapest under the cost model above wins (ties: fewer
    splits).  The reference's heuristic (`_choose_num_kv_splits`,
    kernels/titan_mla.py:432-449) targets its SM80 kernel; any split count it
    would pick can still be passed explicitly as num_kv_splits.
    """
    units = num_tokens * num_head_groups
    if units == 0 or units >= sm_count:
        return 1
    exclusive = {c: e for c, _, e in tables}
    best, best_cost = 1, None
    for S in range(1, sm_count // units + 1):
        C, nc, flat = _launch_layout(units, S, tables)
        rows = -(-index_topk // S)
        cost = max(1, -(-rows // _TILE_ROWS)) * _COST_TILE_US
        cost += _COST_CLUSTER_MERGE_US[C] if C > 1 else 0.0
        if flat:
            cost += _COST_FLAT_MERGE_US + _COST_FLAT_MERGE_PER_PARTIAL_US * S
        elif nc > 1:
            if C >= 2 and nc <= C:
                cost += _COST_SPLIT_MERGE_US + _COST_SPLIT_MERGE_PER_PARTIAL_US * nc
            else:
                cost += _COST_COMBINE_US + _COST_COMBINE_PER_PARTIAL_US * nc
        if units * nc > max(0, exclusive.get(C, 0)):
            cost += _COST_SHARED_SM_US
        if best_cost is None or cost < best_cost - 1e-9:
            best, best_cost = S, cost
    return best


# Per-(device, stream) scratch of split launches: int32 arrival counters (zero
# between calls: every call leaves them at zero) and the fp32 partials
# workspace.  Calls on one stream are ordered, so they can share it; other
# streams get their own.  Buffers are kept for the life of the process, since
# a CUDA graph captured on a stream keeps using that stream's buffers: such a
# graph must not be replayed concurrently with other calls issued on the
# stream it was captured on.  Workspaces above _MAX_CACHED_WORKSPACE are taken
# from the caching allocator per call, like the reference's `mid_out`
# (kernels/titan_mla.py:533-537).
_MAX_CACHED_WORKSPACE = 8 << 20
_scratch = {}
_retired = []
_plans = {}


def _split_scratch(q, dev, stream, ws_bytes, sem_count):
    entry = _scratch.get((dev, stream))
    if entry is not None and entry[0].numel() >= sem_count and entry[1].numel() >= ws_bytes:
        return entry
    if ws_bytes > _MAX_CACHED_WORKSPACE or torch.cuda.is_current_stream_capturing():
        # Not cached: a graph being captured zeroes its own counters on
        # every replay and keeps both buffers in its private pool.
        sem = torch.zeros(sem_count, dtype=torch.int32, device=q.device)
        if entry is not None and entry[0].numel() >= sem_count:
            sem = entry[0]
        return sem, torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    if entry is not None:
        _retired.append(entry)
        sem_count = max(sem_count, entry[0].numel())
        ws_bytes = max(ws_bytes, entry[1].numel())
    entry = (torch.zeros(max(sem_count, 4096), dtype=torch.int32, device=q.device),
             torch.empty(max(ws_bytes, 1 << 20), dtype=torch.uint8, device=q.device))
    _scratch[(dev, stream)] = entry
    return entry


def _plan(dev, num_tokens, num_heads_q, index_topk, num_kv_splits, sm_count):
    """(splits, workspace bytes, counter count) of one call shape, cached."""
    key = (dev, num_tokens, num_heads_q, index_topk, num_kv_splits, sm_count)
    plan = _plans.get(key)
    if plan is None:
        S = num_kv_splits
        if S is None or S == 0:
            groups = _cdiv(num_heads_q, min(_BLOCK_H, num_heads_q))
            S = _choose_kv_splits_b200(num_tokens, groups, index_topk,
                                       num_compute_units(dev) if sm_count is None else sm_count,
                                       _cluster_tables(dev))
        lib = _native.load()
        ws_bytes = lib.titan_mla_workspace_bytes(num_tokens, num_heads_q, S) if num_tokens > 0 else 0
        sem_count = lib.titan_mla_semaphore_count(num_tokens, num_heads_q) if ws_bytes > 0 else 0
        plan = (int(S), ws_bytes, sem_count)
        if len(_plans) < 4096:
            _plans[key] = plan
    return plan


def _destination(out, dev, shape):
    """Device-accessible address of a caller-provided output: a CUDA tensor on
    `dev`, or pinned host memory through its device mapping."""
    assert tuple(out.shape) == shape and out.dtype == torch.bfloat16, \
        f"out must be bf16 {list(shape)}, got {out.dtype} {list(out.shape)}"
    st = out.stride()
    assert st[2] == 1 and out.data_ptr() % 16 == 0 and (st[0] * 2) % 16 == 0 and (st[1] * 2) % 16 == 0, \
        "out needs a contiguous last dim and 16-byte aligned rows"
    if out.is_cuda:
        assert out.get_device() == dev, "out must be on q's device"
        return out.data_ptr()
    assert out.is_pinned(), "a host `out` must be pinned memory (tensor.pin_memory())"
    rc, ptr = _native.entry().device_pointer(out.data_ptr())
    _native.check(rc, "triton_mla_sparse_attention(out=)")
    return ptr


def triton_mla_sparse_attention(
    q: torch.Tensor,
    kv: torch.Tensor,
    indices: torch.Tensor,
    sm_scale: float,
    num_kv_splits: int | None = None,
    sm_count: int | None = None,
    *,
    out: torch.Tensor | None = None,
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
        out:       optional (keyword only; not in the reference signature)
                   [num_tokens, num_heads_q, 512] bf16 destination: a CUDA
                   tensor on q's device or a PINNED host tensor, which the
                   kernel writes through its device mapping (no separate
                   device -> host copy).  Last dim contiguous, 16-byte aligned
                   rows.

    Returns:
        out:   [num_tokens, num_heads_q, 512] bf16 (a new tensor unless `out` is given)
    """
    num_tokens, num_heads_q, dim_qk = q.shape
    # Shape contract of kernels/titan_mla.py:478-488.
    assert dim_qk in (_BLOCK_DMODEL, _DIM_QK), (
        f"sparse MLA kernel requires dim_qk={_BLOCK_DMODEL} (NoPE) or "
        f"{_DIM_QK} (RoPE), got {dim_qk}"
    )
    kv_dtype = kv.dtype
    kv_shape = kv.shape
    assert kv_shape[1] == 1 and kv_shape[2] == (_ROW_BYTES if kv_dtype == torch.int8 else dim_qk)
    index_topk = indices.shape[2]
    assert index_topk % _MIN_BLOCK_N == 0, (
        f"topk ({index_topk}) must be a multiple of the smallest autotune "
        f"BLOCK_N ({_MIN_BLOCK_N})"
    )
    # This build carries the INT8 NoPE path (GLM-5.3, qk_rope_head_dim = 0).
    assert dim_qk == _BLOCK_DMODEL and kv_dtype == torch.int8, (
        "the B200 kernel implements the INT8 NoPE path: dim_qk=512 with a [seq_kv, 1, 528] int8 cache")
    assert q.dtype == torch.bfloat16, "q must be bf16"
    dev = q.get_device()
    assert dev >= 0 and kv.get_device() >= 0 and indices.get_device() >= 0, \
        "sparse MLA runs on CUDA tensors only"
    assert kv.get_device() == dev and indices.get_device() == dev, "q, kv and indices must share a device"

    num_kv_splits, ws_bytes, sem_count = _plan(dev, num_tokens, num_heads_q, index_topk, num_kv_splits,
                                               sm_count)
    if out is None:
        out = q.new_empty((num_tokens, num_heads_q, _BLOCK_DV))
        out_ptr = out.data_ptr()
    else:
        out_ptr = _destination(out, dev, (num_tokens, num_heads_q, _BLOCK_DV))
    if num_tokens == 0:
        return out

    seq_kv = kv_shape[0]
    q_st = q.stride()
    if q_st[2] != 1 or q.data_ptr() % 16 or (q_st[0] * 2) % 16 or (q_st[1] * 2) % 16:
        q = q.contiguous()
        q_st = q.stride()
    idx = indices
    if idx.dtype != torch.int32:
        # Out-of-range wide indices must stay masked after narrowing.
        idx = torch.where((idx >= 0) & (idx < seq_kv), idx, -1).to(torch.int32)
    idx_st = idx.stride()
    if idx_st[2] != 1:
        idx = idx.contiguous()
        idx_st = idx.stride()
    out_st = out.stride()

    lib = _native.entry()
    stream = torch._C._cuda_getCurrentRawStream(dev)
    prev = torch.cuda.current_device()
    if prev != dev:
        torch.cuda.set_device(dev)
    try:
        # indices[:, 0, :] is row t at idx + t * stride(0): no view is needed.
        args = (q.data_ptr(), q_st[0], q_st[1], kv.data_ptr(), kv.stride(0), seq_kv,
                idx.data_ptr(), idx_st[0], index_topk, out_ptr, out_st[0], out_st[1],
                num_tokens, num_heads_q, float(sm_scale), num_kv_splits)
        if ws_bytes > 0:
            # Split launch: partials of a token's clusters are merged by the
            # last CTA to finish (arrival counters), or by a combine kernel.
            sem, ws = _split_scratch(q, dev, stream, ws_bytes, sem_count)
            rc = lib.mla_sem(*args, ws.data_ptr(), ws.numel(), sem.data_ptr(), sem.numel(), stream)
        else:
            rc = lib.mla(*args, None, 0, stream)
    finally:
        if prev != dev:
            torch.cuda.set_device(prev)
    if rc:
        _native.check(rc, "triton_mla_sparse_attention")
    return out


def triton_mla_sparse_attention_paged(
    q: torch.Tensor,
    kv: torch.Tensor,
    token_indices: torch.Tensor,
    req_id_per_token: torch.Tensor,
    block_table: torch.Tensor,
    block_size: int,
    sm_scale: float,
    block_stride_rows: int | None = None,
    num_kv_splits: int | None = None,
    sm_count: int | None = None,
) -> torch.Tensor:
    """Sparse MLA over request-local top-k positions of a paged INT8 cache.

    The reference's backend converts the indexer's request-local positions to
    cache rows and then calls the reader (integration/titan_backend.py:48-54).
    Here the gather does the conversion (one launch, no global-index round
    trip); the result is bit-identical to

        triton_mla_sparse_attention(q, kv, titan_index.triton_convert_req_index_to_global_index(
            req_id_per_token, block_table, token_indices, BLOCK_SIZE=block_size,
            NUM_TOPK_TOKENS=topk, BLOCK_STRIDE_ROWS=block_stride_rows).view(T, 1, -1), ...)

    Args:
        q:             [num_tokens, num_heads_q, 512] bf16
        kv:            [rows, 1, 528] int8: the paged cache viewed as rows
        token_indices: [num_tokens, topk] or [num_tokens, 1, topk] int32 request-local
                       positions (negative = none)
        req_id_per_token: [num_tokens] int32 request of each token
        block_table:   [num_requests, max_blocks] int32 cache block of each request block
        block_size:    positions per block
        block_stride_rows: cache rows from one block to the next (default block_size)
        num_kv_splits, sm_count: as triton_mla_sparse_attention
    """
    num_tokens, num_heads_q, dim_qk = q.shape
    assert dim_qk == _BLOCK_DMODEL and kv.dtype == torch.int8 and kv.shape[1] == 1 and kv.shape[2] == _ROW_BYTES, (
        "the B200 kernel implements the INT8 NoPE path: dim_qk=512 with a [rows, 1, 528] int8 cache")
    assert q.dtype == torch.bfloat16, "q must be bf16"
    ti = token_indices if token_indices.dim() == 2 else token_indices[:, 0, :]
    assert ti.dim() == 2 and ti.shape[0] == num_tokens and ti.dtype == torch.int32, \
        "token_indices must be int32 [num_tokens, topk]"
    index_topk = ti.shape[1]
    assert index_topk % _MIN_BLOCK_N == 0, (
        f"topk ({index_topk}) must be a multiple of the smallest autotune BLOCK_N ({_MIN_BLOCK_N})")
    assert req_id_per_token.dtype == torch.int32 and req_id_per_token.numel() >= num_tokens, \
        "req_id_per_token must be int32 [num_tokens]"
    assert block_table.dtype == torch.int32 and block_table.dim() == 2, "block_table must be int32 [requests, blocks]"
    assert block_size > 0, "block_size must be positive"
    if block_stride_rows is None:
        block_stride_rows = block_size
    dev = q.get_device()
    assert dev >= 0 and all(t.get_device() == dev for t in (kv, ti, req_id_per_token, block_table)), \
        "all tensors must be CUDA tensors on one device"

    num_kv_splits, ws_bytes, sem_count = _plan(dev, num_tokens, num_heads_q, index_topk, num_kv_splits, sm_count)
    out = q.new_empty((num_tokens, num_heads_q, _BLOCK_DV))
    if num_tokens == 0:
        return out
    q_st = q.stride()
    if q_st[2] != 1 or q.data_ptr() % 16 or (q_st[0] * 2) % 16 or (q_st[1] * 2) % 16:
        q = q.contiguous()
        q_st = q.stride()
    if ti.stride(1) != 1:
        ti = ti.contiguous()
    req = req_id_per_token if req_id_per_token.is_contiguous() else req_id_per_token.contiguous()
    bt_st = block_table.stride()
    out_st = out.stride()

    lib = _native.entry()
    stream = torch._C._cuda_getCurrentRawStream(dev)
    with _native.on_device(q.device):
        sem, ws = _split_scratch(q, dev, stream, ws_bytes, sem_count) if ws_bytes > 0 else (None, None)
        rc = lib.mla_paged(
            q.data_ptr(), q_st[0], q_st[1], kv.data_ptr(), kv.stride(0), kv.shape[0],
            ti.data_ptr(), ti.stride(0), index_topk,
            req.data_ptr(), block_table.shape[0], block_table.data_ptr(), bt_st[0], bt_st[1], block_table.shape[1],
            int(block_size), int(block_stride_rows),
            out.data_ptr(), out_st[0], out_st[1], num_tokens, num_heads_q, float(sm_scale), num_kv_splits,
            ws.data_ptr() if ws is not None else None, ws_bytes,
            sem.data_ptr() if sem is not None else None, sem.numel() if sem is not None else 0, stream)
    _native.check(rc, "triton_mla_sparse_attention_paged")
    return out
