# SPDX-License-Identifier: Apache-2.0
"""CPU oracle for the sparse-MLA decode path — TEST INFRASTRUCTURE ONLY.

Restates the reference algorithms on the CPU (numpy for the byte/integer work,
torch-CPU fp32 for attention) so the CUDA path can be checked against them.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module, and only as the checker or the timed CPU baseline: the product
(glm-5.3-kernels_b200/) never imports it.

Pinning: store_int8_rows and moe_align_small are checked bit-exactly against
golden vectors produced by the reference's own code (tests/golden/make_golden.py
runs kernels/titan_kv.py, kernels/titan_moe_align.py and the
benchmarks/moe_align.py oracles); mla_sparse_attention is checked against the
reference MLA kernels' outputs within the path's tolerance.
convert_req_index_to_global is checked bit-exactly against golden vectors
from vLLM's own conversion kernel (the third-party function the reference's
backend calls, run by the Triton interpreter).
"""
import numpy as np
import torch

LATENT_DIM = 512
ROW_BYTES = 528
NUM_EXPERTS = 288
NEG_LARGE = -1.0e30


# --------------------------------------------------------------------- INT8 KV
def bf16_bits_to_f32(bits):
    """uint16 bf16 bit patterns -> float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def tensor_bf16_bits(t):
    """torch bf16 tensor (any device) -> numpy uint16 bit patterns."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def store_int8_rows(x_bits):
    """Quantise bf16 latents [N, 512] (uint16 bit patterns) to 528-byte rows.

    Follows kernels/titan_kv.py:15-21 with IEEE fp32 arithmetic:
      scale = max(max|x| / 127, 1e-12); q = clamp(nearbyint(x / scale), -127, 127)
    Row bytes: [0,512) q as int8, [512,516) scale (fp32 LE), [516,528) zero.
    The reference's max, maximum and minimum (Triton's default
    PropagateNan.NONE: maxnum / minnum on the GPU) drop NaN operands: the row
    max ignores NaN values, an infinite value gives an infinite scale, and a
    NaN quotient (a NaN value, or +-inf / inf) clamps to -127.
    Returns uint8 [N, 528].
    """
    x = bf16_bits_to_f32(np.asarray(x_bits).reshape(-1, LATENT_DIM))
    with np.errstate(invalid="ignore", divide="ignore"):
        a = np.abs(x)
        amax = np.where(np.isnan(a), np.float32(0.0), a).max(axis=1)
        scale = np.fmax(amax / np.float32(127.0), np.float32(1.0e-12)).astype(np.float32)
        q = np.rint(x / scale[:, None])  # np.rint rounds half to even, like nearbyint
    q = np.fmin(np.fmax(q, np.float32(-127)), np.float32(127)).astype(np.int8)
    rows = np.zeros((x.shape[0], ROW_BYTES), dtype=np.uint8)
    rows[:, :LATENT_DIM] = q.view(np.uint8)
    rows[:, LATENT_DIM:LATENT_DIM + 4] = scale.view(np.uint8).reshape(-1, 4)
    return rows


def store_int8(x_bits, cache, slots):
    """In-place oracle of `store_int8(x, cache, slots)` (kernels/titan_kv.py:7-28).

    cache: numpy uint8/int8 [num_blocks, block_size, 528]; slots: integer array.
    Slot s >= 0 writes row s // block_size, s % block_size; s < 0 is skipped.
    """
    slots = np.asarray(slots).reshape(-1).astype(np.int64)
    x_bits = np.asarray(x_bits).reshape(-1, LATENT_DIM)[: slots.size]
    rows = store_int8_rows(x_bits)
    flat = cache.view(np.uint8).reshape(-1, ROW_BYTES)
    block = cache.shape[1]
    keep = slots >= 0
    dest = (slots[keep] // block) * block + slots[keep] % block
    flat[dest] = rows[keep]
    return cache


def dequantize_rows(rows):
    """528-byte rows (uint8/int8 [N, 528]) -> fp32 [N, 512] = int8 * scale."""
    rows = np.ascontiguousarray(np.asarray(rows).view(np.uint8).reshape(-1, ROW_BYTES))
    q = rows[:, :LATENT_DIM].view(np.int8).astype(np.float32)
    scale = rows[:, LATENT_DIM:LATENT_DIM + 4].copy().view(np.float32)
    return q * scale


# ----------------------------------------------------------------- sparse MLA
def choose_num_kv_splits(num_tokens, num_head_groups, index_topk, sm_count):
    """Restatement of kernels/titan_mla.py:432-449."""
    baseline = num_tokens * num_head_groups
    if baseline == 0 or baseline * 4 >= sm_count:
        return 1
    n = max(1, index_topk // 128)
    ideal = 1 if n <= 1 else 1 << (n - 1).bit_length()
    max_splits = max(1, sm_count // baseline)
    max_splits = 1 << (max_splits.bit_length() - 1)
    s = min(ideal, max_splits)
    while s > 1 and index_topk % s != 0:
        s //= 2
    return max(1, s)


def mla_sparse_attention(q, rows, indices, sm_scale, threads=None):
    """FP32 sparse attention over the dequantised cache.

    The exact-arithmetic statement of kernels/titan_mla.py:59-255 and :357-429:
    for each token t and head h, softmax over the valid top-k rows r
    (0 <= r < seq_kv) of (q[t,h] . k_r) * sm_scale, where k_r = int8_r * scale_r,
    then the softmax-weighted sum of the same k_r (NoPE: V = K).  A token with
    no valid row gives zeros (kernels/titan_mla.py:246, :421).  Duplicate
    indices count once per occurrence, as in the reference gather.

    q: [T, H, 512] (torch, any float dtype); rows: uint8/int8 [seq_kv, 528]
    (numpy or torch); indices: [T, topk] or [T, 1, topk] integer.  Returns
    torch.float32 [T, H, 512] on the CPU.
    """
    if threads is not None:
        torch.set_num_threads(threads)
    rows_t = torch.as_tensor(np.ascontiguousarray(np.asarray(
        rows.cpu().numpy() if isinstance(rows, torch.Tensor) else rows).view(np.uint8).reshape(-1, ROW_BYTES)))
    seq_kv = rows_t.shape[0]
    qf = q.detach().cpu().float()
    idx = torch.as_tensor(indices).cpu().reshape(qf.shape[0], -1).long()
    T, H, _ = qf.shape
    out = torch.zeros(T, H, LATENT_DIM, dtype=torch.float32)
    for t in range(T):
        valid = (idx[t] >= 0) & (idx[t] < seq_kv)
        r = idx[t][valid]
        if r.numel() == 0:
            continue
        sel = rows_t[r]
        k = sel[:, :LATENT_DIM].view(torch.int8).float() * sel[:, LATENT_DIM:LATENT_DIM + 4].contiguous().view(torch.float32)
        logits = (qf[t] @ k.T) * sm_scale
        out[t] = torch.softmax(logits, dim=-1) @ k
    return out


def mla_reference_test_metrics(out, q, original_bf16, indices, seq_kv, sm_scale, chunk=64):
    """The reference test's own numerical criteria (tests/verify_mla.py:79-90):
    FP32 softmax attention over the ORIGINAL bf16 latents; returns (nmse, cosine).
    Tokens are processed `chunk` at a time (the gathered latents of a
    4096-token prefill would not fit in host memory at once)."""
    qf = q.detach().cpu().float()
    idx = torch.as_tensor(indices).cpu().reshape(qf.shape[0], -1).long()
    lat = original_bf16.detach().cpu()
    o_all = out.detach().cpu().float()
    err = ref2 = dot = o2 = 0.0
    for t0 in range(0, qf.shape[0], chunk):
        ii = idx[t0:t0 + chunk]
        valid = (ii >= 0) & (ii < seq_kv)
        chosen = lat[ii.clamp(0, seq_kv - 1)].float()
        chosen.masked_fill_(~valid[:, :, None], 0)
        logits = torch.bmm(qf[t0:t0 + chunk], chosen.transpose(1, 2)) * sm_scale
        logits.masked_fill_(~valid[:, None, :], -float("inf"))
        ref = torch.bmm(torch.nan_to_num(logits.softmax(-1), nan=0.0), chosen).double()
        o = o_all[t0:t0 + chunk].double()
        err += (o - ref).square().sum().item()
        ref2 += ref.square().sum().item()
        dot += (o * ref).sum().item()
        o2 += o.square().sum().item()
    nmse = err / max(ref2, 1e-30)
    cos = dot / max((o2 ** 0.5) * (ref2 ** 0.5), 1e-30)
    return nmse, cos


def mla_algorithmic_bytes(indices, seq_kv, num_heads):
    """Bytes one call must move: valid gathered rows x 528 + the int32 indices
    + q and out (bf16), counted per token (duplicates count each time)."""
    idx = np.asarray(torch.as_tensor(indices).cpu()).reshape(np.shape(indices)[0], -1)
    n_valid = int(((idx >= 0) & (idx < seq_kv)).sum())
    T, topk = idx.shape
    return n_valid * ROW_BYTES + T * topk * 4 + 2 * T * num_heads * LATENT_DIM * 2


# --------------------------------------------------------------- MoE align
def moe_align_small(routes):
    """Stable expert-sorted layout of benchmarks/moe_align.py:23-31, vectorised.

    routes: flat integer sequence of R = 8B expert ids.  Returns
    (sorted_ids int32 [8R], expert_ids int32 [R], postpad int32 [1]).
    Padding entries of sorted_ids hold R; unused expert blocks hold -1;
    ids outside [0, 288) are ignored (kernels/titan_moe_align.py:17-46).
    """
    flat = np.asarray(routes, dtype=np.int64).reshape(-1)
    R = flat.size
    valid = (flat >= 0) & (flat < NUM_EXPERTS)
    e = np.where(valid, flat, NUM_EXPERTS)
    counts = np.bincount(e, minlength=NUM_EXPERTS + 1)[:NUM_EXPERTS]
    padded = (counts + 7) // 8 * 8
    offsets = np.cumsum(padded) - padded
    order = np.argsort(e, kind="stable")
    sorted_ids = np.full(R * 8, R, dtype=np.int32)
    expert_ids = np.full(R, -1, dtype=np.int32)
    rank_in_expert = np.zeros(R, dtype=np.int64)
    seen = np.zeros(NUM_EXPERTS + 1, dtype=np.int64)
    for j in order:  # stable: original route order within an expert
        rank_in_expert[j] = seen[e[j]]
        seen[e[j]] += 1
    for j in np.nonzero(valid)[0]:
        sorted_ids[offsets[e[j]] + rank_in_expert[j]] = j
    for ex in np.nonzero(counts)[0]:
        expert_ids[offsets[ex] // 8: offsets[ex] // 8 + padded[ex] // 8] = ex
    return sorted_ids, expert_ids, np.array([padded.sum()], dtype=np.int32)


def moe_align_small_loops(flat):
    """Pure-Python restatement of benchmarks/moe_align.py:23-31 (small cases)."""
    count = len(flat)
    output, experts = [], []
    for expert in range(NUM_EXPERTS):
        members = [i for i, value in enumerate(flat) if value == expert]
        padded = (len(members) + 7) // 8 * 8
        output.extend(members + [count] * (padded - len(members)))
        experts.extend([expert] * (padded // 8))
    postpad = len(output)
    return (output + [count] * (count * 8 - len(output)),
            experts + [-1] * (count - len(experts)), [postpad])


# ------------------------------------------------ MoE split align (prefill)
SPLIT_SIZES = (64, 48, 32, 16)                        # moe_split_align.py:39
SPLIT_COST = {64: 33.3, 48: 26.4, 32: 20.3, 16: 14.1}  # moe_split_align.py:40
SPLIT_UNWRITTEN = -2  # marker for list entries the algorithm leaves untouched


def split_cover_table(max_rows):
    """[max_rows + 1, 4] int32: blocks of each size in SPLIT_SIZES of the cheapest
    cover of r rows (profiles/sm74/titan_prefill/moe_split_align.py:172-185).

    Dynamic programme over r in float64: cost(r) = min over sizes s of
    COST[s] + cost(max(r - s, 0)), ties to the smaller (cost, size) pair.
    """
    best = [0.0] * (max_rows + 1)
    choice = [0] * (max_rows + 1)
    for r in range(1, max_rows + 1):
        best[r], choice[r] = min((SPLIT_COST[s] + best[max(r - s, 0)], s) for s in SPLIT_SIZES)
    table = np.zeros((max_rows + 1, len(SPLIT_SIZES)), dtype=np.int32)
    for r in range(1, max_rows + 1):
        table[r] = table[max(r - choice[r], 0)]
        table[r, SPLIT_SIZES.index(choice[r])] += 1
    return table


def moe_split_align(routes, num_experts, t_max=None, table=None):
    """Split block alignment of profiles/sm74/titan_prefill/moe_split_align.py:204-223.

    routes: integer expert ids of the T = M * topk routed rows (any shape;
    int64 ids are narrowed to int32 first, as :207-209 does).  Returns a list,
    one entry per block size in SPLIT_SIZES, of (block_size, sorted_ids,
    expert_ids, ntpp) where sorted_ids / expert_ids are the full buffers of
    :196-199 (t_max + B*E and (t_max + B*E) // B + 1 entries) with entries the
    algorithm does not write left at SPLIT_UNWRITTEN, and ntpp the list's row
    count.  Steps:
      plan (:73-99)    r_e = valid rows of expert e; n_k = table[r_e, k];
                       rows_k = n_k * B_k; off_k = exclusive prefix over
                       experts; rank boundaries lo1, lo2, lo3; ntpp_k = sum rows_k.
      fill (:102-135)  the last non-empty list of an expert pads its tail with
                       the sentinel T; every list gets its blocks' expert id.
      scatter (:138-169) row j of expert e with stable rank q (flat order) goes
                       to the list whose rank range holds q, at off + q - lo.
    """
    flat = np.asarray(routes).reshape(-1).astype(np.int64)
    flat = ((flat + 2 ** 31) % 2 ** 32 - 2 ** 31)  # ids.to(torch.int32) wraps
    T = flat.size
    E = int(num_experts)
    t_max = T if t_max is None else int(t_max)
    assert 0 < T <= t_max
    table = split_cover_table(t_max) if table is None else np.asarray(table)
    valid = (flat >= 0) & (flat < E)
    r = np.bincount(flat[valid], minlength=E).astype(np.int64)
    rows = np.stack([table[r, k].astype(np.int64) * b for k, b in enumerate(SPLIT_SIZES)])
    off = np.cumsum(rows, axis=1) - rows
    lo1, lo2, lo3 = rows[0], rows[0] + rows[1], rows[0] + rows[1] + rows[2]
    sorted_ids = [np.full(t_max + b * E, SPLIT_UNWRITTEN, dtype=np.int32) for b in SPLIT_SIZES]
    expert_ids = [np.full((t_max + b * E) // b + 1, SPLIT_UNWRITTEN, dtype=np.int32) for b in SPLIT_SIZES]
    for e in range(E):
        b3 = SPLIT_SIZES[3]
        hi3 = lo3[e] + (r[e] + b3 - 1 - lo3[e]) // b3 * b3 if r[e] > lo3[e] else lo3[e]
        last3 = hi3 > lo3[e]
        last2 = lo3[e] > lo2[e] and not last3
        last1 = lo2[e] > lo1[e] and lo3[e] == lo2[e] and not last3
        last0 = lo1[e] > 0 and lo2[e] == lo1[e] and lo3[e] == lo2[e] and not last3
        spans = ((0, lo1[e], last0), (lo1[e], lo2[e], last1), (lo2[e], lo3[e], last2), (lo3[e], hi3, last3))
        for k, (lo, hi, last) in enumerate(spans):
            b = SPLIT_SIZES[k]
            n = hi - lo
            pad = hi - r[e] if last else 0
            start = off[k, e] + n - pad
            for j in range(min(max(pad, 0), 64)):  # :107-108, pad < 64 by construction
                sorted_ids[k][start + j] = T
            for blk in range(n // b):
                expert_ids[k][off[k, e] // b + blk] = e
    seen = np.zeros(E, dtype=np.int64)
    for j in np.nonzero(valid)[0]:
        e = flat[j]
        q = seen[e]
        seen[e] += 1
        k = 3 if q >= lo3[e] else 2 if q >= lo2[e] else 1 if q >= lo1[e] else 0
        base = (0, lo1[e], lo2[e], lo3[e])[k]
        sorted_ids[k][off[k, e] + q - base] = j
    return [(b, sorted_ids[k], expert_ids[k], int(rows[k].sum())) for k, b in enumerate(SPLIT_SIZES)]


# ------------------------------------------------------ paged index conversion
def convert_req_index_to_global(req_id, block_table, token_indices, block_size, block_stride_rows=None):
    """Request-local top-k positions -> global cache rows (int32 [T, topk]).

    Restates vLLM 0.22 v1/attention/backends/mla/sparse_utils.py:11-83
    (`_convert_req_index_to_global_index_kernel`, called by the reference's
    backend at integration/titan_backend.py:49-52 with BLOCK_STRIDE_ROWS):
      blk = tok // block_size, off = tok % block_size
      out = block_table[req, blk] * block_stride_rows + off   (int32 arithmetic)
      out = -1 where tok < 0 or blk >= max_blocks
    plus -1 where req_id[t] is not a row of block_table (vLLM reads out of
    bounds there).  block_stride_rows defaults to block_size (vLLM 0.22).
    """
    req = np.asarray(req_id, dtype=np.int64)
    bt = np.asarray(block_table, dtype=np.int64)
    tok = np.asarray(token_indices, dtype=np.int64)
    stride_rows = block_size if block_stride_rows is None else block_stride_rows
    num_reqs, max_blocks = bt.shape
    blk = np.where(tok >= 0, tok // block_size, -1)
    ok = (tok >= 0) & (blk < max_blocks) & ((req >= 0) & (req < num_reqs))[:, None]
    rr = np.clip(req, 0, max(num_reqs - 1, 0))[:, None]
    base = bt[rr, np.clip(blk, 0, max(max_blocks - 1, 0))] if num_reqs and max_blocks else np.zeros_like(tok)
    val = base * stride_rows + (tok - blk * block_size)
    val = ((val + 2 ** 31) % 2 ** 32) - 2 ** 31          # two's-complement int32 wrap
    return np.where(ok, val, -1).astype(np.int32)


# ------------------------------------------------------- W4A16 MoE GEMM
def moe_w4a16_dequant(q, scales):
    """uint4b8 codes q [E, N, K] (0..15) and bf16 group scales [E, K / 128, N]
    -> float32 [E, N, K] = bf16((q - 8) * scale), the dequantised weight the
    tensor cores consume (Marlin rounds it to the activation type the same way)."""
    q = torch.as_tensor(q).to(torch.int32)
    s = torch.as_tensor(scales).float()
    E, N, K = q.shape
    sk = s.permute(0, 2, 1).repeat_interleave(128, dim=2)            # [E, N, K]
    return ((q - 8).float() * sk).to(torch.bfloat16).float()


def moe_w4a16_gemm(a, w_deq, sorted_ids, expert_ids, ntpp, topk_weights, block_size, top_k,
                   mul_topk_weights, size_m, c):
    """One list GEMM of the split Marlin MoE path (the per-list
    `moe_wna16_marlin_gemm` calls, profiles/sm74/titan_prefill/marlin.py:
    417-444; vLLM's op, not in the reference tree): for each block b <
    ntpp / block_size with expert e = expert_ids[b] and routed rows
    s = sorted_ids[b * block_size + j] < size_m * top_k,
    c[s] = a[s // top_k] @ w_deq[e]^T (times topk_weights[s] when
    mul_topk_weights), accumulated in float64 here and stored as bf16.
    Rows not listed keep their contents.  Modifies and returns c (torch, CPU)."""
    a = torch.as_tensor(a).double()
    sid = np.asarray(torch.as_tensor(sorted_ids).cpu()).astype(np.int64)
    eid = np.asarray(torch.as_tensor(expert_ids).cpu()).astype(np.int64)
    nblocks = int(np.asarray(torch.as_tensor(ntpp).cpu()).reshape(-1)[0]) // block_size
    pad = size_m * top_k
    for b in range(nblocks):
        e = int(eid[b])
        if e < 0 or e >= w_deq.shape[0]:
            continue
        rows = sid[b * block_size:(b + 1) * block_size]
        rows = rows[(rows >= 0) & (rows < pad)]
        if rows.size == 0:
            continue
        r = torch.from_numpy(rows)
        out = a[r // top_k] @ w_deq[e].double().T
        if mul_topk_weights:
            out = out * torch.as_tensor(topk_weights).double().reshape(-1)[r][:, None]
        c[r] = out.to(c.dtype)
    return c


# ------------------------------------------------- indexer pool top-k
def expand_row(pools, seq_len, pool_size, include_tail=True):
    """Restatement of tests/verify_indexer_sharding.py:68-76: pool p ->
    tokens p * pool_size + o (a -1 pool -> -1s), then the tail of the partial
    last pool (pool_size - 1 entries, -1 past seq_len % pool_size)."""
    hist = [p * pool_size + o if p >= 0 else -1 for p in pools for o in range(pool_size)]
    if include_tail:
        start = seq_len // pool_size * pool_size
        hist += [start + o if o < seq_len % pool_size else -1 for o in range(pool_size - 1)]
    return hist


def pool_topk_expand(logits, seq_lens, topk, pool_size, width):
    """Top-`topk` complete pools (p < seq_len // pool_size) by logit, in the
    order of the radix keys a CUDA top-k sorts float32 by (the IEEE bit
    pattern made order-preserving: -0.0 below +0.0, every NaN above +inf),
    descending, equal keys in pool order; then expand_row, then -1 up to
    `width`.  int32 [T, width] (numpy)."""
    lg = np.ascontiguousarray(np.asarray(torch.as_tensor(logits).float().cpu()))
    sl = np.asarray(torch.as_tensor(seq_lens).cpu()).astype(np.int64)
    T, P = lg.shape
    bits = lg.view(np.uint32).astype(np.uint64)
    keys = np.where(bits & 0x80000000, (~bits) & 0xFFFFFFFF, bits | 0x80000000)
    keys = np.where((bits & 0x7FFFFFFF) > 0x7F800000, 0xFFFFFFFF, keys)
    out = np.full((T, width), -1, np.int32)
    for t in range(T):
        n = min(max(int(sl[t]), 0) // pool_size, P)
        order = np.lexsort((np.arange(n), -keys[t, :n].astype(np.int64)))   # key desc, then pool asc
        pools = [int(p) for p in order[:topk]] + [-1] * max(0, topk - n)
        row = expand_row(pools, max(int(sl[t]), 0), pool_size)
        out[t, :len(row)] = row
    return out
