# SPDX-License-Identifier: Apache-2.0
"""Split MoE block alignment for the Marlin W4A16 MoE at whole-expert prefill.

Drop-in for the reference's profiles/sm74/titan_prefill/moe_split_align.py:
the same `SIZES`, `COST`, `cover_table`, `buffers` and `split_align`, with the
same outputs bit for bit.  The routed (token, slot) rows are sorted by expert
into one block list per size in SIZES (64, 48, 32, 16); each expert's r rows
are covered by the cheapest multiset of blocks under the per-block cost model
COST, filled largest size first, only the last (smallest) block padded with the
sentinel T = M * topk.  Rows keep their stable flat order within an expert.

The five Triton kernels of the reference become one launch of one 16-CTA
thread-block cluster, 8 CTAs where the device cannot hold 16
(`titan_moe_split_align` in libtitan_b200.so, csrc/titan_moe_split_align.cu):
per-warp shared-memory histograms, stable ranks from a prefix over warps and
over the cluster's CTAs (distributed shared memory), the plan as a CTA-wide
scan and the fill/scatter in the same kernel.  No host
sync and fixed buffers: CUDA-graph capturable.  Calls that share one buffer
set must be ordered on the GPU (one stream).
"""
from __future__ import annotations

import ctypes
import functools

import torch

try:
    from . import titan_native as _native
except ImportError:
    import titan_native as _native

SIZES = (64, 48, 32, 16)
COST = {64: 33.3, 48: 26.4, 32: 20.3, 16: 14.1}


@functools.lru_cache(maxsize=8)
def _cover_rows(R):
    best = [0.0] * (R + 1)
    choice = [0] * (R + 1)
    for r in range(1, R + 1):
        best[r], choice[r] = min((COST[s] + best[max(r - s, 0)], s) for s in SIZES)
    rows = [(0, 0, 0, 0)]
    for r in range(1, R + 1):
        n = list(rows[max(r - choice[r], 0)])
        n[SIZES.index(choice[r])] += 1
        rows.append(tuple(n))
    return tuple(rows)


def cover_table(R: int) -> torch.Tensor:
    """[R+1, len(SIZES)] int32 (CPU): blocks of each size in the cheapest cover
    of r rows, for r = 0..R (moe_split_align.py:172-185).  A dynamic programme
    over r in float64: cost(r) = min over s of COST[s] + cost(max(r - s, 0)),
    ties to the smaller (cost, size) pair."""
    return torch.tensor(_cover_rows(int(R)), dtype=torch.int32)


def buffers(t_max: int, E: int, device: torch.device) -> dict:
    """All buffers for ``split_align`` at up to ``t_max`` = M*topk routed rows
    (moe_split_align.py:187-201; no histogram scratch is needed here)."""
    if not 1 <= E <= 1024:
        raise ValueError("split_align supports 1..1024 experts")
    return {
        "t_max": t_max,
        "E": E,
        "tab": cover_table(t_max).to(device),
        "s": [torch.empty(t_max + bs * E, device=device, dtype=torch.int32) for bs in SIZES],
        "e": [torch.empty((t_max + bs * E) // bs + 1, device=device, dtype=torch.int32) for bs in SIZES],
        "ntpp": torch.empty(len(SIZES), device=device, dtype=torch.int32),
    }


def split_align(topk_ids: torch.Tensor, E: int, buf: dict):
    """-> [(block_size, sorted_ids, expert_ids, ntpp_1elem)], one per size in
    SIZES, into the fixed buffers ``buf`` (from ``buffers``).

    moe_split_align.py:204-223: ids outside [0, E) are dropped; int64 ids are
    narrowed to int32 first, as the reference's `.to(torch.int32)` does.
    Raises AssertionError when T = topk_ids.numel() is 0 or above buf["t_max"],
    or E differs from buf["E"].
    """
    ids = topk_ids.reshape(-1)
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.to(torch.int32)
    T = ids.numel()
    if not (0 < T <= buf["t_max"] and E == buf["E"]):
        raise AssertionError("split_align buffers too small")
    if not ids.is_cuda:
        raise ValueError("split_align requires CUDA route IDs")
    if any(t.device != ids.device for t in (buf["tab"], buf["ntpp"], *buf["s"], *buf["e"])):
        raise ValueError("split_align buffers must be on the route IDs' device")
    ids = ids.contiguous()  # the kernel reads the flat ids with stride 1
    s, e, ntpp = buf["s"], buf["e"], buf["ntpp"]
    lists_s = (ctypes.c_void_p * 4)(*(t.data_ptr() for t in s))
    lists_e = (ctypes.c_void_p * 4)(*(t.data_ptr() for t in e))
    lib = _native.load()
    with _native.on_device(ids.device):
        rc = lib.titan_moe_split_align(
            ids.data_ptr(), 1 if ids.dtype == torch.int64 else 0, T, E,
            buf["tab"].data_ptr(), buf["tab"].shape[0], buf["t_max"],
            lists_s, lists_e, ntpp.data_ptr(), _native.stream_of(ids))
    _native.check(rc, "split_align")
    return [(bs, s[k], e[k], ntpp[k:k + 1]) for k, bs in enumerate(SIZES)]
