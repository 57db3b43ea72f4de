#!/usr/bin/env python3
# SPDX-License-Identifier: Apache-2.0
"""Benchmark of the GLM-5.3 sparse-MLA decode path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workloads, numbered as in the benchmark configuration list of this path:
1 = the CPU-sized B=1 case (4096-row cache), 2 = production B=1 decode,
3 = B=8 decode, 4 = prefill-shaped T=4096, 5 = MoE route alignment B1..8.

Headline (one JSON line on rank 0): config 2 — B=1 decode, 16 heads,
262,144-row INT8 cache (1024 blocks x 256 x 528 B) filled by store_int8,
2176 indices per token (2048 distinct valid + 128 x -1), sm_scale 512^-0.5.
A step is one call of triton_mla_sparse_attention on one token's index set.
The K timed calls run back to back inside CUDA graphs, like the layers of one
decode step: call j reads cache replica j % 8 (8 x 138 MB, far above the
126 MB L2) with its own index set, and an L2-flushing write precedes every
timed graph replay, so gathered rows come from HBM.  `value` = device time per
call (CUDA events around each replay / calls), whole-job: max over ranks,
divided by the number of ranks (each rank serves its own independent B=1
requests; the path needs no collective).  `e2e` is the same call through the
public API with host buffers, transfers inside the timed region: each step's
q + indices cross from one pinned host staging row to the device (titan_io's
kernel-driven copy) and the attention kernel stores the output into a pinned
host buffer (`out=`); the steps are captured in a CUDA graph, as a decode
engine issues them.  `secondary.e2e_eager_us` is the same loop issued
eagerly (host-bound) and `secondary.e2e_eager_copy_engine_us` the eager loop
with cudaMemcpyAsync-based copies (torch `copy_`) both ways.  Per-call CUDA events tick at 2.048 us on this
platform, so single-call latency (`secondary.isolated_call_us`) is coarse.

Secondary measurements ride along in "secondary": store_int8 cache fill
(config 2 fill, 408.9 MB), B=8 decode sharded over ranks (config 3),
prefill-shaped T=4096 (config 4, sharded over ranks), MoE align B1/2/4/8
(config 5) and the prefill split align of the MoE layer (M = 2304 and 8192
tokens x top-8, 288 experts, uniform and Zipf(1.1) routes).

--impl reference times the reference algorithm's CPU restatement (oracle/,
the only CPU implementation of this path; the reference ships Triton GPU
kernels only) on the host cores for the same config and metric, with the
same protocol as the cpu_baseline key of our arm (time_cpu_port).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "glm-5.3-kernels_b200"
for _p in (str(ROOT), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "sparse MLA decode µs/call + achieved HBM GB/s vs peak at 1/2/4/8 B200"
UNIT = "us/call"
KV_ROWS = 262144
BLOCK = 256
TOPK = 2176
VALID = 2048
HEADS = 16
SM_SCALE = 512 ** -0.5
ROW_BYTES = 528
FLUSH_BYTES = 256 << 20
FALLBACK_HBM_GBS = 6650.0


# ------------------------------------------------------------------ plumbing
def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def token_block(total, world, rank):
    """Contiguous block [lo, hi) of `total` independent requests owned by `rank`
    (the path has no cross-request exchange, so ranks never communicate data)."""
    return total * rank // world, total * (rank + 1) // world


class Dist:
    """torch.distributed for barriers and max-over-ranks timing only (NCCL on
    GPUs; gloo for the CPU tests of this host logic)."""

    def __init__(self, world, rank, local_rank, backend="nccl"):
        self.world, self.rank, self.local_rank = world, rank, local_rank
        self.backend = backend
        self.pg = None
        if world > 1:
            import torch.distributed as dist
            kw = {"device_id": torch.device("cuda", local_rank)} if backend == "nccl" else {}
            dist.init_process_group(backend, timeout=timedelta(seconds=300), **kw)
            self.pg = dist

    def barrier(self):
        if self.pg is not None:
            if self.backend == "nccl":
                self.pg.barrier(device_ids=[self.local_rank])
            else:
                self.pg.barrier()

    def max(self, value):
        if self.pg is None:
            return value
        dev = torch.device("cuda", self.local_rank) if self.backend == "nccl" else torch.device("cpu")
        t = torch.tensor([value], dtype=torch.float64, device=dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            d = json.loads(path.read_text())
            return float(d["hbm_gbs"]), "measured"
        except (ValueError, KeyError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(name):
    """Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) from
    the committed ncu summary profiles/<name>.md, line `traffic_bytes_per_launch: N`."""
    path = ROOT / "profiles" / f"{name}.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed work runs."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.uuid = str(getattr(torch.cuda.get_device_properties(device), "uuid", ""))
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None
        return self

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) != 9:
                    continue
                if self.uuid and self.uuid not in parts[0] and parts[0] not in self.uuid:
                    continue
                rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        busy = [s for s in sm if s > 0]
        return {"sm_mhz": statistics.median(busy) if busy else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


class Flusher:
    """Writes a buffer larger than L2 (126 MB) so every timed call starts cold."""

    def __init__(self, device):
        self.buf = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=device)

    def __call__(self):
        self.buf.fill_(1.0)


def capture(fn):
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()  # warm (and first-call setup) outside capture
        with torch.cuda.graph(graph, stream=s):
            out = fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    return graph, out


def timed_cold(step, n, flush, before=None):
    """n steps; each step: before(k) (untimed), L2 flush (untimed), then events
    around step(k).  Returns per-step device milliseconds."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for k in range(n):
        if before is not None:
            before(k)
        flush()
        evs[k][0].record()
        step(k)
        evs[k][1].record()
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


# --------------------------------------------------------------- workloads
def latents(n, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(n, 512, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)


def decode_sets(batch, sets, seed, kv_rows=KV_ROWS, tail_mode="fixed"):
    """CPU tensors: q [sets, batch, 16, 512] bf16 and indices [sets, batch, 1, 2176] int32."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(sets, batch, HEADS, 512, generator=g).to(torch.bfloat16)
    idx = torch.full((sets, batch, 1, TOPK), -1, dtype=torch.int32)
    for s in range(sets):
        for b in range(batch):
            if tail_mode == "fixed":   # config 2: 2048 distinct + 128 x -1
                idx[s, b, 0, :VALID] = torch.randperm(kv_rows, generator=g)[:VALID].to(torch.int32)
            else:                      # config 3: uniform with a random 0..256 tail of -1
                tail = int(torch.randint(0, 257, (1,), generator=g))
                idx[s, b, 0, :TOPK - tail] = torch.randint(0, kv_rows, (TOPK - tail,), generator=g,
                                                           dtype=torch.int32)
    return q, idx


def prefill_indices(tokens, seed, t0=0):
    """Config 4: token t draws min(t+1, 2176) + 65536 * (t // 1024) candidates
    without replacement, padded to 2176 with -1."""
    g = torch.Generator().manual_seed(seed)
    idx = torch.full((tokens, 1, TOPK), -1, dtype=torch.int32)
    for i in range(tokens):
        t = t0 + i
        pool = min(t + 1, TOPK) + 65536 * (t // 1024)
        k = min(pool, TOPK)
        idx[i, 0, :k] = torch.randperm(pool, generator=g)[:k].to(torch.int32)
    return idx


def alg_bytes(idx_cpu):
    i = idx_cpu.reshape(idx_cpu.shape[0], -1)
    n_valid = int(((i >= 0) & (i < KV_ROWS)).sum())
    return n_valid * ROW_BYTES + i.numel() * 4 + 2 * i.shape[0] * HEADS * 512 * 2


# ------------------------------------------------------------------ our arm
REPLICAS = 8          # KV-cache replicas (one per "layer"), 8 x 138 MB >> 126 MB L2
MAX_CALLS_PER_GRAPH = 512


def graph_calls(k):
    """Calls per captured graph so that k timed calls are whole graph replays."""
    if k <= MAX_CALLS_PER_GRAPH:
        return k
    return max(d for d in range(1, MAX_CALLS_PER_GRAPH + 1) if k % d == 0)


class DecodeBench:
    """`calls` decode calls captured back to back in one CUDA graph, call j on
    cache replica j % REPLICAS with its own index set, like consecutive layers
    of one decode step.  Every timed replay starts after an L2-flushing write,
    and one replay touches calls x ~1.1 MB of distinct rows, so the gathered
    rows come from HBM; q and indices are per call, as the producers leave them."""

    def __init__(self, attn, kvs, batch, calls, seed, tail_mode, sms, splits=None):
        q, idx = decode_sets(batch, calls, seed, tail_mode=tail_mode)
        self.bytes_per_call = statistics.fmean(alg_bytes(idx[j]) for j in range(calls))
        dev = kvs[0].device
        self.q, self.idx = q.to(dev), idx.to(dev)
        self.calls = calls
        kw = {"num_kv_splits": splits} if splits else {"sm_count": sms}

        def run():
            for j in range(calls):
                attn(self.q[j], kvs[j % len(kvs)], self.idx[j], SM_SCALE, **kw)
        self.graph, _ = capture(run)

    def time(self, replays, flush):
        """Device ms of each replay (CUDA events), L2 flushed before each."""
        return timed_cold(lambda k: self.graph.replay(), replays, flush)

    def close(self):
        self.graph.reset()


class PagedBench:
    """Config 2 on a paged layout: the 262,144-row cache as 4096 blocks of 64
    rows and one request whose block table (a random block permutation) is
    shared by all calls, as the layers of one decode step share it, while each
    call has its own 2048 distinct request-local positions + 128 x -1 (the
    per-layer indexer output).
    `fused` times triton_mla_sparse_attention_paged (the gather translates);
    otherwise the conversion kernel runs first and the reader reads its
    output, as the reference's backend does (integration/titan_backend.py:
    49-54).  Calls back to back in one CUDA graph over the cache replicas."""

    BLOCK = 64

    def __init__(self, kvs, calls, seed, sms, fused):
        from kernels.titan_index import triton_convert_req_index_to_global_index as conv
        from kernels.titan_mla import triton_mla_sparse_attention as attn
        from kernels.titan_mla import triton_mla_sparse_attention_paged as attn_paged
        dev = kvs[0].device
        g = torch.Generator().manual_seed(seed)
        nb = KV_ROWS // self.BLOCK
        self.bt = torch.randperm(nb, generator=g).to(torch.int32).view(1, nb).to(dev)
        tok = torch.full((calls, 1, TOPK), -1, dtype=torch.int32)
        for j in range(calls):
            tok[j, 0, :VALID] = torch.randperm(KV_ROWS, generator=g)[:VALID].to(torch.int32)
        self.tok = tok.to(dev)
        self.q = torch.randn(calls, 1, HEADS, 512, generator=g).to(torch.bfloat16).to(dev)
        self.req = torch.zeros(1, dtype=torch.int32, device=dev)

        def run():
            for j in range(calls):
                kv = kvs[j % len(kvs)]
                bt = self.bt
                if fused:
                    attn_paged(self.q[j], kv, self.tok[j], self.req, bt, self.BLOCK, SM_SCALE, sm_count=sms)
                else:
                    glob = conv(self.req, bt, self.tok[j, :, :], BLOCK_SIZE=self.BLOCK, NUM_TOPK_TOKENS=TOPK)
                    attn(self.q[j], kv, glob.view(1, 1, TOPK), SM_SCALE, sm_count=sms)
        self.graph, _ = capture(run)

    def time(self, replays, flush):
        return timed_cold(lambda k: self.graph.replay(), replays, flush)

    def close(self):
        self.graph.reset()


def splits_and_launches(batch, sms, device_index):
    """Split count the B200 policy picks, its cluster size, kernel launches
    per call (the combine kernel runs only when the split kernel cannot merge
    the partials itself: in its clusters, or flat across its CTAs) and how
    the partials are merged."""
    from kernels.titan_mla import _choose_kv_splits_b200, _cluster_tables, _launch_layout
    tables = _cluster_tables(device_index)
    S = _choose_kv_splits_b200(batch, 1, TOPK, sms, tables)
    C, nc, flat = _launch_layout(batch, S, tables)
    if S == 1:
        merge = "single pass"
    elif flat:
        merge = f"flat merge of {S} split CTAs per token"
    elif nc == 1:
        merge = f"cluster merge ({C} CTAs)"
    elif C >= 2 and nc <= C:
        merge = f"cluster merge ({C} CTAs) + last-arriver merge of {nc} clusters"
    else:
        merge = f"combine kernel over {nc} partials"
    return S, C, (1 if nc == 1 or flat or (C >= 2 and nc <= C) else 2), merge


def run_ours(args, dist):
    from kernels import titan_native
    from kernels.titan_kv import store_int8
    from kernels.titan_mla import triton_mla_sparse_attention as attn
    from kernels.titan_moe_align import titan_moe_align_small

    rank, world = dist.rank, dist.world
    dev = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    peak, peak_kind = measured_peaks()
    flush = Flusher(dev)
    K, W = args.steps, args.warmup
    sampler = ClockSampler(dev)

    # ---- caches: config 2 (262,144 rows x 528 B), filled by store_int8; the
    # same seeded replicas on every rank
    lat = latents(KV_ROWS, 1234, dev)
    slots = torch.arange(KV_ROWS, device=dev)
    caches = []
    for r in range(REPLICAS):
        c = torch.empty(KV_ROWS // BLOCK, BLOCK, ROW_BYTES, dtype=torch.int8, device=dev)
        store_int8(latents(KV_ROWS, 1234 + r, dev) if r else lat, c, slots)
        caches.append(c)
    kvs = [c.view(KV_ROWS, 1, ROW_BYTES) for c in caches]
    # Every rank builds the same replicas: compare a checksum of each replica's
    # bytes across ranks (four 16-bit lanes of a wrapping int64 word sum, so
    # the float64 reduction is exact).
    sums = [int(c.view(torch.int64).sum()) for c in caches]
    lanes = [float((x >> (16 * k)) & 0xFFFF) for x in sums for k in range(4)]
    cache_identical = all(dist.max(v) == -dist.max(-v) for v in lanes)
    torch.cuda.synchronize()

    sampler.start()
    dist.barrier()
    # ---- headline: B=1 decode, K calls back to back (CUDA graphs), cold rows
    J = graph_calls(K)
    S1, C1, launches_per_call, merge1 = splits_and_launches(1, sms, dev.index)
    d1 = DecodeBench(attn, kvs, 1, J, 99 + rank, "fixed", sms)
    d1.time(max(1, W // J + 1), flush)                     # warm-up replays (>= W calls)
    dist.barrier()
    ms = d1.time(K // J, flush)
    dist.barrier()
    per_call_ms = sum(ms) / K
    rank_max_ms = dist.max(per_call_ms)
    value_us = rank_max_ms * 1000.0 / world
    bytes_per_call = d1.bytes_per_call
    achieved = dist.max(-(bytes_per_call / (per_call_ms * 1e-3) / 1e9)) * -1.0  # slowest rank
    d1.close()

    # ---- isolated single call (flush, then one call): latency, 2.048-us event ticks
    q1, i1 = decode_sets(1, 16, 7 + rank)
    q1d, i1d = q1.to(dev), i1.to(dev)
    qs, ids = q1d[0].clone(), i1d[0].clone()
    g1, _ = capture(lambda: attn(qs, kvs[0], ids, SM_SCALE, sm_count=sms))

    def load1(k):
        qs.copy_(q1d[k % 16])
        ids.copy_(i1d[k % 16])

    timed_cold(lambda k: g1.replay(), 3, flush, load1)
    iso_us = statistics.fmean(timed_cold(lambda k: g1.replay(), max(10, min(K, 100)), flush, load1)) * 1000
    g1.reset()

    # ---- e2e: public API, pinned host inputs and output inside the timed
    # region.  Each step's q and indices sit back to back in one pinned
    # staging row and cross to the device in ONE transfer; the API is called
    # on device views of that buffer.  Small copy-engine copies cost ~5-8 us
    # of fixed latency each on this platform, so the headline path moves the
    # bytes with the SMs: titan_io.copy_ reads the pinned row through its
    # device mapping, and the attention kernel writes its bf16 output into a
    # pinned host buffer (out=).  The copy-engine loop is timed too.  One
    # staging row (index set) per step of a graph replay, so every step
    # gathers its own rows, from HBM as for `value`.
    sets = max(64, graph_calls(K))
    q_sets, idx_sets = decode_sets(1, sets, 199 + rank)
    q_bytes = q_sets[0].numel() * 2
    staging = torch.cat([q_sets.reshape(sets, -1).view(torch.uint8),
                         idx_sets.reshape(sets, -1).view(torch.uint8)], 1).pin_memory()
    out_host = torch.empty((sets, 1, HEADS, 512), dtype=torch.bfloat16).pin_memory()
    landing = torch.empty(staging.shape[1], dtype=torch.uint8, device=dev)
    qd = landing[:q_bytes].view(torch.bfloat16).view(1, HEADS, 512)
    idd = landing[q_bytes:].view(torch.int32).view(1, 1, TOPK)

    from kernels.titan_io import copy_ as staged_copy

    def e2e_step(k):
        staged_copy(landing, staging[k % sets], src_ready=True)
        attn(qd, kvs[k % REPLICAS], idd, SM_SCALE, sm_count=sms, out=out_host[k % sets])

    def e2e_step_copy_engine(k):
        landing.copy_(staging[k % sets], non_blocking=True)
        o = attn(qd, kvs[k % REPLICAS], idd, SM_SCALE, sm_count=sms)
        out_host[k % sets].copy_(o, non_blocking=True)

    def time_eager(step):
        for k in range(W):
            step(k)
        flush()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for k in range(K):
            step(k)
        b.record()
        torch.cuda.synchronize()
        dist.barrier()
        return dist.max(a.elapsed_time(b) / K) * 1000.0 / world

    # Eager loops (host-bound: each launch costs the host ~3-4 us on this
    # platform), kept for comparison.
    e2e_ce_us = time_eager(e2e_step_copy_engine)
    ref_host = out_host.clone()
    e2e_eager_us = time_eager(e2e_step)
    e2e_same = bool(torch.equal(out_host.view(torch.int16), ref_host.view(torch.int16))) if K + W >= sets else None

    # Headline e2e: the same public-API steps captured in a CUDA graph (how a
    # decode engine issues them), Je steps per replay, step j on staging row
    # j % 64 and cache replica j % 8; an L2-flushing write before every timed
    # replay, as for `value`.
    Je = graph_calls(K)
    out_host.zero_()
    ge, _ = capture(lambda: [e2e_step(j) for j in range(Je)])
    timed_cold(lambda k: ge.replay(), max(1, W // Je + 1), flush)
    dist.barrier()
    ms_e2e = timed_cold(lambda k: ge.replay(), K // Je, flush)
    dist.barrier()
    e2e_us = dist.max(sum(ms_e2e) / K) * 1000.0 / world
    rows_chk = min(Je, sets)
    e2e_same = e2e_same is not False and bool(torch.equal(out_host[:rows_chk].view(torch.int16),
                                                          ref_host[:rows_chk].view(torch.int16)))
    ge.reset()

    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    secondary = {"isolated_call_us": iso_us, "e2e_eager_us": e2e_eager_us, "e2e_eager_copy_engine_us": e2e_ce_us,
                 "e2e_outputs_equal_copy_engine_path": e2e_same}
    # ---- store_int8: config 2 fill, 262,144 rows, 10 fills back to back
    fill_bytes = KV_ROWS * (1024 + ROW_BYTES + 8)
    nf = 10
    for _ in range(2):
        store_int8(lat, caches[0], slots)
    a.record()
    for _ in range(nf):
        store_int8(lat, caches[0], slots)
    b.record()
    torch.cuda.synchronize()
    st_ms = dist.max(a.elapsed_time(b) / nf)
    perm = torch.randperm(KV_ROWS, device=dev)
    for _ in range(2):
        store_int8(lat, caches[1], perm)
    a.record()
    for _ in range(nf):
        store_int8(lat, caches[1], perm)
    b.record()
    torch.cuda.synchronize()
    stp_ms = dist.max(a.elapsed_time(b) / nf)
    secondary["store_int8"] = {
        "rows": KV_ROWS, "bytes": fill_bytes, "us": st_ms * 1000, "GBps": fill_bytes / (st_ms * 1e-3) / 1e9,
        "frac_of_hbm": fill_bytes / (st_ms * 1e-3) / 1e9 / peak, "random_perm_us": stp_ms * 1000,
        "random_perm_GBps": fill_bytes / (stp_ms * 1e-3) / 1e9, "per_rank": True}
    store_int8(lat, caches[0], slots)
    store_int8(latents(KV_ROWS, 1235, dev), caches[1], slots)

    # ---- config 2 on a paged cache: fused translation vs conversion + reader
    paged = {}
    for name, fused in (("fused_us_per_call", True), ("convert_then_reader_us_per_call", False)):
        pb = PagedBench(kvs, 64, 77 + rank, sms, fused)
        pb.time(2, flush)
        ms = pb.time(8, flush)
        pb.close()
        paged[name] = dist.max(statistics.median(ms) * 1000.0 / 64)
    paged["block_size"] = PagedBench.BLOCK
    secondary["paged_decode_b1"] = paged

    # ---- config 3: B=8 decode, tokens sharded contiguously over ranks
    lo, hi = token_block(8, world, rank)
    per = max(1, hi - lo)
    J8 = graph_calls(min(K, 256))
    d8 = DecodeBench(attn, kvs, per, J8, 777 + rank, "random", sms)
    d8.time(1, flush)
    dist.barrier()
    b8_ms = dist.max(sum(d8.time(max(1, min(K, 256) // J8), flush)) / (max(1, min(K, 256) // J8) * J8))
    S8, C8, _, merge8 = splits_and_launches(per, sms, dev.index)
    secondary["decode_b8"] = {
        "tokens_per_rank": per, "us_per_call": b8_ms * 1000, "tokens_per_s": per * world / (b8_ms * 1e-3),
        "GBps_per_rank": d8.bytes_per_call / (b8_ms * 1e-3) / 1e9, "splits": S8, "cluster": C8, "merge": merge8}
    d8.close()

    # ---- config 4: prefill-shaped, T=4096 tokens sharded over ranks
    if not args.skip_prefill:
        t0, t1 = token_block(4096, world, rank)
        tp = t1 - t0
        ip = prefill_indices(tp, 4242 + rank, t0=t0).to(dev)
        qp = torch.randn(tp, HEADS, 512, device=dev, generator=torch.Generator(device=dev).manual_seed(5)).to(
            torch.bfloat16)
        npf = max(3, min(K, 10))
        timed_cold(lambda k: attn(qp, kvs[0], ip, SM_SCALE, sm_count=sms), 2, flush)
        pf_ms = dist.max(statistics.fmean(timed_cold(lambda k: attn(qp, kvs[0], ip, SM_SCALE, sm_count=sms), npf,
                                                     flush)))
        nvalid = int(((ip >= 0) & (ip < KV_ROWS)).sum())
        secondary["prefill_t4096"] = {
            "tokens_per_rank": tp, "ms_per_call": pf_ms, "gathered_GBps": nvalid * ROW_BYTES / (pf_ms * 1e-3) / 1e9,
            "tflops": nvalid * 4 * HEADS * 512 / (pf_ms * 1e-3) / 1e12, "tokens_per_s": tp * world / (pf_ms * 1e-3)}

    # ---- config 5: MoE align.  (a) the reference's methodology, one call per
    # graph replayed 100x (replays are paced by the host and the platform's
    # 2.048-us event/launch granularity here); (b) 100 calls inside one graph.
    moe = {}
    gm = torch.Generator().manual_seed(37)
    for B in (1, 2, 4, 8):
        ids = torch.stack([torch.randperm(288, generator=gm)[:8] for _ in range(B)]).to(torch.int32).to(dev)
        gr, _ = capture(lambda: titan_moe_align_small(ids))
        for _ in range(5):
            gr.replay()
        samples = []
        for _ in range(5):
            a.record()
            for _ in range(100):
                gr.replay()
            b.record()
            torch.cuda.synchronize()
            samples.append(a.elapsed_time(b) * 1000 / 100)
        moe[f"B{B}_us"] = statistics.median(samples)
        gr.reset()
        g100, _ = capture(lambda: [titan_moe_align_small(ids) for _ in range(100)])
        g100.replay()
        samples = []
        for _ in range(5):
            a.record()
            g100.replay()
            b.record()
            torch.cuda.synchronize()
            samples.append(a.elapsed_time(b) * 1000 / 100)
        moe[f"B{B}_in_graph_us"] = statistics.median(samples)
        g100.reset()
        # config 5's second distribution: Zipf(s=1.1) over the 288 experts, no
        # duplicate within a token
        zw = (torch.arange(1, 289, dtype=torch.float64) ** -1.1)
        zids = torch.stack([torch.multinomial(zw, 8, replacement=False, generator=gm) for _ in range(B)])
        zids = zids.to(torch.int32).to(dev)
        gz, _ = capture(lambda: [titan_moe_align_small(zids) for _ in range(100)])
        gz.replay()
        samples = []
        for _ in range(5):
            a.record()
            gz.replay()
            b.record()
            torch.cuda.synchronize()
            samples.append(a.elapsed_time(b) * 1000 / 100)
        moe[f"B{B}_zipf_in_graph_us"] = statistics.median(samples)
        gz.reset()
    secondary["moe_align_graph_replay"] = moe

    # ---- prefill split align (the consumer side of config 5 at whole-expert
    # prefill): M = 2304 tokens x top-8 over 288 experts, uniform and
    # Zipf(1.1); 100 calls on one buffer set inside one graph.
    from kernels import titan_moe_split_align as split_mod
    split = {}
    for M in (2304, 8192):
        sbuf = split_mod.buffers(M * 8, 288, dev)
        for dist_name in ("uniform", "zipf"):
            if dist_name == "uniform":
                sids = torch.randint(0, 288, (M, 8), generator=gm, dtype=torch.int32)
            else:
                zw = (torch.arange(1, 289, dtype=torch.float64) ** -1.1)
                sids = torch.multinomial(zw, M * 8, replacement=True, generator=gm).view(M, 8).to(torch.int32)
            sids = sids.to(dev)
            gs, _ = capture(lambda: [split_mod.split_align(sids, 288, sbuf) for _ in range(100)])
            gs.replay()
            samples = []
            for _ in range(5):
                a.record()
                gs.replay()
                b.record()
                torch.cuda.synchronize()
                samples.append(a.elapsed_time(b) * 1000 / 100)
            split[f"M{M}_{dist_name}_in_graph_us"] = statistics.median(samples)
            gs.reset()
    secondary["moe_split_align"] = split

    # ---- indexer pool top-k + expansion (the producer of the reader's
    # indices): decode, 8 query rows, and a 2048-row prefill chunk, each
    # over 65,536 pools of 4 (a 262,144-token context), k = 512, 2176-wide
    # rows; torch.topk with a torch expansion on the same GPU beside it.
    secondary["pool_topk_expand"] = pool_topk_line(dev, peak, flush)

    # ---- W4A16 MoE GEMM (the consumer of the split align): the gate/up
    # projection of the whole-expert prefill shape, M = 2304 tokens x top-8
    # over 288 experts, 2N = 4096, K = 4096, uint4b8 group-128 weights
    # (profiles/sm74/titan_prefill/marlin.py:417-424), the four list GEMMs
    # back to back in one CUDA graph; Zipf(1.1) routes.  vLLM's Marlin on the
    # same inputs beside it in single-GPU runs only (a comparison line).
    if not args.skip_moe_gemm:
        secondary["moe_w4a16_gemm"] = moe_gemm_line(dev, peak, gm, marlin=world == 1)
    # ---- the reference's own Triton kernels on this B200 (rank 0 of a
    # single-GPU run only; comparison lines, not our path)
    if rank == 0 and world == 1 and not args.skip_reference_triton:
        ref = load_reference_triton()
        if ref is None:
            secondary["reference_triton_b200"] = {"unavailable": "baseline/_ref is not installed"}
        else:
            try:
                secondary["reference_triton_b200"] = reference_triton_b200(ref, kvs, lat, slots, flush, sms, K,
                                                                           caches[0])
            except Exception as exc:  # a Triton compile or launch failure is reported, not fatal
                secondary["reference_triton_b200"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    clocks = sampler.stop()
    dist.barrier()

    err = titan_native.device_error(caches[0])
    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu_baseline:
        cpu = cpu_baseline_b1(caches[0], K, args.cpu_seconds)

    if rank == 0:
        traffic = profile_traffic("mla_decode_b1")
        line = {
            "metric": METRIC, "value": value_us, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": rank_max_ms, "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {
                "workload": "config2: B=1 sparse MLA decode, 16 heads x 512 NoPE latent, 262144-row INT8 "
                            "528-B-row cache filled by store_int8, 2176 indices (2048 distinct valid + 128 x -1)",
                "kv_rows": KV_ROWS, "heads": HEADS, "topk": TOPK, "valid_per_token": VALID,
                "num_kv_splits": S1, "cluster": C1, "sm_count": sms,
                "l2": f"inputs larger than L2: {REPLICAS} cache replicas ({REPLICAS * KV_ROWS * ROW_BYTES / 1e9:.2f} GB) "
                      f"rotated per call and {J} distinct index sets per graph replay, plus a 256 MiB L2-flushing "
                      "write before each timed replay",
                "timing": f"{J} calls back to back per CUDA graph replay, CUDA events per replay, per-call mean, "
                          "max over ranks",
                "parallelism": f"replicas x{world} (independent B=1 requests per GPU, no collective)"},
            "per_gpu_us_per_call": rank_max_ms * 1000.0,
            "tokens_per_s": world / (rank_max_ms * 1e-3),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_kind,
                         "algorithmic_bytes_per_call": bytes_per_call,
                         "kernel": f"sparse_mla_kernel ({S1} splits, {merge1}; {launches_per_call} launch(es) per call), "
                                   "whole call, back to back"},
            "e2e": {"value": e2e_us, "unit": UNIT, "h2d_bytes_per_step": staging.shape[1],
                    "d2h_bytes_per_step": HEADS * 512 * 2,
                    "transfers_per_step": "H2D: q + indices, one pinned staging row, read by titan_copy's kernel "
                                          "through the device mapping; D2H: the attention kernel stores its bf16 "
                                          "output into pinned host memory (out=)",
                    "issue": f"public-API steps captured in a CUDA graph, {Je} per replay, L2 flushed before "
                             "each timed replay; eager loops in secondary"},
            # The sharded workloads (the ones whose 1 -> N curve can bend):
            # config 3 (B=8, tokens split over the ranks) and config 4
            # (prefill T=4096 split over the ranks), max-over-ranks device time.
            "sharded": {
                "decode_b8": {"us_per_call": secondary["decode_b8"]["us_per_call"],
                              "tokens_per_s": secondary["decode_b8"]["tokens_per_s"],
                              "tokens_per_rank": secondary["decode_b8"]["tokens_per_rank"],
                              "per_gpu_roofline_frac": secondary["decode_b8"]["GBps_per_rank"] / peak},
                **({"prefill_t4096": {"ms_per_call": secondary["prefill_t4096"]["ms_per_call"],
                                      "tokens_per_s": secondary["prefill_t4096"]["tokens_per_s"],
                                      "tokens_per_rank": secondary["prefill_t4096"]["tokens_per_rank"],
                                      "per_gpu_tflops": secondary["prefill_t4096"]["tflops"]}}
                   if "prefill_t4096" in secondary else {})},
            "gpu_launches": K * launches_per_call,
            "cache_replicas_identical_across_ranks": cache_identical,
            "clocks": {"sm_mhz": clocks["sm_mhz"], "sm_max_mhz": clocks["sm_max_mhz"], "reasons": clocks["reasons"],
                       "samples": clocks["samples"]},
            "secondary": secondary,
            "device_error_word": err,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)


CPU_INDEX_SEED = 99   # the B=1 index sets both CPU legs time (the headline's rank-0 seed)


def pool_topk_line(dev, peak_gbs, flush):
    """Indexer pool top-k + expansion.  8 rows (a decode step): 64 calls per
    CUDA graph replay, each on its own logits (64 x 2 MB, more than L2), so
    the per-call mean is finer than the 2.048-us event tick; 2048 rows: one
    call per replay.  L2 flushed before each replay; the torch.topk path is
    timed the same way."""
    from kernels.titan_indexer import pool_topk_expand
    P, k, pool, width = 65536, 512, 4, 2176
    out = {}
    for T, J in ((8, 64), (2048, 1)):
        g = torch.Generator(device=dev).manual_seed(T)
        sets = torch.randn(J, T, P, generator=g, device=dev)
        logits = sets[0]
        seq = torch.randint(P * pool - 3, P * pool + 1, (T,), generator=g, device=dev, dtype=torch.int32)
        res = torch.empty(T, width, dtype=torch.int32, device=dev)

        def ours():
            for j in range(J):
                pool_topk_expand(sets[j], seq, k, pool, width, out=res)
        gr, _ = capture(ours)
        timed_cold(lambda i: gr.replay(), 2, flush)
        ms = statistics.median(timed_cold(lambda i: gr.replay(), 5, flush)) / J
        gr.reset()
        pool_topk_expand(logits, seq, k, pool, width, out=res)
        # torch.topk over the pools each row may use, then the expansion
        npool = (seq // pool).clamp(max=P)
        ar = torch.arange(P, device=dev)
        offs = torch.arange(pool, device=dev)

        def torch_path(lg=logits):
            masked = torch.where(ar[None, :] < npool[:, None], lg, torch.full_like(lg, -float("inf")))
            idx = torch.topk(masked, k, dim=1).indices
            tok = (idx[:, :, None] * pool + offs).reshape(T, -1)
            tail = (npool * pool)[:, None] + offs[None, :pool - 1]
            tail = torch.where(offs[None, :pool - 1] < (seq % pool)[:, None], tail, -1)
            pad = torch.full((T, width - k * pool - pool + 1), -1, device=dev, dtype=torch.int64)
            return torch.cat([tok, tail, pad], 1).to(torch.int32)

        def theirs():
            for j in range(J):
                torch_path(sets[j])
        gt, _ = capture(theirs)
        timed_cold(lambda i: gt.replay(), 2, flush)
        ms_t = statistics.median(timed_cold(lambda i: gt.replay(), 5, flush)) / J
        gt.reset()
        nbytes = T * P * 4 + T * width * 4
        out[f"T{T}"] = {"us": ms * 1000, "GBps": nbytes / (ms * 1e-3) / 1e9,
                        "frac_of_hbm": nbytes / (ms * 1e-3) / 1e9 / peak_gbs,
                        "torch_topk_expand_us": ms_t * 1000,
                        "equal_to_torch_path": bool(torch.equal(res, torch_path()))}
        del sets
    out["shape"] = f"T rows x {P} pools of {pool}, k={k}, width={width}, seq_len in [{P * pool - 3}, {P * pool}]"
    out["timing"] = "8 rows: 64 calls per graph replay on 64 logit sets (per-call mean); 2048 rows: one call per replay"
    return out


def moe_gemm_setup(dev, M, N2, K, E=288, top_k=8, seed=5, keep_codes=False):
    """Random uint4b8 expert codes, bf16 group scales, Zipf(1.1) routes split
    by split_align.  Returns (run, useful_flops, weight_bytes_touched, parts):
    run() issues the four list GEMMs into parts["c"]; parts also holds a, the
    lists and, with keep_codes, the codes and scales (for the Marlin line)."""
    from kernels import titan_moe_split_align as split_mod
    from kernels.titan_moe_gemm import moe_w4a16_gemm, pack_weights
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randint(0, 16, (E, N2, K), generator=g, device=dev, dtype=torch.uint8)
    packed = pack_weights(q)
    scales = (torch.rand(E, K // 128, N2, generator=g, device=dev) * 0.02 + 0.002).to(torch.bfloat16)
    gc = torch.Generator().manual_seed(seed)
    w = torch.arange(1, E + 1, dtype=torch.float64) ** -1.1
    routes = torch.stack([torch.multinomial(w, top_k, replacement=False, generator=gc) for _ in range(M)])
    routes = routes.to(torch.int32).to(dev)
    buf = split_mod.buffers(M * top_k, E, dev)
    lists = split_mod.split_align(routes, E, buf)
    a = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
    c = torch.empty(M * top_k, N2, dtype=torch.bfloat16, device=dev)

    def run():
        for bs, s_ids, e_ids, n in lists:
            moe_w4a16_gemm(a, c, packed, scales, s_ids, e_ids, n, None, bs, top_k, False, M, N2, K)
    experts = int(torch.unique(routes).numel())
    parts = {"a": a, "c": c, "lists": lists, "routes": routes, "top_k": top_k}
    if keep_codes:
        parts.update(q=q, scales=scales)
    else:
        del q
    return run, 2.0 * M * top_k * N2 * K, experts * N2 * K // 2 + experts * (K // 128) * N2 * 2, parts


def moe_gemm_line(dev, peak_gbs, gm, marlin=True):
    """us per call of the four list GEMMs (one graph replay, L2 flushed
    before each), useful TFLOP/s and the roofline: time bound = max(useful
    FLOPs / bf16 peak, weight + scale bytes / HBM peak).  With marlin, the
    same codes, scales, activations and lists through vLLM's Marlin MoE GEMM
    (the reference's kernel for this step) on the same GPU, and how far the
    two outputs are apart."""
    M, N2, K = 2304, 4096, 4096
    run, flops, wbytes, parts = moe_gemm_setup(dev, M, N2, K, keep_codes=marlin)
    flush = Flusher(dev)
    g, _ = capture(run)
    timed_cold(lambda k: g.replay(), 2, flush)
    ms = statistics.median(timed_cold(lambda k: g.replay(), 5, flush))
    g.reset()
    tf_peak = 1648.6
    try:
        tf_peak = float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
    except (OSError, ValueError, KeyError):
        pass
    bound_us = max(flops / (tf_peak * 1e12), wbytes / (peak_gbs * 1e9)) * 1e6
    out = {"shape": f"M={M} tokens x top-8, 288 experts, 2N={N2}, K={K}, Zipf(1.1) routes, four lists",
           "us_per_call": ms * 1000, "useful_tflops": flops / (ms * 1e-3) / 1e12,
           "weight_GBps": wbytes / (ms * 1e-3) / 1e9, "roofline_bound_us": bound_us,
           "frac_of_roofline": bound_us / (ms * 1000), "bf16_peak_tflops": tf_peak}
    if marlin:
        try:
            out["vllm_marlin_b200"] = marlin_line(parts, M, N2, K, flush, flops)
        except Exception as exc:  # a library that does not load or launch here is reported, not fatal
            out["vllm_marlin_b200"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    return out


# The reference's thread configuration for its stock split path: block
# size -> (thread_k, thread_n, blocks_per_sm) (profiles/sm74/titan_prefill/
# marlin.py:100-102, :136-140); other block sizes let the op choose.
MARLIN_THREAD_CFG = {64: (64, 256, 1)}


def marlin_weights(q, scales):
    """Codes q (uint8 [E, N, K], 0..15, CUDA) and bf16 scales [E, K/128, N]
    -> vLLM Marlin MoE operands: per expert, GPTQ words int32 [K/8, N]
    (k = 8i + j in bits 4j..4j+3) repacked by gptq_marlin_repack, and the
    scales permuted by marlin_moe_permute_scales."""
    from vllm import _custom_ops as ops
    from vllm.model_executor.layers.quantization.utils.marlin_utils import marlin_moe_permute_scales
    E, N, K = q.shape
    perm = torch.empty(0, dtype=torch.int32, device=q.device)
    shifts = torch.arange(0, 32, 4, dtype=torch.int64, device=q.device)
    w = torch.empty(E, K // 16, N * 2, dtype=torch.int32, device=q.device)
    for e in range(E):
        words = (q[e].t().reshape(K // 8, 8, N).to(torch.int64) << shifts[None, :, None]).sum(1)
        words = torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)
        w[e] = ops.gptq_marlin_repack(words.contiguous(), perm, K, N, 4)
    return w, marlin_moe_permute_scales(scales, K, N, 128)


def marlin_line(parts, M, N2, K, flush, flops):
    """vLLM's moe_wna16_marlin_gemm over the four lists exactly as the
    reference's stock split path calls it (profiles/sm74/titan_prefill/
    marlin.py:427-437, gate/up form), timed like ours; the outputs are
    compared element by element with ours."""
    from vllm import _custom_ops as ops
    from vllm.model_executor.layers.quantization.utils.marlin_utils import marlin_make_workspace_new
    from vllm.scalar_type import scalar_types
    dev = parts["a"].device
    w, s = marlin_weights(parts["q"], parts["scales"])
    del parts["q"]
    a, lists, top_k = parts["a"], parts["lists"], parts["top_k"]
    c = torch.zeros(M * top_k, N2, dtype=torch.bfloat16, device=dev)
    ws = marlin_make_workspace_new(dev, 4)
    tw = torch.ones(M, top_k, dtype=torch.float32, device=dev)

    def run():
        for bs, s_ids, e_ids, n in lists:
            tk, tn, bps = MARLIN_THREAD_CFG.get(bs, (-1, -1, -1))
            ops.moe_wna16_marlin_gemm(
                a, c, w, None, s, None, None, None, None, None, ws, s_ids, e_ids, n, tw,
                moe_block_size=bs, top_k=top_k, mul_topk_weights=False, b_q_type=scalar_types.uint4b8,
                size_m=M, size_n=N2, size_k=K, is_k_full=True, use_atomic_add=False, use_fp32_reduce=True,
                is_zp_float=False, thread_k=tk, thread_n=tn, blocks_per_sm=bps)
    try:
        gr, _ = capture(run)
        step, how = (lambda k: gr.replay()), "one CUDA graph replay of the four calls"
    except Exception:
        gr, step, how = None, (lambda k: run()), "four eager calls"
    timed_cold(step, 2, flush)
    ms = statistics.median(timed_cold(step, 5, flush))
    if gr is not None:
        gr.reset()
    ours = parts["c"].float()
    ref = c.float()
    listed = torch.zeros(M * top_k, dtype=torch.bool, device=dev)
    for bs, s_ids, e_ids, n in lists:
        ids = s_ids[: int(n.item())].long()
        listed[ids[ids < M * top_k]] = True
    d = (ours[listed] - ref[listed]).abs()
    rel = d / ref[listed].abs().clamp_min(1e-30)
    return {"us_per_call": ms * 1000, "useful_tflops": flops / (ms * 1e-3) / 1e12, "timing": how,
            "thread_cfg": "reference table {64: (64, 256, 1)}, others chosen by the op",
            "outputs_max_abs_diff": d.max().item(), "outputs_max_abs": ref[listed].abs().max().item(),
            "outputs_frac_differing": (d > 0).float().mean().item(),
            "outputs_within_one_bf16_step": bool(((rel <= 2 ** -7) | (d <= 2 ** -8 * ref[listed].abs().max())).all())}


def load_reference_triton():
    """The reference's own modules (titan_kv, titan_mla, titan_moe_align) from
    baseline/_ref, the unmodified package pip-installed from the reference
    checkout, loaded under private names; None when it is not installed."""
    import importlib.util
    ref_dir = ROOT / "baseline" / "_ref"
    mods = {}
    for name in ("titan_kv", "titan_mla", "titan_moe_align"):
        path = ref_dir / f"{name}.py"
        if not path.exists():
            return None
        spec = importlib.util.spec_from_file_location(f"reference_{name}", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mods[name] = mod
    return mods


def reference_triton_b200(ref, kvs, lat, slots, flush, sms, K, ours):
    """The reference's Triton kernels JIT-compiled for this B200 and called
    through their public API (its split heuristic, autotuner and merge kernel
    included), on the same inputs and timing protocol as our lines: a
    comparison of the two implementations on one box, not a shipped path
    (the reference targets SM80; no Triton runs on our path)."""
    from kernels.titan_mla import triton_mla_sparse_attention as attn
    mla, kv, moe = ref["titan_mla"], ref["titan_kv"], ref["titan_moe_align"]
    out = {"what": "reference Triton on B200 (not a shipped sm_100 path): baseline/_ref, public API, "
                   "same inputs and protocol as the lines above"}
    dev = kvs[0].device
    # Same inputs, both implementations: outputs within the path tolerance.
    q, idx = decode_sets(8, 1, 4321, tail_mode="random")
    q, idx = q[0].to(dev), idx[0].to(dev)
    a = attn(q, kvs[0], idx, SM_SCALE, sm_count=sms).float()
    b = mla.triton_mla_sparse_attention(q, kvs[0], idx, SM_SCALE, sm_count=sms).float()
    out["b8_outputs_max_abs_diff"] = float((a - b).abs().max())
    out["b8_outputs_within_tolerance"] = bool(((a - b).abs() <= 2e-2 + 1e-2 * b.abs()).all())
    J = graph_calls(K)
    d1 = DecodeBench(mla.triton_mla_sparse_attention, kvs, 1, J, 99, "fixed", sms)
    d1.time(1, flush)
    out["decode_b1_us_per_call"] = sum(d1.time(max(1, K // J), flush)) / (max(1, K // J) * J) * 1000.0
    d1.close()
    J8 = graph_calls(min(K, 256))
    d8 = DecodeBench(mla.triton_mla_sparse_attention, kvs, 8, J8, 777, "random", sms)
    d8.time(1, flush)
    out["decode_b8_us_per_call"] = sum(d8.time(max(1, min(K, 256) // J8), flush)) / (
        max(1, min(K, 256) // J8) * J8) * 1000.0
    d8.close()
    ip = prefill_indices(4096, 4242).to(dev)
    qp = torch.randn(4096, HEADS, 512, device=dev, generator=torch.Generator(device=dev).manual_seed(5)).to(
        torch.bfloat16)
    run = lambda k: mla.triton_mla_sparse_attention(qp, kvs[0], ip, SM_SCALE, sm_count=sms)  # noqa: E731
    timed_cold(run, 2, flush)
    out["prefill_t4096_ms_per_call"] = statistics.fmean(timed_cold(run, 3, flush))
    cache = torch.empty(KV_ROWS // BLOCK, BLOCK, ROW_BYTES, dtype=torch.int8, device=dev)
    a_ev, b_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for perm in (False, True):
        sl = torch.randperm(KV_ROWS, device=dev) if perm else slots
        for _ in range(2):
            kv.store_int8(lat, cache, sl)
        a_ev.record()
        for _ in range(10):
            kv.store_int8(lat, cache, sl)
        b_ev.record()
        torch.cuda.synchronize()
        us = a_ev.elapsed_time(b_ev) * 100.0
        out["store_int8_random_perm_us" if perm else "store_int8_us"] = us
        if not perm:
            out["store_int8_GBps"] = KV_ROWS * (1024 + ROW_BYTES + 8) / (us * 1e-6) / 1e9
            # Bytes against ours: the reference divides with an approximate
            # fp32 division (its own test allows +-1), ours with the IEEE one.
            diff = (cache.view(-1, ROW_BYTES)[:, :512].int() - ours.view(-1, ROW_BYTES)[:, :512].int()).abs()
            out["store_int8_int8_values_differing"] = int((diff > 0).sum())
            out["store_int8_int8_max_abs_diff"] = int(diff.max())
    gm = torch.Generator().manual_seed(37)
    for B in (1, 8):
        ids = torch.stack([torch.randperm(288, generator=gm)[:8] for _ in range(B)]).to(torch.int32).to(dev)
        gr, _ = capture(lambda: moe.titan_moe_align_small(ids))
        for _ in range(5):
            gr.replay()
        samples = []
        for _ in range(5):
            a_ev.record()
            for _ in range(100):
                gr.replay()
            b_ev.record()
            torch.cuda.synchronize()
            samples.append(a_ev.elapsed_time(b_ev) * 1000 / 100)
        out[f"moe_align_B{B}_us"] = statistics.median(samples)
        gr.reset()
        g100, _ = capture(lambda: [moe.titan_moe_align_small(ids) for _ in range(100)])
        g100.replay()
        samples = []
        for _ in range(5):
            a_ev.record()
            g100.replay()
            b_ev.record()
            torch.cuda.synchronize()
            samples.append(a_ev.elapsed_time(b_ev) * 1000 / 100)
        out[f"moe_align_B{B}_in_graph_us"] = statistics.median(samples)
        g100.reset()
    return out


def cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def pin_malloc():
    """Fix glibc's malloc thresholds for the CPU legs.  Each oracle call
    allocates about 13 MB of temporaries (the gathered rows as fp32, the
    products); glibc serves a block from the heap only when it is below its
    mmap threshold, which starts at 128 KB and rises to the size of the
    largest mmapped block freed so far (at most 32 MB).  Left dynamic, the
    temporaries are mmapped and page-faulted afresh on every call in a process
    that never freed a larger block, and recycled in one that did, a 2.6x
    difference in per-call time that depends only on what the process did
    before.  Setting both thresholds makes every process recycle them."""
    import ctypes
    try:
        libc = ctypes.CDLL("libc.so.6")
    except OSError:
        return False
    m_trim_threshold, m_mmap_threshold = -1, -3
    return bool(libc.mallopt(m_mmap_threshold, 32 << 20)) and bool(libc.mallopt(m_trim_threshold, 1 << 30))


def time_cpu_port(rows, steps, seconds, sets=64):
    """One protocol for both CPU legs (the reference arm and the cpu_baseline
    key): the oracle (CPU restatement of the reference algorithm, torch fp32,
    all host threads) on `sets` distinct config-2 B=1 index sets (seed
    CPU_INDEX_SEED); one untimed pass over every set, then blocks of `steps`
    calls (set k % sets) repeated until at least `seconds` have elapsed.
    Returns (us per call, calls timed, seconds timed, threads)."""
    from oracle import oracle as O
    pin_malloc()
    torch.set_num_threads(os.cpu_count() or 1)
    # Both legs time against a fresh copy made by torch's parallel clone, so
    # the 138 MB of rows are first touched (and placed in memory) the same
    # way whichever single-threaded path produced them.
    rows = torch.as_tensor(rows).contiguous().clone()
    q_sets, idx_sets = decode_sets(1, sets, CPU_INDEX_SEED)
    for k in range(sets):
        O.mla_sparse_attention(q_sets[k], rows, idx_sets[k], SM_SCALE)
    n, t0 = 0, time.perf_counter()
    while True:
        for _ in range(steps):
            O.mla_sparse_attention(q_sets[n % sets], rows, idx_sets[n % sets], SM_SCALE)
            n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    return dt / n * 1e6, n, dt, torch.get_num_threads()


def cpu_baseline_b1(cache, steps, seconds):
    """The oracle on the same B=1 workload as the reference arm (same index
    sets, same protocol: time_cpu_port), over the cache the GPU built."""
    rows = cache.view(KV_ROWS, ROW_BYTES).cpu()
    us, n, dt, cores = time_cpu_port(rows, steps, seconds)
    return {"value": us, "unit": UNIT, "cores": cores, "kind": "port", "cpu_model": cpu_model(),
            "sample": f"{n} B=1 calls of oracle.mla_sparse_attention over the 262144-row cache in {dt:.1f} s: "
                      f"64 index sets (seed {CPU_INDEX_SEED}) each run once untimed, then blocks of {steps} calls "
                      "until the time bound (torch CPU fp32, all host threads, glibc malloc thresholds pinned)"}


# ------------------------------------------------------------ reference arm
def run_reference(args):
    """CPU restatement of the reference algorithm (oracle/) on the host cores:
    the cache is filled by the oracle's store_int8 (C restatement) from the
    same-shape latents, then the B=1 calls are timed with time_cpu_port (the
    protocol of the cpu_baseline key of our arm)."""
    import numpy as np
    from oracle import c_oracle
    from oracle import oracle as O
    g = torch.Generator().manual_seed(1234)
    lat = torch.randn(KV_ROWS, 512, generator=g).to(torch.bfloat16)
    bits = np.ascontiguousarray(O.tensor_bf16_bits(lat))
    rows = np.zeros((KV_ROWS, ROW_BYTES), np.uint8)
    t0 = time.perf_counter()
    c_oracle().oracle_store_int8_rows(bits.ctypes.data, KV_ROWS, rows.ctypes.data)
    fill_s = time.perf_counter() - t0
    us, n, dt, cores = time_cpu_port(torch.from_numpy(rows), args.steps, args.cpu_seconds)
    line = {
        "metric": METRIC, "value": us, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": us / 1000, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": "config2: B=1 sparse MLA decode, 16 heads x 512 NoPE latent, 262144-row INT8 "
                               "528-B-row cache filled by store_int8, 2176 indices (2048 distinct valid + 128 x -1)",
                   "index_sets": 64},
        "cpu_baseline": {"value": us, "unit": UNIT, "cores": cores, "kind": "port", "cpu_model": cpu_model(),
                         "sample": f"{n} B=1 calls of the CPU restatement (torch fp32) in {dt:.1f} s: 64 index "
                                   f"sets (seed {CPU_INDEX_SEED}) each run once untimed, then blocks of "
                                   f"{args.steps} calls until the time bound (glibc malloc thresholds pinned); cache fill "
                                   "by the C restatement "
                                   f"of store_int8 took {fill_s:.2f} s single-threaded"},
        "e2e": {"value": us, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_profile(args):
    """Only the chosen workload's calls, eager and without L2 flushes (ncu
    flushes caches itself between replay passes); prints nothing.  Used as the
    target of the ncu captures summarised under profiles/."""
    from kernels.titan_kv import store_int8
    from kernels.titan_mla import triton_mla_sparse_attention as attn
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n = args.warmup + args.steps
    if args.profile == "pool_topk":  # decode shape: 8 rows x 65,536 pools
        from kernels.titan_indexer import pool_topk_expand
        logits = torch.randn(8, 65536, device=dev)
        seq = torch.full((8,), 262144, dtype=torch.int32, device=dev)
        for _ in range(n):
            pool_topk_expand(logits, seq)
        torch.cuda.synchronize()
        return
    if args.profile == "moe_gemm":  # the four list GEMMs; small: M = 512 tokens, 2N = 1024, K = 4096
        run, _, _, _ = moe_gemm_setup(dev, 512, 1024, 4096)
        for _ in range(n):
            run()
        torch.cuda.synchronize()
        return
    if args.profile == "moe_align":  # config 5: B = 1 and B = 8 decode tokens x top-8 of 288 experts
        from kernels.titan_moe_align import titan_moe_align_small
        gm = torch.Generator().manual_seed(37)
        sets = [torch.stack([torch.randperm(288, generator=gm)[:8] for _ in range(B)]).to(torch.int32).to(dev)
                for B in (1, 8)]
        for _ in range(n):
            for ids in sets:
                titan_moe_align_small(ids)
        torch.cuda.synchronize()
        return
    if args.profile == "split_align":  # M = 2304 tokens x top-8, 288 uniform experts
        from kernels import titan_moe_split_align as split_mod
        g = torch.Generator().manual_seed(1)
        ids = torch.randint(0, 288, (2304, 8), generator=g, dtype=torch.int32).to(dev)
        sbuf = split_mod.buffers(2304 * 8, 288, dev)
        for _ in range(n):
            split_mod.split_align(ids, 288, sbuf)
        torch.cuda.synchronize()
        return
    lat = latents(KV_ROWS, 1234, dev)
    cache = torch.zeros(KV_ROWS // BLOCK, BLOCK, ROW_BYTES, dtype=torch.int8, device=dev)
    slots = torch.arange(KV_ROWS, device=dev)
    store_int8(lat, cache, slots)
    kv = cache.view(KV_ROWS, 1, ROW_BYTES)
    if args.profile == "store_int8":
        for _ in range(n):
            store_int8(lat, cache, slots)
    elif args.profile in ("decode_b1", "decode_b8"):
        batch = 1 if args.profile == "decode_b1" else 8
        q, idx = decode_sets(batch, 8, 99, tail_mode="fixed" if batch == 1 else "random")
        q, idx = q.to(dev), idx.to(dev)
        for k in range(n):
            attn(q[k % 8], kv, idx[k % 8], SM_SCALE)
    elif args.profile == "paged_b1":
        from kernels.titan_index import triton_convert_req_index_to_global_index as conv
        from kernels.titan_mla import triton_mla_sparse_attention_paged as attn_paged
        g = torch.Generator().manual_seed(77)
        bt = torch.randperm(KV_ROWS // 64, generator=g).to(torch.int32).view(1, -1).to(dev)
        tok = torch.full((1, TOPK), -1, dtype=torch.int32)
        tok[0, :VALID] = torch.randperm(KV_ROWS, generator=g)[:VALID].to(torch.int32)
        tok = tok.to(dev)
        req = torch.zeros(1, dtype=torch.int32, device=dev)
        q1 = torch.randn(1, HEADS, 512, generator=g).to(torch.bfloat16).to(dev)
        for _ in range(n):  # fused call, then conversion + reader
            attn_paged(q1, kv, tok, req, bt, 64, SM_SCALE)
            glob = conv(req, bt, tok, BLOCK_SIZE=64, NUM_TOPK_TOKENS=TOPK)
            attn(q1, kv, glob.view(1, 1, TOPK), SM_SCALE)
    elif args.profile == "prefill":
        tp = 512
        ip = prefill_indices(tp, 4242, t0=1024).to(dev)
        qp = torch.randn(tp, HEADS, 512, device=dev).to(torch.bfloat16)
        for _ in range(n):
            attn(qp, kv, ip, SM_SCALE)
    torch.cuda.synchronize()


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=None)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="time bound of both CPU legs (reference arm and cpu_baseline)")
    ap.add_argument("--skip-prefill", action="store_true")
    ap.add_argument("--skip-cpu-baseline", action="store_true")
    ap.add_argument("--skip-moe-gemm", action="store_true")
    ap.add_argument("--skip-reference-triton", action="store_true",
                    help="skip the secondary lines of the reference's Triton kernels run on this GPU")
    ap.add_argument("--profile", choices=("decode_b1", "decode_b8", "store_int8", "prefill", "paged_b1", "split_align",
                                          "moe_gemm", "pool_topk", "moe_align"),
                    default=None,
                    help="run only this workload (warmup + steps calls) as an ncu target; prints nothing")
    args = ap.parse_args()
    rank, world, local_rank = env_rank()
    if args.gpus is None:
        args.gpus = world
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.profile is not None:
        run_profile(args)
        return 0
    if args.impl == "reference":
        if rank == 0:
            run_reference(args)
        return 0
    dist = Dist(world, rank, local_rank)
    try:
        run_ours(args, dist)
    finally:
        dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
