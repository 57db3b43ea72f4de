// Split MoE block alignment for whole-expert prefill (Marlin W4A16 MoE).
//
// Output contract of profiles/sm74/titan_prefill/moe_split_align.py:204-223
// (`split_align`, five Triton kernels :44-169).  The T = M * topk routed rows
// are sorted by expert into four block lists, one per block size B_k in
// {64, 48, 32, 16}:
//   r_e            valid rows of expert e (ids narrowed to int32, then 0 <= id < E)
//   n_k(e)         cover_tab[r_e][k], the cheapest multiset of blocks covering r_e
//   rows_k(e)      n_k * B_k;  off_k(e) = exclusive prefix of rows_k over experts
//   lo1, lo2, lo3  rank boundaries rows_0, rows_0 + rows_1, rows_0 + rows_1 + rows_2
//   ntpp[k]        sum over experts of rows_k
//   fill (:102-135)  the last non-empty list of an expert pads its tail with the
//                    sentinel T; each list's blocks get the expert id
//   scatter (:138-169) the row with flat index j and stable rank q within its
//                    expert goes to list k = the range [lo_k, lo_k+1) holding q,
//                    at sorted_k[off_k(e) + q - lo_k] = j
// Entries outside what the algorithm writes are left untouched.
//
// B200 design: ONE launch of one thread-block cluster (16 CTAs of 1024
// threads where the device holds such a cluster, else 8) instead of five
// kernels with a global histogram.  Warp w of the cluster (CTA-major order)
// owns the w-th contiguous slice of the routes; its expert counts live in a
// private shared-memory histogram (no atomics: peer masks of equal ids,
// built from one ballot per id bit, give in-group ranks; the group leader
// adds the popcount).  Each CTA sums its
// warps' counts per expert and publishes the totals in its shared memory;
// after a cluster barrier every CTA reads the lower CTAs' totals through
// distributed shared memory, so prefix (CTA) + prefix (warp) is each slice's
// stable-rank base and the sum over CTAs is r_e.  Every CTA computes the
// plan (a CTA-wide scan of four counters per expert, E <= 1024) itself; the
// fill takes one warp per expert across the cluster.  Fill and scatter need
// no barrier between them (they write disjoint entries); a split cluster
// barrier (arrive after the last remote read, wait at the end) keeps every
// CTA resident until its peers' remote reads are done.  Each lane loads eight
// groups of route ids before using them.
#include "titan_common.cuh"

#include <cstdlib>

namespace titan {

constexpr int kSplitThreads = 1024;
constexpr int kSplitWarps = kSplitThreads / 32;
constexpr int kSplitMaxExperts = TITAN_SPLIT_ALIGN_MAX_EXPERTS;
constexpr int kSplitBatch = 8;  // route groups loaded per lane before use
// Shared memory: 32 warp histograms (rows of E | 1 words: an odd stride, so
// one expert's column is read without bank conflicts) + per expert the CTA
// total, r, the lower CTAs' rows, 4 list offsets and 3 rank boundaries.
constexpr int kSplitWordsPerExpert = 1 + 1 + 1 + 4 + 3;
__host__ __device__ constexpr int split_hist_stride(int E) { return E | 1; }
constexpr int kSplitClusterMax = 16;

// Full cluster barrier: release this CTA's prior memory operations, acquire
// the peers'.
__device__ __forceinline__ void split_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t split_cluster_size() {
  uint32_t n;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
  return n;
}
__device__ __forceinline__ int split_ld_dsmem(uint32_t addr) {
  int v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

struct SplitLists {
  int32_t *s0, *s1, *s2, *s3;
  int32_t *e0, *e1, *e2, *e3;
};

// Lanes of the warp holding the same valid expert id as this lane (e >= 0),
// else this lane alone: the peer mask of a match-any over the ids, built from
// one ballot per id bit (nbits = bits of E - 1), which on this GPU is far
// cheaper than match-any over ~30 distinct values.
__device__ __forceinline__ unsigned split_peers(int e, int nbits, int lane) {
  unsigned m = __ballot_sync(0xffffffffu, e >= 0);
  for (int b = 0; b < nbits; ++b) {  // warp-uniform trip count
    const bool bit = (e >> b) & 1;
    const unsigned v = __ballot_sync(0xffffffffu, bit);
    m &= bit ? v : ~v;
  }
  return e >= 0 ? m : (1u << lane);
}

__device__ __forceinline__ int split_block_size(int k) { return k == 0 ? 64 : k == 1 ? 48 : k == 2 ? 32 : 16; }

template <typename IdT>
__device__ __forceinline__ int split_route_expert(const IdT *ids, int j, int end, int E) {
  if (j >= end) return -1;
  // The reference narrows the ids to int32 before validating them (:207-209).
  const int v = (int)(uint32_t)(unsigned long long)(long long)ids[j];
  return (v >= 0 && v < E) ? v : -1;
}

__device__ __forceinline__ void split_fill_list(int k, int expert, int r, int off, int lo, int hi, bool last,
                                                int T, int64_t cap_s, int64_t cap_e, int32_t *s, int32_t *e,
                                                int lane) {
  const int bs = split_block_size(k);
  const int rows = hi - lo;
  const int pad = last ? hi - r : 0;
  const int pad_n = min(pad, 64);  // the reference pads at most 64 entries (:107-108)
  for (int j = lane; j < pad_n; j += 32) {
    const int64_t p = (int64_t)off + rows - pad + j;
    if (p >= 0 && p < cap_s) s[p] = T;
  }
  const int nblk = rows / bs;
  for (int b = lane; b < nblk; b += 32) {
    const int64_t p = (int64_t)(off / bs) + b;
    if (p >= 0 && p < cap_e) e[p] = expert;
  }
}

template <typename IdT>
__global__ void __launch_bounds__(kSplitThreads, 1)
    moe_split_align_kernel(const IdT *__restrict__ ids, int T, int E, const int32_t *__restrict__ cover_tab,
                           int64_t t_max, SplitLists out, int32_t *__restrict__ ntpp) {
  extern __shared__ int split_smem[];
  const int hs = split_hist_stride(E);
  int *hist = split_smem;                // [32][hs]: slice counts, then rank bases within the CTA
  int *total = hist + kSplitWarps * hs;  // [E]      this CTA's rows per expert (read by peers)
  int *count = total + E;                // [E]      r_e
  int *below = count + E;                // [E]      rows of this expert in lower CTAs
  int *off = below + E;                  // [4][E]   list offsets
  int *lo = off + 4 * E;                 // [3][E]   lo1, lo2, lo3
  __shared__ int4 warp_total[kSplitWarps];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cta = (int)cluster_ctarank(), ncta = (int)split_cluster_size();
  const int gwarp = cta * kSplitWarps + warp, nwarps = ncta * kSplitWarps;
  const unsigned lower = (1u << lane) - 1u;
  const int nbits = E > 1 ? 32 - __clz(E - 1) : 0;
  pdl_launch_dependents();
  for (int i = tid; i < kSplitWarps * hs; i += kSplitThreads) hist[i] = 0;
  pdl_wait_primary();  // the route ids come from earlier kernels; the lists are rewritten below
  __syncthreads();

  // Pass 1: per-slice expert counts.
  const int per_warp = (T + nwarps - 1) / nwarps;
  const int beg = min(gwarp * per_warp, T), end = min(beg + per_warp, T);
  int *my_hist = hist + warp * hs;
  for (int g0 = beg; g0 < end; g0 += 32 * kSplitBatch) {
    int ex[kSplitBatch];
#pragma unroll
    for (int b = 0; b < kSplitBatch; ++b) ex[b] = split_route_expert(ids, g0 + 32 * b + lane, end, E);
#pragma unroll
    for (int b = 0; b < kSplitBatch; ++b) {
      if (g0 + 32 * b >= end) break;  // warp-uniform
      const unsigned peers = split_peers(ex[b], nbits, lane);  // invalid lanes match nobody
      if (ex[b] >= 0 && (peers & lower) == 0) my_hist[ex[b]] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();

  // Per expert (one warp per expert, lane w = slice w): exclusive prefix of
  // the slice counts over this CTA's warps, and the CTA total.
  // Four experts at a time, so their shuffle chains overlap.
  for (int x0 = warp; x0 < E; x0 += 4 * kSplitWarps) {
    int h[4], inc[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int x = x0 + u * kSplitWarps;
      h[u] = x < E ? hist[lane * hs + x] : 0;
      inc[u] = h[u];
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = __shfl_up_sync(0xffffffffu, inc[u], o);
        if (lane >= o) inc[u] += t;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int x = x0 + u * kSplitWarps;
      if (x < E) {
        hist[lane * hs + x] = inc[u] - h[u];
        if (lane == 31) total[x] = inc[u];
      }
    }
  }
  split_cluster_sync();  // every CTA's totals are published
  // Rows of lower CTAs come first (added to the rank in the scatter); the sum
  // over all CTAs is r_e.
  for (int x = tid; x < E; x += kSplitThreads) {
    int v[kSplitClusterMax];
#pragma unroll
    for (int c = 0; c < kSplitClusterMax; ++c)  // all remote loads in flight at once
      v[c] = c < ncta ? split_ld_dsmem(dsmem_addr(&total[x], (uint32_t)c)) : 0;
    int lower_rows = 0, r = 0;
#pragma unroll
    for (int c = 0; c < kSplitClusterMax; ++c) {
      lower_rows += c < cta ? v[c] : 0;
      r += v[c];
    }
    below[x] = lower_rows;
    count[x] = r;
  }
  // This CTA reads no peer's shared memory after this point; the matching
  // wait at the end keeps every CTA resident until all peers got here.
  cluster_arrive_relaxed();
  __syncthreads();

  // Plan: rows_k per expert from the cover table, exclusive prefix over experts
  // (one expert per thread, E <= 1024), componentwise over the four lists.
  int4 rows = make_int4(0, 0, 0, 0);
  if (tid < E) {
    const int64_t r = count[tid];
    const int32_t *n = cover_tab + 4 * r;
    rows = make_int4(__ldg(n) * 64, __ldg(n + 1) * 48, __ldg(n + 2) * 32, __ldg(n + 3) * 16);
  }
  int4 inc = rows;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ax = __shfl_up_sync(0xffffffffu, inc.x, o), ay = __shfl_up_sync(0xffffffffu, inc.y, o);
    const int az = __shfl_up_sync(0xffffffffu, inc.z, o), aw = __shfl_up_sync(0xffffffffu, inc.w, o);
    if (lane >= o) inc = make_int4(inc.x + ax, inc.y + ay, inc.z + az, inc.w + aw);
  }
  if (lane == 31) warp_total[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int4 t = warp_total[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ax = __shfl_up_sync(0xffffffffu, t.x, o), ay = __shfl_up_sync(0xffffffffu, t.y, o);
      const int az = __shfl_up_sync(0xffffffffu, t.z, o), aw = __shfl_up_sync(0xffffffffu, t.w, o);
      if (lane >= o) t = make_int4(t.x + ax, t.y + ay, t.z + az, t.w + aw);
    }
    warp_total[lane] = t;
  }
  __syncthreads();
  if (tid < E) {
    const int4 base = warp > 0 ? warp_total[warp - 1] : make_int4(0, 0, 0, 0);
    off[tid] = base.x + inc.x - rows.x;
    off[E + tid] = base.y + inc.y - rows.y;
    off[2 * E + tid] = base.z + inc.z - rows.z;
    off[3 * E + tid] = base.w + inc.w - rows.w;
    lo[tid] = rows.x;
    lo[E + tid] = rows.x + rows.y;
    lo[2 * E + tid] = rows.x + rows.y + rows.z;
  }
  if (cta == 0 && tid == 0) {
    const int4 all = warp_total[kSplitWarps - 1];
    ntpp[0] = all.x;
    ntpp[1] = all.y;
    ntpp[2] = all.z;
    ntpp[3] = all.w;
  }
  __syncthreads();

  // Fill: one warp per expert; sentinel tail of the last non-empty list and
  // the expert id of every block.
  const int64_t cap_s[4] = {t_max + 64ll * E, t_max + 48ll * E, t_max + 32ll * E, t_max + 16ll * E};
  for (int x = gwarp; x < E; x += nwarps) {
    const int r = count[x], lo1 = lo[x], lo2 = lo[E + x], lo3 = lo[2 * E + x];
    const int hi3 = r > lo3 ? lo3 + (r + 15 - lo3) / 16 * 16 : lo3;
    const bool last3 = hi3 > lo3;
    const bool last2 = lo3 > lo2 && !last3;
    const bool last1 = lo2 > lo1 && lo3 == lo2 && !last3;
    const bool last0 = lo1 > 0 && lo2 == lo1 && lo3 == lo2 && !last3;
    split_fill_list(0, x, r, off[x], 0, lo1, last0, T, cap_s[0], cap_s[0] / 64 + 1, out.s0, out.e0, lane);
    split_fill_list(1, x, r, off[E + x], lo1, lo2, last1, T, cap_s[1], cap_s[1] / 48 + 1, out.s1, out.e1, lane);
    split_fill_list(2, x, r, off[2 * E + x], lo2, lo3, last2, T, cap_s[2], cap_s[2] / 32 + 1, out.s2, out.e2, lane);
    split_fill_list(3, x, r, off[3 * E + x], lo3, hi3, last3, T, cap_s[3], cap_s[3] / 16 + 1, out.s3, out.e3, lane);
  }
  // Fill and scatter write disjoint entries: the sentinels of an expert's
  // last list start at its rank r, and its rows go below r.

  // Pass 2: stable ranks and the scatter into the lists.
  for (int g0 = beg; g0 < end; g0 += 32 * kSplitBatch) {
    int ex[kSplitBatch];
#pragma unroll
    for (int b = 0; b < kSplitBatch; ++b) ex[b] = split_route_expert(ids, g0 + 32 * b + lane, end, E);
#pragma unroll
    for (int b = 0; b < kSplitBatch; ++b) {
      if (g0 + 32 * b >= end) break;  // warp-uniform
      const int e = ex[b];
      const unsigned peers = split_peers(e, nbits, lane);
      const int q = e >= 0 ? below[e] + my_hist[e] + __popc(peers & lower) : 0;
      __syncwarp();
      if (e >= 0 && (peers & lower) == 0) my_hist[e] += __popc(peers);
      __syncwarp();
      if (e >= 0) {
        const int lo1 = lo[e], lo2 = lo[E + e], lo3 = lo[2 * E + e];
        const int k = q >= lo3 ? 3 : q >= lo2 ? 2 : q >= lo1 ? 1 : 0;
        const int base = k == 3 ? lo3 : k == 2 ? lo2 : k == 1 ? lo1 : 0;
        int32_t *s = k == 3 ? out.s3 : k == 2 ? out.s2 : k == 1 ? out.s1 : out.s0;
        const int64_t p = (int64_t)off[k * E + e] + q - base;
        if (p >= 0 && p < t_max + (int64_t)split_block_size(k) * E) s[p] = g0 + 32 * b + lane;
      }
    }
  }
  cluster_wait();
}

}  // namespace titan

extern "C" int64_t titan_moe_split_align_smem_bytes(int64_t num_experts) {
  return ((int64_t)titan::kSplitWarps * (num_experts | 1) + (int64_t)titan::kSplitWordsPerExpert * num_experts) * 4;
}

extern "C" int titan_moe_split_align(const void *topk_ids, int ids_is_int64, int64_t num_routes,
                                     int64_t num_experts, const int32_t *cover_tab, int64_t cover_rows,
                                     int64_t t_max, int32_t *const *sorted_ids, int32_t *const *expert_ids,
                                     int32_t *ntpp, titan_stream_t stream) {
  using namespace titan;
  if (num_routes < 1 || num_routes > t_max || t_max > (int64_t)INT32_MAX / 2)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_split_align: need 0 < num_routes (%lld) <= t_max (%lld) < 2^30",
                (long long)num_routes, (long long)t_max);
  if (num_experts < 1 || num_experts > kSplitMaxExperts)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_split_align: num_experts must be in [1, %d], got %lld",
                kSplitMaxExperts, (long long)num_experts);
  if (cover_rows < num_routes + 1)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_split_align: cover table has %lld rows, needs num_routes + 1 = %lld",
                (long long)cover_rows, (long long)num_routes + 1);
  if (t_max + 64 * num_experts > (int64_t)INT32_MAX)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_split_align: list buffers exceed int32 indexing");
  if (topk_ids == nullptr || cover_tab == nullptr || sorted_ids == nullptr || expert_ids == nullptr ||
      ntpp == nullptr)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_split_align: null pointer");
  SplitLists out{sorted_ids[0], sorted_ids[1], sorted_ids[2], sorted_ids[3],
                 expert_ids[0], expert_ids[1], expert_ids[2], expert_ids[3]};
  for (int k = 0; k < 4; ++k)
    if (sorted_ids[k] == nullptr || expert_ids[k] == nullptr)
      return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_split_align: null list pointer %d", k);

  // Per device, once: the shared-memory opt-in for the largest expert count,
  // 16-CTA clusters allowed, and the cluster size (16 if the device can hold
  // one such cluster of 1024-thread CTAs, else the portable 8).
  static std::atomic<int> dev_cluster[64];  // 0 = not set up
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "moe_split_align: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(TITAN_ERR_CUDA, "moe_split_align: device ordinal %d out of range", dev);
  const int max_smem = (int)titan_moe_split_align_smem_bytes(kSplitMaxExperts);
  int cluster = dev_cluster[dev].load(std::memory_order_acquire);
  if (cluster == 0) {
    std::lock_guard<std::mutex> lock(setup_mutex());
    cluster = dev_cluster[dev].load(std::memory_order_relaxed);
    if (cluster == 0) {
      e = cudaSuccess;
      for (auto k : {(const void *)moe_split_align_kernel<int32_t>, (const void *)moe_split_align_kernel<long long>}) {
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      }
      if (e != cudaSuccess)
        return fail(TITAN_ERR_CUDA, "moe_split_align: device setup: %s", cudaGetErrorString(e));
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(kSplitClusterMax);
      q.blockDim = dim3(kSplitThreads);
      q.dynamicSmemBytes = (size_t)max_smem;
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = kSplitClusterMax;
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = 1;
      q.attrs = qa;
      q.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, moe_split_align_kernel<int32_t>, &q) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
      cluster = n >= 1 ? kSplitClusterMax : 8;
      // TITAN_SPLIT_ALIGN_CLUSTER=8, read here once per device, forces the
      // portable 8-CTA cluster (the fallback of devices that cannot hold 16),
      // so that path can be tested on a device that can.
      const char *force = getenv("TITAN_SPLIT_ALIGN_CLUSTER");
      if (force != nullptr && atoi(force) == 8) cluster = 8;
      dev_cluster[dev].store(cluster, std::memory_order_release);
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)cluster);
  cfg.blockDim = dim3(kSplitThreads);
  cfg.dynamicSmemBytes = (size_t)titan_moe_split_align_smem_bytes(num_experts);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const int T = (int)num_routes, E = (int)num_experts;
  if (ids_is_int64)
    e = cudaLaunchKernelEx(&cfg, moe_split_align_kernel<long long>, static_cast<const long long *>(topk_ids), T, E,
                           cover_tab, t_max, out, ntpp);
  else
    e = cudaLaunchKernelEx(&cfg, moe_split_align_kernel<int32_t>, static_cast<const int32_t *>(topk_ids), T, E,
                           cover_tab, t_max, out, ntpp);
  if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "moe_split_align launch: %s", cudaGetErrorString(e));
  return check_launch("moe_split_align launch");
}
