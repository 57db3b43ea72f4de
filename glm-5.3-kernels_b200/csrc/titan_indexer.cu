// Pool top-k of the sparse indexer and its expansion to token positions: the
// step that produces the MLA reader's 2176 indices per query token.
//
// For query row t with seq_len = position + 1 tokens (pools of `pool` tokens):
//   valid pools p < min(seq_len / pool, ld) (complete pools; the partial last
//   pool's tokens come from the tail below);
//   pools_t = the k valid pools of largest logits[t, p], ordered by logit
//   (descending; equal logits: smaller pool first; NaN ranks above every
//   number), -1 where fewer than k pools are valid;
//   out[t, pool i + o] = pools_t[i] pool + o   (-1 for a -1 pool), i < k, o < pool
//   out[t, k pool + o] = (seq_len / pool) pool + o if o < seq_len % pool, else -1,
//                        o < pool - 1  (the tail);
//   out[t, j] = -1 for the remaining columns up to `width`.
// The expansion is the reference's (tests/verify_indexer_sharding.py:68-76,
// `expand_row`; the finish block of integration/patch_indexer_sharding.py:
// 85-104 writes it into the 2176-wide index buffer); the selection is the
// CUDA top-k that precedes it (integration/patch_decode_indexer.py:49-104).
//
// B200 design: one CTA of 1024 threads per query row.  The logits become
// order-preserving unsigned keys.  Fast path: one pass over the row (eight
// loads in flight per thread) builds a histogram of the keys' top 11 bits in
// eight private copies (few hot bins would otherwise serialise the shared
// atomics); the bin holding the k-th largest key follows from a suffix scan;
// a second pass appends every key of that bin or above to a candidate list
// (warp-aggregated); one refinement pass over the candidates and bitonic
// sorts (key descending, pool ascending; unrolled networks in registers) put
// the k selected pools first, in their final order.  The cluster form (few rows) keeps each CTA's
// share of the row in registers between the two passes.  When
// more than 4096 keys reach the candidate list (heavy ties or a degenerate
// distribution), the exact multi-pass selection runs instead: three radix
// passes (11 + 11 + 10 bits) find the k-th key, keys above it are collected,
// keys equal to it are taken in pool order, and the k pairs are sorted.
#include "titan_common.cuh"

namespace titan {
namespace idx {

constexpr int kThreads = 1024;
constexpr int kMaxK = 1024;
constexpr int kBins = 2048;
constexpr int kHistCopies = 8;   // private histograms, four warps each
constexpr int kCandCap = 4096;   // candidate list of the fast path
constexpr int kUnroll = 8;       // loads in flight per thread in a pass over the row

// Float -> key whose unsigned order is the float order; every NaN (either
// sign) maps to the largest key, above +inf.
__device__ __forceinline__ uint32_t float_key(float x) {
  const uint32_t b = __float_as_uint(x);
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) return 0xFFFFFFFFu;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

struct Smem {
  uint32_t hist[kHistCopies][kBins];  // copy 0 also serves the multi-pass selection
  uint32_t key[kCandCap];             // candidates, or the selected pairs (first kMaxK)
  int32_t pool[kCandCap];
  uint32_t slice[kBins / 8];          // cluster form: this CTA's slice of the row's histogram
  uint32_t warp_sum[32];
  uint32_t bin, above, cnt;           // cnt is also the scan's total (block_exclusive_scan)
  uint32_t ccnt;                      // cluster form: CTA 0's candidate count (nothing else writes it)
  uint32_t bcnt;                      // boundary-bin entries of the split selection
};

constexpr int kClusterMax = 16;       // CTAs per row in the cluster form
constexpr int kRegVec = 2;            // cluster form: 16-byte vectors per thread kept in registers (8192 pools per CTA)
// Slice-sum rounds of the cluster form: S = kBins / C bins per CTA, kThreads / C
// of them per round, for both cluster sizes (8 and 16).
constexpr int kSliceRounds = kBins / kThreads;
static_assert((kBins / 8) / (kThreads / 8) == kSliceRounds && (kBins / 16) / (kThreads / 16) == kSliceRounds,
              "slice rounds");
static_assert(kBins / 8 >= kBins / kClusterMax && kBins % kClusterMax == 0, "histogram slices");

// Block-wide exclusive scan of one value per thread (1024 threads).
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, Smem &sm, uint32_t &total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) sm.warp_sum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = sm.warp_sum[lane], wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    sm.warp_sum[lane] = wi - w;  // exclusive prefix of the warps
    if (lane == 31) sm.cnt = wi;
  }
  __syncthreads();
  total = sm.cnt;
  const uint32_t r = sm.warp_sum[warp] + incl - v;
  __syncthreads();  // warp_sum and cnt are reused by the next call
  return r;
}

// The bin of hist (nb bins) that holds the remaining-th largest key, counting
// from the top bin: sm.bin, and the keys in the bins above it: sm.above.
__device__ __forceinline__ void find_bin(const uint32_t *hist, int nb, uint32_t remaining, Smem &sm) {
  const int tid = threadIdx.x;
  // Suffix counts from the top bin down: thread j owns bins nb - 1 - 2j and
  // nb - 2 - 2j (2048 bins over 1024 threads).
  const int b0 = nb - 1 - 2 * tid, b1 = b0 - 1;
  const uint32_t c0 = b0 >= 0 ? hist[b0] : 0u, c1 = b1 >= 0 ? hist[b1] : 0u;
  uint32_t total;
  const uint32_t above0 = block_exclusive_scan(c0 + c1, sm, total);  // keys in bins above b0
  if (b0 >= 0 && above0 < remaining && remaining <= above0 + c0) {
    sm.bin = (uint32_t)b0;
    sm.above = above0;
  }
  if (b1 >= 0 && above0 + c0 < remaining && remaining <= above0 + c0 + c1) {
    sm.bin = (uint32_t)b1;
    sm.above = above0 + c0;
  }
  __syncthreads();
}

__device__ __forceinline__ bool first_ordered(uint32_t ka, int32_t pa, uint32_t kb, int32_t pb) {
  return ka > kb || (ka == kb && pa < pb);
}

static_assert(2 * kMaxK <= kBins, "sort exchange buffers fit one histogram copy each");

// Bitonic network over the first s (<= W) pairs of keys / pools (key
// descending, pool ascending), sorted in place.  E elements per thread in
// threads lt = 0 .. W / E - 1 of the calling group (active; the others only
// take the barriers): element e = E lt + r, entries past s sort last.
// Partners closer than E are in the same thread, closer than 32 E in the
// same warp (shuffles), farther ones are exchanged through two alternating
// buffers xk / xp (2 W words each; one block barrier per such sub-stage,
// taken by every thread of the block).  Unrolled at full width: with
// run-time strides the in-thread partners became run-time register selects
// and a 1024-wide sort took ~10 us longer.  A network of W <= 32 E has no
// barrier and may run in one warp.
template <int W, int E>
__device__ __forceinline__ void sort_net(uint32_t *keys, int32_t *pools, int s, int lt, bool active, uint32_t *xk,
                                         int32_t *xp) {
  constexpr int T = W / E;
  static_assert(E == 1 || E == 2 || E == 4, "elements per thread");
  uint32_t key[E];
  int32_t pl[E];
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const int e = E * lt + r;
    key[r] = active && e < s ? keys[e] : 0u;
    pl[r] = active && e < s ? pools[e] : 0x7fffffff;
  }
  int buf = 0;
#pragma unroll
  for (int size = 2; size <= W; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride < E) {  // partner in this thread: pairs (a, a + stride), a & stride == 0
        if (active) {
#pragma unroll
          for (int a = 0; a < E; ++a) {
            if (a & stride) continue;
            const int b = a + stride;
            const bool asc = ((E * lt + a) & size) == 0;  // this pair's lower slot takes the first-ordered
            if (first_ordered(key[a], pl[a], key[b], pl[b]) != asc) {
              const uint32_t tk = key[a];
              key[a] = key[b];
              key[b] = tk;
              const int32_t tp = pl[a];
              pl[a] = pl[b];
              pl[b] = tp;
            }
          }
        }
        continue;
      }
      const int ts = stride / E;  // partner thread: lt ^ ts, same r
      uint32_t ok[E];
      int32_t op[E];
      if (ts < 32) {
        if (active) {
#pragma unroll
          for (int r = 0; r < E; ++r) {
            ok[r] = __shfl_xor_sync(0xffffffffu, key[r], ts);
            op[r] = __shfl_xor_sync(0xffffffffu, pl[r], ts);
          }
        }
      } else {
        if (active) {
#pragma unroll
          for (int r = 0; r < E; ++r) {
            xk[(buf * T + lt) * E + r] = key[r];
            xp[(buf * T + lt) * E + r] = pl[r];
          }
        }
        __syncthreads();
        if (active) {
#pragma unroll
          for (int r = 0; r < E; ++r) {
            ok[r] = xk[(buf * T + (lt ^ ts)) * E + r];
            op[r] = xp[(buf * T + (lt ^ ts)) * E + r];
          }
        }
        buf ^= 1;
      }
      if (active) {
        // This thread's slots take the pair's first-ordered element when they
        // are the lower slots of a "first-ordered first" block (or the upper
        // slots of a reversed one); size > stride >= E, the same for all r.
        const bool lower = (lt & ts) == 0;
        const bool ascending_block = ((E * lt) & size) == 0;
#pragma unroll
        for (int r = 0; r < E; ++r) {
          const bool me_first = first_ordered(key[r], pl[r], ok[r], op[r]);
          if ((lower == ascending_block) != me_first) {
            key[r] = ok[r];
            pl[r] = op[r];
          }
        }
      }
    }
  }
  if (active) {
#pragma unroll
    for (int r = 0; r < E; ++r) {
      const int e = E * lt + r;
      if (e < s) {
        keys[e] = key[r];
        pools[e] = pl[r];
      }
    }
  }
}

// Sort of the first s (<= kMaxK) pairs of sm.key / sm.pool, key descending,
// pool ascending, in place: a 512-wide network (two per thread, 256 threads,
// 45 sub-stages, 6 behind barriers) when s <= 512, else a 1024-wide one (four
// per thread, 55 sub-stages, 6 behind barriers).  The exchange buffers are
// in the histogram's space, free by now.
__device__ __forceinline__ void sort_pairs(Smem &sm, int s) {
  const int tid = threadIdx.x;
  __syncthreads();  // the pairs were written by other threads; the histogram space is free
  uint32_t *xk = &sm.hist[0][0];
  int32_t *xp = reinterpret_cast<int32_t *>(&sm.hist[1][0]);
  if (s <= kMaxK / 2)
    sort_net<kMaxK / 2, 2>(sm.key, sm.pool, s, tid, tid < kMaxK / 4, xk, xp);
  else
    sort_net<kMaxK, 4>(sm.key, sm.pool, s, tid, tid < kMaxK / 4, xk, xp);
  __syncthreads();
}

// Visits the row in groups of four elements: f(i, v, nv) gets elements i ..
// i + 3 in v (nv of them below n, the rest to be ignored), with eight loads
// of 16 bytes in flight per thread when the row is 16-byte aligned (scalar
// loads, one element per group, otherwise).  The loop bound is uniform
// across each warp and f is called for all lanes (nv = 0 past the row), so
// f may use warp collectives.
template <typename F>
__device__ __forceinline__ void visit_row(const float *__restrict__ row, int n, F &&f) {
  const int tid = threadIdx.x, lane = tid & 31;
  if ((reinterpret_cast<uintptr_t>(row) & 15u) == 0) {
    const float4 *r4 = reinterpret_cast<const float4 *>(row);
    const int n4 = (n + 3) >> 2;  // the last vector may run past n (same 16-byte line)
    for (int c0 = tid; c0 - lane < n4; c0 += kThreads * kUnroll) {
      float4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * kThreads;
        v[u] = c < n4 ? __ldg(r4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i = 4 * (c0 + u * kThreads);
        f(i, v[u], max(0, min(4, n - i)));
      }
    }
  } else {
    for (int i0 = tid; i0 - lane < n; i0 += kThreads * kUnroll) {
      float v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i = i0 + u * kThreads;
        v[u] = i < n ? __ldg(row + i) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) f(i0 + u * kThreads, make_float4(v[u], 0.f, 0.f, 0.f), i0 + u * kThreads < n ? 1 : 0);
    }
  }
}

// Exact multi-pass selection of the k largest keys of the n > k pools:
// three radix passes over the row find the k-th key; keys above it are
// collected in any order, then the keys equal to it in pool order.  Leaves
// the k pairs in sm.key / sm.pool [0, k).
__device__ void select_multipass(const float *__restrict__ row, int n, int k, Smem &sm) {
  const int tid = threadIdx.x;
  uint32_t *hist = sm.hist[0];
  uint32_t prefix = 0, mask = 0;
  uint32_t remaining = (uint32_t)k;
#pragma unroll 1
  for (int ps = 0; ps < 3; ++ps) {  // bits 31..21, 20..10, 9..0
    const int sh = ps == 0 ? 21 : (ps == 1 ? 10 : 0), nb = ps == 2 ? 1024 : 2048;
    for (int b = tid; b < nb; b += kThreads) hist[b] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += kThreads) {
      const uint32_t key = float_key(__ldg(row + i));
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> sh) & (uint32_t)(nb - 1)], 1u);
    }
    __syncthreads();
    find_bin(hist, nb, remaining, sm);
    remaining -= sm.above;
    prefix |= sm.bin << sh;
    mask |= (uint32_t)(nb - 1) << sh;
    __syncthreads();
  }
  const uint32_t thresh = prefix;
  const int need = (int)remaining;  // keys equal to thresh to take
  if (tid == 0) sm.cnt = 0;
  __syncthreads();
  for (int i = tid; i < n; i += kThreads) {
    const uint32_t key = float_key(__ldg(row + i));
    if (key > thresh) {
      const uint32_t pos = atomicAdd(&sm.cnt, 1u);
      sm.key[pos] = key;
      sm.pool[pos] = i;
    }
  }
  __syncthreads();
  const int base = (int)sm.cnt;  // = k - need
  __syncthreads();
  int taken = 0;
  for (int i0 = 0; i0 < n && taken < need; i0 += kThreads) {  // uniform loop
    const int i = i0 + tid;
    const bool eq = i < n && float_key(__ldg(row + i)) == thresh;
    uint32_t total;
    const uint32_t rank = block_exclusive_scan(eq ? 1u : 0u, sm, total);
    if (eq && taken + (int)rank < need) {
      sm.key[base + taken + rank] = thresh;
      sm.pool[base + taken + rank] = i;
    }
    taken += (int)total;
  }
  __syncthreads();
}

// Histogram of the top 11 bits of the keys of elements [0, n) of `row`
// (private copies, then summed into sm.hist[0]).
__device__ __forceinline__ void histogram_top11(const float *__restrict__ row, int n, Smem &sm) {
  const int tid = threadIdx.x, warp = tid >> 5;
  for (int b = tid; b < kHistCopies * kBins; b += kThreads) (&sm.hist[0][0])[b] = 0;
  __syncthreads();
  uint32_t *h = sm.hist[warp >> 2];
  visit_row(row, n, [&](int, float4 v, int nv) {
    if (nv > 0) atomicAdd(&h[float_key(v.x) >> 21], 1u);
    if (nv > 1) atomicAdd(&h[float_key(v.y) >> 21], 1u);
    if (nv > 2) atomicAdd(&h[float_key(v.z) >> 21], 1u);
    if (nv > 3) atomicAdd(&h[float_key(v.w) >> 21], 1u);
  });
  __syncthreads();
  for (int b = tid; b < kBins; b += kThreads) {
    uint32_t sum = 0;
#pragma unroll
    for (int c = 0; c < kHistCopies; ++c) sum += sm.hist[c][b];
    sm.hist[0][b] = sum;
  }
  __syncthreads();
}

// Appends every element of [0, n) of `row` whose key's top 11 bits are >=
// thr to a candidate list: push(key, row index) per kept element, called
// by the lanes of a warp together with the base of the warp's block of
// slots reserved through reserve(count) by lane 0.
template <typename Reserve, typename Put>
__device__ __forceinline__ void collect_candidates(const float *__restrict__ row, int n, uint32_t thr,
                                                   Reserve &&reserve, Put &&put) {
  const int lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  visit_row(row, n, [&](int i, float4 v, int nv) {
    const uint32_t kk[4] = {float_key(v.x), float_key(v.y), float_key(v.z), float_key(v.w)};
    bool any = false;
#pragma unroll
    for (int q = 0; q < 4; ++q) any |= q < nv && (kk[q] >> 21) >= thr;
    if (__ballot_sync(0xffffffffu, any) == 0) return;  // the common case: nothing to keep
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const bool take = q < nv && (kk[q] >> 21) >= thr;
      const uint32_t m = __ballot_sync(0xffffffffu, take);
      if (m) {
        uint32_t base = 0;
        if (lane == 0) base = reserve((uint32_t)__popc(m));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (take) put(base + (uint32_t)__popc(m & lt), kk[q], i + q);
      }
    }
  });
}

// From c candidates in sm.key / sm.pool (every key whose top 11 bits are >=
// thr; `above` of them in higher bins), the k selected pairs in their final
// order in sm.key / sm.pool [0, k): one radix pass over the candidates (the
// next 11 bits) finds the bin B of the k-th key; every candidate in B or
// above it (k plus the few others that share B) is kept and sorted.  With
// more than kMaxK of them (ties), the multi-pass selection over the row.
__device__ void select_from_candidates(Smem &sm, int c, uint32_t thr, uint32_t above, int k,
                                       const float *__restrict__ row, int n) {
  const int tid = threadIdx.x;
  uint32_t *h0 = sm.hist[0];
  __syncthreads();  // the candidates are complete; the histogram space is free
  for (int b = tid; b < kBins; b += kThreads) h0[b] = 0;
  __syncthreads();
  for (int i = tid; i < c; i += kThreads) {
    const uint32_t key = sm.key[i];
    if ((key >> 21) == thr) atomicAdd(&h0[(key >> 10) & (uint32_t)(kBins - 1)], 1u);
  }
  __syncthreads();
  find_bin(h0, kBins, (uint32_t)k - above, sm);
  // Keys >= T are the candidates of bin (thr, sm.bin) or above it.
  const uint32_t T = (thr << 21) | (sm.bin << 10);
  const int sel = (int)(above + sm.above + h0[sm.bin]);
  __syncthreads();
  if (sel > kMaxK) {
    select_multipass(row, n, k, sm);
    sort_pairs(sm, k);
    return;
  }
  constexpr int kPer = kCandCap / kThreads;  // candidates per thread
  uint32_t kept_key[kPer];
  int32_t kept_pool[kPer];
  bool keep[kPer];
  uint32_t nk = 0;
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    const int i = tid + q * kThreads;
    keep[q] = i < c && sm.key[i] >= T;
    kept_key[q] = keep[q] ? sm.key[i] : 0u;
    kept_pool[q] = keep[q] ? sm.pool[i] : 0;
    nk += keep[q] ? 1u : 0u;
  }
  // Split selection: the a keys above the boundary bin (bits 31..10 of T)
  // all precede its b keys, and a < k <= a + b.  With a <= 512 and b <= 32
  // the a keys are sorted by a 512-wide network while one warp sorts the
  // boundary bin and appends its first k - a, instead of one 1024-wide sort
  // of all a + b (which the usual ~530 kept keys need).
  const int a_above = (int)(above + sm.above);
  const int b_bin = (int)h0[sm.bin];
  const bool split = a_above <= kMaxK / 2 && b_bin <= 32;
  if (tid == 0) {
    sm.cnt = 0;
    sm.bcnt = 0;
  }
  __syncthreads();  // every candidate has been read before the list is rewritten
  if (!split) {
    uint32_t pos = nk ? atomicAdd(&sm.cnt, nk) : 0u;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      if (keep[q]) {
        sm.key[pos] = kept_key[q];
        sm.pool[pos] = kept_pool[q];
        ++pos;
      }
    }
    sort_pairs(sm, sel);  // the first k (ties by smaller pool) are the selection
    return;
  }
  // Above the bin -> [0, a); in the bin -> [kBinSlot, kBinSlot + b).
  constexpr int kBinSlot = kCandCap / 2;
  const uint32_t tb = T >> 10;
  uint32_t na = 0, nb = 0;
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    na += keep[q] && (kept_key[q] >> 10) > tb ? 1u : 0u;
    nb += keep[q] && (kept_key[q] >> 10) == tb ? 1u : 0u;
  }
  uint32_t pa = na ? atomicAdd(&sm.cnt, na) : 0u;
  uint32_t pb = nb ? atomicAdd(&sm.bcnt, nb) : 0u;
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    if (!keep[q]) continue;
    const uint32_t slot = (kept_key[q] >> 10) > tb ? pa++ : kBinSlot + pb++;
    sm.key[slot] = kept_key[q];
    sm.pool[slot] = kept_pool[q];
  }
  __syncthreads();
  if ((tid >> 5) == kThreads / 32 - 1) {  // the last warp: the boundary bin, then the a-sort's barriers
    const int lane = tid & 31;
    sort_net<32, 1>(sm.key + kBinSlot, sm.pool + kBinSlot, b_bin, lane, true, nullptr, nullptr);
    __syncwarp();
    if (lane < k - a_above) {
      sm.key[a_above + lane] = sm.key[kBinSlot + lane];
      sm.pool[a_above + lane] = sm.pool[kBinSlot + lane];
    }
  }
  sort_net<kMaxK / 2, 2>(sm.key, sm.pool, a_above, tid, tid < kMaxK / 4, &sm.hist[0][0],
                         reinterpret_cast<int32_t *>(&sm.hist[1][0]));
  __syncthreads();
}

// The index row: pools sm.pool[0, nsel) expanded to their tokens, the tail
// of the partial last pool, -1 up to `width`.
__device__ __forceinline__ void expand_into(const Smem &sm, int nsel, int k, int pool, int seq_len,
                                            int32_t *__restrict__ orow, int width) {
  const int span = k * pool;
  const int tail_start = (seq_len > 0 ? seq_len / pool : 0) * pool;
  const int tail_len = seq_len > 0 ? seq_len % pool : 0;
  const bool pow2 = (pool & (pool - 1)) == 0;  // shifts instead of a division per entry
  const int sh = __ffs(pool) - 1;
  for (int j = threadIdx.x; j < width; j += kThreads) {
    int v = -1;
    if (j < span) {
      const int i = pow2 ? j >> sh : j / pool, o = pow2 ? j & (pool - 1) : j - (j / pool) * pool;
      if (i < nsel) v = sm.pool[i] * pool + o;
    } else if (j < span + pool - 1) {
      const int o = j - span;
      if (o < tail_len) v = tail_start + o;
    }
    orow[j] = v;
  }
}

// Every valid pool selected (n <= k): load and sort them.
__device__ __forceinline__ void select_all(const float *__restrict__ row, int n, Smem &sm) {
  for (int i = threadIdx.x; i < n; i += kThreads) {
    sm.key[i] = float_key(__ldg(row + i));
    sm.pool[i] = i;
  }
  sort_pairs(sm, n);
}

// One CTA per query row (many rows).
__global__ void __launch_bounds__(kThreads, 1)
    pool_topk_expand_kernel(const float *__restrict__ logits, int64_t ld, const int32_t *__restrict__ seq_lens, int k,
                            int pool, int32_t *__restrict__ out, int64_t out_stride, int width) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
  const int t = blockIdx.x, tid = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait_primary();  // the logits and lengths come from earlier kernels
  const float *row = logits + (int64_t)t * ld;
  const int seq_len = __ldg(seq_lens + t);
  const int64_t n64 = seq_len > 0 ? (int64_t)(seq_len / pool) : 0;
  const int n = (int)(n64 < ld ? n64 : ld);
  const int nsel = n < k ? n : k;

  if (n <= k) {
    select_all(row, n, sm);
  } else {
    histogram_top11(row, n, sm);
    find_bin(sm.hist[0], kBins, (uint32_t)k, sm);
    const uint32_t thr = sm.bin, above = sm.above;
    const uint32_t cand = above + sm.hist[0][thr];  // keys in the bin or above it
    if (cand <= (uint32_t)kCandCap) {
      if (tid == 0) sm.cnt = 0;
      __syncthreads();
      collect_candidates(
          row, n, thr, [&](uint32_t cnt) { return atomicAdd(&sm.cnt, cnt); },
          [&](uint32_t pos, uint32_t key, int i) {
            if (pos < (uint32_t)kCandCap) {  // pos < cand <= kCandCap by construction
              sm.key[pos] = key;
              sm.pool[pos] = i;
            } else {
              atomicCAS(&g_device_error, 0, kDevErrCapacity);
            }
          });
      __syncthreads();
      select_from_candidates(sm, (int)min(sm.cnt, (uint32_t)kCandCap), thr, above, k, row, n);
    } else {
      select_multipass(row, n, k, sm);
      sort_pairs(sm, nsel);
    }
  }
  expand_into(sm, nsel, k, pool, seq_len, out + (int64_t)t * out_stride, width);
}

// Distributed shared memory of the cluster form.
__device__ __forceinline__ uint32_t ld_cluster_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_cluster_u32(uint32_t addr, uint32_t v) {
  uint32_t old;
  asm volatile("atom.shared::cluster.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(addr), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t v;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(v));
  return v;
}

// Cluster form (few rows): the C CTAs of a cluster share one row.  CTA r
// histograms its contiguous share of the pools; each CTA then sums one
// slice of the bins over the cluster's histograms and every CTA reads the
// summed slices back, so all find the same threshold bin; the CTAs append
// their candidates straight into CTA 0's shared memory (one remote atomic
// per warp and keep), and CTA 0 refines, sorts and expands.  The cluster
// barriers are reached by every thread of every CTA on uniform control flow
// (the row and its sizes are uniform across the cluster).
__global__ void __launch_bounds__(kThreads, 1)
    pool_topk_cluster_kernel(const float *__restrict__ logits, int64_t ld, const int32_t *__restrict__ seq_lens,
                             int k, int pool, int32_t *__restrict__ out, int64_t out_stride, int width) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
  const int C = (int)cluster_size(), r = (int)cluster_ctarank();
  const int t = blockIdx.x / C, tid = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait_primary();  // the logits and lengths come from earlier kernels
  const float *row = logits + (int64_t)t * ld;
  const int seq_len = __ldg(seq_lens + t);
  const int64_t n64 = seq_len > 0 ? (int64_t)(seq_len / pool) : 0;
  const int n = (int)(n64 < ld ? n64 : ld);
  const int nsel = n < k ? n : k;
  int32_t *orow = out + (int64_t)t * out_stride;

  if (n <= k) {  // uniform across the cluster: CTA 0 alone
    if (r == 0) {
      select_all(row, n, sm);
      expand_into(sm, nsel, k, pool, seq_len, orow, width);
    }
    return;
  }
  // This CTA's share of the pools: [lo, hi), lo a multiple of 4 (16-byte
  // loads stay aligned when the row is).
  const int per = ((n + C - 1) / C + 3) & ~3;
  const int lo = min(n, r * per), hi = min(n, lo + per);
  const int m = hi - lo;
  // A share of at most kRegVec 16-byte vectors per thread (an aligned row)
  // stays in registers, as keys, from the histogram to the candidate pass:
  // no second read of the row.  Its loads are issued before the histogram
  // copies are cleared, so the clearing hides their latency.
  const bool in_regs = m <= kRegVec * 4 * kThreads && (reinterpret_cast<uintptr_t>(row + lo) & 15u) == 0;
  uint32_t kk[kRegVec][4];
  int nv[kRegVec];
  if (in_regs) {
    const float4 *r4 = reinterpret_cast<const float4 *>(row + lo);
    const int n4 = (m + 3) >> 2;  // the last vector may run past m (same 16-byte line)
    float4 v[kRegVec];
#pragma unroll
    for (int j = 0; j < kRegVec; ++j) {
      const int c = tid + j * kThreads;
      v[j] = c < n4 ? __ldg(r4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      nv[j] = max(0, min(4, m - 4 * c));
    }
    for (int b = tid; b < kHistCopies * kBins; b += kThreads) (&sm.hist[0][0])[b] = 0;
#pragma unroll
    for (int j = 0; j < kRegVec; ++j) {
      kk[j][0] = float_key(v[j].x);
      kk[j][1] = float_key(v[j].y);
      kk[j][2] = float_key(v[j].z);
      kk[j][3] = float_key(v[j].w);
    }
    __syncthreads();
    uint32_t *h = sm.hist[(tid >> 5) >> 2];
#pragma unroll
    for (int j = 0; j < kRegVec; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (q < nv[j]) atomicAdd(&h[kk[j][q] >> 21], 1u);
    __syncthreads();
    for (int b = tid; b < kBins; b += kThreads) {
      uint32_t sum = 0;
#pragma unroll
      for (int c = 0; c < kHistCopies; ++c) sum += sm.hist[c][b];
      sm.hist[0][b] = sum;
    }
    __syncthreads();
  } else {
    histogram_top11(row + lo, m, sm);
  }
  if (tid == 0) sm.ccnt = 0;  // CTA 0's candidate counter (every CTA clears its own)
  cluster_sync_all();         // every CTA's histogram (sm.hist[0]) is complete
  // Slice sums: CTA r owns bins [r S, r S + S).  C consecutive lanes (C
  // divides 32) load one bin from the C CTAs at once and add by shuffles.
  // (kSliceRounds rounds of kThreads / C bins; every remote load is issued
  // before the first sum, one round trip instead of one per round.)
  const int S = kBins / C;
  {
    uint32_t v[kSliceRounds];
#pragma unroll
    for (int j = 0; j < kSliceRounds; ++j) {
      const int b = j * (kThreads / C) + tid / C, q = tid % C;
      v[j] = 0;
      if (b < S) {
        uint32_t a;
        asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(&sm.hist[0][r * S + b])), "r"(q));
        v[j] = ld_cluster_u32(a);
      }
    }
#pragma unroll
    for (int j = 0; j < kSliceRounds; ++j) {
      const int b = j * (kThreads / C) + tid / C, q = tid % C;
      for (int o = C >> 1; o > 0; o >>= 1) v[j] += __shfl_down_sync(0xffffffffu, v[j], o, C);
      if (q == 0 && b < S) sm.slice[b] = v[j];
    }
  }
  cluster_sync_all();  // every slice is summed
  // The row's histogram, read back from the slices into sm.hist[1] (both
  // remote loads of a thread in flight together).
  {
    uint32_t v[kBins / kThreads];
#pragma unroll
    for (int j = 0; j < kBins / kThreads; ++j) {
      const int b = tid + j * kThreads;
      uint32_t a;
      asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(&sm.slice[b % S])), "r"(b / S));
      v[j] = ld_cluster_u32(a);
    }
#pragma unroll
    for (int j = 0; j < kBins / kThreads; ++j) sm.hist[1][tid + j * kThreads] = v[j];
  }
  __syncthreads();
  find_bin(sm.hist[1], kBins, (uint32_t)k, sm);
  const uint32_t thr = sm.bin, above = sm.above;
  const uint32_t cand = above + sm.hist[1][thr];
  const bool fast = cand <= (uint32_t)kCandCap;  // uniform across the cluster
  if (fast) {
    const uint32_t cnt0 = [&] {
      uint32_t a;
      asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(&sm.ccnt)), "r"(0));
      return a;
    }();
    uint32_t key0, pool0;
    asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(key0) : "r"(smem_u32(&sm.key[0])), "r"(0));
    asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(pool0) : "r"(smem_u32(&sm.pool[0])), "r"(0));
    auto put = [&](uint32_t pos, uint32_t key, int i) {
      // pos < cand <= kCandCap by construction; checked, not trusted
      if (pos < (uint32_t)kCandCap) {
        st_cluster_u32(key0 + 4 * pos, key);
        st_cluster_u32(pool0 + 4 * pos, (uint32_t)(lo + i));
      } else {
        atomicCAS(&g_device_error, 0, kDevErrCapacity);
      }
    };
    if (in_regs) {
      // One remote atomic per warp reserves the slots of all its keeps: one
      // ballot per key slot, offsets by popcount.
      const int lane = tid & 31;
      const uint32_t lt = (1u << lane) - 1u;
      uint32_t ball[kRegVec][4];
      uint32_t total = 0;
#pragma unroll
      for (int j = 0; j < kRegVec; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          ball[j][q] = __ballot_sync(0xffffffffu, q < nv[j] && (kk[j][q] >> 21) >= thr);
          total += (uint32_t)__popc(ball[j][q]);
        }
      if (total) {  // warp-uniform
        uint32_t base = 0;
        if (lane == 0) base = atom_add_cluster_u32(cnt0, total);
        base = __shfl_sync(0xffffffffu, base, 0);
#pragma unroll
        for (int j = 0; j < kRegVec; ++j)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if ((ball[j][q] >> lane) & 1u) put(base + (uint32_t)__popc(ball[j][q] & lt), kk[j][q], 4 * (tid + j * kThreads) + q);
            base += (uint32_t)__popc(ball[j][q]);
          }
      }
    } else {
      collect_candidates(row + lo, m, thr, [&](uint32_t c) { return atom_add_cluster_u32(cnt0, c); }, put);
    }
  }
  // The candidates have reached CTA 0, and no CTA reads a peer's slice any
  // more: the others may exit.
  cluster_sync_all();
  if (r != 0) return;
  if (fast) {
    select_from_candidates(sm, (int)min(sm.ccnt, (uint32_t)kCandCap), thr, above, k, row, n);
  } else {
    select_multipass(row, n, k, sm);
    sort_pairs(sm, nsel);
  }
  expand_into(sm, nsel, k, pool, seq_len, orow, width);
}

}  // namespace idx

namespace {
std::atomic<int> g_topk_ready[64];
std::atomic<int> g_topk_clusters[64][2];  // clusters of 16 / 8 CTAs the device runs at once
}  // namespace
}  // namespace titan

extern "C" int titan_pool_topk_expand(const float *logits, int64_t ld, const int32_t *seq_lens, int64_t num_rows,
                                      int k, int pool_size, int32_t *out, int64_t out_stride, int width,
                                      titan_stream_t stream) {
  using namespace titan;
  if (num_rows < 0 || num_rows > 0x7fffffffLL)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "pool_topk_expand: invalid row count");
  if (k < 1 || k > idx::kMaxK) return fail(TITAN_ERR_INVALID_ARGUMENT, "pool_topk_expand: k must be in [1, %d]", idx::kMaxK);
  if (pool_size < 1 || pool_size > 64) return fail(TITAN_ERR_INVALID_ARGUMENT, "pool_topk_expand: pool size must be in [1, 64]");
  if (ld < 0 || width < k * pool_size + pool_size - 1 || out_stride < width)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "pool_topk_expand: width %d below k * pool + pool - 1 = %d, or a bad stride",
                width, k * pool_size + pool_size - 1);
  if (num_rows == 0) return TITAN_OK;
  if (seq_lens == nullptr || out == nullptr || (logits == nullptr && ld > 0))
    return fail(TITAN_ERR_INVALID_ARGUMENT, "pool_topk_expand: null pointer");
  const size_t smem = sizeof(idx::Smem);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "pool_topk_expand: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(TITAN_ERR_CUDA, "pool_topk_expand: device ordinal %d out of range", dev);
  // One-time set-up per device: shared-memory opt-in for both kernels,
  // 16-CTA clusters allowed, and how many clusters of each size fit.
  if (!g_topk_ready[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(setup_mutex());
    if (!g_topk_ready[dev].load(std::memory_order_relaxed)) {
      e = cudaFuncSetAttribute(idx::pool_topk_expand_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(idx::pool_topk_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(idx::pool_topk_cluster_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "pool_topk_expand: setup: %s", cudaGetErrorString(e));
      // How many clusters of 16 and of 8 CTAs the device runs at once.
      for (int ci = 0; ci < 2; ++ci) {
        const int csize = ci == 0 ? idx::kClusterMax : 8;
        cudaLaunchConfig_t q = {};
        q.gridDim = dim3((unsigned)csize);
        q.blockDim = dim3(idx::kThreads);
        q.dynamicSmemBytes = smem;
        cudaLaunchAttribute qa[1];
        qa[0].id = cudaLaunchAttributeClusterDimension;
        qa[0].val.clusterDim.x = (unsigned)csize;
        qa[0].val.clusterDim.y = 1;
        qa[0].val.clusterDim.z = 1;
        q.attrs = qa;
        q.numAttrs = 1;
        int nclusters = 0;
        if (cudaOccupancyMaxActiveClusters(&nclusters, idx::pool_topk_cluster_kernel, &q) != cudaSuccess) {
          cudaGetLastError();
          nclusters = 0;
        }
        g_topk_clusters[dev][ci].store(nclusters, std::memory_order_relaxed);
      }
      g_topk_ready[dev].store(1, std::memory_order_release);
    }
  }
  const int n16 = g_topk_clusters[dev][0].load(std::memory_order_relaxed);
  const int n8 = g_topk_clusters[dev][1].load(std::memory_order_relaxed);
  // Few rows: a cluster per row (16 CTAs when the rows' clusters all run at
  // once, else 8), so a decode step's rows spread over the SMs; many rows:
  // one CTA per row.
  const int cluster = num_rows <= n16 ? idx::kClusterMax : (num_rows <= n8 ? 8 : 0);
  if (cluster > 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(num_rows * cluster));
    cfg.blockDim = dim3(idx::kThreads);
    cfg.dynamicSmemBytes = smem;
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
    e = cudaLaunchKernelEx(&cfg, idx::pool_topk_cluster_kernel, logits, ld, seq_lens, k, pool_size, out, out_stride,
                           width);
    if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "pool_topk_expand launch: %s", cudaGetErrorString(e));
    return check_launch("pool_topk_expand launch");
  }
  e = launch_pdl(idx::pool_topk_expand_kernel, dim3((unsigned)num_rows), dim3(idx::kThreads), smem,
                 reinterpret_cast<cudaStream_t>(stream), logits, ld, seq_lens, k, pool_size, out, out_stride, width);
  if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "pool_topk_expand launch: %s", cudaGetErrorString(e));
  return check_launch("pool_topk_expand launch");
}
