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
// (warp-aggregated); a bitonic sort of the candidates (key descending, pool
// ascending) puts the k selected pools first, in their final order.  When
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
  uint32_t warp_sum[32];
  uint32_t bin, above, cnt;
};

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

// Bitonic sort of the first s (<= kMaxK) pairs of sm.key / sm.pool: key
// descending, pool ascending; the result goes back to sm.key / sm.pool
// [0, s).  Thread t holds element t in registers (entries past s sort last).
// Partners closer than 32 are exchanged by shuffles; farther ones through
// two alternating shared-memory buffers (in the histogram's space, free by
// now), one block barrier per such sub-stage.
__device__ __forceinline__ void sort_pairs(Smem &sm, int s) {
  const int tid = threadIdx.x;
  int sw = 1;
  while (sw < s) sw <<= 1;
  __syncthreads();  // the pairs were written by other threads; the histogram space is free
  uint32_t key = tid < s ? sm.key[tid] : 0u;
  int32_t pl = tid < s ? sm.pool[tid] : 0x7fffffff;
  uint32_t *xk = &sm.hist[0][0];                              // [2][kThreads] keys
  int32_t *xp = reinterpret_cast<int32_t *>(&sm.hist[1][0]);  // [2][kThreads] pools
  int buf = 0;
  for (int size = 2; size <= sw; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      uint32_t ok;
      int32_t op;
      if (stride < 32) {
        ok = __shfl_xor_sync(0xffffffffu, key, stride);
        op = __shfl_xor_sync(0xffffffffu, pl, stride);
      } else {
        xk[buf * kThreads + tid] = key;
        xp[buf * kThreads + tid] = pl;
        __syncthreads();
        ok = xk[buf * kThreads + (tid ^ stride)];
        op = xp[buf * kThreads + (tid ^ stride)];
        buf ^= 1;
      }
      // This thread's slot takes the pair's first-ordered element when it is
      // the lower slot of a "first-ordered first" block (or the upper slot
      // of a reversed one).
      const bool lower = (tid & stride) == 0;
      const bool ascending_block = (tid & size) == 0;
      const bool me_first = key > ok || (key == ok && pl < op);
      if ((lower == ascending_block) != me_first) {
        key = ok;
        pl = op;
      }
    }
  }
  if (tid < s) {
    sm.key[tid] = key;
    sm.pool[tid] = pl;
  }
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

__global__ void __launch_bounds__(kThreads, 1)
    pool_topk_expand_kernel(const float *__restrict__ logits, int64_t ld, const int32_t *__restrict__ seq_lens, int k,
                            int pool, int32_t *__restrict__ out, int64_t out_stride, int width) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float *row = logits + (int64_t)t * ld;
  const int seq_len = __ldg(seq_lens + t);
  const int64_t n64 = seq_len > 0 ? (int64_t)(seq_len / pool) : 0;
  const int n = (int)(n64 < ld ? n64 : ld);
  const int nsel = n < k ? n : k;

  if (n <= k) {
    // Every valid pool is selected.
    for (int i = tid; i < n; i += kThreads) {
      sm.key[i] = float_key(__ldg(row + i));
      sm.pool[i] = i;
    }
  } else {
    // ---- fast path, pass 1: histograms of the keys' top 11 bits
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
    find_bin(sm.hist[0], kBins, (uint32_t)k, sm);
    const uint32_t thr = sm.bin;
    const uint32_t cand = sm.above + sm.hist[0][thr];  // keys in the bin or above it
    if (cand <= (uint32_t)kCandCap) {
      // ---- pass 2: every key of the threshold bin or above joins the list
      if (tid == 0) sm.cnt = 0;
      __syncthreads();
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
            if (lane == 0) base = atomicAdd(&sm.cnt, (uint32_t)__popc(m));
            base = __shfl_sync(0xffffffffu, base, 0);
            if (take) {
              const uint32_t pos = base + (uint32_t)__popc(m & lt);
              sm.key[pos] = kk[q];
              sm.pool[pos] = i + q;
            }
          }
        }
      });
      __syncthreads();
      const int c = (int)sm.cnt;
      // ---- refine within the threshold bin on the candidates (two radix
      // passes over at most kCandCap keys in shared memory): the exact k-th
      // key T and how many keys equal to T to take.
      uint32_t *h0 = sm.hist[0];
      uint32_t prefix = thr << 21, mask = 0xFFE00000u;
      uint32_t remaining = (uint32_t)k - sm.above;
      uint32_t ties = 0;
#pragma unroll 1
      for (int ps = 0; ps < 2; ++ps) {
        const int sh = ps == 0 ? 10 : 0, nb = ps == 0 ? 2048 : 1024;
        for (int b = tid; b < nb; b += kThreads) h0[b] = 0;
        __syncthreads();
        for (int i = tid; i < c; i += kThreads) {
          const uint32_t key = sm.key[i];
          if ((key & mask) == prefix) atomicAdd(&h0[(key >> sh) & (uint32_t)(nb - 1)], 1u);
        }
        __syncthreads();
        find_bin(h0, nb, remaining, sm);
        remaining -= sm.above;
        prefix |= sm.bin << sh;
        mask |= (uint32_t)(nb - 1) << sh;
        if (ps == 1) ties = h0[sm.bin];  // candidates equal to T
        __syncthreads();
      }
      const uint32_t T = prefix;
      const int sel = k - (int)remaining + (int)ties;  // keys above T, and every key equal to T
      if (sel <= kMaxK) {
        // ---- keep the keys >= T (at most kMaxK), sort them; the first k
        // (ties by smaller pool) are the selection.
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
        if (tid == 0) sm.cnt = 0;
        __syncthreads();  // every candidate has been read before the list is rewritten
        uint32_t pos = nk ? atomicAdd(&sm.cnt, nk) : 0u;
#pragma unroll
        for (int q = 0; q < kPer; ++q) {
          if (keep[q]) {
            sm.key[pos] = kept_key[q];
            sm.pool[pos] = kept_pool[q];
            ++pos;
          }
        }
        sort_pairs(sm, sel);
      } else {
        select_multipass(row, n, k, sm);
        sort_pairs(sm, nsel);
      }
    } else {
      select_multipass(row, n, k, sm);
      sort_pairs(sm, nsel);
    }
  }
  if (n <= k) sort_pairs(sm, nsel);
  // Expansion into the index row.
  int32_t *orow = out + (int64_t)t * out_stride;
  const int span = k * pool;
  const int tail_start = (seq_len > 0 ? seq_len / pool : 0) * pool;
  const int tail_len = seq_len > 0 ? seq_len % pool : 0;
  for (int j = tid; j < width; j += kThreads) {
    int v = -1;
    if (j < span) {
      const int i = j / pool, o = j - (j / pool) * pool;
      if (i < nsel) v = sm.pool[i] * pool + o;
    } else if (j < span + pool - 1) {
      const int o = j - span;
      if (o < tail_len) v = tail_start + o;
    }
    orow[j] = v;
  }
}

}  // namespace idx

namespace {
std::atomic<int> g_topk_ready[64];
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
  if (!g_topk_ready[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(setup_mutex());
    if (!g_topk_ready[dev].load(std::memory_order_relaxed)) {
      e = cudaFuncSetAttribute(idx::pool_topk_expand_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "pool_topk_expand: setup: %s", cudaGetErrorString(e));
      g_topk_ready[dev].store(1, std::memory_order_release);
    }
  }
  idx::pool_topk_expand_kernel<<<(unsigned)num_rows, idx::kThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      logits, ld, seq_lens, k, pool_size, out, out_stride, width);
  return check_launch("pool_topk_expand launch");
}
