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
// order-preserving unsigned keys; a three-pass radix select (11 + 11 + 10
// bits, shared-memory histograms, suffix scan over the bins) finds the k-th
// largest key; keys above it are collected unordered, keys equal to it are
// taken in pool order by a block-wide ordered scan, and the k selected
// (key, pool) pairs are sorted by a bitonic sort in shared memory.  Each pass
// reads the row's logits from L2 (256 KB at 65,536 pools).
#include "titan_common.cuh"

namespace titan {
namespace idx {

constexpr int kThreads = 1024;
constexpr int kMaxK = 1024;
constexpr int kBins = 2048;

// Float -> key whose unsigned order is the float order; every NaN (either
// sign) maps to the largest key, above +inf.
__device__ __forceinline__ uint32_t float_key(float x) {
  const uint32_t b = __float_as_uint(x);
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) return 0xFFFFFFFFu;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

struct Smem {
  uint32_t hist[kBins];
  uint32_t key[kMaxK];
  int32_t pool[kMaxK];
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

__global__ void __launch_bounds__(kThreads, 1)
    pool_topk_expand_kernel(const float *__restrict__ logits, int64_t ld, const int32_t *__restrict__ seq_lens, int k,
                            int pool, int32_t *__restrict__ out, int64_t out_stride, int width) {
  __shared__ Smem sm;
  const int t = blockIdx.x, tid = threadIdx.x;
  const float *row = logits + (int64_t)t * ld;
  const int seq_len = __ldg(seq_lens + t);
  const int64_t n64 = seq_len > 0 ? (int64_t)(seq_len / pool) : 0;
  const int n = (int)(n64 < ld ? n64 : ld);
  const int nsel = n < k ? n : k;

  uint32_t thresh = 0;  // keys >= thresh candidates; exactly (nsel - need) keys > thresh
  int need = 0;         // keys equal to thresh to take (in pool order)
  if (n <= k) {
    // Every valid pool is selected: threshold below every key.
    thresh = 0;
    need = 0;
  } else {
    uint32_t prefix = 0, mask = 0;
    uint32_t remaining = (uint32_t)k;
#pragma unroll 1
    for (int ps = 0; ps < 3; ++ps) {  // bits 31..21, 20..10, 9..0
      const int sh = ps == 0 ? 21 : (ps == 1 ? 10 : 0), nb = ps == 2 ? 1024 : 2048;
      for (int b = tid; b < nb; b += kThreads) sm.hist[b] = 0;
      __syncthreads();
      for (int i = tid; i < n; i += kThreads) {
        const uint32_t key = float_key(__ldg(row + i));
        if ((key & mask) == prefix) atomicAdd(&sm.hist[(key >> sh) & (uint32_t)(nb - 1)], 1u);
      }
      __syncthreads();
      // Suffix counts from the top bin down: thread j owns bins nb - 1 - 2j
      // and nb - 2 - 2j (2048 bins over 1024 threads).
      const int b0 = nb - 1 - 2 * tid, b1 = b0 - 1;
      const uint32_t c0 = b0 >= 0 ? sm.hist[b0] : 0u, c1 = b1 >= 0 ? sm.hist[b1] : 0u;
      uint32_t total;
      const uint32_t above0 = block_exclusive_scan(c0 + c1, sm, total);  // keys in bins above b0
      // The bin holding the remaining-th largest key: above < remaining <= above + count.
      if (b0 >= 0 && above0 < remaining && remaining <= above0 + c0) {
        sm.bin = (uint32_t)b0;
        sm.above = above0;
      }
      if (b1 >= 0 && above0 + c0 < remaining && remaining <= above0 + c0 + c1) {
        sm.bin = (uint32_t)b1;
        sm.above = above0 + c0;
      }
      __syncthreads();
      remaining -= sm.above;
      prefix |= sm.bin << sh;
      mask |= (uint32_t)(nb - 1) << sh;
      __syncthreads();
    }
    thresh = prefix;
    need = (int)remaining;  // keys equal to thresh to take
  }

  // Collect keys above the threshold (any order), then the first `need`
  // keys equal to it in pool order.
  if (tid == 0) sm.cnt = 0;
  __syncthreads();
  if (n <= k) {
    for (int i = tid; i < n; i += kThreads) {
      sm.key[i] = float_key(__ldg(row + i));
      sm.pool[i] = i;
    }
  } else {
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
  }
  // Pad to the sort width with entries that sort last.
  int sw = 1;
  while (sw < nsel) sw <<= 1;
  for (int i = nsel + tid; i < sw; i += kThreads) {
    sm.key[i] = 0u;
    sm.pool[i] = 0x7fffffff;
  }
  __syncthreads();
  // Bitonic sort: key descending, pool ascending.
  for (int size = 2; size <= sw; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < sw; i += kThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const uint32_t ki = sm.key[i], kj = sm.key[j];
          const int pi = sm.pool[i], pj = sm.pool[j];
          // i before j in the final order when (ki > kj) or (ki == kj and pi < pj)
          const bool i_first = ki > kj || (ki == kj && pi < pj);
          const bool ascending_block = (i & size) == 0;  // this block sorts "first-ordered first"
          if (ascending_block != i_first) {
            sm.key[i] = kj;
            sm.key[j] = ki;
            sm.pool[i] = pj;
            sm.pool[j] = pi;
          }
        }
      }
      __syncthreads();
    }
  }
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
  idx::pool_topk_expand_kernel<<<(unsigned)num_rows, idx::kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      logits, ld, seq_lens, k, pool_size, out, out_stride, width);
  return check_launch("pool_topk_expand launch");
}
