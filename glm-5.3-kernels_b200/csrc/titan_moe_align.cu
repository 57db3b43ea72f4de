// Small stable MoE route alignment: B1..8 tokens x top-8, 288 experts, block 8.
//
// Output contract of kernels/titan_moe_align.py:12-46 (the reference
// `_align_small`), equal to the stable argsort layout of
// benchmarks/moe_align.py:23-31 (`cpu_reference`):
//   rank_j   = #{k < j valid : e_k == e_j}           count_e = #{valid : e}
//   pad_e    = ceil(count_e / 8) * 8                  off_e   = sum of pad over experts < e
//   sorted_ids[off_e + rank_j] = j  (rest = R),  expert_ids[off_e/8 + b] = e (rest = -1),
//   postpad  = sum pad_e.
//
// B200 design: one warp computes everything in registers; nothing scales with
// the 288 experts, only with the R <= 64 routes.  Routes j and j + 32 live in
// lane j.  Every lane walks the R routes once by warp shuffles (the ids of
// route k broadcast from lane k & 31) and counts, for each of its routes,
// the equal experts before it (its rank) and in total (its count); a route
// of rank 0 "leads" its expert and carries the expert's padded count.  A
// second walk sums, for each route, the padded counts of the leaders of
// smaller experts: that is its expert's offset.  The layout is assembled in
// shared memory and written with 16-byte stores (4-byte stores when an
// output is not 16-byte aligned).  Removing the 288-entry count table, its
// zeroing and its scan shortens the single warp's serial chain.
#include "titan_common.cuh"

#include <type_traits>

namespace titan {

constexpr int kMoeMaxRoutes = 64;  // B <= 8, top-8
constexpr int kMoeExperts = TITAN_MOE_NUM_EXPERTS;

template <typename IdT, int R>
__global__ void __launch_bounds__(128) moe_align_small_kernel(const IdT *__restrict__ ids,
                                                              int32_t *__restrict__ sorted_ids,
                                                              int32_t *__restrict__ expert_ids,
                                                              int32_t *__restrict__ postpad, bool vec_out) {
  constexpr bool kTwoHalves = R > 32;
  // The whole layout is built by warp 0: no CTA-wide barrier sits on the
  // critical path, which starts with the route-id loads.  Extra warps (the
  // caller's num_warps) have nothing to do.
  // Launched as a programmatic dependent: the next kernel on the stream may
  // launch at once (it waits for this grid before reading its outputs), and
  // this one waits for the previous grid (the router writing the ids, or the
  // previous call writing the same outputs) only before its first global
  // access, after the shared-memory set-up.
  pdl_launch_dependents();
  if (threadIdx.x >= 32) return;
  __shared__ __align__(16) int s_sorted[kMoeMaxRoutes * 8];
  __shared__ __align__(16) int s_experts[kMoeMaxRoutes];
  const int lane = threadIdx.x;

  // Initialise: padding = R, unused blocks = -1.
  const int4 pad4 = make_int4(R, R, R, R);
  for (int i = lane; i < 2 * R; i += 32) reinterpret_cast<int4 *>(s_sorted)[i] = pad4;  // 8R ints
  for (int i = lane; i < R; i += 32) s_experts[i] = -1;

  pdl_wait_primary();
  // Route lane (half 0) and lane + 32 (half 1).  Validity is decided on the
  // full-width id, before narrowing (an int64 id of 2^32 + 5 is invalid).
  long long raw0 = -1, raw1 = -1;
  if (lane < R) raw0 = (long long)ids[lane];
  if (kTwoHalves && lane + 32 < R) raw1 = (long long)ids[lane + 32];

  // Invalid routes (and lanes past R) get expert -1: they match no valid
  // route, lead nothing and never scatter.
  const int e0 = (raw0 >= 0 && raw0 < kMoeExperts) ? (int)raw0 : -1;
  const int e1 = (raw1 >= 0 && raw1 < kMoeExperts) ? (int)raw1 : -1;
  const int j1 = lane + 32;
  int rank0 = 0, cnt0 = 0, rank1 = 0, cnt1 = 0;
#pragma unroll
  for (int k = 0; k < R; ++k) {  // unrolled: the R shuffles are independent and pipeline
    const int ek = __shfl_sync(0xffffffffu, (!kTwoHalves || k < 32) ? e0 : e1, k & 31);
    const int same0 = (int)(ek == e0), same1 = (int)(ek == e1);
    cnt0 += same0;
    rank0 += same0 & (int)(k < lane);
    if (kTwoHalves) {
      cnt1 += same1;
      rank1 += same1 & (int)(k < j1);
    }
  }
  // Padded count carried by the leader (rank 0) of each valid expert.
  const int lead0 = (e0 >= 0 && rank0 == 0) ? (cnt0 + 7) & ~7 : 0;
  const int lead1 = (kTwoHalves && e1 >= 0 && rank1 == 0) ? (cnt1 + 7) & ~7 : 0;
  int off0 = 0, off1 = 0;
#pragma unroll
  for (int k = 0; k < R; ++k) {
    const bool lo = !kTwoHalves || k < 32;
    const int ek = __shfl_sync(0xffffffffu, lo ? e0 : e1, k & 31);
    const int pk = __shfl_sync(0xffffffffu, lo ? lead0 : lead1, k & 31);
    off0 += ek < e0 ? pk : 0;  // leaders of smaller experts (pk = 0 unless k leads)
    if (kTwoHalves) off1 += ek < e1 ? pk : 0;
  }
  int total = lead0 + lead1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
  __syncwarp();  // the initialisation above is complete before the scatter
  // Scatter: route j goes to off_e + rank_j.  Offsets are multiples of 8, so
  // the route whose rank is a multiple of 8 opens block (off_e + rank_j) / 8
  // of its expert: exactly ceil(count_e / 8) blocks per expert, no loop.
  if (e0 >= 0) {
    const int pos = off0 + rank0;
    s_sorted[pos] = lane;
    if ((rank0 & 7) == 0) s_experts[pos >> 3] = e0;
  }
  if (kTwoHalves && e1 >= 0) {
    const int pos = off1 + rank1;
    s_sorted[pos] = j1;
    if ((rank1 & 7) == 0) s_experts[pos >> 3] = e1;
  }
  __syncwarp();
  if (vec_out) {
    for (int i = lane; i < 2 * R; i += 32)
      reinterpret_cast<int4 *>(sorted_ids)[i] = reinterpret_cast<const int4 *>(s_sorted)[i];
    for (int i = lane; i < R / 4; i += 32)
      reinterpret_cast<int4 *>(expert_ids)[i] = reinterpret_cast<const int4 *>(s_experts)[i];
  } else {
    for (int i = lane; i < 8 * R; i += 32) sorted_ids[i] = s_sorted[i];
    for (int i = lane; i < R; i += 32) expert_ids[i] = s_experts[i];
  }
  if (lane == 0) postpad[0] = total;
}

}  // namespace titan

extern "C" int titan_moe_align_small(const void *topk_ids, int ids_is_int64, int64_t num_routes,
                                     int32_t *sorted_ids, int32_t *expert_ids, int32_t *postpad, int num_warps,
                                     titan_stream_t stream) {
  using namespace titan;
  if (num_routes < 8 || num_routes > kMoeMaxRoutes || num_routes % 8 != 0)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_align_small: num_routes must be 8*B with B in 1..8, got %lld",
                (long long)num_routes);
  if (num_warps != 1 && num_warps != 2 && num_warps != 4)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_align_small: num_warps must be 1, 2 or 4");
  if (topk_ids == nullptr || sorted_ids == nullptr || expert_ids == nullptr || postpad == nullptr)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_align_small: null pointer");
  const int R = (int)num_routes;
  const bool vec_out = (uintptr_t)sorted_ids % 16 == 0 && (uintptr_t)expert_ids % 16 == 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32 * num_warps);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaSuccess;
  // One instantiation per route count (R = 8 B): the route walks unroll.
  auto launch = [&](auto ids) {
    using IdT = std::remove_const_t<std::remove_pointer_t<decltype(ids)>>;
    auto go = [&](auto kernel) { e = cudaLaunchKernelEx(&cfg, kernel, ids, sorted_ids, expert_ids, postpad, vec_out); };
    switch (R) {
      case 8: go(moe_align_small_kernel<IdT, 8>); break;
      case 16: go(moe_align_small_kernel<IdT, 16>); break;
      case 24: go(moe_align_small_kernel<IdT, 24>); break;
      case 32: go(moe_align_small_kernel<IdT, 32>); break;
      case 40: go(moe_align_small_kernel<IdT, 40>); break;
      case 48: go(moe_align_small_kernel<IdT, 48>); break;
      case 56: go(moe_align_small_kernel<IdT, 56>); break;
      default: go(moe_align_small_kernel<IdT, 64>); break;
    }
  };
  if (ids_is_int64)
    launch(static_cast<const long long *>(topk_ids));
  else
    launch(static_cast<const int32_t *>(topk_ids));
  if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "moe_align_small launch: %s", cudaGetErrorString(e));
  return check_launch("moe_align_small launch");
}
