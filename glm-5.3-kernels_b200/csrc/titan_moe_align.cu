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
// B200 design: one warp computes everything with warp primitives instead of
// the reference's R x R pairwise compare.  Routes j and j + 32 live in lane j.
// Ranks come from __match_any_sync (peer mask) and a popcount of the lower
// lanes; the 288 expert counts live in shared memory; the padded offsets are
// a warp prefix scan with 9 experts per lane (32 x 9 = 288).  The result is
// assembled in shared memory and written with 16-byte stores (4-byte stores
// when an output is not 16-byte aligned).
#include "titan_common.cuh"

namespace titan {

constexpr int kMoeMaxRoutes = 64;  // B <= 8, top-8
constexpr int kMoeExperts = TITAN_MOE_NUM_EXPERTS;
constexpr int kMoePerLane = kMoeExperts / 32;  // 9
static_assert(kMoePerLane * 32 == kMoeExperts, "expert count must split evenly over a warp");

template <typename IdT>
__global__ void __launch_bounds__(128) moe_align_small_kernel(const IdT *__restrict__ ids, int R,
                                                              int32_t *__restrict__ sorted_ids,
                                                              int32_t *__restrict__ expert_ids,
                                                              int32_t *__restrict__ postpad, bool vec_out) {
  // The whole layout is built by warp 0: no CTA-wide barrier sits on the
  // critical path, which starts with the route-id loads.  Extra warps (the
  // caller's num_warps) have nothing to do.
  if (threadIdx.x >= 32) return;
  __shared__ __align__(16) int s_count[kMoeExperts];
  __shared__ __align__(16) int s_offset[kMoeExperts];
  __shared__ __align__(16) int s_sorted[kMoeMaxRoutes * 8];
  __shared__ __align__(16) int s_experts[kMoeMaxRoutes];
  const int lane = threadIdx.x;
  const unsigned lt = (1u << lane) - 1u;

  // Route lane (half 0) and lane + 32 (half 1).  Validity is decided on the
  // full-width id, before narrowing (an int64 id of 2^32 + 5 is invalid).
  long long raw0 = -1, raw1 = -1;
  if (lane < R) raw0 = (long long)ids[lane];
  if (lane + 32 < R) raw1 = (long long)ids[lane + 32];

  // Initialise while the loads are in flight: padding = R, unused blocks = -1.
  const int4 pad4 = make_int4(R, R, R, R);
  for (int i = lane; i < 2 * R; i += 32) reinterpret_cast<int4 *>(s_sorted)[i] = pad4;  // 8R ints
  for (int i = lane; i < R; i += 32) s_experts[i] = -1;
  for (int i = lane; i < kMoeExperts; i += 32) s_count[i] = 0;
  __syncwarp();

  const int e0 = (raw0 >= 0 && raw0 < kMoeExperts) ? (int)raw0 : -1;
  const int e1 = (raw1 >= 0 && raw1 < kMoeExperts) ? (int)raw1 : -1;
  // Invalid routes get a key no valid expert uses; they never scatter.
  const unsigned m0 = __match_any_sync(0xffffffffu, e0 >= 0 ? e0 : 0x7fffffff);
  const int rank0 = __popc(m0 & lt);
  if (e0 >= 0 && rank0 == 0) s_count[e0] = __popc(m0);
  __syncwarp();
  const int base1 = e1 >= 0 ? s_count[e1] : 0;  // routes of half 0 precede half 1
  const unsigned m1 = __match_any_sync(0xffffffffu, e1 >= 0 ? e1 : 0x7fffffff);
  const int rank1 = base1 + __popc(m1 & lt);
  __syncwarp();
  if (e1 >= 0 && __popc(m1 & lt) == 0) s_count[e1] = base1 + __popc(m1);
  __syncwarp();

  // Exclusive prefix of padded counts: lane owns experts [9 lane, 9 lane + 9).
  int local[kMoePerLane];
  int sum = 0;
#pragma unroll
  for (int k = 0; k < kMoePerLane; ++k) {
    local[k] = sum;
    sum += (s_count[kMoePerLane * lane + k] + 7) & ~7;
  }
  int incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  const int excl = incl - sum;
#pragma unroll
  for (int k = 0; k < kMoePerLane; ++k) s_offset[kMoePerLane * lane + k] = excl + local[k];
  __syncwarp();
  // Scatter: route j goes to off_e + rank_j.  Offsets are multiples of 8, so
  // the route whose rank is a multiple of 8 opens block (off_e + rank_j) / 8
  // of its expert: exactly ceil(count_e / 8) blocks per expert, no loop.
  if (e0 >= 0) {
    const int pos = s_offset[e0] + rank0;
    s_sorted[pos] = lane;
    if ((rank0 & 7) == 0) s_experts[pos >> 3] = e0;
  }
  if (e1 >= 0) {
    const int pos = s_offset[e1] + rank1;
    s_sorted[pos] = lane + 32;
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
  if (lane == 31) postpad[0] = incl;
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
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int R = (int)num_routes;
  const bool vec_out = (uintptr_t)sorted_ids % 16 == 0 && (uintptr_t)expert_ids % 16 == 0;
  if (ids_is_int64)
    moe_align_small_kernel<long long><<<1, 32 * num_warps, 0, s>>>(static_cast<const long long *>(topk_ids), R,
                                                                  sorted_ids, expert_ids, postpad, vec_out);
  else
    moe_align_small_kernel<int32_t><<<1, 32 * num_warps, 0, s>>>(static_cast<const int32_t *>(topk_ids), R,
                                                                 sorted_ids, expert_ids, postpad, vec_out);
  return check_launch("moe_align_small launch");
}
