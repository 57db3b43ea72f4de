// W4A16 MoE GEMM over the split-align block lists, on the 5th-generation
// tensor cores (tcgen05, accumulators in tensor memory).
//
// The consumer of titan_moe_split_align's lists: one call per list, as the
// reference runs one `moe_wna16_marlin_gemm` per list
// (profiles/sm74/titan_prefill/marlin.py:417-444).  For each of the
// ntpp / block_size blocks b of the list, with e = expert_ids[b] and the
// block's routed rows s_j = sorted_ids[b * block_size + j]:
//   C[s_j, n] = sum_k A[s_j / top_k, k] * W_e[n, k]   (s_j < size_m * top_k;
//                                                       larger ids are padding)
//   W_e[n, k] = bf16((q[e, n, k] - 8) * scale[e, k / 128, n])   (uint4b8,
//                                                       group size 128)
// and, with mul_topk_weights, C[s_j, :] *= topk_weights[s_j].  Products and
// sums in fp32, C in bf16.  The dequantised weight is rounded to bf16 before
// the MMA, as Marlin's W4A16 dequantisation does.
//
// B200 design, one persistent CTA of 15 warps per SM, work item = (block b,
// 256 output features: two MMA tiles of M = 128 sharing the activation
// tile), pipeline step = 128 k (one scale group):
//  * warps 0 and 14 (producers): they gather the block's activation rows
//    with TMA tile::gather4 (four 128-byte rows per load, two 64-k halves)
//    straight into 128B-swizzled K-major tiles, padding rows as out-of-map
//    rows that read as zeros; the gathers of a step are split between the
//    two warps, because lanes of one warp issue them one after another
//    (one warp: 2360 us at the bench shape, two: 1948, four: 2048, six:
//    2096).  Warp 0's lane 0 also bulk-copies the step's packed int4
//    weights (16 KB for the tile pair) and group scales.  Everything lands
//    on one mbarrier per stage, six stages;
//  * warps 2..9 (dequantisation): thread = feature row of one tile; the
//    step's 128 k become 64 columns of bf16 pairs in tensor memory (two
//    tcgen05.st), two buffers; the weights never pass through shared memory
//    in bf16;
//  * warp 1 (one lane): sixteen tcgen05.mma kind::f16 per step (2 tiles x
//    8 x K16, A = the dequantised weights in tensor memory, B = the rows)
//    into double-buffered accumulators, then one tcgen05.commit that frees
//    the stage and the weight buffer together.  The MMA lane waits on one
//    barrier per step (the dequantisation warps have seen the stage land),
//    so a round of synchronisation serves sixteen MMAs;
//  * warps 10..13: tcgen05.ld of the accumulator (one lane quarter each),
//    topk weighting, bf16 stores of the block's rows.
// Every wait is an mbarrier wait bounded in time; a wait that gives up sets
// the device error word and the CTA abandons its remaining work items, then
// waits (bounded) for its copies in flight and its MMAs before it releases
// tensor memory and exits.
#include "titan_common.cuh"

namespace titan {
namespace moeg {

constexpr int kBM = 128;           // output features per MMA tile (M)
constexpr int kNT = 2;             // MMA tiles per work item, sharing one activation tile
constexpr int kBK = 128;           // K per pipeline step (one scale group)
constexpr int kHalfK = 64;         // K per 128-byte swizzled row: the activation tile is two halves
constexpr int kStages = 6;         // stages (packed weights, scales, activation rows)
constexpr int kWBufs = 2;          // dequantised weight buffers in tensor memory
constexpr int kMaxBS = 64;         // block rows (MMA N)
constexpr int kDeqWarps = 8;
constexpr int kGatherWarps = 2;    // warps issuing the row gathers: 0 and 14
constexpr int kWarps = 15;         // 0 producer, 1 MMA, 2..9 dequantisation, 10..13 epilogue, 14 gathers
constexpr int kThreads = kWarps * 32;
constexpr int kStepWBytes = kBM * kBK / 2;   // packed int4 of one tile per step: 8 KB
constexpr int kHalfBytes = kMaxBS * 128;     // one 64-k half of the activation tile: 8 KB
constexpr int kTmemCols = 512;
constexpr int kColAcc = 0;         // accumulators: [2 sets][kNT tiles][64 fp32 columns]
constexpr int kColA = 256;         // dequantised weights: [kWBufs][kNT tiles][64 columns of bf16 pairs]

struct Smem {
  alignas(1024) uint8_t act[kStages][2][kHalfBytes];       // bf16 rows, SW128 K-major, two 64-k halves
  alignas(128) uint8_t wraw[kStages][kNT * kStepWBytes];   // the pair's packed int4 of the step
  alignas(16) uint16_t sscale[kStages][kNT * kBM];         // the step's group scales (bf16 bits)
  alignas(8) uint64_t full[kStages];                        // weights + scales + rows landed (tx bytes)
  uint64_t done[kStages];                                   // the step's MMAs completed (commit)
  uint64_t deq[kWBufs];                                     // dequantised tiles written (8 warps)
  uint64_t acc_full[2];                                     // accumulators ready (MMA commit)
  uint64_t acc_empty[2];                                    // accumulators read out (4 warps)
  uint64_t drain;                                           // every MMA of this CTA completed
  uint32_t tmem_base;
  int abort_flag;                                           // a bounded wait gave up
};

struct Params {
  int64_t a_stride;                  // elements between activation rows (the tensor map holds the rows)
  const uint8_t *wq;                 // packed weights: per expert, tile pairs x k steps x 8 KB tiles
  const __nv_bfloat16 *scales;       // [E][K/128][N]
  const int32_t *sorted_ids;
  const int32_t *expert_ids;
  const int32_t *ntpp;
  const float *topk_weights;         // [size_m * top_k] when mul_topk_weights
  __nv_bfloat16 *c;
  int64_t c_stride;                  // elements between rows of C
  int size_m, top_k, N, K, bs, mul_topk, num_experts;
  int64_t max_blocks;                // capacity of expert_ids
};

// --------------------------------------------------------------- tcgen05 PTX
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] . B[smem desc]^T, kind::f16 (bf16 in, fp32 accumulate).
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] . B[smem desc]^T, kind::f16; A: M = 128 lanes (rows),
// each 32-bit column two consecutive k (bf16), K = 16 = eight columns.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 consecutive 32-bit columns of this thread's lane (this warp's lane quarter).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// The mbarrier completes once every tcgen05.mma issued before by this thread has.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 16 consecutive fp32 columns of this warp's 32 lanes (lane quarter warp % 4).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzle
// layout: rows of 128 bytes (64 bf16), 8-row atoms of 1024 bytes stacked
// densely (stride 1024 B), atoms 1024-byte aligned.  Fields: start address
// >> 4 (bits 0-13), leading-dimension byte offset >> 4 = 1 (unused by the
// swizzled K-major layout), stride byte offset >> 4 (bits 32-45), the
// descriptor version 1 of this architecture (bits 46-47) and the layout type
// 2 = 128-byte swizzle (bits 61-63).  The MMA's K = 16 slice k of a 64-wide
// row starts 32 k bytes further (the swizzle is applied to the address).
__device__ __forceinline__ uint64_t sw128_desc(const void *tile, int k_bytes) {
  const uint64_t start = (uint64_t)((smem_u32(tile) + (uint32_t)k_bytes) >> 4) & 0x3FFFull;
  return start | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulator (bits 4-5 = 1), A
// and B bf16 (bits 7-9 = 1, bits 10-12 = 1), both K-major, N >> 3 in bits
// 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Byte offset of (row r, 16-byte chunk c) in a 128B-swizzled K-major tile.
__device__ __forceinline__ int sw128_offset(int r, int c) { return (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4); }

// Four packed nibble pairs of one 32-bit word -> four bf16x2 of (q - 8):
// nibble positions (0,4), (1,5), (2,6), (3,7) hold consecutive k (the
// packing interleaves them), so one LOP3 per pair builds the bf16 bits of
// 128 + q (0x4300 | q), one packed subtraction of 136 leaves q - 8 exactly.
__device__ __forceinline__ void nibbles_to_bf16x8(uint32_t w, uint32_t (&out)[4]) {
  const uint32_t bias = 0x43084308u;  // bf16x2 {136, 136}
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t x = ((w >> (4 * i)) & 0x000F000Fu) | 0x43004300u;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(out[i]) : "r"(x), "r"(bias));
  }
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Wait with the CTA-wide abort flag: once one role has given up, the others
// stop waiting at their next wait.  Bounded like mbar_wait_bounded, but the
// clock is read once per 32 polls, so waiting warps take fewer issue slots
// from the dequantisation warps.
__device__ __forceinline__ bool wait_or_abort(Smem &sm, uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (*reinterpret_cast<volatile int *>(&sm.abort_flag)) return false;
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > kLongWaitCycles) {
      atomicCAS(&g_device_error, 0, kDevErrMbarrierTimeout);
      *reinterpret_cast<volatile int *>(&sm.abort_flag) = 1;
      return false;
    }
  }
}

// Bounded wait for a stage's copies at exit (they land in microseconds).
constexpr long long kDrainWaitCycles = 20000000LL;

__global__ void __launch_bounds__(kThreads, 1)
    moe_w4a16_gemm_kernel(const Params p, const __grid_constant__ CUtensorMap amap) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The dynamic window is 16-byte aligned by contract; align the tiles to 1024.
  Smem &sm = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);   // the producer's expect-tx arrival; the copies complete the bytes
      mbar_init(&sm.done[s], 1);
    }
    for (int w = 0; w < kWBufs; ++w) mbar_init(&sm.deq[w], kDeqWarps);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 4);
    }
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (tid == 32) prefetch_tensormap(&amap);
  if (warp == 1) {  // tensor-memory owner
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  pdl_wait_primary();  // the lists and activations come from earlier kernels
  const int bs = p.bs;
  const int64_t nb_raw = (int64_t)__ldg(p.ntpp) / bs;
  const int64_t nblocks = nb_raw < 0 ? 0 : (nb_raw > p.max_blocks ? p.max_blocks : nb_raw);
  const int ntn = p.N / kBM, nk = p.K / kBK;
  const int npairs = (ntn + kNT - 1) / kNT;  // work items per block: pairs of 128-feature tiles
  const int64_t items = nblocks * npairs;
  const int64_t pad_id = (int64_t)p.size_m * p.top_k;
  // Item = (block b, feature tiles kNT np .. kNT np + nts - 1).
  auto tiles_of = [&](int np) { return min(kNT, ntn - kNT * np); };

  if (warp == 0 || warp >= 2 + kDeqWarps + 4) {
    // --------------------------------------------------------- producers
    // Gather l < bs / 2 of each step (half h = l / (bs / 4), rows 4 i .. 4 i
    // + 3 with i = l % (bs / 4)) is issued by lane l / kGatherWarps of
    // producer warp l % kGatherWarps.
    // Warp 0 also arms the stage's barrier and bulk-copies the weights.
    const int pw = warp == 0 ? 0 : warp - (2 + kDeqWarps + 4) + 1;
    const int ng = bs >> 2;
    const int l = kGatherWarps * lane + pw;
    const bool gl = l < 2 * ng;
    const int gh = gl ? l / ng : 0, gi = gl ? l % ng : 0;
    uint32_t g = 0;  // step counter of this CTA
    bool ok = true;
    for (int64_t item = blockIdx.x; item < items && ok; item += gridDim.x) {
      const int64_t b = item / npairs;
      const int np = (int)(item - b * npairs), nts = tiles_of(np);
      const int e = __ldg(p.expert_ids + b);
      if (e < 0 || e >= p.num_experts) continue;
      // Activation row of block rows lane and lane + 32 (size_m: padding,
      // outside the map, reads as zeros), then this lane's four gather rows.
      int row_lo, row_hi;
      {
        const int64_t s0 = lane < bs ? __ldg(p.sorted_ids + b * bs + lane) : -1;
        const int64_t s1 = lane + 32 < bs ? __ldg(p.sorted_ids + b * bs + lane + 32) : -1;
        row_lo = (s0 >= 0 && s0 < pad_id) ? (int)(s0 / p.top_k) : p.size_m;
        row_hi = (s1 >= 0 && s1 < pad_id) ? (int)(s1 / p.top_k) : p.size_m;
      }
      int gr[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int j = 4 * gi + m;
        const int lo = __shfl_sync(0xffffffffu, row_lo, j & 31);
        const int hi = __shfl_sync(0xffffffffu, row_hi, j & 31);
        gr[m] = j < 32 ? lo : hi;
      }
      // Packed weights of the pair: per step, its nts tiles' 8 KB back to back.
      const uint8_t *wsrc = p.wq + ((int64_t)e * ntn * nk + (int64_t)kNT * np * nk) * kStepWBytes;
      const __nv_bfloat16 *ssrc = p.scales + (int64_t)e * nk * p.N + kNT * np * kBM;
      const uint32_t bytes = (uint32_t)(nts * (kStepWBytes + kBM * 2) + 2 * bs * 128);
      for (int kc = 0; kc < nk; ++kc, ++g) {
        const int s = (int)(g % kStages);
        const uint32_t use = g / kStages;
        if (use > 0) ok = wait_or_abort(sm, &sm.done[s], (use - 1) & 1u);
        if (!ok) break;
        if (pw == 0 && lane == 0) {
          mbar_arrive_expect_tx(&sm.full[s], bytes);
          bulk_g2s(sm.wraw[s], wsrc + (int64_t)kc * nts * kStepWBytes, (uint32_t)(nts * kStepWBytes), &sm.full[s]);
          bulk_g2s(sm.sscale[s], ssrc + (int64_t)kc * p.N, (uint32_t)(nts * kBM * 2), &sm.full[s]);
        }
        if (gl)
          tma_gather4(&sm.act[s][gh][gi * 512], &amap, kc * kBK + gh * kHalfK, gr[0], gr[1], gr[2], gr[3],
                      &sm.full[s]);
      }
    }
    // Copies issued and not consumed (after an abort) land before the CTA
    // releases its shared memory: each producer warp waits for the last
    // phase of every stage it issued into.
    if (lane == 0) {
      const uint32_t first = g > (uint32_t)kStages ? g - kStages : 0u;
      for (uint32_t gg = first; gg < g; ++gg)
        mbar_wait_bounded(&sm.full[gg % kStages], (gg / kStages) & 1u, kDrainWaitCycles);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    const uint32_t idesc = idesc_bf16(kBM, bs);
    uint32_t g = 0;
    int it = 0;
    bool ok = true;
    for (int64_t item = blockIdx.x; item < items && ok; item += gridDim.x) {
      const int64_t b = item / npairs;
      const int np = (int)(item - b * npairs), nts = tiles_of(np);
      const int e = __ldg(p.expert_ids + b);
      if (e < 0 || e >= p.num_experts) continue;
      const int ab = it & 1;
      const uint32_t use_acc = (uint32_t)(it >> 1);
      if (use_acc > 0) ok = wait_or_abort(sm, &sm.acc_empty[ab], (use_acc - 1) & 1u);
      tc_fence_after();
      for (int kc = 0; kc < nk && ok; ++kc, ++g) {
        const int s = (int)(g % kStages), wb = (int)(g % kWBufs);
        // The dequantisation warps arrive only after they have seen the
        // stage land, so this one wait covers the rows as well.
        ok = wait_or_abort(sm, &sm.deq[wb], (g / kWBufs) & 1u);
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) {
          for (int t = 0; t < nts; ++t) {
            const uint32_t d = tmem + (uint32_t)(kColAcc + ab * (kNT * 64) + t * 64);
            const uint32_t aw = tmem + (uint32_t)(kColA + wb * (kNT * 64) + t * 64);
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k)
              umma_bf16_ts(d, aw + 8 * k, sw128_desc(sm.act[s][k >> 2], 32 * (k & 3)), idesc,
                           (kc > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&sm.done[s]);  // frees the stage and the weight buffer
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&sm.acc_full[ab]);
      __syncwarp();
      ++it;
    }
    // Every MMA issued (also after an abort) completes before tensor memory
    // is released.
    if (lane == 0) umma_commit(&sm.drain);
    __syncwarp();
    mbar_wait_bounded(&sm.drain, 0u, kLongWaitCycles);
  } else if (warp < 2 + kDeqWarps) {
    // ---------------------------------------------------- dequantisation
    // Warp w writes tensor-memory lanes 32 (w % 4) .. + 31: thread = feature
    // row r of tile t, its 128 dequantised k of the step as 64 columns of
    // bf16 pairs (two tcgen05.st).
    const int r = 32 * (warp & 3) + lane;
    const int t = (warp - 2) >> 2;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    uint32_t g = 0;
    bool ok = true;
    for (int64_t item = blockIdx.x; item < items && ok; item += gridDim.x) {
      const int64_t b = item / npairs;
      const int np = (int)(item - b * npairs), nts = tiles_of(np);
      const int e = __ldg(p.expert_ids + b);
      if (e < 0 || e >= p.num_experts) continue;
      for (int kc = 0; kc < nk; ++kc, ++g) {
        const int s = (int)(g % kStages), wb = (int)(g % kWBufs);
        ok = wait_or_abort(sm, &sm.full[s], (g / kStages) & 1u);
        // Buffer wb was last read by the MMAs of step g - kWBufs.
        if (ok && g >= (uint32_t)kWBufs) {
          const uint32_t gp = g - kWBufs;
          ok = wait_or_abort(sm, &sm.done[gp % kStages], (gp / kStages) & 1u);
        }
        if (!ok) break;
        tc_fence_after();
        if (t < nts) {
          // Packed layout of a tile step: [quarter c][row r][16 bytes],
          // quarter c = the row's k 32 c .. 32 c + 31 (four 32-bit words of
          // eight k each).
          const uint8_t *raw = sm.wraw[s] + t * kStepWBytes + r * 16;
          const uint32_t sc = sm.sscale[s][t * kBM + r];
          const uint32_t sc2 = sc | (sc << 16);
          const uint32_t col = (uint32_t)(kColA + wb * (kNT * 64) + t * 64);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const uint4 w0 = *reinterpret_cast<const uint4 *>(raw + (2 * hh) * 2048);
            const uint4 w1 = *reinterpret_cast<const uint4 *>(raw + (2 * hh + 1) * 2048);
            const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            uint32_t v[32];
#pragma unroll
            for (int c = 0; c < 8; ++c) {  // word c = k 8c .. 8c + 7 of this half = columns 4c .. 4c + 3
              uint32_t x[4];
              nibbles_to_bf16x8(words[c], x);
#pragma unroll
              for (int i = 0; i < 4; ++i) v[4 * c + i] = bf16x2_mul(x[i], sc2);
            }
            tmem_st32(tmem + lane_base + col + 32u * hh, v);
          }
          tmem_st_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.deq[wb]);
      }
    }
  } else {
    // -------------------------------------------------------- epilogue
    const int q = warp & 3;             // lane quarter this warp may read
    const int f = q * 32 + lane;        // feature row within a tile
    int it = 0;
    for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
      const int64_t b = item / npairs;
      const int np = (int)(item - b * npairs), nts = tiles_of(np);
      const int e = __ldg(p.expert_ids + b);
      if (e < 0 || e >= p.num_experts) continue;
      const int ab = it & 1;
      // The block's sorted ids, held by every epilogue warp itself (lane l:
      // rows l and l + 32), so no barrier ties the four warps together.
      const int id_lo = lane < bs ? __ldg(p.sorted_ids + b * bs + lane) : -1;
      const int id_hi = lane + 32 < bs ? __ldg(p.sorted_ids + b * bs + lane + 32) : -1;
      if (!wait_or_abort(sm, &sm.acc_full[ab], (uint32_t)(it >> 1) & 1u)) break;
      tc_fence_after();
      // One tile at a time (64 registers of accumulator); the accumulator
      // set is released after the last tile's load.
#pragma unroll 1
      for (int t = 0; t < nts; ++t) {
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(kColAcc + ab * (kNT * 64) + t * 64);
        float v[kMaxBS];
#pragma unroll
        for (int j0 = 0; j0 < kMaxBS; j0 += 16) {
          if (j0 < bs) {
            float x[16];
            tmem_ld16(taddr + (uint32_t)j0, x);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[j0 + i] = x[i];
          }
        }
        tmem_ld_wait();
        if (t == nts - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.acc_empty[ab]);
        }
        __nv_bfloat16 *col = p.c + (int64_t)(kNT * np + t) * kBM + f;
#pragma unroll
        for (int j = 0; j < kMaxBS; ++j) {
          if (j < bs) {
            const int64_t sid = __shfl_sync(0xffffffffu, j < 32 ? id_lo : id_hi, j & 31);
            if (sid >= 0 && sid < pad_id) {
              const float wgt = p.mul_topk ? __ldg(p.topk_weights + sid) : 1.0f;
              col[sid * p.c_stride] = __float2bfloat16_rn(v[j] * wgt);
            }
          }
        }
      }
      ++it;
    }
  }

  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace moeg

namespace {
std::atomic<int> g_moeg_ready[64];

// Tensor map of the activations for the row gather: bf16 [size_m][k], rows
// a_stride elements apart, boxes of 64 elements (one 128-byte swizzled row)
// by one row; row size_m and beyond (the padding rows' coordinate) read as
// zeros.  The last encoding of each host thread is reused.
int act_tensor_map(const void *a, int64_t size_m, int64_t k, int64_t a_stride, CUtensorMap *out) {
  const EncodeTiledFn encode = tensor_map_encoder();
  if (encode == nullptr) return fail(TITAN_ERR_CUDA, "moe_w4a16_gemm: cuTensorMapEncodeTiled is unavailable");
  static thread_local const void *last_a = nullptr;
  static thread_local int64_t last_m = -1, last_k = -1, last_stride = -1;
  static thread_local CUtensorMap last_map;
  if (a == last_a && size_m == last_m && k == last_k && a_stride == last_stride) {
    *out = last_map;
    return TITAN_OK;
  }
  const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)size_m};
  const cuuint64_t strides[1] = {(cuuint64_t)a_stride * 2};
  const cuuint32_t box[2] = {64, 1};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = encode(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(a), dims, strides, box, elem,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TITAN_ERR_CUDA, "moe_w4a16_gemm: cuTensorMapEncodeTiled failed (%d) for rows=%lld k=%lld stride=%lld",
                (int)r, (long long)size_m, (long long)k, (long long)a_stride);
  last_a = a;
  last_m = size_m;
  last_k = k;
  last_stride = a_stride;
  last_map = *out;
  return TITAN_OK;
}
std::atomic<int> g_moeg_sms[64];
}  // namespace
}  // namespace titan

extern "C" int64_t titan_moe_w4a16_packed_bytes(int64_t num_experts, int64_t n, int64_t k) {
  if (num_experts <= 0 || n <= 0 || k <= 0 || n % 128 || k % 128) return -1;
  return num_experts * n * k / 2;
}

extern "C" int titan_moe_w4a16_gemm(const void *a, int64_t a_stride, int64_t size_m, void *c, int64_t c_stride,
                                    const void *wq_packed, const void *scales, const int32_t *sorted_ids,
                                    const int32_t *expert_ids, int64_t max_blocks, const int32_t *ntpp,
                                    const float *topk_weights, int block_size, int top_k, int mul_topk_weights,
                                    int64_t num_experts, int64_t n, int64_t k, titan_stream_t stream) {
  using namespace titan;
  using namespace titan::moeg;
  if (block_size != 16 && block_size != 32 && block_size != 48 && block_size != 64)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_w4a16_gemm: block_size must be 16, 32, 48 or 64, got %d", block_size);
  if (n <= 0 || k <= 0 || n % kBM || k % 128 || n > (1 << 20) || k > (1 << 20))
    return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_w4a16_gemm: N must be a multiple of 128 and K of 128 (N=%lld K=%lld)",
                (long long)n, (long long)k);
  if (size_m < 0 || top_k < 1 || num_experts < 1 || max_blocks < 0 || size_m * top_k > 0x7fffffffLL)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_w4a16_gemm: invalid sizes");
  if (a == nullptr || c == nullptr || wq_packed == nullptr || scales == nullptr || sorted_ids == nullptr ||
      expert_ids == nullptr || ntpp == nullptr || (mul_topk_weights && topk_weights == nullptr))
    return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_w4a16_gemm: null pointer");
  if ((uintptr_t)a % 16 || (a_stride * 2) % 16 || a_stride < k || (uintptr_t)wq_packed % 16 || (uintptr_t)scales % 16)
    return fail(TITAN_ERR_INVALID_ARGUMENT,
                "moe_w4a16_gemm: A rows, packed weights and scales must be 16-byte aligned");
  if (c_stride < n) return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_w4a16_gemm: C rows shorter than N");
  if (size_m == 0 || max_blocks == 0) return TITAN_OK;

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "moe_w4a16_gemm: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(TITAN_ERR_CUDA, "moe_w4a16_gemm: device ordinal %d out of range", dev);
  const size_t smem = sizeof(Smem) + 1024;  // + alignment slack
  if (!g_moeg_ready[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(setup_mutex());
    if (!g_moeg_ready[dev].load(std::memory_order_relaxed)) {
      e = cudaFuncSetAttribute(moe_w4a16_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      int sms = 0;
      if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "moe_w4a16_gemm: setup: %s", cudaGetErrorString(e));
      g_moeg_sms[dev].store(sms, std::memory_order_relaxed);
      g_moeg_ready[dev].store(1, std::memory_order_release);
    }
  }
  CUtensorMap amap;
  const int rc = act_tensor_map(a, size_m, k, a_stride, &amap);
  if (rc != TITAN_OK) return rc;
  Params prm;
  prm.a_stride = a_stride;
  prm.wq = static_cast<const uint8_t *>(wq_packed);
  prm.scales = static_cast<const __nv_bfloat16 *>(scales);
  prm.sorted_ids = sorted_ids;
  prm.expert_ids = expert_ids;
  prm.ntpp = ntpp;
  prm.topk_weights = topk_weights;
  prm.c = static_cast<__nv_bfloat16 *>(c);
  prm.c_stride = c_stride;
  prm.size_m = (int)size_m;
  prm.top_k = top_k;
  prm.N = (int)n;
  prm.K = (int)k;
  prm.bs = block_size;
  prm.mul_topk = mul_topk_weights ? 1 : 0;
  prm.num_experts = (int)num_experts;
  prm.max_blocks = max_blocks;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)g_moeg_sms[dev].load(std::memory_order_relaxed));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, moe_w4a16_gemm_kernel, prm, amap);
  if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "moe_w4a16_gemm launch: %s", cudaGetErrorString(e));
  return TITAN_OK;
}
