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
// B200 design, one persistent CTA of 10 warps per SM, work item = (block b,
// 128 output features); the MMA computes D[128 features x bs rows] =
// W_e[128 x K] . A_rows[bs x K]^T with M = 128 and N = bs in {16..64}:
//  * warp 0 (one lane): per 64-wide K step, a bulk copy of the step's 4 KB
//    of packed int4 weights and a TMA tile::gather4 of the block's activation
//    rows (row s / top_k; padding rows read as zeros) into a 128B-swizzled,
//    K-major shared tile, four pipeline stages;
//  * warps 2..5: dequantise the weights into a 128B-swizzled K-major bf16
//    tile (one thread per feature row; nibbles pre-interleaved by
//    titan_moe_w4a16_pack so one LOP3 yields a bf16 pair);
//  * warp 1 (one lane): four tcgen05.mma kind::f16 (K = 16 each) per step
//    into a double-buffered tensor-memory accumulator (2 x 64 columns),
//    tcgen05.commit frees the stage / publishes the accumulator;
//  * warps 6..9: tcgen05.ld of the accumulator (one lane quarter each),
//    topk weighting, bf16 stores of the block's rows.
// Every wait is an mbarrier wait bounded in time; a wait that gives up sets
// the device error word and the CTA abandons its remaining work items.
#include "titan_common.cuh"

namespace titan {
namespace moeg {

constexpr int kBM = 128;           // output features per work item (MMA M)
constexpr int kBK = 64;            // K per pipeline step: one 128-byte bf16 row
constexpr int kStages = 4;
constexpr int kMaxBS = 64;         // block rows (MMA N)
constexpr int kWarps = 10;
constexpr int kThreads = kWarps * 32;
constexpr int kStepWBytes = kBM * kBK / 2;  // packed int4 weights of one step: 4 KB
constexpr int kTmemCols = 128;     // two accumulators of up to 64 fp32 columns

struct Smem {
  alignas(1024) uint8_t wtile[kStages][kBM * kBK * 2];     // 16 KB per stage, bf16, SW128 K-major
  alignas(1024) uint8_t atile[kStages][kMaxBS * kBK * 2];  // 8 KB per stage, bf16, SW128 K-major
  alignas(128) uint8_t wraw[kStages][kStepWBytes];         // 4 KB per stage, packed int4
  alignas(16) uint16_t sscale[kStages][kBM];               // the step's group scales (bf16 bits)
  alignas(8) uint64_t full_a[kStages];                     // activation rows landed (tx bytes)
  uint64_t full_w[kStages];                                // packed weights landed (tx bytes)
  uint64_t deq[kStages];                                   // dequantised tile written (4 warps)
  uint64_t empty[kStages];                                 // stage consumed by the MMAs (commit)
  uint64_t acc_full[2];                                    // accumulator ready (commit)
  uint64_t acc_empty[2];                                   // accumulator read out (4 warps)
  uint64_t drain;                                          // every MMA of this CTA completed
  int rows_p[kMaxBS];                                      // producer: gather row of each block row
  uint32_t tmem_base;
  int abort_flag;                                          // a bounded wait gave up
};

struct Params {
  const uint8_t *wq;                 // packed weights, [E][N/128][K/64][4096 B]
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
// stop waiting at their next wait.
__device__ __forceinline__ bool wait_or_abort(Smem &sm, uint64_t *bar, uint32_t parity) {
  if (*reinterpret_cast<volatile int *>(&sm.abort_flag)) return false;
  if (mbar_wait_bounded(bar, parity, kLongWaitCycles)) return true;
  *reinterpret_cast<volatile int *>(&sm.abort_flag) = 1;
  return false;
}

__global__ void __launch_bounds__(kThreads, 1)
    moe_w4a16_gemm_kernel(const Params p, const __grid_constant__ CUtensorMap a_map) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The dynamic window is 16-byte aligned by contract; align the tiles to 1024.
  Smem &sm = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full_a[s], 1);
      mbar_init(&sm.full_w[s], 1);
      mbar_init(&sm.deq[s], 4);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 4);
    }
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {  // tensor-memory owner
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) prefetch_tensormap(&a_map);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  pdl_wait_primary();  // the lists and activations come from earlier kernels
  const int bs = p.bs;
  const int64_t nb_raw = (int64_t)__ldg(p.ntpp) / bs;
  const int64_t nblocks = nb_raw < 0 ? 0 : (nb_raw > p.max_blocks ? p.max_blocks : nb_raw);
  const int ntn = p.N / kBM, nk = p.K / kBK;
  const int64_t items = nblocks * ntn;
  const int64_t pad_id = (int64_t)p.size_m * p.top_k;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    uint32_t g = 0;  // global step counter of this CTA
    for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
      const int64_t b = item / ntn;
      const int nt = (int)(item - b * ntn);
      const int e = __ldg(p.expert_ids + b);
      if (e < 0 || e >= p.num_experts) continue;
      int *rows = sm.rows_p;  // the gathers take rows as operands: reusable once issued
      for (int j = lane; j < bs; j += 32) {
        const int64_t sid = __ldg(p.sorted_ids + b * bs + j);
        rows[j] = (sid >= 0 && sid < pad_id) ? (int)(sid / p.top_k) : -1;
      }
      __syncwarp();
      const uint8_t *wsrc = p.wq + ((int64_t)e * ntn + nt) * nk * (int64_t)kStepWBytes;
      const __nv_bfloat16 *ssrc = p.scales + (int64_t)e * (p.K / 128) * p.N + nt * kBM;
      for (int kc = 0; kc < nk; ++kc, ++g) {
        const int s = (int)(g % kStages);
        const uint32_t use = g / kStages;
        bool ok = true;
        if (use > 0) ok = wait_or_abort(sm, &sm.empty[s], (use - 1) & 1u);
        if (!ok) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&sm.full_w[s], (uint32_t)(kStepWBytes + kBM * 2));
          bulk_g2s(sm.wraw[s], wsrc + (int64_t)kc * kStepWBytes, (uint32_t)kStepWBytes, &sm.full_w[s]);
          bulk_g2s(sm.sscale[s], ssrc + (int64_t)(kc >> 1) * p.N, (uint32_t)(kBM * 2), &sm.full_w[s]);
          mbar_arrive_expect_tx(&sm.full_a[s], (uint32_t)(bs * kBK * 2));
          for (int j = 0; j < bs; j += 4)
            tma_gather4(sm.atile[s] + j * (kBK * 2), &a_map, kc * kBK, rows[j], rows[j + 1], rows[j + 2], rows[j + 3],
                        &sm.full_a[s]);
        }
        __syncwarp();
      }
      if (*reinterpret_cast<volatile int *>(&sm.abort_flag)) break;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    const uint32_t idesc = idesc_bf16(kBM, bs);
    uint32_t g = 0;
    int it = 0;
    for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
      const int64_t b = item / ntn;
      const int e = __ldg(p.expert_ids + b);
      if (e < 0 || e >= p.num_experts) continue;
      const int buf = it & 1;
      const uint32_t use_acc = (uint32_t)(it >> 1);
      bool ok = true;
      if (use_acc > 0) ok = wait_or_abort(sm, &sm.acc_empty[buf], (use_acc - 1) & 1u);
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(buf * 64);
      for (int kc = 0; kc < nk && ok; ++kc, ++g) {
        const int s = (int)(g % kStages);
        const uint32_t use = g / kStages;
        ok = wait_or_abort(sm, &sm.full_a[s], use & 1u) && wait_or_abort(sm, &sm.deq[s], use & 1u);
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_bf16(d, sw128_desc(sm.wtile[s], 32 * k), sw128_desc(sm.atile[s], 32 * k), idesc,
                      (kc > 0 || k > 0) ? 1u : 0u);
          umma_commit(&sm.empty[s]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&sm.acc_full[buf]);
      __syncwarp();
      ++it;
    }
    // Every MMA issued (also after an abort) completes before tensor memory
    // is released.
    if (lane == 0) umma_commit(&sm.drain);
    __syncwarp();
    mbar_wait_bounded(&sm.drain, 0u, kLongWaitCycles);
  } else if (warp < 6) {
    // ---------------------------------------------------- dequantisation
    const int r = tid - 64;  // feature row of the tile, 0..127
    uint32_t g = 0;
    for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
      const int64_t b = item / ntn;
      const int e = __ldg(p.expert_ids + b);
      if (e < 0 || e >= p.num_experts) continue;
      bool ok = true;
      for (int kc = 0; kc < nk; ++kc, ++g) {
        const int s = (int)(g % kStages);
        const uint32_t use = g / kStages;
        ok = wait_or_abort(sm, &sm.full_w[s], use & 1u);
        if (!ok) break;
        const uint32_t sc = sm.sscale[s][r];  // scale of group kc / 2, feature r
        // Packed layout of a step: [half h][row r][16 bytes] (64 nibbles of row r).
        const uint4 w0 = *reinterpret_cast<const uint4 *>(&sm.wraw[s][r * 16]);
        const uint4 w1 = *reinterpret_cast<const uint4 *>(&sm.wraw[s][2048 + r * 16]);
        const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const uint32_t sc2 = sc | (sc << 16);
        uint8_t *dst = sm.wtile[s];
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // chunk c = k 8c .. 8c + 7
          uint32_t v[4];
          nibbles_to_bf16x8(words[c], v);
          *reinterpret_cast<uint4 *>(dst + sw128_offset(r, c)) =
              make_uint4(bf16x2_mul(v[0], sc2), bf16x2_mul(v[1], sc2), bf16x2_mul(v[2], sc2), bf16x2_mul(v[3], sc2));
        }
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.deq[s]);
      }
      if (!ok) break;
    }
  } else {
    // -------------------------------------------------------- epilogue
    const int q = warp & 3;             // lane quarter this warp may read
    const int f = q * 32 + lane;        // feature row of the tile
    int it = 0;
    for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
      const int64_t b = item / ntn;
      const int nt = (int)(item - b * ntn);
      const int e = __ldg(p.expert_ids + b);
      if (e < 0 || e >= p.num_experts) continue;
      const int buf = it & 1;
      // The block's sorted ids, held by every epilogue warp itself (lane l:
      // rows l and l + 32), so no barrier ties the four warps together.
      const int id_lo = lane < bs ? __ldg(p.sorted_ids + b * bs + lane) : -1;
      const int id_hi = lane + 32 < bs ? __ldg(p.sorted_ids + b * bs + lane + 32) : -1;
      if (!wait_or_abort(sm, &sm.acc_full[buf], (uint32_t)(it >> 1) & 1u)) break;
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 64);
      float v[kMaxBS];
#pragma unroll
      for (int j0 = 0; j0 < kMaxBS; j0 += 16) {
        if (j0 < bs) {
          float t[16];
          tmem_ld16(taddr + (uint32_t)j0, t);
#pragma unroll
          for (int i = 0; i < 16; ++i) v[j0 + i] = t[i];
        }
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
      const int n = nt * kBM + f;
#pragma unroll
      for (int j = 0; j < kMaxBS; ++j) {
        if (j < bs) {
          const int64_t sid = __shfl_sync(0xffffffffu, j < 32 ? id_lo : id_hi, j & 31);
          if (sid >= 0 && sid < pad_id) {
            float x = v[j];
            if (p.mul_topk) x *= __ldg(p.topk_weights + sid);
            p.c[sid * p.c_stride + n] = __float2bfloat16_rn(x);
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
typedef CUresult (*EncodeTiledFnG)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFnG encoder_fn() {
  static const EncodeTiledFnG fn = [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFnG>(f);
    cudaGetLastError();
    return static_cast<EncodeTiledFnG>(nullptr);
  }();
  return fn;
}
std::atomic<int> g_moeg_ready[64];
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
  if ((uintptr_t)a % 16 || (a_stride * 2) % 16 || a_stride < k || (uintptr_t)wq_packed % 16)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "moe_w4a16_gemm: A rows and packed weights must be 16-byte aligned");
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
  EncodeTiledFnG encode = encoder_fn();
  if (encode == nullptr) return fail(TITAN_ERR_CUDA, "moe_w4a16_gemm: cuTensorMapEncodeTiled is unavailable");
  // A as a 2-D bf16 tensor [size_m rows][k], rows a_stride elements apart;
  // boxes of 64 elements (128 bytes) by one row, 128-byte swizzle: a
  // tile::gather4 of four rows lands as four rows of the swizzled K-major tile.
  CUtensorMap amap;
  const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)size_m};
  const cuuint64_t strides[1] = {(cuuint64_t)(a_stride * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, 1};
  const cuuint32_t elem[2] = {1, 1};
  CUresult r = encode(&amap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(a), dims, strides, box, elem,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TITAN_ERR_CUDA, "moe_w4a16_gemm: cuTensorMapEncodeTiled failed (%d)", (int)r);

  Params prm;
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
