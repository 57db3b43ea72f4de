// INT8 latent KV writer: each warp quantises four token rows.
//
// Follows kernels/titan_kv.py:7-21 (the reference `_store_int8`):
//   scale = max(max|x| / 127, 1e-12)            (fp32, IEEE division)
//   q     = clamp(nearbyint(x / scale), -127, 127)
//   row   = cache + (slot / block) * stride0 + (slot % block) * stride1
//   bytes [0,512) = q, bytes [512,528) = fp32 {scale, 0, 0, 0}; slot < 0 skips.
//   max / maximum / minimum drop NaN operands, as Triton's default forms do on
//   the GPU: NaN values are ignored by the row max and store -127; an inf
//   makes the scale inf (finite values store 0, +-inf stores -127).
//
// Layout of the work: for each of its rows, lane l of the warp owns latent
// values [16 l, 16 l + 16): two 16-byte loads of bf16, one 16-byte store of int8.
// Lane 0 also writes the 16-byte scale block.  The amax is a warp-shuffle max.
// HBM traffic per row: 1024 B read + 528 B written + 8 B slot.
#include "titan_common.cuh"

#include <algorithm>

namespace titan {

constexpr int kKvWarpsPerCta = 8;
constexpr int kKvRowsPerWarp = 4;

// 1.5 * 2^23: adding it to |y| < 2^22 rounds y to an integer (round to
// nearest even, the fp32 addition's own rounding) and leaves that integer's
// two's-complement low byte in the low byte of the sum's bit pattern.
constexpr float kRoundMagic = 12582912.0f;

// Quantise 16 values to 4 packed int8 words: q = rint(v / scale) with the
// correctly rounded quotient.  With r = fl(1/scale), y = fl(v * r) satisfies
// |y - v/scale| <= |v/scale| (2u + u^2) <= 1.52e-5 (u = 2^-24, |v/scale| <=
// 127.00002), and the correctly rounded quotient is within half an ulp
// (<= 3.9e-6) of v/scale, so |y - fl(v/scale)| < 1.91e-5.  rint(y) therefore
// equals rint(fl(v/scale)) unless y lies within 1.91e-5 of a half-integer; such
// values (window 2^-14 = 6.1e-5, ~3x margin) are recomputed one by one with
// the IEEE division.  |q| <= 127 needs no clamp: scale >= fl(amax / 127) keeps
// |v / scale| <= 127 (1 + 2^-24), which rounds to at most 127.
__device__ __forceinline__ void quant16(const float (&v)[16], float scale, float rcp, uint32_t (&out)[4]) {
  float m[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float y = v[i] * rcp;
    m[i] = y + kRoundMagic;
    const float r = m[i] - kRoundMagic;
    if (fabsf(y - r) > 0.49993896484375f) m[i] = __fdiv_rn(v[i], scale) + kRoundMagic;  // 0.5 - 2^-14
  }
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t lo = prmt(__float_as_uint(m[4 * w + 0]), __float_as_uint(m[4 * w + 1]), 0x0040u);
    const uint32_t hi = prmt(__float_as_uint(m[4 * w + 2]), __float_as_uint(m[4 * w + 3]), 0x0040u);
    out[w] = prmt(lo, hi, 0x5410u);
  }
}

// Cache row of a slot: block = slot / block_size, offset = slot % block_size;
// a shift when the block size is a power of two (block_shift >= 0).
__device__ __forceinline__ void split_slot(int64_t slot, int64_t block, int block_shift, int64_t &blk, int64_t &off) {
  if (block_shift >= 0) {
    blk = slot >> block_shift;
    off = slot & (block - 1);
  } else {
    blk = slot / block;
    off = slot - blk * block;
  }
}

__device__ __forceinline__ void bf16x2_to_f32(uint32_t w, float &lo, float &hi) {
  lo = __uint_as_float(w << 16);
  hi = __uint_as_float(w & 0xFFFF0000u);
}

__device__ __forceinline__ float warp_amax(float a) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  return a;
}

// scale = max(max|x| / 127, 1e-12) with the IEEE quotient (kernels/titan_kv.py:16),
// without a division: y0 = fl(amax * c), c = fl(1/127), corrected once with
// the exact FMA residual (Markstein, "Computation of elementary functions on
// the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990).  amax is
// the magnitude of a bf16 value, so every possible input can be and is checked
// exhaustively (tests/test_kv_scale_exact.py): the result after the 1e-12
// floor equals the IEEE quotient for all 32,640 non-negative finite bf16.
constexpr float kInv127 = 0.007874015718698502f;  // fl(1/127)
__device__ __forceinline__ float row_scale(float amax) {
  const float y0 = __fmul_rn(amax, kInv127);
  const float r = __fmaf_rn(-y0, 127.0f, amax);
  return fmaxf(__fmaf_rn(r, kInv127, y0), 1.0e-12f);
}

// Rows holding NaN or inf (rare; taken by whole warps so the fast paths keep
// their arithmetic).  The reference's max, maximum and minimum drop NaN
// operands (Triton's default PropagateNan.NONE lowers them to maxnum /
// minnum), so the row max ignores NaN values, an infinite row max gives an
// infinite scale, and a NaN quotient (a NaN value, or +-inf / inf) clamps to
// -127 — CUDA's fmaxf / fminf have the same NaN rule.  A finite row gets the
// same bytes here as on the fast paths: IEEE division throughout.
__device__ __forceinline__ float nonfinite_row_scale(float amax_without_nan) {
  return isinf(amax_without_nan) ? __int_as_float(0x7F800000) : row_scale(amax_without_nan);
}

__device__ __forceinline__ uint32_t quant4_exact(float a, float b, float c, float d, float scale) {
  auto q = [scale](float v) {
    return (uint32_t)__float2int_rn(fminf(fmaxf(rintf(__fdiv_rn(v, scale)), -127.0f), 127.0f)) & 0xFFu;
  };
  return q(a) | q(b) << 8 | q(c) << 16 | q(d) << 24;
}

// True when |v| is inf or NaN.
__device__ __forceinline__ bool not_finite(float v) { return !(fabsf(v) < __int_as_float(0x7F800000)); }

// Each warp quantises kKvRowsPerWarp rows; every row's two 16-byte loads per
// lane are issued before any arithmetic so ~4 KB per warp is in flight.
template <typename SlotT>
__global__ void __launch_bounds__(kKvWarpsPerCta * 32)
    store_int8_vec_kernel(const __nv_bfloat16 *__restrict__ x, int64_t x_row_stride, int8_t *__restrict__ cache,
                          int64_t num_blocks, int64_t block, int block_shift, int64_t cs0, int64_t cs1,
                          const SlotT *__restrict__ slots, int64_t n) {
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t row0 = ((int64_t)blockIdx.x * kKvWarpsPerCta + (threadIdx.x >> 5)) * kKvRowsPerWarp;
  pdl_wait_primary();  // the latents and slots come from earlier kernels
  int64_t slot[kKvRowsPerWarp];
  uint4 a[kKvRowsPerWarp], b[kKvRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kKvRowsPerWarp; ++r) {
    const int64_t row = row0 + r;
    slot[r] = -1;
    a[r] = b[r] = make_uint4(0, 0, 0, 0);
    if (row < n) {
      slot[r] = (int64_t)slots[row];
      const uint8_t *src = reinterpret_cast<const uint8_t *>(x + row * x_row_stride) + lane * 32;
      a[r] = ld_global_nc_v4(src);
      b[r] = ld_global_nc_v4(src + 16);
    }
  }
#pragma unroll
  for (int r = 0; r < kKvRowsPerWarp; ++r) {
    if (slot[r] < 0) continue;
    int64_t blk, off;
    split_slot(slot[r], block, block_shift, blk, off);
    if (blk >= num_blocks) continue;
    float v[16];
    bf16x2_to_f32(a[r].x, v[0], v[1]);
    bf16x2_to_f32(a[r].y, v[2], v[3]);
    bf16x2_to_f32(a[r].z, v[4], v[5]);
    bf16x2_to_f32(a[r].w, v[6], v[7]);
    bf16x2_to_f32(b[r].x, v[8], v[9]);
    bf16x2_to_f32(b[r].y, v[10], v[11]);
    bf16x2_to_f32(b[r].z, v[12], v[13]);
    bf16x2_to_f32(b[r].w, v[14], v[15]);
    float amax = 0.0f;  // fmaxf drops NaN: the max of the non-NaN magnitudes
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      amax = fmaxf(amax, fabsf(v[i]));
      bad |= not_finite(v[i]);
    }
    amax = warp_amax(amax);
    uint32_t q[4];
    float scale;
    if (__any_sync(0xffffffffu, bad)) {  // the row (one per warp here) holds NaN or inf
      scale = nonfinite_row_scale(amax);
#pragma unroll
      for (int w = 0; w < 4; ++w) q[w] = quant4_exact(v[4 * w], v[4 * w + 1], v[4 * w + 2], v[4 * w + 3], scale);
    } else {
      scale = row_scale(amax);
      quant16(v, scale, __frcp_rn(scale), q);
    }
    int8_t *dst = cache + blk * cs0 + off * cs1;
    *reinterpret_cast<uint4 *>(dst + lane * 16) = make_uint4(q[0], q[1], q[2], q[3]);
    if (lane == 0) *reinterpret_cast<uint4 *>(dst + 512) = make_uint4(__float_as_uint(scale), 0u, 0u, 0u);
  }
}

// Streaming kernel for 16-byte-aligned rows.  Persistent CTAs; every warp
// independently quantises two rows per step (one per half-warp), streaming
// its rows through a private 4-stage shared-memory ring filled with cp.async
// (16 bytes per lane per copy), so ~8 KB per warp stay in flight without
// holding registers.  Lane j of a half-warp owns 16-byte chunks j, j+16, j+32,
// j+48 of its row (values [8j, 8j+8) + 128 k): conflict-free shared loads and
// four coalesced 8-byte stores.  The abs-max runs on bf16 bit patterns
// (max.u16x2), the quantisation on packed f32x2 arithmetic.
constexpr int kKvStreamWarps = 8;
constexpr int kKvStreamStages = 4;
constexpr int kKvStageBytes = 2 * 1024;  // two rows
constexpr size_t kKvStreamSmem = (size_t)kKvStreamWarps * kKvStreamStages * kKvStageBytes;

// Packed bf16 max of magnitudes: |result| = max(|a|, |b|) per half (the
// sign is the XOR of the inputs' signs and is masked off by the caller); a
// NaN operand gives NaN (0x7FFF after masking), so a non-finite row is seen.
__device__ __forceinline__ uint32_t bf16x2_absmax(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// 32 values (16 bf16x2 words) of one row held by one lane -> 8 packed int8
// words, four values at a time, on packed f32x2 arithmetic.  With
// rcp = fl(1/scale) the product p = v * rcp is taken exactly inside an FMA
// and rounded once to an integer by adding 1.5 * 2^23: m = RN(p + magic)
// holds rint(p), ties to even.  |p - v/scale| <= |v/scale| 2^-24 <= 7.6e-6
// and the correctly rounded quotient Q = fl(v/scale) is within 2^-18 of
// v/scale, so |p - Q| < 1.15e-5: rint(p) = rint(Q) unless p lies within
// 1.15e-5 of a half-integer.  The residual d = RN(p - rint(p)) (again one
// FMA) flags such values, |d| > 0.5 - 2^-14 (window 6.1e-5, ~5x margin);
// their group of four is recomputed with the IEEE division.  The window test
// stays per group of four values: a warp executes the exact path whenever
// any of its lanes needs it, so wider groups would multiply the divisions.
__device__ __forceinline__ void quant32(const uint32_t (&w)[16], float scale, float rcp, uint32_t (&out)[8]) {
  const float2 rcp2 = make_float2(rcp, rcp);
  const float2 mag2 = make_float2(kRoundMagic, kRoundMagic);
  const float2 neg1 = make_float2(-1.0f, -1.0f);
  constexpr float kWindow = 0.49993896484375f;  // 0.5 - 2^-14
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float2 m[2];
    bool near_half = false;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const uint32_t wd = w[2 * k + e];
      const float2 v = make_float2(__uint_as_float(wd << 16), __uint_as_float(wd & 0xFFFF0000u));
      m[e] = __ffma2_rn(v, rcp2, mag2);                      // magic + rint(v * rcp)
      const float2 nr = __ffma2_rn(m[e], neg1, mag2);         // -rint(v * rcp), exact
      const float2 d = __ffma2_rn(v, rcp2, nr);               // RN(v * rcp - rint(v * rcp))
      near_half |= (fabsf(d.x) > kWindow) | (fabsf(d.y) > kWindow);
    }
    if (near_half) {  // a value within 2^-14 of a half-integer: exact quotient
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint32_t wd = w[2 * k + e];
        m[e].x = __fdiv_rn(__uint_as_float(wd << 16), scale) + kRoundMagic;
        m[e].y = __fdiv_rn(__uint_as_float(wd & 0xFFFF0000u), scale) + kRoundMagic;
      }
    }
    const uint32_t lo = prmt(__float_as_uint(m[0].x), __float_as_uint(m[0].y), 0x0040u);
    const uint32_t hi = prmt(__float_as_uint(m[1].x), __float_as_uint(m[1].y), 0x0040u);
    out[k] = prmt(lo, hi, 0x5410u);
  }
}

template <typename SlotT>
__global__ void __launch_bounds__(kKvStreamWarps * 32, 3)
    store_int8_stream_kernel(const __nv_bfloat16 *__restrict__ x, int64_t x_row_stride, int8_t *__restrict__ cache,
                             int64_t num_blocks, int64_t block, int block_shift, int64_t cs0, int64_t cs1,
                             const SlotT *__restrict__ slots, int64_t n) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane >> 4, j = lane & 15;
  uint8_t *ring = smem + (size_t)warp * kKvStreamStages * kKvStageBytes;
  const int64_t gwarp = (int64_t)blockIdx.x * kKvStreamWarps + warp;
  const int64_t nwarps = (int64_t)gridDim.x * kKvStreamWarps;
  const int64_t pairs = (n + 1) / 2;
  const int64_t my_steps = gwarp < pairs ? (pairs - 1 - gwarp) / nwarps + 1 : 0;
  pdl_launch_dependents();
  pdl_wait_primary();  // the latents and slots come from earlier kernels
  // Step i of this warp covers rows 2 (gwarp + i nwarps) + {0, 1}.
  auto row_of = [&](int64_t i) { return 2 * (gwarp + i * nwarps) + half; };
  auto fetch = [&](int64_t i) {  // this lane's 4 chunks of its row of step i
    if (i < my_steps) {
      const int64_t row = row_of(i);
      if (row < n) {
        const uint8_t *src = reinterpret_cast<const uint8_t *>(x + row * x_row_stride);
        uint8_t *dst = ring + (int)(i % kKvStreamStages) * kKvStageBytes + half * 1024;
#pragma unroll
        for (int k = 0; k < 4; ++k) cp_async_16(dst + (j + 16 * k) * 16, src + (j + 16 * k) * 16);
      }
    }
    cp_async_commit();  // empty groups keep the group count uniform
  };
#pragma unroll
  for (int i = 0; i < kKvStreamStages - 1; ++i) fetch(i);
  int64_t slot_next = (my_steps > 0 && row_of(0) < n) ? (int64_t)slots[row_of(0)] : -1;
  for (int64_t i = 0; i < my_steps; ++i) {
    fetch(i + kKvStreamStages - 1);
    const int64_t slot = slot_next;
    slot_next = (i + 1 < my_steps && row_of(i + 1) < n) ? (int64_t)slots[row_of(i + 1)] : -1;
    cp_async_wait<kKvStreamStages - 1>();
    __syncwarp();
    const uint8_t *row = ring + (int)(i % kKvStreamStages) * kKvStageBytes + half * 1024;
    uint32_t w[16];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint4 c = *reinterpret_cast<const uint4 *>(row + (j + 16 * k) * 16);
      w[4 * k + 0] = c.x;
      w[4 * k + 1] = c.y;
      w[4 * k + 2] = c.z;
      w[4 * k + 3] = c.w;
    }
    uint32_t mx = w[0];
#pragma unroll
    for (int k = 1; k < 16; ++k) mx = bf16x2_absmax(mx, w[k]);
    mx = max(mx & 0x7FFFu, (mx >> 16) & 0x7FFFu);  // |x| as bf16 bits; integer order = value order
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    uint32_t q[8];
    float scale;
    // Bits >= 0x7F80 (inf, or NaN, which outranks every number): a row of
    // this warp holds a non-finite value, and both half-warps take the exact
    // path (same bytes for a finite row).
    if (__any_sync(0xffffffffu, mx >= 0x7F80u)) {
      float amax = 0.0f;  // fmaxf drops NaN
#pragma unroll
      for (int k = 0; k < 16; ++k)
        amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(w[k] << 16)), fabsf(__uint_as_float(w[k] & 0xFFFF0000u))));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      scale = nonfinite_row_scale(amax);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        q[k] = quant4_exact(__uint_as_float(w[2 * k] << 16), __uint_as_float(w[2 * k] & 0xFFFF0000u),
                            __uint_as_float(w[2 * k + 1] << 16), __uint_as_float(w[2 * k + 1] & 0xFFFF0000u), scale);
    } else {
      scale = row_scale(__uint_as_float(mx << 16));
      quant32(w, scale, __frcp_rn(scale), q);
    }
    __syncwarp();  // the stage may be refilled once every lane has read it
    int64_t blk = 0, off = 0;
    if (slot >= 0) split_slot(slot, block, block_shift, blk, off);
    if (slot >= 0 && blk < num_blocks) {
      int8_t *dst = cache + blk * cs0 + off * cs1;
#pragma unroll
      for (int k = 0; k < 4; ++k) *reinterpret_cast<uint2 *>(dst + 8 * j + 128 * k) = make_uint2(q[2 * k], q[2 * k + 1]);
      if (j == 0) *reinterpret_cast<uint4 *>(dst + 512) = make_uint4(__float_as_uint(scale), 0u, 0u, 0u);
    }
  }
  cp_async_wait<0>();
}

// Unaligned fallback (x rows or cache rows not 16-byte aligned): lane l owns
// values l + 32 k, byte stores.  Same arithmetic.
template <typename SlotT>
__global__ void __launch_bounds__(kKvWarpsPerCta * 32)
    store_int8_scalar_kernel(const __nv_bfloat16 *__restrict__ x, int64_t x_row_stride, int8_t *__restrict__ cache,
                             int64_t num_blocks, int64_t block, int block_shift, int64_t cs0, int64_t cs1,
                             const SlotT *__restrict__ slots, int64_t n) {
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kKvWarpsPerCta + (threadIdx.x >> 5);
  if (row >= n) return;
  pdl_wait_primary();  // the latents and slots come from earlier kernels
  const int64_t slot = (int64_t)slots[row];
  if (slot < 0) return;
  int64_t blk, off;
  split_slot(slot, block, block_shift, blk, off);
  if (blk >= num_blocks) return;
  const __nv_bfloat16 *src = x + row * x_row_stride;
  float v[16];
  float amax = 0.0f;  // fmaxf drops NaN
  bool bad = false;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    v[k] = __bfloat162float(src[lane + 32 * k]);
    amax = fmaxf(amax, fabsf(v[k]));
    bad |= not_finite(v[k]);
  }
  amax = warp_amax(amax);
  uint32_t q[4];
  float scale;
  if (__any_sync(0xffffffffu, bad)) {
    scale = nonfinite_row_scale(amax);
#pragma unroll
    for (int w = 0; w < 4; ++w) q[w] = quant4_exact(v[4 * w], v[4 * w + 1], v[4 * w + 2], v[4 * w + 3], scale);
  } else {
    scale = row_scale(amax);
    quant16(v, scale, __frcp_rn(scale), q);
  }
  int8_t *dst = cache + blk * cs0 + off * cs1;
#pragma unroll
  for (int k = 0; k < 16; ++k) dst[lane + 32 * k] = (int8_t)((q[k >> 2] >> (8 * (k & 3))) & 0xFF);
  if (lane < 16) {
    const uint32_t bits = lane < 4 ? __float_as_uint(scale) : 0u;
    dst[512 + lane] = (int8_t)((bits >> (8 * (lane & 3))) & 0xFF);
  }
}

}  // namespace titan

extern "C" int titan_store_int8(const void *x, int64_t x_row_stride, void *cache, int64_t num_blocks,
                                int64_t block_size, int64_t cache_stride0, int64_t cache_stride1,
                                const void *slots, int slots_is_int64, int64_t n_slots, titan_stream_t stream) {
  using namespace titan;
  if (n_slots < 0) return fail(TITAN_ERR_INVALID_ARGUMENT, "store_int8: negative slot count");
  if (n_slots == 0) return TITAN_OK;
  if (x == nullptr || cache == nullptr || slots == nullptr)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "store_int8: null pointer");
  if (block_size <= 0 || num_blocks < 0)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "store_int8: invalid cache geometry");
  const int64_t rows_per_cta_vec = kKvWarpsPerCta * kKvRowsPerWarp;
  int block_shift = -1;
  if ((block_size & (block_size - 1)) == 0) {
    block_shift = 0;
    while ((int64_t(1) << block_shift) < block_size) ++block_shift;
  }
  const bool aligned = ((uintptr_t)x % 16 == 0) && ((x_row_stride * 2) % 16 == 0) && ((uintptr_t)cache % 16 == 0) &&
                       (cache_stride0 % 16 == 0) && (cache_stride1 % 16 == 0);
  const int64_t ctas = aligned ? (n_slots + rows_per_cta_vec - 1) / rows_per_cta_vec
                               : (n_slots + kKvWarpsPerCta - 1) / kKvWarpsPerCta;
  if (ctas > 0x7fffffffLL) return fail(TITAN_ERR_INVALID_ARGUMENT, "store_int8: too many rows");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (aligned && cache_stride1 % 8 == 0 && n_slots >= 1024) {
    // Large batches: persistent streaming kernel, three CTAs per SM.
    // Per device, once: the kernels' shared-memory opt-in and the SM count.
    static std::atomic<int> dev_sms[64];  // 0 = not set up
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64)
      return fail(TITAN_ERR_CUDA, "store_int8: cudaGetDevice: %s", cudaGetErrorString(e));
    int sms = dev_sms[dev].load(std::memory_order_acquire);
    if (sms == 0) {
      std::lock_guard<std::mutex> lock(setup_mutex());
      sms = dev_sms[dev].load(std::memory_order_relaxed);
      if (sms == 0) {
        e = cudaFuncSetAttribute(store_int8_stream_kernel<int64_t>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kKvStreamSmem);
        if (e == cudaSuccess)
          e = cudaFuncSetAttribute(store_int8_stream_kernel<int32_t>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kKvStreamSmem);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess || sms <= 0)
          return fail(TITAN_ERR_CUDA, "store_int8: device setup: %s", cudaGetErrorString(e));
        dev_sms[dev].store(sms, std::memory_order_release);
      }
    }
    const int64_t warps_needed = (n_slots + 1) / 2;
    const int64_t ctas_needed = (warps_needed + kKvStreamWarps - 1) / kKvStreamWarps;
    const unsigned grid_s = (unsigned)std::min<int64_t>(ctas_needed, 3 * (int64_t)sms);
    const __nv_bfloat16 *xb = static_cast<const __nv_bfloat16 *>(x);
    int8_t *cb = static_cast<int8_t *>(cache);
    if (slots_is_int64)
      e = launch_pdl(store_int8_stream_kernel<int64_t>, dim3(grid_s), dim3(kKvStreamWarps * 32), kKvStreamSmem, s, xb,
                     x_row_stride, cb, num_blocks, block_size, block_shift, cache_stride0, cache_stride1,
                     static_cast<const int64_t *>(slots), n_slots);
    else
      e = launch_pdl(store_int8_stream_kernel<int32_t>, dim3(grid_s), dim3(kKvStreamWarps * 32), kKvStreamSmem, s, xb,
                     x_row_stride, cb, num_blocks, block_size, block_shift, cache_stride0, cache_stride1,
                     static_cast<const int32_t *>(slots), n_slots);
    if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "store_int8 (stream) launch: %s", cudaGetErrorString(e));
    return check_launch("store_int8 (stream) launch");
  }
  const dim3 grid((unsigned)ctas), block(kKvWarpsPerCta * 32);
  const __nv_bfloat16 *xb = static_cast<const __nv_bfloat16 *>(x);
  int8_t *cb = static_cast<int8_t *>(cache);
  cudaError_t le;
  if (slots_is_int64) {
    const int64_t *sl = static_cast<const int64_t *>(slots);
    le = aligned ? launch_pdl(store_int8_vec_kernel<int64_t>, grid, block, 0, s, xb, x_row_stride, cb, num_blocks,
                              block_size, block_shift, cache_stride0, cache_stride1, sl, n_slots)
                 : launch_pdl(store_int8_scalar_kernel<int64_t>, grid, block, 0, s, xb, x_row_stride, cb, num_blocks,
                              block_size, block_shift, cache_stride0, cache_stride1, sl, n_slots);
  } else {
    const int32_t *sl = static_cast<const int32_t *>(slots);
    le = aligned ? launch_pdl(store_int8_vec_kernel<int32_t>, grid, block, 0, s, xb, x_row_stride, cb, num_blocks,
                              block_size, block_shift, cache_stride0, cache_stride1, sl, n_slots)
                 : launch_pdl(store_int8_scalar_kernel<int32_t>, grid, block, 0, s, xb, x_row_stride, cb, num_blocks,
                              block_size, block_shift, cache_stride0, cache_stride1, sl, n_slots);
  }
  if (le != cudaSuccess) return fail(TITAN_ERR_CUDA, "store_int8 launch: %s", cudaGetErrorString(le));
  return check_launch("store_int8 launch");
}
