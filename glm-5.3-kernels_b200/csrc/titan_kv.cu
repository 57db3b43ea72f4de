// INT8 latent KV writer: each warp quantises four token rows.
//
// Follows kernels/titan_kv.py:7-21 (the reference `_store_int8`):
//   scale = max(max|x| / 127, 1e-12)            (fp32, IEEE division)
//   q     = clamp(nearbyint(x / scale), -127, 127)
//   row   = cache + (slot / block) * stride0 + (slot % block) * stride1
//   bytes [0,512) = q, bytes [512,528) = fp32 {scale, 0, 0, 0}; slot < 0 skips.
//
// Layout of the work: for each of its rows, lane l of the warp owns latent
// values [16 l, 16 l + 16): two 16-byte loads of bf16, one 16-byte store of int8.
// Lane 0 also writes the 16-byte scale block.  The amax is a warp-shuffle max.
// HBM traffic per row: 1024 B read + 528 B written + 8 B slot.
#include "titan_common.cuh"

namespace titan {

constexpr int kKvWarpsPerCta = 8;
constexpr int kKvRowsPerWarp = 4;

// 1.5 * 2^23: adding it to |y| < 2^22 rounds y to an integer (round to
// nearest even, the fp32 addition's own rounding) and leaves that integer's
// two's-complement low byte in the low byte of the sum's bit pattern.
constexpr float kRoundMagic = 12582912.0f;

// Quantise 16 values to 4 packed int8 words: q = rint(v / scale) with the
// correctly rounded quotient.  y = v * fl(1/scale) differs from v / scale by
// less than 2^-22 relative (|y| <= 127.1, so < 2^-15 absolute), hence
// rint(y) == rint(fl(v / scale)) unless y lies within 2^-10 of a
// half-integer; any lane that meets such a value recomputes its 16 values with
// the IEEE division.  |q| <= 127 needs no clamp: scale >= fl(amax / 127)
// keeps |v / scale| <= 127 (1 + 2^-24), which rounds to at most 127.
__device__ __forceinline__ void quant16(const float (&v)[16], float scale, float rcp, uint32_t (&out)[4]) {
  float m[16];
  bool near_half = false;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float y = v[i] * rcp;
    m[i] = y + kRoundMagic;
    const float r = m[i] - kRoundMagic;
    near_half |= fabsf(y - r) > 0.4990234375f;  // 0.5 - 2^-10
  }
  if (near_half) {
#pragma unroll
    for (int i = 0; i < 16; ++i) m[i] = __fdiv_rn(v[i], scale) + kRoundMagic;
  }
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t lo = prmt(__float_as_uint(m[4 * w + 0]), __float_as_uint(m[4 * w + 1]), 0x0040u);
    const uint32_t hi = prmt(__float_as_uint(m[4 * w + 2]), __float_as_uint(m[4 * w + 3]), 0x0040u);
    out[w] = prmt(lo, hi, 0x5410u);
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

// scale = max(max|x| / 127, 1e-12) with the IEEE quotient (kernels/titan_kv.py:16).
__device__ __forceinline__ float row_scale(float amax) { return fmaxf(__fdiv_rn(amax, 127.0f), 1.0e-12f); }

// Each warp quantises kKvRowsPerWarp rows; every row's two 16-byte loads per
// lane are issued before any arithmetic so ~4 KB per warp is in flight.
template <typename SlotT>
__global__ void __launch_bounds__(kKvWarpsPerCta * 32)
    store_int8_vec_kernel(const __nv_bfloat16 *__restrict__ x, int64_t x_row_stride, int8_t *__restrict__ cache,
                          int64_t num_blocks, int64_t block, int64_t cs0, int64_t cs1,
                          const SlotT *__restrict__ slots, int64_t n) {
  const int lane = threadIdx.x & 31;
  const int64_t row0 = ((int64_t)blockIdx.x * kKvWarpsPerCta + (threadIdx.x >> 5)) * kKvRowsPerWarp;
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
    const int64_t blk = slot[r] / block;
    if (blk >= num_blocks) continue;
    const int64_t off = slot[r] - blk * block;
    float v[16];
    bf16x2_to_f32(a[r].x, v[0], v[1]);
    bf16x2_to_f32(a[r].y, v[2], v[3]);
    bf16x2_to_f32(a[r].z, v[4], v[5]);
    bf16x2_to_f32(a[r].w, v[6], v[7]);
    bf16x2_to_f32(b[r].x, v[8], v[9]);
    bf16x2_to_f32(b[r].y, v[10], v[11]);
    bf16x2_to_f32(b[r].z, v[12], v[13]);
    bf16x2_to_f32(b[r].w, v[14], v[15]);
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float scale = row_scale(warp_amax(amax));
    uint32_t q[4];
    quant16(v, scale, __frcp_rn(scale), q);
    int8_t *dst = cache + blk * cs0 + off * cs1;
    *reinterpret_cast<uint4 *>(dst + lane * 16) = make_uint4(q[0], q[1], q[2], q[3]);
    if (lane == 0) *reinterpret_cast<uint4 *>(dst + 512) = make_uint4(__float_as_uint(scale), 0u, 0u, 0u);
  }
}

// Unaligned fallback (x rows or cache rows not 16-byte aligned): lane l owns
// values l + 32 k, byte stores.  Same arithmetic.
template <typename SlotT>
__global__ void __launch_bounds__(kKvWarpsPerCta * 32)
    store_int8_scalar_kernel(const __nv_bfloat16 *__restrict__ x, int64_t x_row_stride, int8_t *__restrict__ cache,
                             int64_t num_blocks, int64_t block, int64_t cs0, int64_t cs1,
                             const SlotT *__restrict__ slots, int64_t n) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kKvWarpsPerCta + (threadIdx.x >> 5);
  if (row >= n) return;
  const int64_t slot = (int64_t)slots[row];
  if (slot < 0) return;
  const int64_t blk = slot / block;
  if (blk >= num_blocks) return;
  const int64_t off = slot - blk * block;
  const __nv_bfloat16 *src = x + row * x_row_stride;
  float v[16];
  float amax = 0.0f;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    v[k] = __bfloat162float(src[lane + 32 * k]);
    amax = fmaxf(amax, fabsf(v[k]));
  }
  const float scale = row_scale(warp_amax(amax));
  uint32_t q[4];
  quant16(v, scale, __frcp_rn(scale), q);
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
  const bool aligned = ((uintptr_t)x % 16 == 0) && ((x_row_stride * 2) % 16 == 0) && ((uintptr_t)cache % 16 == 0) &&
                       (cache_stride0 % 16 == 0) && (cache_stride1 % 16 == 0);
  const int64_t ctas = aligned ? (n_slots + rows_per_cta_vec - 1) / rows_per_cta_vec
                               : (n_slots + kKvWarpsPerCta - 1) / kKvWarpsPerCta;
  if (ctas > 0x7fffffffLL) return fail(TITAN_ERR_INVALID_ARGUMENT, "store_int8: too many rows");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)ctas), block(kKvWarpsPerCta * 32);
  const __nv_bfloat16 *xb = static_cast<const __nv_bfloat16 *>(x);
  int8_t *cb = static_cast<int8_t *>(cache);
  if (slots_is_int64) {
    const int64_t *sl = static_cast<const int64_t *>(slots);
    if (aligned)
      store_int8_vec_kernel<int64_t><<<grid, block, 0, s>>>(xb, x_row_stride, cb, num_blocks, block_size,
                                                            cache_stride0, cache_stride1, sl, n_slots);
    else
      store_int8_scalar_kernel<int64_t><<<grid, block, 0, s>>>(xb, x_row_stride, cb, num_blocks, block_size,
                                                               cache_stride0, cache_stride1, sl, n_slots);
  } else {
    const int32_t *sl = static_cast<const int32_t *>(slots);
    if (aligned)
      store_int8_vec_kernel<int32_t><<<grid, block, 0, s>>>(xb, x_row_stride, cb, num_blocks, block_size,
                                                            cache_stride0, cache_stride1, sl, n_slots);
    else
      store_int8_scalar_kernel<int32_t><<<grid, block, 0, s>>>(xb, x_row_stride, cb, num_blocks, block_size,
                                                               cache_stride0, cache_stride1, sl, n_slots);
  }
  return check_launch("store_int8 launch");
}
