// INT8 latent KV writer: one warp per token row.
//
// Follows kernels/titan_kv.py:7-21 (the reference `_store_int8`):
//   scale = max(max|x| / 127, 1e-12)            (fp32, IEEE division)
//   q     = clamp(nearbyint(x / scale), -127, 127)
//   row   = cache + (slot / block) * stride0 + (slot % block) * stride1
//   bytes [0,512) = q, bytes [512,528) = fp32 {scale, 0, 0, 0}; slot < 0 skips.
//
// Layout of the work: lane l of the row's warp owns latent values
// [16 l, 16 l + 16): two 16-byte loads of bf16, one 16-byte store of int8.
// Lane 0 also writes the 16-byte scale block.  The amax is a warp-shuffle max.
// HBM traffic per row: 1024 B read + 528 B written + 8 B slot.
#include "titan_common.cuh"

namespace titan {

constexpr int kKvWarpsPerCta = 8;

// q = clamp(rint(v / scale)) with the exact IEEE quotient.  A multiply by the
// reciprocal is tried first: its error is below 2^-22 relative, so rint() of it
// equals rint() of the correctly rounded quotient unless the product lies
// within 2^-10 of a half-integer; only then is the IEEE division evaluated.
__device__ __forceinline__ int quant_one(float v, float scale, float rcp) {
  float y = v * rcp;
  const float frac = fabsf(y - truncf(y));
  if (fabsf(frac - 0.5f) < 9.765625e-4f) y = __fdiv_rn(v, scale);
  y = rintf(y);
  y = fminf(fmaxf(y, -127.0f), 127.0f);
  return __float2int_rn(y);
}

__device__ __forceinline__ void bf16x2_to_f32(uint32_t w, float &lo, float &hi) {
  lo = __uint_as_float(w << 16);
  hi = __uint_as_float(w & 0xFFFF0000u);
}

template <typename SlotT>
__global__ void __launch_bounds__(kKvWarpsPerCta * 32)
    store_int8_vec_kernel(const __nv_bfloat16 *__restrict__ x, int64_t x_row_stride, int8_t *__restrict__ cache,
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

  const uint8_t *src = reinterpret_cast<const uint8_t *>(x + row * x_row_stride) + lane * 32;
  const uint4 a = ld_global_nc_v4(src);
  const uint4 b = ld_global_nc_v4(src + 16);
  float v[16];
  bf16x2_to_f32(a.x, v[0], v[1]);
  bf16x2_to_f32(a.y, v[2], v[3]);
  bf16x2_to_f32(a.z, v[4], v[5]);
  bf16x2_to_f32(a.w, v[6], v[7]);
  bf16x2_to_f32(b.x, v[8], v[9]);
  bf16x2_to_f32(b.y, v[10], v[11]);
  bf16x2_to_f32(b.z, v[12], v[13]);
  bf16x2_to_f32(b.w, v[14], v[15]);

  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));

  const float scale = fmaxf(__fdiv_rn(amax, 127.0f), 1.0e-12f);
  const float rcp = __frcp_rn(scale);

  uint32_t packed[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const int q0 = quant_one(v[4 * w + 0], scale, rcp);
    const int q1 = quant_one(v[4 * w + 1], scale, rcp);
    const int q2 = quant_one(v[4 * w + 2], scale, rcp);
    const int q3 = quant_one(v[4 * w + 3], scale, rcp);
    packed[w] = (uint32_t)(q0 & 0xFF) | ((uint32_t)(q1 & 0xFF) << 8) | ((uint32_t)(q2 & 0xFF) << 16) |
                ((uint32_t)(q3 & 0xFF) << 24);
  }
  int8_t *dst = cache + blk * cs0 + off * cs1;
  *reinterpret_cast<uint4 *>(dst + lane * 16) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  if (lane == 0) *reinterpret_cast<uint4 *>(dst + 512) = make_uint4(__float_as_uint(scale), 0u, 0u, 0u);
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
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = fmaxf(__fdiv_rn(amax, 127.0f), 1.0e-12f);
  const float rcp = __frcp_rn(scale);
  int8_t *dst = cache + blk * cs0 + off * cs1;
#pragma unroll
  for (int k = 0; k < 16; ++k) dst[lane + 32 * k] = (int8_t)quant_one(v[k], scale, rcp);
  if (lane < 16) {
    const uint32_t bits = lane < 4 ? __float_as_uint(scale) : 0u;
    const int byte = lane & 3;
    dst[512 + lane] = (int8_t)((bits >> (8 * byte)) & 0xFF);
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
  const int64_t ctas = (n_slots + kKvWarpsPerCta - 1) / kKvWarpsPerCta;
  if (ctas > 0x7fffffffLL) return fail(TITAN_ERR_INVALID_ARGUMENT, "store_int8: too many rows");
  const bool aligned = ((uintptr_t)x % 16 == 0) && ((x_row_stride * 2) % 16 == 0) && ((uintptr_t)cache % 16 == 0) &&
                       (cache_stride0 % 16 == 0) && (cache_stride1 % 16 == 0);
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
