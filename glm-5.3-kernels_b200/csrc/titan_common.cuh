// Shared helpers for the sm_100a kernels: host-side error reporting, the
// device error word, bf16/int8 packing and the PTX wrappers for mbarriers and
// bulk (TMA) copies.
#pragma once

#include <cuda.h>  // CUtensorMap
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <mutex>

#include "../../include/titan_b200.h"

namespace titan {

// ---------------------------------------------------------------- host side
void set_error(const char *fmt, ...);
// Serialises the one-time per-device setup of the launchers (kernel
// attributes, capacity queries, symbol lookups); readers check an atomic
// ready flag first, so steady-state launches take no lock.
std::mutex &setup_mutex();
int fail(int code, const char *fmt, ...);
int check_launch(const char *what);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda); nullptr when the driver does not provide it.
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
inline EncodeTiledFn tensor_map_encoder() {
  static const EncodeTiledFn encode = [] {  // looked up once (thread-safe static initialisation)
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(fn);
    cudaGetLastError();
    return static_cast<EncodeTiledFn>(nullptr);
  }();
  return encode;
}

// Device error word (one per device, in this module; the library is a single
// translation unit, titan_b200.cu).  Bounded waits that give up write a
// non-zero code here instead of trapping.
enum DeviceError : int {
  kDevErrNone = 0,
  kDevErrMbarrierTimeout = 1,
  kDevErrCapacity = 2,  // a count past a fixed-size list; the excess is dropped
  kDevErrSpinTimeout = 3,  // a CTA gave up waiting for the other CTAs of its barrier
};
__device__ int g_device_error = 0;

// --------------------------------------------------------------- device side
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Arrive once and add `tx_bytes` to the expected transaction count.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t tx_bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(tx_bytes)
      : "memory");
}

// Plain arrival (release at CTA scope).
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after ~`limit_cycles` SM clocks, records the failure
// in the device error word and returns false.  Never traps, never spins forever.
// Bulk copies land in microseconds; a wait allows ~0.1 s (kLongWaitCycles).
// After a give-up the caller stops issuing copies and drains the ones already
// in flight with kShortWaitCycles waits (~0.5 ms each), so a CTA with a lost
// copy ends quickly instead of stalling the grid.
constexpr long long kLongWaitCycles = 200000000LL;
constexpr long long kShortWaitCycles = 1000000LL;

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, long long limit_cycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > limit_cycles) {
      atomicCAS(&g_device_error, 0, kDevErrMbarrierTimeout);
      return false;
    }
  }
}

// Launch as a programmatic dependent of the previous work on the stream: the
// kernel may start while that work finishes and must call pdl_wait_primary()
// before touching memory the earlier work reads or writes.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// PDL (programmatic dependent launch) controls.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_primary() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Four int8 in one word -> two bf16x2 words (bytes 0,1 -> lo; bytes 2,3 -> hi),
// exactly.  Each byte is biased to an unsigned value u = x + 128 and placed in
// the low mantissa bits of 2^23 (fp32 bits 0x4B0000uu = 2^23 + u); subtracting
// 2^23 + 128 recovers x as an fp32 integer, whose top 16 bits are its bf16
// encoding because |x| <= 128 needs at most 8 significant bits.
__device__ __forceinline__ void i8x4_to_bf16x4(uint32_t w, uint32_t &lo, uint32_t &hi) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t magic = 0x4B000000u;
  float2 f01 = make_float2(__uint_as_float(prmt(u, magic, 0x7540u)), __uint_as_float(prmt(u, magic, 0x7541u)));
  float2 f23 = make_float2(__uint_as_float(prmt(u, magic, 0x7542u)), __uint_as_float(prmt(u, magic, 0x7543u)));
  const float2 bias = make_float2(-8388736.0f, -8388736.0f);
  f01 = __fadd2_rn(f01, bias);
  f23 = __fadd2_rn(f23, bias);
  lo = prmt(__float_as_uint(f01.x), __float_as_uint(f01.y), 0x7632u);
  hi = prmt(__float_as_uint(f23.x), __float_as_uint(f23.y), 0x7632u);
}

// Four int8 in one word -> two f16x2 words (bytes 0,1 -> lo; bytes 2,3 ->
// hi), exactly: each byte is biased to u = x + 128 and placed in the low
// mantissa byte of 1024 (f16 bits 0x64uu = 1024 + u, ulp 1 in [1024, 2048));
// one packed f16 add of -1152 then leaves x, exact since |x| <= 128.
__device__ __forceinline__ void i8x4_to_f16x4(uint32_t w, uint32_t &lo, uint32_t &hi) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t magic = 0x64646464u;
  const uint32_t bias = 0xE480E480u;  // f16x2 {-1152, -1152}
  const uint32_t a = prmt(u, magic, 0x4140u), b = prmt(u, magic, 0x4342u);
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(a), "r"(bias));
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(b), "r"(bias));
}

// 2^e as a float, exact, for -126 <= e <= 127 (0 below).
__device__ __forceinline__ float exp2i(int e) { return e < -126 ? 0.0f : __int_as_float((e + 127) << 23); }

// Four 8x8 b16 matrices from shared memory (lane i gives the address of row
// i % 8 of matrix i / 8); lane (g, c) receives the pair (row g, cols 2c, 2c+1)
// of each: with matrices (rows 0-7, cols 0-7), (8-15, 0-7), (0-7, 8-15),
// (8-15, 8-15) that is the A fragment of m16n8k16.
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&d)[4], const void *row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
               : "r"(smem_u32(row))
               : "memory");
}

// 8x8 b16 matrix transpose across the warp (standard fragment layout).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

// D += A * B, m16n8k16, bf16 inputs, fp32 accumulate.  Not volatile: the
// compiler may interleave independent accumulator chains.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D += A * B, m16n8k16, f16 inputs, fp32 accumulate (exact products).
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

// 16-byte asynchronous global -> shared copy (per thread), grouped per thread.
__device__ __forceinline__ void cp_async_16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// 4 bytes global -> shared, zero-filling the destination beyond `src_bytes`
// (0 = nothing is read: the source address is not accessed).
__device__ __forceinline__ void cp_async_4_zfill(void *dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int kPending>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kPending) : "memory");
}

// Thread-block cluster helpers (distributed shared memory).
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Split cluster barrier: arrive early (non-blocking), wait later.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// Shared::cluster address of the same shared-memory variable in CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(const void *p, uint32_t rank) {
  uint32_t r;
  asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

// Asynchronous remote stores into a peer CTA's shared memory that complete
// (in bytes) on the peer's mbarrier; the sender never waits.
__device__ __forceinline__ void st_async_f32x2(uint32_t addr, float2 v, uint32_t mbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(addr),
               "f"(v.x), "f"(v.y), "r"(mbar)
               : "memory");
}

// Bulk copy (TMA engine) from this CTA's shared memory into a peer CTA's shared
// memory, completing in bytes on the peer's mbarrier.  dst/src 16-byte aligned,
// bytes a multiple of 16.  The source must stay untouched until
// bulk_wait_read_all() returns.
__device__ __forceinline__ void bulk_s2cluster(uint32_t dst_cluster, const void *src, uint32_t bytes,
                                               uint32_t mbar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst_cluster),
      "r"(smem_u32(src)), "r"(bytes), "r"(mbar_cluster)
      : "memory");
}
// TMA gather of four rows of a 2-D tensor map (box one row high): rows r0..r3
// at column x land back to back at dst (128-byte aligned), completing in bytes
// on `bar`.  Rows outside the map read as zeros.  x * element size must be a
// multiple of 16 bytes.
__device__ __forceinline__ void tma_gather4(void *dst, const void *tmap, int x, int r0, int r1, int r2, int r3,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(smem_u32(bar))
      : "memory");
}

// Pull a TMA descriptor (kernel parameter or global) into the descriptor cache.
__device__ __forceinline__ void prefetch_tensormap(const void *tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Arrival ticket with release (prior writes of this thread and of those
// ordered before it by a CTA barrier) and acquire semantics at GPU scope.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int *p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ int atom_add_relaxed_gpu(int *p, int v) {
  int old;
  asm volatile("atom.relaxed.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void st_relaxed_gpu(int *p, int v) {
  asm volatile("st.relaxed.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_gpu(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded spin until the counter at p reaches `target` (acquire: what the
// arriving CTAs released before their increments is visible afterwards).
// Acquire loads in the loop: relaxed polls with one fence.acq_rel after the
// value is seen were 0.3 us slower per flat-merge call.
// Gives up after ~`limit_cycles` SM clocks, recording kDevErrSpinTimeout.
// Only for counters whose arrivals come from CTAs of the same grid that are
// resident together with the waiting one.
__device__ __forceinline__ bool spin_until_at_least(const int *p, int target, long long limit_cycles) {
  if (ld_acquire_gpu(p) >= target) return true;
  const long long t0 = clock64();
  while (true) {
    if (ld_acquire_gpu(p) >= target) return true;
    if (clock64() - t0 > limit_cycles) {
      atomicCAS(&g_device_error, 0, kDevErrSpinTimeout);
      return false;
    }
  }
}

__device__ __forceinline__ uint4 ld_global_nc_v4(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

}  // namespace titan
