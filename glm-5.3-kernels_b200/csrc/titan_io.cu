// Host <-> device staging for latency-bound calls (no counterpart in the
// reference: its callers keep every operand on the GPU).
//
// A decode call moves ~25 KB in (q + indices) and 16 KB out.  Through the
// copy engine each small pinned copy costs several microseconds of fixed
// latency, more than the attention kernel itself.  Here the SMs move the
// bytes instead: titan_copy launches a kernel that reads (or writes) pinned
// host memory directly through its device mapping, 16 bytes per thread with
// every load in flight at once, so the transfer costs about one PCIe round
// trip.  Kernels that already write their result (the MLA reader's `out`)
// can equally be handed a mapped pinned pointer, resolved with
// titan_device_pointer, and store straight into host memory.
//
// Pinned allocations made with cudaHostAlloc / cudaMallocHost (torch's
// pin_memory) are mapped into the device address space under unified
// addressing; pageable memory is not, and is rejected on the host.
#include "titan_common.cuh"

namespace titan {

constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 4;  // 16-byte words per thread per round, all loaded before any store

// Device-accessible address of `p`: device and managed memory as is, pinned
// host memory through its device mapping.  Returns nullptr (and sets the
// error message) for pageable or unknown memory.
static void *device_view(const void *p, const char *what) {
  cudaPointerAttributes a;
  cudaError_t e = cudaPointerGetAttributes(&a, p);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    set_error("%s: cudaPointerGetAttributes: %s", what, cudaGetErrorString(e));
    return nullptr;
  }
  switch (a.type) {
    case cudaMemoryTypeDevice:
    case cudaMemoryTypeManaged:
      return const_cast<void *>(p);
    case cudaMemoryTypeHost:
      if (a.devicePointer == nullptr) set_error("%s: pinned host memory without a device mapping", what);
      return a.devicePointer;
    default:
      set_error("%s: pageable host memory (pin it, e.g. cudaHostAlloc / tensor.pin_memory())", what);
      return nullptr;
  }
}

// grid-stride copy of n16 16-byte words, then the byte tail (bytes % 16).
// `vec` = both pointers 16-byte aligned; otherwise bytes only.  The
// destination may still be read by the previous grid on the stream (e.g. the
// reader of the last call's landing buffer), so nothing is stored before the
// programmatic-dependency wait.  With `early_read` (the source is not written
// by earlier work on the stream) the first round of loads is issued before
// that wait, overlapping the source's latency with the previous grid's tail.
__global__ void __launch_bounds__(kCopyThreads)
    staged_copy_kernel(uint8_t *__restrict__ dst, const uint8_t *__restrict__ src, int64_t bytes, bool vec,
                       bool early_read) {
  const int64_t nthreads = (int64_t)gridDim.x * kCopyThreads;
  const int64_t tid = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x;
  pdl_launch_dependents();  // the next kernel may start its own set-up; it still waits for this grid
  if (!early_read) pdl_wait_primary();
  int64_t done = 0;
  if (vec) {
    const int64_t n16 = bytes >> 4;
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    for (int64_t base = 0; base < n16; base += nthreads * kCopyUnroll) {
      uint4 v[kCopyUnroll];
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t i = base + u * nthreads + tid;
        if (i < n16) v[u] = s[i];
      }
      if (early_read && base == 0) pdl_wait_primary();
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t i = base + u * nthreads + tid;
        if (i < n16) d[i] = v[u];
      }
    }
    done = n16 << 4;
  }
  if (early_read && done == 0) pdl_wait_primary();  // no vector round ran
  for (int64_t i = done + tid; i < bytes; i += nthreads) dst[i] = src[i];
}

}  // namespace titan

extern "C" int titan_device_pointer(const void *ptr, void **device_ptr_out) {
  using namespace titan;
  if (device_ptr_out == nullptr) return fail(TITAN_ERR_INVALID_ARGUMENT, "device_pointer: null output");
  *device_ptr_out = nullptr;
  if (ptr == nullptr) return fail(TITAN_ERR_INVALID_ARGUMENT, "device_pointer: null pointer");
  void *v = device_view(ptr, "device_pointer");
  if (v == nullptr) return TITAN_ERR_INVALID_ARGUMENT;
  *device_ptr_out = v;
  return TITAN_OK;
}

extern "C" int titan_copy(void *dst, const void *src, int64_t bytes, titan_stream_t stream) {
  return titan_copy_ex(dst, src, bytes, 0, stream);
}

extern "C" int titan_copy_ex(void *dst, const void *src, int64_t bytes, int flags, titan_stream_t stream) {
  using namespace titan;
  if (flags & ~TITAN_COPY_SRC_READY) return fail(TITAN_ERR_INVALID_ARGUMENT, "copy: unknown flags 0x%x", flags);
  if (bytes < 0) return fail(TITAN_ERR_INVALID_ARGUMENT, "copy: negative size");
  if (bytes == 0) return TITAN_OK;
  if (dst == nullptr || src == nullptr) return fail(TITAN_ERR_INVALID_ARGUMENT, "copy: null pointer");
  void *d = device_view(dst, "copy dst");
  if (d == nullptr) return TITAN_ERR_INVALID_ARGUMENT;
  const void *s = device_view(src, "copy src");
  if (s == nullptr) return TITAN_ERR_INVALID_ARGUMENT;
  const uint8_t *s8 = static_cast<const uint8_t *>(s);
  uint8_t *d8 = static_cast<uint8_t *>(d);
  if (d8 < s8 + bytes && s8 < d8 + bytes) return fail(TITAN_ERR_INVALID_ARGUMENT, "copy: overlapping buffers");
  const bool vec = (uintptr_t)d8 % 16 == 0 && (uintptr_t)s8 % 16 == 0;
  // One 16-byte word per thread for small copies (latency: every load in
  // flight at once); larger ones loop, kCopyUnroll words per thread per round.
  const int64_t words = vec ? (bytes + 15) / 16 : bytes;
  int64_t blocks = (words + kCopyThreads - 1) / kCopyThreads;
  if (blocks > 1184) blocks = 1184;  // 148 SMs x 8 resident blocks of 256 threads
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(kCopyThreads);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const bool early_read = (flags & TITAN_COPY_SRC_READY) != 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, staged_copy_kernel, d8, s8, bytes, vec, early_read);
  if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "copy launch: %s", cudaGetErrorString(e));
  return TITAN_OK;
}
