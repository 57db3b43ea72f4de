// ABI plumbing shared by the three launchers: per-thread error message,
// the device error word and its query.
#include "titan_common.cuh"

#include <string.h>

namespace titan {

static thread_local char t_last_error[512] = "";

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
}

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

std::mutex &setup_mutex() {
  static std::mutex m;
  return m;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return TITAN_OK;
}

}  // namespace titan

extern "C" int titan_abi_version(void) { return 100; }

extern "C" const char *titan_last_error(void) { return titan::t_last_error; }

extern "C" int titan_device_error(int *error_out, int clear_after, titan_stream_t stream) {
  if (error_out == nullptr) return titan::fail(TITAN_ERR_INVALID_ARGUMENT, "error_out is null");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return titan::fail(TITAN_ERR_CUDA, "stream sync: %s", cudaGetErrorString(e));
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, titan::g_device_error, sizeof(int));
  if (e != cudaSuccess) return titan::fail(TITAN_ERR_CUDA, "read error word: %s", cudaGetErrorString(e));
  if (clear_after && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(titan::g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return titan::fail(TITAN_ERR_CUDA, "clear error word: %s", cudaGetErrorString(e));
  }
  *error_out = v;
  return TITAN_OK;
}

namespace titan {

// One warp waits on an mbarrier that nothing arrives at, with the same
// bounded wait the kernels use: it gives up after `limit_cycles`, records
// kDevErrMbarrierTimeout in the device error word and returns.
__global__ void selftest_bounded_wait_kernel(long long limit_cycles) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  mbar_wait_bounded(&bar, 0u, limit_cycles);  // phase 0 never completes
}

// A counter that no kernel writes: the spin self-test waits for it to reach 1.
__device__ int g_selftest_counter = 0;

__global__ void selftest_bounded_spin_kernel(long long limit_cycles) {
  if (threadIdx.x == 0) spin_until_at_least(&g_selftest_counter, 1, limit_cycles);
}

}  // namespace titan

extern "C" int titan_selftest_bounded_spin(long long limit_cycles, titan_stream_t stream) {
  if (limit_cycles < 1 || limit_cycles > 4000000000LL)
    return titan::fail(TITAN_ERR_INVALID_ARGUMENT, "selftest: limit_cycles must be in [1, 4e9]");
  titan::selftest_bounded_spin_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(limit_cycles);
  return titan::check_launch("selftest_bounded_spin launch");
}

extern "C" int titan_selftest_bounded_wait(long long limit_cycles, titan_stream_t stream) {
  if (limit_cycles < 1 || limit_cycles > 4000000000LL)
    return titan::fail(TITAN_ERR_INVALID_ARGUMENT, "selftest: limit_cycles must be in [1, 4e9]");
  titan::selftest_bounded_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(limit_cycles);
  return titan::check_launch("selftest_bounded_wait launch");
}
