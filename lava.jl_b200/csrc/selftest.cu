// selftest.cu — exercises the failure path every kernel of the library shares: a bounded
// mbarrier wait that runs out records LVB_ERR_TIMEOUT (with the wait site) in the device
// status word and the kernel returns, leaving the context usable. Nothing arrives at the
// barrier here, so the wait always runs out after the given limit; no fault, no hang.
#include "lvb_internal.h"

namespace lvb {

constexpr int kSelftestSite = 99;

__global__ void wait_selftest_kernel(DevStatus* status, unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    bar_init(&bar, 1);  // one arrival expected, none will come
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const WaitGuard g{status, &abort_flag, timeout_ns};
    wait_bar(&bar, 0, g, kSelftestSite, 0);
  }
  __syncthreads();
}

int selftest_launch(DevStatus* status, int32_t timeout_ms, cudaStream_t stream, const char* op) {
  if (timeout_ms <= 0 || timeout_ms > 2000)
    return fail(LVB_ERR_INVALID_ARG, op, "timeout_ms must be in 1..2000");
  wait_selftest_kernel<<<1, 32, 0, stream>>>(status, (unsigned long long)timeout_ms * 1000000ull);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LVB_OK : fail_cuda(e, op, "kernel launch");
}

}  // namespace lvb

using namespace lvb;

extern "C" int lvb_selftest_wait_timeout(int32_t timeout_ms, void* stream) {
  const char* op = "lvb_selftest_wait_timeout";
  if (timeout_ms <= 0 || timeout_ms > 2000)
    return fail(LVB_ERR_INVALID_ARG, op, "timeout_ms must be in 1..2000");
  DeviceState* dev = current_device_state(op);
  if (!dev) return LVB_ERR_NO_DEVICE;
  return selftest_launch(dev->status, timeout_ms, reinterpret_cast<cudaStream_t>(stream), op);
}

// The same against lvb_gemm_noalloc's own status word (the head of its static array), which
// lvb_gemm_noalloc_status reads. Allocates nothing.
extern "C" int lvb_gemm_noalloc_selftest_wait_timeout(int32_t timeout_ms, void* stream) {
  const char* op = "lvb_gemm_noalloc_selftest_wait_timeout";
  if (timeout_ms <= 0 || timeout_ms > 2000)
    return fail(LVB_ERR_INVALID_ARG, op, "timeout_ms must be in 1..2000");
  DevStatus* word = nullptr;
  int st = noalloc_status_word(&word, op);
  if (st) return st;
  return selftest_launch(word, timeout_ms, reinterpret_cast<cudaStream_t>(stream), op);
}
