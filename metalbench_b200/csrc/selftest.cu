// Self-test of the bounded-wait machinery, without faulting or hanging a GPU:
// one CTA waits on an mbarrier that nothing ever arrives on, with a short
// limit. The wait must give up, record MB_DEV_TIMEOUT_SELFTEST in the device
// status word and return; the host then sees MB_ERR_TIMEOUT from the status
// check and the context stays usable.
#include "common.cuh"

namespace {
__global__ void bounded_wait_kernel(uint32_t* status, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbd::mbar_init(&bar, 1);  // expects one arrival that never comes
    mbd::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbd::mbar_wait(&bar, 0, status, MB_DEV_TIMEOUT_SELFTEST, nullptr, limit_ns);
  __syncthreads();
}
}  // namespace

extern "C" int mb_selftest_bounded_wait(int timeout_us, void* stream) {
  MB_REQUIRE(timeout_us > 0 && timeout_us <= 1000000, "selftest: timeout_us must be in (0, 1e6]");
  uint32_t* st = mb::device_status_ptr();
  if (!st) {
    mb::set_error("selftest: no device status word (mb_init first)");
    return MB_ERR_NOT_INIT;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  bounded_wait_kernel<<<1, 32, 0, s>>>(st, (uint64_t)timeout_us * 1000ull);
  MB_CUDA(cudaGetLastError());
  return mb::check_device_status(s);
}
