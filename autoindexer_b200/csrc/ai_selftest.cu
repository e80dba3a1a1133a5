// ai_attn_selftest_wait: the device-side failure path, exercised without a
// fault.  One CTA waits on an mbarrier that nothing completes, with the same
// bounded wait (ptx::mbar_wait) every kernel of the library uses; when the
// limit runs out it records AI_ERR_DEV_TIMEOUT in the status word, exactly as
// a kernel whose wait expired does, and returns.  Nothing asynchronous (TMA,
// tcgen05) is in flight, so giving up cannot leave work behind.

#include <cuda_runtime.h>

#include "../../include/ai_attn.h"
#include "ai_common.cuh"
#include "sm100_ptx.cuh"

namespace {

__global__ void selftest_wait_kernel(int32_t* status, long long max_cycles) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = ai::ptx::smem_u32(&bar);
  if (threadIdx.x == 0) {
    ai::ptx::mbar_init(b, 1);
    ai::ptx::fence_mbar_init();
  }
  __syncthreads();
  if (!ai::ptx::mbar_wait(b, 0, max_cycles)) ai::report(status, AI_ERR_DEV_TIMEOUT);
  __syncthreads();
  if (threadIdx.x == 0) ai::ptx::mbar_arrive(b);  // complete the phase before the CTA exits
}

}  // namespace

extern "C" int ai_attn_selftest_wait(int32_t* status, long long max_cycles, void* stream) {
  if (!status) return AI_ERR_NULL;
  if (max_cycles <= 0 || max_cycles > 2000000000LL) return AI_ERR_SHAPE;
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major != 10) {
    cudaGetLastError();
    return AI_ERR_NO_DEVICE;
  }
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, max_cycles);
  return cudaGetLastError() == cudaSuccess ? AI_OK : AI_ERR_LAUNCH;
}
