// Test hook for the failure path every kernel here shares: a bounded wait on
// an mbarrier that nothing arrives on.  The wait runs out after limit_ns,
// records kDevTimeout in the device status word and returns, so the kernel
// ends, the context stays usable and the host reads the error through
// tq_device_status -- what a lost producer would look like to any of the
// GEMM, LoRA or loss kernels, made on purpose and without a fault.
#include "tq_ptx.cuh"
#include "tq_runtime.h"

namespace tq {
namespace {

__global__ void wait_selftest_kernel(uint64_t limit_ns, int* status) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    fence_mbar_init();
  }
  __syncwarp();
  // Nobody arrives: phase 0 never completes.
  if (threadIdx.x == 0) mbar_wait(b, 0, status, limit_ns);
  __syncwarp();
}

}  // namespace
}  // namespace tq

extern "C" int tq_wait_selftest(int64_t limit_ns, void* stream) {
  using namespace tq;
  if (limit_ns < 1000000 || limit_ns > 10000000000ll)
    return fail(TQ_ERR_INVALID, "wait_selftest: limit_ns must be within [1 ms, 10 s], got %lld",
                (long long)limit_ns);
  int rc = TQ_OK;
  int* status = device_status_ptr(&rc);
  if (!status) return rc;
  wait_selftest_kernel<<<1, 32, 0, as_stream(stream)>>>(static_cast<uint64_t>(limit_ns), status);
  return check_cuda(cudaGetLastError(), "wait_selftest launch");
}
