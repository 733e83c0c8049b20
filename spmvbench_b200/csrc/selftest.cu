// Failure-path self test of the bounded mbarrier wait (mbar_wait in
// common.cuh) and of the context's device error word: one thread arms an
// mbarrier for 16 bytes that no copy will ever deliver, waits with a short
// limit, records the timeout in the error word and returns. No copy is
// issued, so nothing is left in flight.
#include "internal.hpp"
#include "common.cuh"

namespace spmvb {

__global__ void wait_timeout_probe(int* __restrict__ err, uint32_t limit) {
  __shared__ __align__(8) unsigned long long bar;
  const uint32_t b = smem_addr(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_expect_tx(b, 16);
  const bool ok = mbar_wait(b, 0, limit);
  if (__syncthreads_or(!ok)) {
    if (threadIdx.x == 0) atomicExch(err, 2);
    return;
  }
}

}  // namespace spmvb

using namespace spmvb;

extern "C" spmvb_status spmvb_selftest_wait_timeout(spmvb_context ctx) {
  clear_error();
  if (!ctx) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null context");
  DeviceGuard g(ctx->device);
  wait_timeout_probe<<<1, 32>>>(ctx->err.as<int>(), 64);
  count_launch();
  SPMVB_TRY_CUDA(cudaGetLastError());
  return spmvb_context_check(ctx);
}
