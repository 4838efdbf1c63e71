// Failure-detection self-test: one kernel waits on an mbarrier that nothing ever completes, with the same bounded
// wait every pipeline in this library uses. When the limit passes, the wait sets the CTA's abort flag, ORs
// DC_DEVERR_WAIT_PROBE into the context's device error word and returns, the kernel ends normally, and the next
// dc_sync reports DC_ETIMEOUT (clearing the word): the context stays usable. Nothing faults, traps or hangs.
#include <cuda_runtime.h>

#include "dc_internal.h"
#include "dc_ptx.cuh"

using namespace dcx;

namespace {

__global__ void wait_probe_kernel(uint32_t *err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    mbar_init_fence();
  }
  __syncthreads();
  // phase 0 of a fresh barrier with an arrival count of 1 completes only on an arrival, which never comes
  if (threadIdx.x == 0) mbar_wait(smem_u32(&bar), 0, &abort_flag, err, DC_DEVERR_WAIT_PROBE, limit_ns);
}

}  // namespace

int ops_wait_probe(dc_ctx *ctx, int limit_us) {
  wait_probe_kernel<<<1, 32, 0, ctx->stream>>>(ctx->d_err, 1000ull * (unsigned long long)limit_us);
  return dc_launch_check("self-test wait");
}
