// selftest.cu -- exercises the bounded mbarrier wait that every kernel of
// this library uses, on a barrier that nothing ever completes.
//
// Each role of the decode kernels waits on mbarriers with mbar_wait
// (common.cuh): after kWaitLimitCycles SM cycles (about 2 s) the wait gives
// up, raises the CTA's abort flag, writes a code into the caller's device
// status word and returns false, so a lost arrival (a bug, a peer that died)
// ends the kernel with an error the host can read instead of hanging the GPU.
// This kernel runs exactly that path with nothing else in flight: one warp
// waits on a fresh barrier that no thread, copy or MMA will ever arrive on.
#include "common.cuh"
#include "flagattn_b200.h"

namespace fa {

__global__ void selftest_wait_timeout_kernel(int *status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;  // one waiter: it alone owns the status word
  mbar_init(smem_u32(&bar), 1);
  abort_flag = 0;
  // phase 0 never completes: the bounded wait must give up and report
  if (mbar_wait(smem_u32(&bar), 0, &abort_flag, status, kDevTimeoutSelfTest))
    atomicExch(status, -1);  // would mean a phase completed with no arrival
}

}  // namespace fa

extern "C" int fa_selftest_wait_timeout(int32_t *status, void *stream) {
  if (status == nullptr) return FA_ERR_INVALID_ARGUMENT;
  fa::selftest_wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_CUDA;
}
