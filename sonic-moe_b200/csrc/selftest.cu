// Self-test of the bounded waits every pipelined kernel of this library relies on.
//
// Each mbarrier wait in the GEMMs gives up after kWaitTimeoutNs, records a code in the caller's
// error word and lets the kernel return, so a lost arrival shows up as an error status instead of
// a hung GPU.  This kernel exercises that path on purpose with a barrier nothing ever arrives on:
// the wait runs out (about 2 s), the code is recorded, the kernel exits, and the context stays
// usable.  No memory is touched beyond the error word.
#include "../../include/sonic_b200.h"
#include "common.cuh"
#include "sonic_internal.h"

namespace smb {

__global__ void __launch_bounds__(32) bounded_wait_selftest_kernel(int* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) (void)mbar_wait(&bar, 0, err, kErrSelfTestWait);  // no arrival: gives up
  __syncwarp();
}

}  // namespace smb

extern "C" int sm_selftest_bounded_wait(int32_t* err, void* stream) {
  if (!err) return smb::set_last_error(SM_EINVAL, "selftest: null error word");
  smb::bounded_wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(err);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return smb::set_last_error(SM_EIO, "selftest: %s", cudaGetErrorString(e));
  return SM_OK;
}
