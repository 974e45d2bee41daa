// k_selftest.cu — self-test of the bounded waits every kernel here relies on.
//
// One CTA of two warps does what a tcgen05 kernel of this library does when
// a wait runs out: warp 0 takes TMEM columns, warp 1 waits on an mbarrier
// that nothing arrives at, with the caller's (short) limit, and records
// kDevErrWaitTimeout in the device error flag and raises the CTA's abort
// flag; warp 0, itself parked in a wait with the kernels' own 4 s limit on a
// second barrier nothing arrives at, sees the abort flag and gives up; then
// warp 0 frees its TMEM and the CTA exits.  The GPU is never left waiting:
// both waits end by %globaltimer or by the abort flag.
#include "ts_common.cuh"
#include "ts_kernels.h"

namespace ts {

__global__ void __launch_bounds__(64, 1) wait_selftest_kernel(int* err, unsigned long long limit_ns, int* result) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag_s;
  volatile int* abort_flag = &abort_flag_s;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  if (threadIdx.x == 32) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  int ok = 1;
  if (warp == 1) {
    // the wait that runs out: nothing ever arrives at bars[0]
    if (lane == 0) ok = wait_or_abort(&bars[0], 0, err, abort_flag, limit_ns) ? 1 : 0;
    if (lane == 0 && result) result[0] = ok;
  } else {
    // another role parked on its own barrier: released by the abort flag
    if (lane == 0) ok = wait_or_abort(&bars[1], 0, err, abort_flag) ? 1 : 0;
    if (lane == 0 && result) result[1] = ok;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) {
    __syncwarp();
    tmem_dealloc(tmem_slot, 32);
  }
}

cudaError_t launch_wait_selftest(int* err, unsigned long long limit_ns, int* result, cudaStream_t st) {
  wait_selftest_kernel<<<1, 64, 0, st>>>(err, limit_ns, result);
  return cudaGetLastError();
}

}  // namespace ts
