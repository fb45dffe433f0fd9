// Probe of the bounded device waits that every tcgen05 kernel uses (mbar_wait_spin /
// mbar_wait in tc_common.cuh): one thread waits on an mbarrier that nothing will ever complete,
// with a short limit, so the expiry path runs for real: the wait gives up, records the device
// error code and the kernel returns.  The host then sees FLETCHER_ERR_DEVICE_WAIT at the next
// synchronisation, and the context stays usable.  Nothing faults and nothing hangs: the wait
// ends after `limit` cycles (at most the production limit, about 2 s).
#include "kernels.cuh"
#include "tc_common.cuh"

namespace fl {
using namespace tc;

__global__ void k_wait_probe(int32_t* err, long long limit, int sleeping) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival expected; none comes
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    volatile int* abort = &abort_flag;
    const bool ok = sleeping ? mbar_wait(&bar, 0, abort, err, limit) : mbar_wait_spin(&bar, 0, abort, err, limit);
    if (ok) atomicExch(err, 2);  // the phase cannot complete: report it as a distinct code
  }
}

}  // namespace fl

using namespace fl;

extern "C" {

int32_t Cuda_Debug_WaitTimeoutProbe(CudaContextRef ctx, int64_t limit_cycles, int32_t sleeping) {
  Ctx* c = reinterpret_cast<Ctx*>(ctx);
  if (!c) return FLETCHER_ERR_INVALID;
  DeviceGuard g(c);
  FL_CHECK(c, limit_cycles > 0 && limit_cycles <= kWaitLimitCycles, "WaitTimeoutProbe: limit %lld out of (0, %lld]",
           (long long)limit_cycles, (long long)kWaitLimitCycles);
  k_wait_probe<<<1, 32, 0, c->stream>>>(c->d_err, (long long)limit_cycles, sleeping);
  FL_LAUNCH(c);
  FL_CUDA(c, cudaStreamSynchronize(c->stream));
  return check_device_flag(c);
}

}  // extern "C"
