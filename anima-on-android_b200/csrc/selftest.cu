// selftest.cu -- exercises the library's bounded-wait failure path on the device.
//
// Every kernel wait in this library (mbarrier waits on TMA copies, MMA commits and
// softmax hand-offs) gives up after a time limit, records ANIMA_ERR_TIMEOUT in the
// device status word and returns instead of hanging.  This kernel runs that exact path
// on purpose with a short limit: it waits on an mbarrier that nothing will ever arrive
// on, so the wait runs out, the status word is set, and the kernel returns normally.
// The CUDA context stays usable; no fault, trap or unbounded spin is involved.
#include "common.cuh"

namespace anima {

__global__ void selftest_wait_kernel(int* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // expects one arrival that never comes
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long t0 = globaltimer_ns();
    while (!mbar_try_wait(&bar, 0)) {
      if (globaltimer_ns() - t0 > limit_ns) {
        atomicCAS(status, 0, ANIMA_ERR_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
}

int selftest_wait_launch(int* status, unsigned timeout_us, cudaStream_t st) {
  if (timeout_us == 0 || timeout_us > 1000000u) return ANIMA_ERR_ARG;
  selftest_wait_kernel<<<1, 32, 0, st>>>(status, (unsigned long long)timeout_us * 1000ull);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

}  // namespace anima
