// Self-test of the bounded-wait path used by every pipelined kernel: one
// block waits on an mbarrier that nothing ever completes, with a short limit,
// and must give up, count the timeout and return (the context stays usable).
// No copy is issued, so nothing is in flight when the block exits.
#include "tma.cuh"

B2K_DEFINE_TIMEOUT_COUNTER()

namespace b2k {

__global__ void selftest_wait_kernel(unsigned long long limit_ns, int* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival expected; none will come
    fence_barrier_init();
  }
  __syncthreads();
  const bool done = mbar_wait(&bar, 0u, limit_ns);
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!done) atomicAdd(&b2k_tu_timeouts, 1u);
    *status = done ? 0 : 1;
  }
}

}  // namespace b2k

extern "C" int b2k_selftest_bounded_wait(unsigned long long limit_ns, int* status,
                                         void* stream) {
  B2K_REQUIRE(status != nullptr, "b2k_selftest_bounded_wait: null status");
  B2K_REQUIRE(limit_ns <= 10000000000ull, "b2k_selftest_bounded_wait: limit above 10 s");
  b2k::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, status);
  return b2k::check_launch("b2k_selftest_bounded_wait");
}
