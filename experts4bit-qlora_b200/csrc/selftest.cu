// Self-test of the failure path of the library's bounded waits (no counterpart in
// the reference). One CTA arms an mbarrier for a copy that is never issued and
// waits on it with the same bounded wait every TMA consumer here uses; the wait
// gives up after its iteration cap, the kernel records E4B_ERR_TIMEOUT in the
// workspace's error word and returns normally, leaving the context usable. Used
// by the tests to check that a wait that runs out is reported, not hung.
#include "async.cuh"
#include "common.cuh"

namespace e4b {
namespace {

__global__ void wait_timeout_kernel(int* err, int* outcome) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_proxy_async();
    mbar_arrive_expect_tx(&bar, 16);  // 16 bytes that no copy will deliver
    const bool done = mbar_wait(&bar, 0);
    *outcome = done ? 1 : 0;
    if (!done) raise_error(err, E4B_ERR_TIMEOUT);
  }
}

}  // namespace
}  // namespace e4b

extern "C" e4b_status e4b_selftest_wait_timeout(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes < e4b::kErrBytes) return E4B_ERR_WORKSPACE;
  cudaStream_t s = (cudaStream_t)stream;
  int* err = static_cast<int*>(workspace);
  if (cudaMemsetAsync(err, 0, 2 * sizeof(int), s) != cudaSuccess) return E4B_ERR_CUDA;
  e4b::wait_timeout_kernel<<<1, 32, 0, s>>>(err, err + 1);
  return e4b::launch_status();
}
