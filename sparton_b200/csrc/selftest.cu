// selftest.cu — sparton_selftest_wait_timeout: makes the bounded device wait of
// ptx.cuh run out on purpose, so a test can check that a stuck wait ends with
// a status code instead of a hang, and that the context stays usable.
//
// Upstream has no counterpart (its Triton kernels never wait on one another).
// The kernels of this library wait on mbarriers that TMA copies and tensor-core
// MMAs complete; a correct launch never comes near the wait limit, so the
// timeout path cannot be reached through them without breaking a kernel on
// purpose. This kernel reaches it with no fault: it waits on barriers that
// nobody arrives on, through the same mbar_wait_bounded the production kernels
// use, with a short limit.
//
// One CTA, two warps, two barriers that nothing completes:
//   warp 0 waits on barrier 0 with `limit_ns`; when the limit passes it raises
//          the CTA's abort flag and records SPARTON_DEV_TIMEOUT_SELFTEST in the
//          status word (the first code recorded wins, as in every kernel);
//   warp 1 waits on barrier 1 with the production limit and must leave early,
//          through the abort flag raised by warp 0: the path by which the other
//          roles of a kernel unwind after one role timed out.
// Workspace words: [0] status, [1] microseconds warp 0 waited, [2] 1 when warp
// 1 left through the abort flag before its own limit.
#include "internal.h"
#include "ptx.cuh"

namespace sparton {
namespace {

__global__ void __launch_bounds__(64) wait_selftest_kernel(uint64_t limit_ns,
                                                           unsigned int* words) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(smem_addr(&bars[0]), 1);
    mbar_init(smem_addr(&bars[1]), 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  volatile int* flag = &abort_flag;
  const uint64_t t0 = global_timer_ns();
  if (warp == 0) {
    const bool done = mbar_wait_bounded_warp(smem_addr(&bars[0]), 0, flag, words,
                                             SPARTON_DEV_TIMEOUT_SELFTEST, limit_ns);
    if (threadIdx.x == 0)
      words[1] = done ? 0u : static_cast<unsigned int>((global_timer_ns() - t0) / 1000ull);
  } else {
    const bool done = mbar_wait_bounded_warp(smem_addr(&bars[1]), 0, flag, words,
                                             SPARTON_DEV_TIMEOUT_EPILOGUE);
    const bool early = global_timer_ns() - t0 < kWaitTimeoutNs;
    if (threadIdx.x == 32) words[2] = (!done && early) ? 1u : 0u;
  }
}

}  // namespace
}  // namespace sparton

extern "C" int sparton_selftest_wait_timeout(uint32_t limit_us, void* workspace,
                                             size_t workspace_size, void* stream) {
  if (limit_us < 1 || limit_us > 1000000)
    return sparton::fail(SPARTON_ERR_INVALID_ARGUMENT, "limit_us=%u must lie in [1, 1000000]",
                         limit_us);
  if (workspace == nullptr || workspace_size < 256)
    return sparton::fail(SPARTON_ERR_WORKSPACE, "workspace of 256 bytes needed, %zu given",
                         workspace_size);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return sparton::fail(SPARTON_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  const int st = sparton::check_device();
  if (st != SPARTON_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned int* words = static_cast<unsigned int*>(workspace);
  cudaError_t e = cudaMemsetAsync(words, 0, 16, s);
  if (e != cudaSuccess) return sparton::cuda_fail(e, "cudaMemsetAsync");
  sparton::wait_selftest_kernel<<<1, 64, 0, s>>>(static_cast<uint64_t>(limit_us) * 1000ull, words);
  e = cudaGetLastError();
  if (e != cudaSuccess) return sparton::cuda_fail(e, "wait_selftest_kernel launch");
  return SPARTON_OK;
}
