// wait_probe.cu -- a test hook for the bounded device-side waits every kernel of
// this library uses (tc::mbar_wait): one CTA waits on an mbarrier that nothing
// ever arrives on, with a caller-given budget, and records the site code in a
// device error word when the wait gives up -- the path a real kernel takes when
// a copy or a peer never completes, exercised without any copy in flight.
#include "kb200_internal.h"
#include "tc_common.cuh"

namespace {
__global__ void wait_probe_kernel(int* err, long long budget) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    kb::tc::mbar_init(&bar, 1);
    kb::tc::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !kb::tc::mbar_wait(&bar, 0, budget)) atomicCAS(err, 0, 99);
}
}  // namespace

extern "C" int kb200_wait_probe(void* err_word, int64_t budget_cycles, void* stream) {
  if (!err_word || budget_cycles < 0 || budget_cycles > 4000000000LL)
    return kb::set_error(KB200_ERR_INVALID, "wait_probe: need an error word and 0 <= budget <= 4e9 cycles");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(err_word, 0, sizeof(int), st) != cudaSuccess) return kb::check_launch("wait_probe reset");
  wait_probe_kernel<<<1, 32, 0, st>>>(static_cast<int*>(err_word), budget_cycles);
  return kb::check_launch("wait_probe_kernel");
}

extern "C" int kb200_read_error_word(const void* err_word, void* stream) {
  if (!err_word) return kb::set_error(KB200_ERR_INVALID, "read_error_word: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int code = 0;
  if (cudaMemcpyAsync(&code, err_word, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return kb::check_launch("read_error_word");
  if (code != 0) return kb::set_error(KB200_ERR_TIMEOUT, "a device-side wait gave up (site %d)", code);
  return KB200_OK;
}
