// Diagnostics: a kernel that exercises the bounded-wait timeout path of the
// tcgen05 kernels on purpose, so the path can be tested without a GPU fault.
//
// wait_probe_kernel initialises an mbarrier, allocates TMEM like the real
// kernels, and then waits on the barrier through wait_bounded with the
// caller's cycle limit.  With `complete` = 0 nothing ever arrives on the
// barrier, so the wait runs out: the waiter records (kernel_id << 16 | site)
// in the status word and raises the CTA's abort flag, the other warps see the
// flag and leave their own bounded waits, TMEM is freed and the kernel
// returns.  With `complete` = 1 one thread arrives first and the wait succeeds
// (the control case).  No trap, no device assert, no endless loop: every spin
// is bounded by `limit_cycles`.
#include <cstdio>

#include "common.cuh"

namespace mt {
namespace {

constexpr uint32_t kProbeKernelId = 15;
constexpr uint32_t kProbeSite = 1;

__global__ void __launch_bounds__(128, 1) wait_probe_kernel(uint32_t* status, long long limit_cycles, int complete) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int warp = warp_id();
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  WaitCtx wc{status, &abort_flag, kProbeKernelId};
  wc.limit = limit_cycles;
  if (threadIdx.x == 32 && complete) mbar_arrive(&bar);
  // every warp's lane 0 waits; the first to give up raises the abort flag
  // and the others return as soon as they see it
  if ((threadIdx.x & 31) == 0) wait_bounded(wc, &bar, 0, kProbeSite);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

}  // namespace
}  // namespace mt

using namespace mt;

extern "C" int mt_debug_wait_timeout(int64_t limit_cycles, int complete, uint32_t* status, void* stream) {
  if (status == nullptr || limit_cycles <= 0 || limit_cycles > kWaitCycles) return MT_ERR_INVALID_ARGUMENT;
  int st = bind_device_of(status);
  if (st != MT_OK) return st;
  if ((st = check_arch()) != MT_OK) return st;
  auto s = static_cast<cudaStream_t>(stream);
  wait_probe_kernel<<<1, 128, 0, s>>>(status, (long long)limit_cycles, complete ? 1 : 0);
  if ((st = check_launch("wait_probe_kernel")) != MT_OK) return st;
  // test-only entry: wait for the kernel and report the status word
  cudaError_t err = cudaStreamSynchronize(s);
  if (err != cudaSuccess) {
    set_last_error("cudaStreamSynchronize(wait probe)", err);
    return MT_ERR_LAUNCH;
  }
  uint32_t word = 0;
  err = cudaMemcpy(&word, status, sizeof(word), cudaMemcpyDeviceToHost);
  if (err != cudaSuccess) {
    set_last_error("cudaMemcpy(status word)", err);
    return MT_ERR_LAUNCH;
  }
  if (word != 0) {
    char text[128];
    snprintf(text, sizeof(text), "device wait gave up: kernel %u, site %u", word >> 16, word & 0xFFFFu);
    set_last_error_text(text);
    return MT_ERR_DEVICE_TIMEOUT;
  }
  return MT_OK;
}
