// Self-test of the bounded-wait protocol every pipelined kernel here follows.
//
// The kernels' waits on mbarriers (TMA stage full / empty, accumulator
// ready) poll for a bounded time; on timeout the waiting thread records a
// code in the per-device error word and the CTA unwinds: the producer waits
// (again bounded) for its own copies in flight, the TMEM owner frees the
// columns after a block-wide fence, and the kernel returns, so the CUDA
// context stays usable and the host reads the code. This kernel runs exactly
// that protocol with a wait that cannot complete: its consumer warp waits on
// an mbarrier that no thread ever arrives on, with a short caller-given
// limit, while a producer has a bulk copy in flight and a TMEM allocation is
// held. Nothing faults, traps or hangs: every wait ends.
#include "internal.h"
#include "ptx.cuh"

namespace tfx {
namespace {

constexpr int kCopyBytes = 4096;
__device__ __align__(128) uint4 g_selftest_src[kCopyBytes / 16];

__global__ void __launch_bounds__(96, 1)
    bounded_wait_selftest_kernel(long long limit_cycles, int* err) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ __align__(128) uint8_t buf[kCopyBytes];
  __shared__ __align__(8) uint64_t full;
  __shared__ __align__(8) uint64_t never;  // no thread arrives on it
  __shared__ uint32_t tmem_slot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&full, 1);
    mbar_init(&never, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (warp == 0 && lane == 0) {
    // Producer: one copy in flight; whatever happens to the consumer, it
    // lands before the CTA may exit.
    mbar_arrive_expect_tx(&full, kCopyBytes);
    bulk_load(buf, g_selftest_src, kCopyBytes, &full);
    mbar_wait_for(&full, 0, err, kDevTimeoutFull, limit_cycles);
  } else if (warp == 2) {
    // Consumer: the wait that cannot complete. The outcome is made
    // warp-uniform before anything warp-collective, as in the real kernels.
    const bool ok =
        __all_sync(0xffffffffu, mbar_wait_for(&never, 0, err, kDevTimeoutAccum, limit_cycles));
    (void)ok;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 32);
}

}  // namespace
}  // namespace tfx

using namespace tfx;

extern "C" {

int tfx_selftest_bounded_wait(int64_t limit_cycles, tfx_stream_t stream) {
  if (limit_cycles <= 0 || limit_cycles > kWaitLimitCycles)
    return fail(TFX_ERR_INVALID_ARGUMENT,
                "tfx_selftest_bounded_wait: limit_cycles must be in (0, %lld]", kWaitLimitCycles);
  int* err = device_error_word();
  if (err == nullptr) return fail(TFX_ERR_CUDA, "device error word unavailable");
  launch_pdl(bounded_wait_selftest_kernel, dim3(1), dim3(96), 0,
             reinterpret_cast<cudaStream_t>(stream), static_cast<long long>(limit_cycles), err);
  return check_launch("bounded_wait_selftest_kernel");
}

}  // extern "C"
