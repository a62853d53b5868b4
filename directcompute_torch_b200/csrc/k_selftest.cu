// Self-test of the device-side failure path: a bounded wait that runs out.
//
// One block initialises an mbarrier that expects one arrival and waits for its
// phase 0 with a bounded poll count; nothing ever arrives, so the wait gives up,
// sets DCT_DEVERR_WAIT_TIMEOUT in the library's mapped error word and the
// kernel returns normally (no trap, no fault, no copy in flight).  The host
// then sees the error at its next wait and the context stays usable.
#include "dct_common.cuh"
#include "dct_tma.cuh"
#include "runtime_internal.h"
#include "../../include/dct_cuda.h"

namespace dct {
namespace {

__global__ void k_selftest_wait(uint32_t spins, uint32_t* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, err, spins);
  __syncthreads();
}

}  // namespace
}  // namespace dct

extern "C" DCT_API int dct_selftest_bounded_wait(uint32_t spins) {
  using namespace dct;
  std::lock_guard<std::recursive_mutex> lk(rt_mutex());
  if (!rt_init()) return DCT_ERR_NO_DEVICE;
  uint32_t* err = device_error_word();
  if (!err) return DCT_ERR_NO_DEVICE;
  if (spins == 0) spins = 1;
  k_selftest_wait<<<1, 32, 0, rt_stream()>>>(spins, err);
  return rt_cuda_ok(cudaGetLastError(), "dct_selftest_bounded_wait") ? 0 : DCT_ERR_CUDA;
}
