// BatchNorm training forward that allocates nothing.
//
// Why it exists: some callers of this library cannot let it allocate device
// memory at the moment they run BatchNorm.  A serving or training process that
// has handed all of HBM to its own caching allocator or arena up front would
// see an allocation from here fail, or fragment memory it does not own; a
// caller working to a fixed memory budget must know every byte before its loop
// starts.  The ordinary entry point, dct_batchnorm_forward_train, takes its
// per-plane float64 partial sums from the library's workspace, which grows with
// cudaMallocAsync.  This variant takes the same inputs and outputs as raw
// device pointers and keeps its scratch in a file-scope device array instead.
//
// The array: `g_bn_noalloc_scratch`, 2 MiB + 64 KiB of doubles, enough for
// N*C <= 131072 (n, c) planes and C <= 4096 channels.  Every GPU that loads
// this library holds it until the process exits.  Larger shapes are rejected
// with DCT_ERR_SIZE and a message naming the limit; nothing is launched.
//
// Set-up: the first call on each device looks up the array's device address
// with cudaGetSymbolAddress (host code cannot use the array's name as an
// address) and caches it per device; make that first call on a device before
// any stream capture.  No call of this entry point uses cudaMalloc, cudaFree
// or any allocating library routine.
//
// Sharing: every call uses the same array, and the array keeps the last call's
// contents.  Nothing in it has to start at zero: each plane's sums are written
// by exactly one warp and each channel's fold overwrites its slot, so stale
// values are never read.  Calls that overlap on the GPU (for example on two
// streams at once) race on the array; serialise them.
#include <cuda_runtime.h>
#include <mutex>
#include <stdio.h>

#include "dct_common.cuh"
#include "kernels.h"
#include "../../include/dct_cuda.h"

namespace dct {

void note_error(int code, const char* msg);     // runtime.cu

namespace {

constexpr uint32_t kMaxPlanes = 131072;           // N * C
constexpr uint32_t kMaxChannels = 4096;           // C
constexpr size_t kScratchDoubles = 2ull * kMaxPlanes + 2ull * kMaxChannels;

static __device__ __align__(256) double g_bn_noalloc_scratch[kScratchDoubles];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
double* g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of the scratch array for the current device (looked up once).
int scratch_for_current_device(double** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    note_error(DCT_ERR_NO_DEVICE, "dct_batchnorm_forward_train_noalloc: no usable current CUDA device");
    return DCT_ERR_NO_DEVICE;
  }
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_bn_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      char msg[256];
      snprintf(msg, sizeof(msg), "dct_batchnorm_forward_train_noalloc: cudaGetSymbolAddress failed: %s",
               cudaGetErrorString(e));
      note_error(DCT_ERR_CUDA, msg);
      return DCT_ERR_CUDA;
    }
    g_scratch_addr[dev] = static_cast<double*>(p);
  }
  *out = g_scratch_addr[dev];
  return DCT_OK;
}

}  // namespace
}  // namespace dct

extern "C" DCT_API int dct_batchnorm_forward_train_noalloc(const float* x, const float* gamma, const float* beta,
                                                           float* running_mean, float* running_var,
                                                           float* batch_mean, float* batch_var, float* y,
                                                           uint32_t N, uint32_t C, uint32_t S, float eps,
                                                           float momentum, void* stream) {
  using namespace dct;
  if (!x || !gamma || !beta || !running_mean || !running_var || !batch_mean || !batch_var || !y) {
    note_error(DCT_ERR_ARG, "dct_batchnorm_forward_train_noalloc: a device pointer is null");
    return DCT_ERR_ARG;
  }
  const uint64_t planes = (uint64_t)N * C;
  if (planes > kMaxPlanes || C > kMaxChannels) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "dct_batchnorm_forward_train_noalloc: N*C = %llu planes and C = %u exceed the fixed scratch "
             "(at most %u planes and %u channels); use dct_batchnorm_forward_train",
             (unsigned long long)planes, C, kMaxPlanes, kMaxChannels);
    note_error(DCT_ERR_SIZE, msg);
    return DCT_ERR_SIZE;
  }
  // an empty batch (N or S zero) runs the same launches as dct_batchnorm_forward_train:
  // statistics over no elements (0 / 0) and their running update
  if (C == 0) return DCT_OK;
  double* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != DCT_OK) return rc;
  double* plane_sums = scratch;                        // [N*C][2]
  double* chan = scratch + 2ull * kMaxPlanes;          // [C][2]
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_bn_plane_sums(x, nullptr, N, C, S, plane_sums, st);
  if (e == cudaSuccess) e = launch_bn_fold(plane_sums, N, C, chan, st);
  if (e == cudaSuccess)
    e = launch_bn_stats_final(chan, C, (double)N * S, batch_mean, batch_var, running_mean, running_var, true,
                              momentum, st);
  if (e == cudaSuccess)
    e = launch_bn_forward(x, batch_mean, batch_var, gamma, beta, y, N, C, S, eps, planes * S, st);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "dct_batchnorm_forward_train_noalloc: launch failed: %s", cudaGetErrorString(e));
    note_error(DCT_ERR_CUDA, msg);
    return DCT_ERR_CUDA;
  }
  return DCT_OK;
}
