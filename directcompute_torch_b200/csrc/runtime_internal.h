// Engine internals shared between runtime.cu and the other host-side
// translation units of libdct_cuda (dist.cu).  Not exported.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace dct {

struct Buffer {
  uint32_t magic;
  int32_t ref;
  uint64_t count;          // fp32 elements
  float* d;
  bool owned;              // false: wraps caller memory (dct_wrap_device_ptr)
  // an index buffer made by MaxPoolForwardFused: its pooling geometry (bc, inH,
  // inW, pool, stride, outH, outW); cleared whenever the buffer is handed out
  bool has_pool_geom = false;
  uint32_t pool_geom[7] = {};
};

std::recursive_mutex& rt_mutex();
bool rt_init();                                 // InitEngine semantics
Buffer* rt_buf(void* handle);                   // live buffer or null (call under rt_mutex)
cudaStream_t rt_stream();
bool rt_ensure_ws(size_t bytes);                // grow the scratch workspace (stream-ordered)
void* rt_ws();
double* rt_host_scratch();                      // pinned, 8 doubles
bool rt_cuda_ok(cudaError_t e, const char* where);
void note_error(int code, const char* msg);
// Waits for the library stream.  With a distributed communicator active this
// polls (stream status, communicator async error, deadline) instead of
// blocking, and aborts the communicator on failure.
bool rt_wait_stream(const char* where);

// hooks installed by dist.cu while a communicator is active
struct DistHooks {
  bool (*async_error)(char* msg, int len) = nullptr;   // true: the communicator failed
  void (*abort)() = nullptr;
  double timeout_s = 120.0;
};
DistHooks& rt_dist_hooks();

}  // namespace dct
