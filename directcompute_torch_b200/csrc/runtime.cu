// libdct_cuda: the C-ABI drop-in for directcompute_torch's native engine.
//
// The reference binds `engine.dll` with ctypes (nn_engine.py:42-119) and drives
// it through 32 extern "C" entry points (engine.cpp).  This file exports the
// same names with the same argument meaning, on CUDA for one B200 per process:
//
//   device + stream      InitEngine / GetGPUInfo / FlushGPU / SyncGPU
//   buffers              CreateBuffer / AddRefBuffer / UpdateBuffer / ReleaseBuffer /
//                        ReleaseBufferBatch / ReadBuffer / ClearBuffer (refcounted
//                        handles over cudaMallocAsync memory, size-keyed pool with
//                        the reference's per-size caps, engine.cpp:181-290)
//   kernels by name      CompileShader (name -> built-in CUDA kernel; the HLSL file
//                        is not read) / RunShader / RunShaderRaw / RunShaderAlloc(2) /
//                        ResolveShader / RunSequence(WithSGD)
//   optimizers           SGDBatch / SGDBatchClipped as multi-tensor launches
//   pool                 WarmPool / GetPoolStats / ResetPoolStats / GetPoolMemory / DrainPool
//   pooling              MaxPoolForwardFused / MaxPoolBackwardFused
//   out of scope         MatMulAlloc / Conv*Fused: exported stubs (return null,
//                        record an error)
//
// and extension entry points prefixed dct_ (NumPy-broadcast binary ops, unary
// ops, axis/full reductions, fused softmax+CE, fused Adam, BatchNorm, device
// timing, errors, raw-pointer interop, NCCL sharding).
//
// Errors never cross the ABI as exceptions: like the reference, calls fail
// quietly (null / false / no-op) -- and, unlike it, record a message that
// dct_last_error() returns and dct_error_code() numbers.  Handles are checked
// against the live-handle set before use, so a stale or foreign pointer is
// rejected instead of dereferenced.  Every entry point holds one mutex
// (ctypes drops the GIL during calls).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <stdarg.h>
#include <stddef.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <mutex>
#include <thread>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "dct_common.cuh"
#include "kernels.h"
#include "runtime_internal.h"
#include "../../include/dct_cuda.h"

namespace dct {

// ---------------------------------------------------------------------------
// engine state
// ---------------------------------------------------------------------------
constexpr uint32_t kBufMagic = 0xDC7B0F01u;
static_assert(sizeof(DctSeqCmd) == 200 && offsetof(DctSeqCmd, cbData) == 128 && offsetof(DctSeqCmd, cbSize) == 192,
              "DctSeqCmd must match the reference's SeqCmd field layout");
static_assert(sizeof(DctGPUInfo) == 160 && offsetof(DctGPUInfo, description) == 28, "GPUInfo layout");

struct Engine {
  bool init = false;
  DevInfo info;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  std::unordered_set<Buffer*> live;
  std::unordered_map<uint64_t, std::vector<Buffer*>> pool;
  uint64_t hits = 0, misses = 0, pool_bytes = 0;
  void* ws = nullptr;             // reduction scratch
  size_t ws_bytes = 0;
  float* host_small = nullptr;    // pinned 64-byte staging for scalar readbacks
  uint32_t* dev_err_host = nullptr;   // mapped error word written by device code
  uint32_t* dev_err_dev = nullptr;
  uint32_t* flags = nullptr;          // kDeviceFlags zeroed device words (the maxpool fix-up flag)
  char name[128] = {0};
  // error state
  int err_code = 0;
  std::string err;
};

static Engine g;
static std::recursive_mutex g_mu;
#define LOCK std::lock_guard<std::recursive_mutex> _lk(g_mu)

// Launch geometry of the engine's device; before InitEngine (callers of the
// allocation-free entry point may never initialise the engine) it is read
// from the current device's attributes, which allocates nothing.
const DevInfo& dev_info() {
  if (g.init) return g.info;
  static thread_local DevInfo local;
  int d = 0;
  if (cudaGetDevice(&d) == cudaSuccess && local.device != d) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d) == cudaSuccess && v > 0) local.sm_count = v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxThreadsPerMultiProcessor, d) == cudaSuccess && v > 0)
      local.max_threads_per_sm = v;
    local.device = d;
  }
  cudaGetLastError();
  return local;
}

static void set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g.err_code = code;
  g.err = buf;
}

uint32_t* device_error_word() { return g.dev_err_dev; }
uint32_t* device_flags() { return g.init ? g.flags : nullptr; }

// error recording for entry points that live outside this file
void note_error(int code, const char* msg) {
  LOCK;
  g.err_code = code;
  g.err = msg ? msg : "";
}

static bool cuda_ok(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return true;
  set_error(DCT_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
  return false;
}

static bool ensure_init();

static DistHooks g_hooks;           // the sharding layer's wait hooks (set while a communicator is active)

// Device code reports bounded-wait timeouts through a mapped host word; surface
// them after every wait on the stream.
static bool check_device_errors() {
  if (!g.dev_err_host) return true;
  const uint32_t e = *(volatile uint32_t*)g.dev_err_host;
  if (!e) return true;
  *(volatile uint32_t*)g.dev_err_host = 0;
  if (e & DCT_DEVERR_PEER_WAIT) {
    // the ranks' exchange epochs no longer agree: the communicator cannot be used again
    set_error(DCT_ERR_DIST, "sharded op: a peer rank's record did not arrive before the deadline (a rank is "
              "gone or behind; error bits 0x%x); results are invalid; communicator aborted", e);
    if (g_hooks.abort) g_hooks.abort();
  }
  else if (e & DCT_DEVERR_PEER_INVALID)
    set_error(DCT_ERR_DIST, "sharded op: a rank's shard was invalid (bad handle, size or count on that rank; "
              "error bits 0x%x); results are invalid", e);
  else
    set_error(DCT_ERR_CUDA, "device: a bounded wait in a kernel timed out (error bits 0x%x); results are invalid", e);
  return false;
}

// ---------------------------------------------------------------------------
// buffers and pool (engine.cpp:181-290 semantics)
// ---------------------------------------------------------------------------
static size_t max_pool_for_size(uint64_t count) {          // engine.cpp:186-197
  const uint64_t bytes = count * sizeof(float);
  const uint64_t usable = g.info.total_mem;
  if (usable > 0 && bytes >= usable / 4) return 4;
  if (bytes >= 4ull * 1024 * 1024) return 6;
  if (bytes >= 256ull * 1024) return 8;
  return 16;
}

static Buffer* buf_of(void* h) {
  Buffer* b = static_cast<Buffer*>(h);
  if (!b || g.live.find(b) == g.live.end() || b->magic != kBufMagic) return nullptr;
  return b;
}

static Buffer* create_buffer(const float* host, uint64_t count) {
  if (!ensure_init()) return nullptr;
  if (count == 0) {
    set_error(DCT_ERR_ARG, "CreateBuffer: zero-length buffer");
    return nullptr;
  }
  Buffer* b = nullptr;
  auto it = g.pool.find(count);
  if (it != g.pool.end() && !it->second.empty()) {
    b = it->second.back();
    it->second.pop_back();
    g.pool_bytes -= count * sizeof(float);
    g.hits++;
  } else {
    g.misses++;
    void* d = nullptr;
    const size_t bytes = ((count * sizeof(float)) + 255) & ~size_t(255);
    if (!cuda_ok(cudaMallocAsync(&d, bytes, g.stream), "CreateBuffer(cudaMallocAsync)")) return nullptr;
    b = new Buffer{kBufMagic, 0, count, static_cast<float*>(d), true};
  }
  b->ref = 1;
  b->has_pool_geom = false;
  g.live.insert(b);
  if (host) {
    cudaPointerAttributes at{};
    const bool pinned = cudaPointerGetAttributes(&at, host) == cudaSuccess && at.type == cudaMemoryTypeHost;
    cudaGetLastError();
    cuda_ok(cudaMemcpyAsync(b->d, host, count * sizeof(float), cudaMemcpyHostToDevice, g.stream), "CreateBuffer(H2D)");
    if (pinned) rt_wait_stream("CreateBuffer");      // caller may reuse its memory on return
  }
  return b;
}

static void destroy(Buffer* b) {
  if (b->owned && b->d) cudaFreeAsync(b->d, g.stream);
  b->magic = 0;
  delete b;
}

static void release_internal(Buffer* b) {                   // engine.cpp:267-290
  g.live.erase(b);
  if (!b->owned) { destroy(b); return; }
  auto& lst = g.pool[b->count];
  if (lst.size() < max_pool_for_size(b->count)) {
    lst.push_back(b);
    g.pool_bytes += b->count * sizeof(float);
  } else {
    destroy(b);
  }
}

static void release_handle(void* h) {
  Buffer* b = buf_of(h);
  if (!b) {
    if (h) set_error(DCT_ERR_HANDLE, "ReleaseBuffer: unknown handle %p", h);
    return;
  }
  if (--b->ref <= 0) release_internal(b);
}

static bool g_capturing = false;    // RunSequence is capturing the stream into a CUDA graph

static bool ensure_ws(size_t bytes) {
  if (bytes <= g.ws_bytes) return true;
  if (g_capturing) {                 // an allocation inside a capture would belong to the graph
    set_error(DCT_ERR_CUDA, "workspace growth during graph capture");
    return false;
  }
  size_t want = std::max(bytes, g.ws_bytes * 2);
  want = (want + (1 << 20) - 1) & ~size_t((1 << 20) - 1);
  if (g.ws) cudaFreeAsync(g.ws, g.stream);
  g.ws = nullptr;
  g.ws_bytes = 0;
  if (!cuda_ok(cudaMallocAsync(&g.ws, want, g.stream), "workspace(cudaMallocAsync)")) return false;
  g.ws_bytes = want;
  return true;
}

// ---------------------------------------------------------------------------
// internal API for the other translation units (runtime_internal.h)
// ---------------------------------------------------------------------------
DistHooks& rt_dist_hooks() { return g_hooks; }
std::recursive_mutex& rt_mutex() { return g_mu; }
Buffer* rt_buf(void* h) { return buf_of(h); }
cudaStream_t rt_stream() { return g.stream; }
bool rt_ensure_ws(size_t bytes) { return ensure_ws(bytes); }
void* rt_ws() { return g.ws; }
double* rt_host_scratch() { return reinterpret_cast<double*>(g.host_small); }
bool rt_cuda_ok(cudaError_t e, const char* where) { return cuda_ok(e, where); }

bool rt_wait_stream(const char* where) {
  if (!g_hooks.async_error) {
    if (!cuda_ok(cudaStreamSynchronize(g.stream), where)) return false;
    return check_device_errors();
  }
  // a peer that died must not hang this process: poll with a deadline
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaStreamQuery(g.stream);
    if (q == cudaSuccess) return check_device_errors();
    if (q != cudaErrorNotReady) return cuda_ok(q, where);
    char msg[256] = {0};
    const double limit = g_hooks.timeout_s;
    if (g_hooks.async_error(msg, sizeof(msg))) {
      if (g_hooks.abort) g_hooks.abort();       // clears the hooks
      set_error(DCT_ERR_DIST, "%s: communicator failed: %s", where, msg);
      return false;
    }
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > limit) {
      if (g_hooks.abort) g_hooks.abort();
      set_error(DCT_ERR_DIST, "%s: no progress within %.0f s (a peer rank is gone?); communicator aborted", where,
                limit);
      return false;
    }
    // poll hot for the first 2 ms (short waits stay short), then back off
    if (el < 2e-3) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

// ---------------------------------------------------------------------------
// init / device
// ---------------------------------------------------------------------------
static bool init_engine() {
  if (g.init) return true;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    set_error(DCT_ERR_NO_DEVICE, "InitEngine: no CUDA device visible");
    return false;
  }
  int dev = -1;
  const char* e = getenv("DCT_DEVICE");
  if (!e) e = getenv("LOCAL_RANK");
  if (e) dev = atoi(e) % n;
  if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  if (!cuda_ok(cudaSetDevice(dev), "InitEngine(cudaSetDevice)")) return false;
  cudaDeviceProp p{};
  if (!cuda_ok(cudaGetDeviceProperties(&p, dev), "InitEngine(props)")) return false;
  g.info.device = dev;
  g.info.sm_count = p.multiProcessorCount;
  g.info.max_threads_per_sm = p.maxThreadsPerMultiProcessor;
  g.info.smem_optin = p.sharedMemPerBlockOptin;
  g.info.total_mem = p.totalGlobalMem;
  snprintf(g.name, sizeof(g.name), "%.127s", p.name);   // GPUInfo::description holds 128 bytes
  if (!cuda_ok(cudaStreamCreateWithFlags(&g.stream, cudaStreamNonBlocking), "InitEngine(stream)")) return false;
  cudaEventCreate(&g.ev0);
  cudaEventCreate(&g.ev1);
  // keep freed blocks in the stream-ordered pool instead of returning them to the driver
  cudaMemPool_t mp;
  if (cudaDeviceGetDefaultMemPool(&mp, dev) == cudaSuccess) {
    uint64_t thr = UINT64_MAX;
    cudaMemPoolSetAttribute(mp, cudaMemPoolAttrReleaseThreshold, &thr);
  }
  cudaGetLastError();
  if (!cuda_ok(cudaMallocHost(&g.host_small, 64), "InitEngine(pinned staging)")) return false;
  if (!cuda_ok(cudaHostAlloc((void**)&g.dev_err_host, 64, cudaHostAllocMapped), "InitEngine(error word)")) return false;
  *g.dev_err_host = 0;
  if (!cuda_ok(cudaHostGetDevicePointer((void**)&g.dev_err_dev, g.dev_err_host, 0), "InitEngine(error word)"))
    return false;
  if (!cuda_ok(cudaMalloc(&g.flags, kDeviceFlags * sizeof(uint32_t)), "InitEngine(flags)")) return false;
  if (!cuda_ok(cudaMemset(g.flags, 0, kDeviceFlags * sizeof(uint32_t)), "InitEngine(flags)")) return false;
  g.init = true;
  return true;
}

static bool ensure_init() {
  if (g.init) return true;
  if (init_engine()) return true;
  return false;
}
bool rt_init() {
  LOCK;
  return ensure_init();
}

// ---------------------------------------------------------------------------
// shader registry
// ---------------------------------------------------------------------------
struct Disp {
  Buffer* srv[16];
  uint32_t nsrv;
  Buffer* uav[16];
  uint32_t nuav;
  uint32_t gx, gy, gz;
  uint32_t u[16];          // cbuffer words, zero padded
  uint32_t cbsize;
  const char* name;
};
typedef bool (*Handler)(const Disp&);

struct Shader {
  const char* name;
  Handler fn;
  bool always;             // extension kernels: usable without CompileShader
  bool compiled;
  uint32_t magic;
};
constexpr uint32_t kShaderMagic = 0x5EADC0DEu;

static float f_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint64_t lim(uint64_t count, uint32_t groups, uint32_t tpg = 256) {
  return std::min<uint64_t>(count, (uint64_t)groups * tpg);
}

// argument checks: handles present and large enough
static bool need(const Disp& d, uint32_t ns, uint32_t nu) {
  if (d.nsrv < ns || d.nuav < nu) {
    set_error(DCT_ERR_ARG, "%s: needs %u SRVs / %u UAVs, got %u / %u", d.name, ns, nu, d.nsrv, d.nuav);
    return false;
  }
  for (uint32_t i = 0; i < ns; ++i)
    if (!d.srv[i]) { set_error(DCT_ERR_HANDLE, "%s: SRV t%u is not a live buffer", d.name, i); return false; }
  for (uint32_t i = 0; i < nu; ++i)
    if (!d.uav[i]) { set_error(DCT_ERR_HANDLE, "%s: UAV u%u is not a live buffer", d.name, i); return false; }
  return true;
}
static bool fits(const Disp& d, const Buffer* b, uint64_t n, const char* what) {
  if (b->count >= n) return true;
  set_error(DCT_ERR_SIZE, "%s: %s holds %llu floats, the dispatch touches %llu", d.name, what,
            (unsigned long long)b->count, (unsigned long long)n);
  return false;
}
#define FITS(b, n, what) if (!fits(d, b, n, what)) return false
#define LAUNCH(expr) return cuda_ok((expr), d.name)

// ---- elementwise -----------------------------------------------------------
static bool h_add_bias_impl(const Disp& d, bool relu) {     // nn_add_bias.hlsl / nn_bias_relu.hlsl
  if (!need(d, 2, 1)) return false;
  const uint64_t M = d.u[0], N = d.u[1];
  const uint64_t n = lim(M * N, d.gx);
  if (n == 0 || N == 0) return true;
  FITS(d.srv[0], n, "A"); FITS(d.uav[0], n, "C"); FITS(d.srv[1], std::min<uint64_t>(N, n), "B");
  const uint64_t full = n / N, rem = n % N;
  cudaError_t e = cudaSuccess;
  if (full) e = launch_add_bias(d.srv[0]->d, d.srv[1]->d, d.uav[0]->d, full, N, relu, g.stream);
  if (e == cudaSuccess && rem)
    e = launch_add_bias(d.srv[0]->d + full * N, d.srv[1]->d, d.uav[0]->d + full * N, 1, rem, relu, g.stream);
  LAUNCH(e);
}
static bool h_add_bias(const Disp& d) { return h_add_bias_impl(d, false); }
static bool h_bias_relu(const Disp& d) { return h_add_bias_impl(d, true); }

static bool h_relu(const Disp& d) {                           // nn_relu.hlsl: no cb, no bounds check
  if (!need(d, 1, 1)) return false;
  const uint64_t n_out = lim(d.uav[0]->count, d.gx);
  LAUNCH(launch_relu_bounded(d.srv[0]->d, d.srv[0]->count, d.uav[0]->d, n_out, g.stream));
}

static bool unary_n(const Disp& d, int op, float alpha) {
  if (!need(d, 1, 1)) return false;
  const uint64_t n = lim(d.u[0], d.gx);
  FITS(d.srv[0], n, "input"); FITS(d.uav[0], n, "output");
  LAUNCH(launch_unary(op, d.srv[0]->d, d.uav[0]->d, n, alpha, g.stream));
}
static bool binary_n(const Disp& d, int op, uint64_t count, float al, float be) {
  if (!need(d, 2, 1)) return false;
  const uint64_t n = lim(count, d.gx);
  FITS(d.srv[0], n, "t0"); FITS(d.srv[1], n, "t1"); FITS(d.uav[0], n, "u0");
  LAUNCH(launch_binary_same(op, d.srv[0]->d, d.srv[1]->d, d.uav[0]->d, n, al, be, g.stream));
}
static bool h_relu6(const Disp& d) { return unary_n(d, EW_RELU6, 0.f); }
static bool h_leaky_relu(const Disp& d) { return unary_n(d, EW_LEAKY_RELU, f_of(d.u[1])); }
static bool h_sigmoid(const Disp& d) { return unary_n(d, EW_SIGMOID, 0.f); }
static bool h_relu_grad(const Disp& d) { return binary_n(d, EW_RELU_GRAD, d.u[0], 0.f, 0.f); }
static bool h_relu6_grad(const Disp& d) { return binary_n(d, EW_RELU6_GRAD, d.u[0], 0.f, 0.f); }
static bool h_leaky_relu_grad(const Disp& d) { return binary_n(d, EW_LEAKY_RELU_GRAD, d.u[0], f_of(d.u[1]), 0.f); }
static bool h_sigmoid_grad(const Disp& d) { return binary_n(d, EW_SIGMOID_GRAD, d.u[0], 0.f, 0.f); }
static bool h_add(const Disp& d) { return binary_n(d, EW_ADD, (uint64_t)d.u[0] * d.u[1], 0.f, 0.f); }
static bool h_scale_add(const Disp& d) { return binary_n(d, EW_SCALE_ADD, d.u[0], f_of(d.u[1]), f_of(d.u[2])); }

static bool h_grad_accum(const Disp& d) {                     // accum = accum + grad
  if (!need(d, 1, 1)) return false;
  const uint64_t n = lim(d.u[0], d.gx);
  FITS(d.srv[0], n, "grad"); FITS(d.uav[0], n, "accum");
  LAUNCH(launch_binary_same(EW_ADD, d.uav[0]->d, d.srv[0]->d, d.uav[0]->d, n, 0.f, 0.f, g.stream));
}

static bool h_gap_backward(const Disp& d) {
  if (!need(d, 1, 1)) return false;
  const uint64_t S = d.u[2];
  const uint64_t n = lim((uint64_t)d.u[0] * d.u[1] * S, d.gx);
  if (n == 0) return true;
  FITS(d.uav[0], n, "dx"); FITS(d.srv[0], (n + S - 1) / S, "grad_output");
  LAUNCH(launch_gap_backward(d.srv[0]->d, d.uav[0]->d, n, (uint32_t)S, g.stream));
}

static bool h_accumulate_scalar(const Disp& d) {
  if (!need(d, 1, 1)) return false;
  LAUNCH(launch_accumulate_scalar(d.srv[0]->d, d.uav[0]->d, g.stream));
}

// ---- reductions ------------------------------------------------------------
static bool reduce_strided(const Disp& d, int op, const float* x, uint64_t outer, uint64_t len, uint64_t inner,
                           uint64_t so, uint64_t sl, uint64_t si, float* out, int32_t* idx) {
  const size_t ws = reduce_strided_ws_bytes(outer, len, inner, so, sl, si);
  if (ws && !ensure_ws(ws)) return false;
  LAUNCH(launch_reduce_strided(op, x, outer, len, inner, so, sl, si, out, idx, g.ws, g.ws_bytes, g.stream));
}

static bool h_bias_grad(const Disp& d) {                      // nn_bias_grad.hlsl:8-29
  if (!need(d, 1, 1)) return false;
  const uint64_t B = d.u[0], K = std::min<uint64_t>(d.u[1], d.gx), si = d.u[2], sc = d.u[3];
  if (K == 0) return true;
  FITS(d.uav[0], K, "grad_bias");
  if (B == 0) LAUNCH(cudaMemsetAsync(d.uav[0]->d, 0, K * sizeof(float), g.stream));
  FITS(d.srv[0], (B - 1) * si + (K - 1) * sc + 1, "grad_out");
  const float* x = d.srv[0]->d;
  if (sc == 1) return reduce_strided(d, RED_SUM, x, 1, B, K, 0, si, 1, d.uav[0]->d, nullptr);
  if (si == 1) return reduce_strided(d, RED_SUM, x, K, B, 1, sc, 1, 1, d.uav[0]->d, nullptr);
  return reduce_strided(d, RED_SUM, x, 1, B, K, 0, si, sc, d.uav[0]->d, nullptr);
}

static bool h_gap(const Disp& d) {                            // nn_global_avg_pool.hlsl:16-35
  if (!need(d, 1, 1)) return false;
  const uint64_t S = d.u[2];
  const uint64_t rows = std::min<uint64_t>((uint64_t)d.u[0] * d.u[1], d.gx);
  if (rows == 0 || S == 0) return true;
  FITS(d.srv[0], rows * S, "input"); FITS(d.uav[0], rows, "output");
  return reduce_strided(d, RED_MEAN, d.srv[0]->d, rows, S, 1, S, 1, 1, d.uav[0]->d, nullptr);
}

static bool h_rms(const Disp& d) {                            // nn_rms.hlsl:7-24
  if (!need(d, 1, 1)) return false;
  const uint64_t n = d.u[0];
  FITS(d.srv[0], n, "A");
  if (!ensure_ws(full_reduce_ws_bytes())) return false;
  LAUNCH(launch_rms(d.srv[0]->d, n, d.uav[0]->d, g.ws, g.stream));
}

static bool h_grad_sq_reduce(const Disp& d) {                 // nn_grad_sq_reduce.hlsl:16-30
  if (!need(d, 1, 1)) return false;
  const uint64_t count = d.u[0], off = d.u[1], ng = d.gx;
  FITS(d.srv[0], std::min<uint64_t>(count, ng * 256), "grad");
  FITS(d.uav[0], off + ng, "partials");
  LAUNCH(launch_grad_sq_reduce(d.srv[0]->d, std::min<uint64_t>(count, ng * 256), d.uav[0]->d, off, ng, g.stream));
}

static bool h_grad_norm_final(const Disp& d) {                // nn_grad_norm_final.hlsl:16-35
  if (!need(d, 1, 1)) return false;
  FITS(d.srv[0], d.u[0], "partials"); FITS(d.uav[0], 2, "normScale");
  LAUNCH(launch_grad_norm_final(d.srv[0]->d, d.u[0], f_of(d.u[1]), d.uav[0]->d, g.stream));
}

static bool h_dice_loss(const Disp& d) {
  if (!need(d, 2, 1)) return false;
  const uint32_t b = std::min<uint32_t>(d.u[0], d.gx), size = d.u[1];
  FITS(d.srv[0], (uint64_t)b * size, "Pred"); FITS(d.srv[1], (uint64_t)b * size, "Target"); FITS(d.uav[0], b, "Out");
  if (!ensure_ws(dice_ws_bytes(b, size))) return false;
  LAUNCH(launch_dice_sums(d.srv[0]->d, d.srv[1]->d, b, size, d.uav[0]->d, 1, g.ws, g.ws_bytes, g.stream));
}
static bool h_dice_loss_sums(const Disp& d) {
  if (!need(d, 2, 1)) return false;
  const uint32_t b = std::min<uint32_t>(d.u[0], d.gx), size = d.u[1];
  FITS(d.srv[0], (uint64_t)b * size, "Pred"); FITS(d.srv[1], (uint64_t)b * size, "Target");
  FITS(d.uav[0], 3ull * b, "Sums");
  if (!ensure_ws(dice_ws_bytes(b, size))) return false;
  LAUNCH(launch_dice_sums(d.srv[0]->d, d.srv[1]->d, b, size, d.uav[0]->d, 0, g.ws, g.ws_bytes, g.stream));
}
static bool h_dice_loss_grad(const Disp& d) {
  if (!need(d, 3, 1)) return false;
  const uint32_t batch = d.u[0], size = d.u[1];
  const uint64_t n = lim((uint64_t)batch * size, d.gx);
  if (n == 0) return true;
  FITS(d.srv[0], n, "Pred"); FITS(d.srv[1], n, "Target"); FITS(d.uav[0], n, "DX");
  FITS(d.srv[2], 3 * ((n - 1) / size + 1), "Sums");
  LAUNCH(launch_dice_grad(d.srv[0]->d, d.srv[1]->d, d.srv[2]->d, d.uav[0]->d, batch, size, n, g.stream));
}

// ---- layout ops beside the path ------------------------------------------------------
// The shaders index with 32-bit `uint`; an index space past 2^32 is refused, as
// is a buffer smaller than the largest index the dispatch touches.
static bool idx32(const Disp& d, uint64_t v, const char* what) {
  if (v <= 0xFFFFFFFFull) return true;
  set_error(DCT_ERR_ARG, "%s: %s needs %llu elements, past the shader's 32-bit index space", d.name, what,
            (unsigned long long)v);
  return false;
}

static bool h_upsample(const Disp& d) {                       // nn_upsample.hlsl:15-33
  if (!need(d, 1, 1)) return false;
  const uint64_t B = d.u[0], C = d.u[1], inH = d.u[2], inW = d.u[3], oH = d.u[4], oW = d.u[5], sH = d.u[6],
                 sW = d.u[7];
  const uint64_t total = B * C * oH * oW;
  if (!idx32(d, total, "the output")) return false;
  const uint64_t n = lim(total, d.gx);
  if (n == 0) return true;
  if (sH == 0 || sW == 0) { set_error(DCT_ERR_ARG, "%s: a scale factor is 0", d.name); return false; }
  // largest source index over outputs [0, n): the last output, the end of the
  // row before it and the end of the plane before it (each term is monotone)
  auto src = [&](uint64_t i) {
    const uint64_t w = i % oW, r = i / oW, h = r % oH, bc = r / oH;
    return (bc * inH + h / sH) * inW + w / sW;
  };
  const uint64_t last = n - 1, row0 = last - last % oW, plane0 = (last / (oH * oW)) * oH * oW;
  uint64_t hi = src(last);
  if (row0 > 0) hi = std::max(hi, src(row0 - 1));
  if (plane0 > 0) hi = std::max(hi, src(plane0 - 1));
  if (!idx32(d, hi + 1, "the input")) return false;
  FITS(d.srv[0], hi + 1, "X"); FITS(d.uav[0], n, "Out");
  LAUNCH(launch_upsample(d.srv[0]->d, d.uav[0]->d, (uint32_t)n, (uint32_t)total, (uint32_t)inH, (uint32_t)inW,
                         (uint32_t)oH, (uint32_t)oW, (uint32_t)sH, (uint32_t)sW, g.stream));
}

static bool h_upsample_backward(const Disp& d) {              // nn_upsample_backward.hlsl:15-45
  if (!need(d, 1, 1)) return false;
  const uint64_t B = d.u[0], C = d.u[1], inH = d.u[2], inW = d.u[3], oH = d.u[4], oW = d.u[5], sH = d.u[6],
                 sW = d.u[7];
  const uint64_t total = B * C * inH * inW;
  if (!idx32(d, total, "the input gradient") || !idx32(d, B * C * oH * oW, "the output gradient") ||
      !idx32(d, inH * sH, "inH * scaleH") || !idx32(d, inW * sW, "inW * scaleW"))
    return false;
  const uint64_t n = lim(total, d.gx);
  if (n == 0) return true;
  FITS(d.uav[0], n, "DX");
  if (sH && sW) FITS(d.srv[0], ((n - 1) / (inH * inW) + 1) * oH * oW, "DY");   // reads stay in their plane
  LAUNCH(launch_upsample_backward(d.srv[0]->d, d.uav[0]->d, (uint32_t)n, (uint32_t)total, (uint32_t)inH,
                                  (uint32_t)inW, (uint32_t)oH, (uint32_t)oW, (uint32_t)sH, (uint32_t)sW, g.stream));
}

// nn_concat_insert.hlsl:12-27 (slice = false) and nn_slice.hlsl:12-27 (slice = true)
static bool channel_copy(const Disp& d, bool slice) {
  if (!need(d, 1, 1)) return false;
  const uint64_t B = d.u[0], c_in = d.u[1], S = d.u[2], c_out = d.u[3], c_off = d.u[4];
  const uint64_t L = c_in * S, total = B * L, pitch = c_out * S, off = c_off * S;
  if (!idx32(d, total, "the copied block") || !idx32(d, pitch, "c_out * spatial") ||
      !idx32(d, off, "c_offset * spatial"))
    return false;
  const uint64_t n = lim(total, d.gx);
  if (n == 0) return true;
  // largest strided index over [0, n): the last element and the end of the row before it
  const uint64_t q = (n - 1) / L, r = (n - 1) - q * L;
  uint64_t hi = q * pitch + off + r;
  if (q > 0) hi = std::max(hi, (q - 1) * pitch + off + L - 1);
  if (!idx32(d, hi + 1, "the strided tensor")) return false;
  if (slice) { FITS(d.srv[0], hi + 1, "DY"); FITS(d.uav[0], n, "DX"); }
  else { FITS(d.srv[0], n, "X"); FITS(d.uav[0], hi + 1, "Out"); }
  LAUNCH(launch_channel_copy(slice, d.srv[0]->d, d.uav[0]->d, (uint32_t)n, (uint32_t)L, (uint32_t)pitch,
                             (uint32_t)off, g.stream));
}
static bool h_concat_insert(const Disp& d) { return channel_copy(d, false); }
static bool h_slice(const Disp& d) { return channel_copy(d, true); }

// outputs the 16x16-thread groups reach: ow < lw, oh < lh, bc < lb
struct PoolCover {
  uint64_t lw, lh, lb, last;                                  // last = largest output index + 1
};
static PoolCover pool_cover(const Disp& d, uint64_t bc, uint64_t oH, uint64_t oW) {
  PoolCover c;
  c.lw = std::min<uint64_t>(oW, (uint64_t)d.gx * 16);
  c.lh = std::min<uint64_t>(oH, (uint64_t)d.gy * 16);
  c.lb = std::min<uint64_t>(bc, d.gz);
  c.last = (c.lw && c.lh && c.lb) ? (c.lb - 1) * oH * oW + (c.lh - 1) * oW + c.lw : 0;
  return c;
}

static bool h_maxpool_forward(const Disp& d) {                // nn_maxpool_forward.hlsl:16-52
  if (!need(d, 1, 2)) return false;
  const uint64_t B = d.u[0], C = d.u[1], inH = d.u[2], inW = d.u[3], p = d.u[4], s = d.u[5], oH = d.u[6],
                 oW = d.u[7];
  if (!idx32(d, B * C * oH * oW, "the output") || !idx32(d, B * C * inH * inW, "the input")) return false;
  const PoolCover c = pool_cover(d, B * C, oH, oW);
  if (c.last == 0) return true;
  if (!idx32(d, (c.lh - 1) * s + p, "the window rows") || !idx32(d, (c.lw - 1) * s + p, "the window columns"))
    return false;
  FITS(d.uav[0], c.last, "output"); FITS(d.uav[1], c.last, "indices");
  if (p && inH && inW) {
    const uint64_t hi = (c.lb - 1) * inH * inW + std::min(inH - 1, (c.lh - 1) * s + p - 1) * inW +
                        std::min(inW - 1, (c.lw - 1) * s + p - 1);
    FITS(d.srv[0], hi + 1, "input");
  }
  const PoolShape gs{(uint32_t)(B * C), (uint32_t)inH, (uint32_t)inW, (uint32_t)p, (uint32_t)s, (uint32_t)oH,
                     (uint32_t)oW};
  LAUNCH(launch_maxpool_forward(d.srv[0]->d, d.uav[0]->d, reinterpret_cast<uint32_t*>(d.uav[1]->d), (uint32_t)c.lw,
                                (uint32_t)c.lh, (uint32_t)c.lb, gs, g.stream));
}

static bool h_maxpool_backward(const Disp& d) {               // nn_maxpool_backward.hlsl:12-25
  if (!need(d, 2, 1)) return false;
  const uint64_t B = d.u[0], C = d.u[1], oH = d.u[2], oW = d.u[3];
  if (!idx32(d, B * C * oH * oW, "the output gradient")) return false;
  const PoolCover c = pool_cover(d, B * C, oH, oW);
  if (c.last == 0) return true;
  FITS(d.srv[0], c.last, "dZ"); FITS(d.srv[1], c.last, "indices");
  LAUNCH(launch_maxpool_scatter(d.srv[0]->d, reinterpret_cast<const uint32_t*>(d.srv[1]->d), d.uav[0]->d,
                                d.uav[0]->count, (uint32_t)c.lw, (uint32_t)c.lh, (uint32_t)c.lb, (uint32_t)oH,
                                (uint32_t)oW, g.stream));
}

// Largest [b][oc][pixel] index over columns bp < lbp of row oc = loc - 1 (the
// last column and the end of the image before it).
static uint64_t nchw_hi(uint64_t lbp, uint64_t loc, uint64_t OC, uint64_t P) {
  auto at = [&](uint64_t bp) { return (bp / P) * OC * P + (loc - 1) * P + bp % P; };
  uint64_t hi = at(lbp - 1);
  if (lbp - 1 >= P) hi = std::max(hi, at(((lbp - 1) / P) * P - 1));
  return hi;
}

static bool h_conv_reshape(const Disp& d) {                   // nn_conv_reshape.hlsl:13-30
  if (!need(d, 2, 1)) return false;
  const uint64_t B = d.u[0], OC = d.u[1], P = (uint64_t)d.u[2] * d.u[3], BP = B * P;
  if (!idx32(d, OC * BP, "the output")) return false;
  const uint64_t lbp = std::min<uint64_t>(BP, (uint64_t)d.gx * 16), loc = std::min<uint64_t>(OC, (uint64_t)d.gy * 16);
  if (lbp == 0 || loc == 0) return true;
  FITS(d.srv[0], (loc - 1) * BP + lbp, "matmul_res"); FITS(d.srv[1], loc, "bias");
  FITS(d.uav[0], nchw_hi(lbp, loc, OC, P) + 1, "output");
  LAUNCH(launch_conv_reshape(d.srv[0]->d, d.srv[1]->d, d.uav[0]->d, (uint32_t)B, (uint32_t)OC, (uint32_t)P,
                             (uint32_t)lbp, (uint32_t)loc, d.u[4], g.stream));
}

// nn_conv_grad_reshape.hlsl:16-28 / nn_conv_grad_reshape_relu.hlsl:21-39: the
// cbuffer's fifth word (`ks`) carries outC, words 8 and 9 outH and outW
static bool conv_grad_reshape(const Disp& d, bool relu) {
  if (!need(d, relu ? 2 : 1, 1)) return false;
  const uint64_t B = d.u[0], OC = d.u[4], P = (uint64_t)d.u[7] * d.u[8], BP = B * P;
  if (!idx32(d, OC * BP, "the gradient")) return false;
  const uint64_t lbp = std::min<uint64_t>(BP, (uint64_t)d.gx * 16), loc = std::min<uint64_t>(OC, (uint64_t)d.gy * 16);
  if (lbp == 0 || loc == 0) return true;
  const uint64_t hi = nchw_hi(lbp, loc, OC, P) + 1;
  FITS(d.srv[0], hi, "dZ");
  if (relu) FITS(d.srv[1], hi, "fwd_output");
  FITS(d.uav[0], (loc - 1) * BP + lbp, "output");
  LAUNCH(launch_conv_grad_reshape(d.srv[0]->d, relu ? d.srv[1]->d : nullptr, d.uav[0]->d, (uint32_t)B, (uint32_t)OC,
                                  (uint32_t)P, (uint32_t)lbp, (uint32_t)loc, g.stream));
}
static bool h_conv_grad_reshape(const Disp& d) { return conv_grad_reshape(d, false); }
static bool h_conv_grad_reshape_relu(const Disp& d) { return conv_grad_reshape(d, true); }

// ---- softmax / CE -------------------------------------------------------------
static bool run_softmax_ce(const Disp& d, SoftmaxCEArgs a) {
  a.err = g.dev_err_dev;
  const size_t ws = softmax_ce_ws_bytes(a.rows, a.K);
  if (!ensure_ws(ws)) return false;
  LAUNCH(launch_softmax_ce(a, g.ws, g.stream));
}

static bool h_softmax(const Disp& d) {                        // nn_softmax.hlsl:5-13 (16 rows / group)
  if (!need(d, 1, 1)) return false;
  const uint32_t K = d.u[1];
  const uint32_t rows = (uint32_t)std::min<uint64_t>(d.u[0], (uint64_t)d.gx * 16);
  FITS(d.srv[0], (uint64_t)rows * K, "input"); FITS(d.uav[0], (uint64_t)rows * K, "output");
  SoftmaxCEArgs a;
  a.logits = d.srv[0]->d; a.rows = rows; a.K = K; a.probs = d.uav[0]->d; a.ref_max_init = true;
  return run_softmax_ce(d, a);
}

static bool h_loss(const Disp& d) {                           // nn_loss.hlsl:11-43
  if (!need(d, 2, 1)) return false;
  const uint32_t B = d.u[0], K = d.u[1];
  FITS(d.srv[0], (uint64_t)B * K, "logits"); FITS(d.srv[1], B, "labels"); FITS(d.uav[0], 1, "loss");
  SoftmaxCEArgs a;
  a.logits = d.srv[0]->d; a.labels = d.srv[1]->d; a.rows = B; a.K = K;
  a.loss = d.uav[0]->d; a.loss_div = (double)(float)B; a.ref_max_init = true;
  return run_softmax_ce(d, a);
}

static bool h_softmax_ce_grad(const Disp& d) {                // nn_softmax_ce_grad.hlsl:6-11 (16x16 groups)
  if (!need(d, 2, 1)) return false;
  const uint32_t B = d.u[0], K = d.u[1];
  const uint32_t cols = (uint32_t)std::min<uint64_t>(K, (uint64_t)d.gx * 16);
  const uint32_t rows = (uint32_t)std::min<uint64_t>(B, (uint64_t)d.gy * 16);
  FITS(d.srv[0], (uint64_t)B * K, "softmax_out"); FITS(d.srv[1], rows, "labels");
  FITS(d.uav[0], (uint64_t)B * K, "grad_in");
  LAUNCH(launch_softmax_ce_grad(d.srv[0]->d, d.srv[1]->d, d.uav[0]->d, B, K, rows, cols, g.stream));
}

static bool h_argmax_correct(const Disp& d) {                 // nn_argmax_correct.hlsl:10-26
  if (!need(d, 2, 1)) return false;
  const uint32_t K = d.u[1];
  const uint32_t rows = (uint32_t)lim(d.u[0], d.gx);
  FITS(d.srv[0], (uint64_t)rows * K, "logits"); FITS(d.srv[1], rows, "labels");
  LAUNCH(launch_argmax_correct(d.srv[0]->d, d.srv[1]->d, rows, K, reinterpret_cast<uint32_t*>(d.uav[0]->d), g.stream));
}

// ---- optimizers ----------------------------------------------------------------
static bool h_sgd(const Disp& d) {                            // nn_sgd.hlsl:5-11
  if (!need(d, 1, 1)) return false;
  const uint64_t n = lim(d.u[0], d.gx);
  FITS(d.srv[0], n, "grad"); FITS(d.uav[0], n, "weight");
  LAUNCH(launch_sgd(d.uav[0]->d, d.srv[0]->d, n, f_of(d.u[1]), f_of(d.u[2]), g.stream));
}

static bool h_sgd_clipped(const Disp& d) {                    // nn_sgd_clipped.hlsl:15-20
  if (!need(d, 2, 1)) return false;
  const uint64_t n = lim(d.u[0], d.gx);
  FITS(d.srv[0], n, "grad"); FITS(d.srv[1], 2, "normScale"); FITS(d.uav[0], n, "weight");
  LAUNCH(launch_sgd_clipped(d.uav[0]->d, d.srv[0]->d, n, f_of(d.u[1]), d.srv[1]->d, g.stream));
}

static bool h_adam(const Disp& d) {                           // nn_adam.hlsl:18-34
  if (!need(d, 1, 3)) return false;
  const uint64_t n = lim(d.u[0], d.gx);
  FITS(d.srv[0], n, "grad"); FITS(d.uav[0], n, "weight"); FITS(d.uav[1], n, "m"); FITS(d.uav[2], n, "v");
  AdamParams p{f_of(d.u[1]), f_of(d.u[2]), f_of(d.u[3]), f_of(d.u[4]), f_of(d.u[5]), f_of(d.u[6])};
  LAUNCH(launch_adam(d.uav[0]->d, d.uav[1]->d, d.uav[2]->d, d.srv[0]->d, n, p, g.stream));
}

// ---- batchnorm -------------------------------------------------------------------
static bool bn_stats(const Disp& d, const float* x, uint32_t N, uint32_t C, uint32_t S, float* mean, float* var,
                     float* rm, float* rv, bool training, float momentum, uint32_t c_eff);

static bool h_bn_mean_var(const Disp& d) {                    // nn_batchnorm_mean_var.hlsl:19-60
  if (!need(d, 1, 4)) return false;
  const uint32_t N = d.u[0], C = d.u[1], S = d.u[2];
  const bool training = d.u[3] == 1;
  const uint32_t c_eff = std::min<uint32_t>(C, d.gx);
  FITS(d.srv[0], (uint64_t)N * C * S, "x");
  for (int i = 0; i < 4; ++i) FITS(d.uav[i], c_eff, "stats");
  return bn_stats(d, d.srv[0]->d, N, C, S, d.uav[0]->d, d.uav[1]->d, d.uav[2]->d, d.uav[3]->d, training,
                  f_of(d.u[4]), c_eff);
}

static bool h_bn_forward(const Disp& d) {                     // nn_batchnorm_forward.hlsl:18-34
  if (!need(d, 5, 1)) return false;
  const uint32_t N = d.u[0], C = d.u[1], S = d.u[2];
  const uint64_t total = (uint64_t)N * C * S, n = lim(total, d.gx);
  FITS(d.srv[0], n, "x"); FITS(d.uav[0], n, "y");
  for (int i = 1; i < 5; ++i) FITS(d.srv[i], C, "per-channel");
  LAUNCH(launch_bn_forward(d.srv[0]->d, d.srv[1]->d, d.srv[2]->d, d.srv[3]->d, d.srv[4]->d, d.uav[0]->d, N, C, S,
                           f_of(d.u[3]), n, g.stream));
}

static bool h_bn_backward_reduce(const Disp& d) {             // nn_batchnorm_backward_reduce.hlsl:21-60
  if (!need(d, 4, 2)) return false;
  const uint32_t N = d.u[0], C = d.u[1], S = d.u[2];
  const uint32_t c_eff = std::min<uint32_t>(C, d.gx);
  FITS(d.srv[0], (uint64_t)N * C * S, "x"); FITS(d.srv[1], (uint64_t)N * C * S, "dy");
  FITS(d.srv[2], C, "mean"); FITS(d.srv[3], C, "var"); FITS(d.uav[0], c_eff, "dgamma"); FITS(d.uav[1], c_eff, "dbeta");
  if (!ensure_ws(bn_ws_bytes(N, C))) return false;
  double* ps = (double*)g.ws;
  double* chan = ps + (size_t)N * C * 2;
  cudaError_t e = launch_bn_plane_sums(d.srv[0]->d, d.srv[1]->d, N, C, S, ps, g.stream);
  if (e == cudaSuccess) e = launch_bn_fold(ps, N, C, chan, g.stream);
  if (e == cudaSuccess)
    e = launch_bn_bwd_final(chan, c_eff, d.srv[2]->d, d.srv[3]->d, f_of(d.u[3]), d.uav[0]->d, d.uav[1]->d, g.stream);
  LAUNCH(e);
}

static bool h_bn_backward_dx(const Disp& d) {                 // nn_batchnorm_backward_dx.hlsl:20-38
  if (!need(d, 7, 1)) return false;
  const uint32_t N = d.u[0], C = d.u[1], S = d.u[2];
  const uint64_t total = (uint64_t)N * C * S, n = lim(total, d.gx);
  FITS(d.srv[0], n, "x"); FITS(d.srv[1], n, "dy"); FITS(d.uav[0], n, "dx");
  for (int i = 2; i < 7; ++i) FITS(d.srv[i], C, "per-channel");
  LAUNCH(launch_bn_backward_dx(d.srv[0]->d, d.srv[1]->d, d.srv[2]->d, d.srv[3]->d, d.srv[4]->d, d.srv[5]->d,
                               d.srv[6]->d, d.uav[0]->d, N, C, S, f_of(d.u[3]), n, g.stream));
}

// ---- extension kernels (new names, same RunShader signature) ---------------------
// dct_unary      cb {op, count, alpha_bits}         t0 x        u0 y
// dct_binary     cb {op, ndim, a_mask, b_mask, shape[ndim]} (ndim <= 8; a mask bit d = the
//                operand has extent 1 along output dim d)  t0 a, t1 b  u0 out
// dct_reduce     cb {op, outer, len, inner}          t0 x        u0 out [, u1 int32 idx]
// dct_reduce_all cb {op, count}                      t0 x        u0 out[1]
// dct_softmax_ce cb {rows, K, flags, loss_div_bits, grad_div_bits}  t0 logits, t1 labels
//                u0 probs, u1 dlogits, u2 loss[1], u3 logprobs (any may be null);
//                flags bit0: labels are int32
static bool binary_from_masks(const Disp& d, int op, uint32_t ndim, uint32_t am, uint32_t bm, const uint32_t* shp,
                              const Buffer* A, const Buffer* B, Buffer* O);

static bool h_dct_unary(const Disp& d) {
  if (!need(d, 1, 1)) return false;
  const uint64_t n = d.u[1];
  FITS(d.srv[0], n, "x"); FITS(d.uav[0], n, "y");
  LAUNCH(launch_unary((int)d.u[0], d.srv[0]->d, d.uav[0]->d, n, f_of(d.u[2]), g.stream));
}

static bool h_dct_binary(const Disp& d) {
  if (!need(d, 2, 1)) return false;
  const uint32_t ndim = d.u[1];
  if (ndim > 8) { set_error(DCT_ERR_ARG, "dct_binary: ndim %u > 8", ndim); return false; }
  return binary_from_masks(d, (int)d.u[0], ndim, d.u[2], d.u[3], &d.u[4], d.srv[0], d.srv[1], d.uav[0]);
}

static bool h_dct_reduce(const Disp& d) {
  if (!need(d, 1, 1)) return false;
  const int op = (int)d.u[0];
  const uint64_t outer = d.u[1], len = d.u[2], inner = d.u[3];
  FITS(d.srv[0], outer * len * inner, "x"); FITS(d.uav[0], outer * inner, "out");
  int32_t* idx = nullptr;
  if (d.nuav > 1 && d.uav[1]) { FITS(d.uav[1], outer * inner, "idx"); idx = reinterpret_cast<int32_t*>(d.uav[1]->d); }
  float* out = d.uav[0]->d;
  if (len == 0 && outer * inner > 0) {
    // NumPy: the sum over an empty axis is 0 and the mean NaN; the extremes and
    // their indices have no identity (NumPy raises)
    if (op == RED_SUM || op == RED_MEAN)
      return cuda_ok(cudaMemsetAsync(out, op == RED_SUM ? 0 : 0xFF, outer * inner * sizeof(float), g.stream),
                     "dct_reduce(empty axis)");
    set_error(DCT_ERR_ARG, "dct_reduce: op %d over a zero-length axis has no identity", op);
    return false;
  }
  int op_run = op;
  if (op == RED_ARGMAX || op == RED_ARGMIN) {
    // the index is the product; values are not requested
    if (!idx) { idx = reinterpret_cast<int32_t*>(out); out = nullptr; }
  } else if ((op == RED_MAX || op == RED_MIN) && idx) {
    op_run = op == RED_MAX ? RED_ARGMAX : RED_ARGMIN;       // values and indices in one pass
  }
  if (len > 0x7fffffffull && (op == RED_ARGMAX || op == RED_ARGMIN)) {
    set_error(DCT_ERR_ARG, "dct_reduce: arg reductions need len < 2^31");
    return false;
  }
  const size_t ws = reduce3d_ws_bytes(op, outer, len, inner);
  if (ws && !ensure_ws(ws)) return false;
  LAUNCH(launch_reduce3d(op_run, d.srv[0]->d, outer, len, inner, out, idx, g.ws, g.stream));
}

static bool h_dct_reduce_all(const Disp& d) {
  if (!need(d, 1, 1)) return false;
  const uint64_t n = d.u[1];
  FITS(d.srv[0], n, "x"); FITS(d.uav[0], 1, "out");
  if (n == 0 && (d.u[0] == RED_MAX || d.u[0] == RED_MIN)) {
    set_error(DCT_ERR_ARG, "dct_reduce_all: max/min of an empty vector has no identity");
    return false;
  }
  if (!ensure_ws(full_reduce_ws_bytes())) return false;
  LAUNCH(launch_full_reduce((int)d.u[0], d.srv[0]->d, n, d.uav[0]->d, nullptr, g.ws, g.stream));
}

static bool h_dct_softmax_ce(const Disp& d) {
  if (d.nsrv < 1 || !d.srv[0]) { set_error(DCT_ERR_ARG, "dct_softmax_ce: logits missing"); return false; }
  const uint32_t rows = d.u[0], K = d.u[1];
  FITS(d.srv[0], (uint64_t)rows * K, "logits");
  SoftmaxCEArgs a;
  a.logits = d.srv[0]->d;
  a.rows = rows; a.K = K;
  if (d.nsrv > 1 && d.srv[1]) { FITS(d.srv[1], rows, "labels"); a.labels = d.srv[1]->d; }
  a.labels_int32 = (d.u[2] & 1u) != 0;
  Buffer* o[4] = {nullptr, nullptr, nullptr, nullptr};
  for (uint32_t i = 0; i < 4 && i < d.nuav; ++i) o[i] = d.uav[i];
  if (o[0]) { FITS(o[0], (uint64_t)rows * K, "probs"); a.probs = o[0]->d; }
  if (o[1]) { FITS(o[1], (uint64_t)rows * K, "dlogits"); a.dlogits = o[1]->d; }
  if (o[2]) { FITS(o[2], 1, "loss"); a.loss = o[2]->d; }
  if (o[3]) { FITS(o[3], (uint64_t)rows * K, "logprobs"); a.logprobs = o[3]->d; }
  a.loss_div = d.u[3] ? (double)f_of(d.u[3]) : (double)rows;
  a.grad_div = d.u[4] ? f_of(d.u[4]) : (float)rows;
  if ((a.dlogits || a.loss) && !a.labels) { set_error(DCT_ERR_ARG, "dct_softmax_ce: labels required"); return false; }
  return run_softmax_ce(d, a);
}

static Shader g_shaders[] = {
    {"add_bias", h_add_bias, false, false, kShaderMagic},
    {"bias_relu", h_bias_relu, false, false, kShaderMagic},
    {"relu", h_relu, false, false, kShaderMagic},
    {"relu_grad", h_relu_grad, false, false, kShaderMagic},
    {"relu6", h_relu6, false, false, kShaderMagic},
    {"relu6_grad", h_relu6_grad, false, false, kShaderMagic},
    {"leaky_relu", h_leaky_relu, false, false, kShaderMagic},
    {"leaky_relu_grad", h_leaky_relu_grad, false, false, kShaderMagic},
    {"sigmoid", h_sigmoid, false, false, kShaderMagic},
    {"sigmoid_grad", h_sigmoid_grad, false, false, kShaderMagic},
    {"add", h_add, false, false, kShaderMagic},
    {"scale_add", h_scale_add, false, false, kShaderMagic},
    {"grad_accum", h_grad_accum, false, false, kShaderMagic},
    {"bias_grad", h_bias_grad, false, false, kShaderMagic},
    {"global_avg_pool", h_gap, false, false, kShaderMagic},
    {"global_avg_pool_backward", h_gap_backward, false, false, kShaderMagic},
    {"softmax", h_softmax, false, false, kShaderMagic},
    {"loss", h_loss, false, false, kShaderMagic},
    {"softmax_ce_grad", h_softmax_ce_grad, false, false, kShaderMagic},
    {"argmax_correct", h_argmax_correct, false, false, kShaderMagic},
    {"accumulate_scalar", h_accumulate_scalar, false, false, kShaderMagic},
    {"rms", h_rms, false, false, kShaderMagic},
    {"grad_sq_reduce", h_grad_sq_reduce, false, false, kShaderMagic},
    {"grad_norm_final", h_grad_norm_final, false, false, kShaderMagic},
    {"sgd", h_sgd, false, false, kShaderMagic},
    {"sgd_clipped", h_sgd_clipped, false, false, kShaderMagic},
    {"adam", h_adam, false, false, kShaderMagic},
    {"batchnorm_mean_var", h_bn_mean_var, false, false, kShaderMagic},
    {"batchnorm_forward", h_bn_forward, false, false, kShaderMagic},
    {"batchnorm_backward_reduce", h_bn_backward_reduce, false, false, kShaderMagic},
    {"batchnorm_backward_dx", h_bn_backward_dx, false, false, kShaderMagic},
    {"dice_loss", h_dice_loss, false, false, kShaderMagic},
    {"dice_loss_sums", h_dice_loss_sums, false, false, kShaderMagic},
    {"dice_loss_grad", h_dice_loss_grad, false, false, kShaderMagic},
    {"upsample", h_upsample, false, false, kShaderMagic},
    {"upsample_backward", h_upsample_backward, false, false, kShaderMagic},
    {"concat_insert", h_concat_insert, false, false, kShaderMagic},
    {"slice", h_slice, false, false, kShaderMagic},
    {"maxpool_forward", h_maxpool_forward, false, false, kShaderMagic},
    {"maxpool_backward", h_maxpool_backward, false, false, kShaderMagic},
    {"conv_reshape", h_conv_reshape, false, false, kShaderMagic},
    {"conv_grad_reshape", h_conv_grad_reshape, false, false, kShaderMagic},
    {"conv_grad_reshape_relu", h_conv_grad_reshape_relu, false, false, kShaderMagic},
    {"dct_unary", h_dct_unary, true, false, kShaderMagic},
    {"dct_binary", h_dct_binary, true, false, kShaderMagic},
    {"dct_reduce", h_dct_reduce, true, false, kShaderMagic},
    {"dct_reduce_all", h_dct_reduce_all, true, false, kShaderMagic},
    {"dct_softmax_ce", h_dct_softmax_ce, true, false, kShaderMagic},
};
constexpr int kNumShaders = sizeof(g_shaders) / sizeof(g_shaders[0]);

static Shader* find_shader(const char* name) {
  if (!name) return nullptr;
  for (int i = 0; i < kNumShaders; ++i)
    if (strcmp(g_shaders[i].name, name) == 0) return &g_shaders[i];
  return nullptr;
}

static bool is_shader_ptr(const void* p) {
  const Shader* s = static_cast<const Shader*>(p);
  return s >= g_shaders && s < g_shaders + kNumShaders && s->magic == kShaderMagic;
}

static bool make_disp(Disp& d, Shader* s, void** srvs, uint32_t nsrv, void** uavs, uint32_t nuav,
                      const uint32_t* groups, const void* cb, uint32_t cbsize) {
  memset(&d, 0, sizeof(d));
  d.name = s->name;
  if (nsrv > 16 || nuav > 16) { set_error(DCT_ERR_ARG, "%s: too many views", s->name); return false; }
  d.nsrv = nsrv;
  d.nuav = nuav;
  for (uint32_t i = 0; i < nsrv; ++i) {
    d.srv[i] = srvs ? buf_of(srvs[i]) : nullptr;
    if (srvs && srvs[i] && !d.srv[i]) { set_error(DCT_ERR_HANDLE, "%s: SRV t%u %p is not a live buffer", s->name, i, srvs[i]); return false; }
  }
  for (uint32_t i = 0; i < nuav; ++i) {
    d.uav[i] = uavs ? buf_of(uavs[i]) : nullptr;
    if (uavs && uavs[i] && !d.uav[i]) { set_error(DCT_ERR_HANDLE, "%s: UAV u%u %p is not a live buffer", s->name, i, uavs[i]); return false; }
  }
  d.gx = groups ? groups[0] : 1;
  d.gy = groups ? groups[1] : 1;
  d.gz = groups ? groups[2] : 1;
  d.cbsize = cbsize;
  if (cb && cbsize) memcpy(d.u, cb, std::min<uint32_t>(cbsize, sizeof(d.u)));
  return true;
}

static bool dispatch(Shader* s, void** srvs, uint32_t nsrv, void** uavs, uint32_t nuav, const uint32_t* groups,
                     const void* cb, uint32_t cbsize) {
  if (!ensure_init()) return false;
  Disp d;
  if (!make_disp(d, s, srvs, nsrv, uavs, nuav, groups, cb, cbsize)) return false;
  return s->fn(d);
}

// Peepholes of RunSequence: an elementwise dispatch over a [B, K] row-major
// matrix directly followed by bias_grad over its output (column sums, row
// stride K) runs as one pass that writes the matrix and its column sums, with
// the same results as the dispatches (the column kernel keeps bias_grad's
// plan).  Each returns false, launching nothing, when the commands do not have
// that form.

// bias_grad (b) over the whole [B, K] matrix a just wrote to a.uav[0] (n floats).
static bool colsum_of(const Disp& a, const Disp& b, uint64_t n, uint64_t& B, uint64_t& K) {
  if (strcmp(b.name, "bias_grad") != 0 || b.nsrv < 1 || b.nuav < 1 || !b.srv[0] || !b.uav[0]) return false;
  if (!a.uav[0] || b.srv[0] != a.uav[0]) return false;             // bias_grad reads what a just wrote
  B = b.u[0];
  K = std::min<uint64_t>(b.u[1], b.gx);
  return K > 0 && B > 0 && b.u[3] == 1 && b.u[2] == K && B * K == n && b.uav[0]->count >= K;
}

// grad_accum (c) adding exactly the K column sums in db to its accumulator.
static Buffer* accum_of(const Disp* c, const Buffer* db, uint64_t K) {
  if (!c || strcmp(c->name, "grad_accum") != 0 || c->nsrv < 1 || c->nuav < 1) return nullptr;
  if (c->srv[0] != db || !c->uav[0] || c->uav[0] == db) return nullptr;
  if (lim(c->u[0], c->gx) != K || c->uav[0]->count < K) return nullptr;
  return c->uav[0];
}

// relu_grad (grad, y -> dx), then bias_grad over dx (the backward of bias +
// ReLU, nn_engine.py:1091-1106), and when c is grad_accum over those column
// sums, that too (*used = 3).
static bool try_fused_relu_bias_grad(const Disp& a, const Disp& b, const Disp* c, bool& ok, int* used) {
  if (strcmp(a.name, "relu_grad") != 0 || a.nsrv < 2 || a.nuav < 1) return false;
  if (!a.srv[0] || !a.srv[1] || !a.uav[0]) return false;
  const uint64_t n = lim(a.u[0], a.gx);
  uint64_t B, K;
  if (!colsum_of(a, b, n, B, K)) return false;
  Buffer *bg = a.srv[0], *by = a.srv[1], *bdx = a.uav[0], *bdb = b.uav[0];
  if (bdb == bg || bdb == by || bdb == bdx) return false;
  if (bg->count < n || by->count < n || bdx->count < n) return false;
  Buffer* acc = accum_of(c, bdb, K);
  if (acc && (acc == bg || acc == by || acc == bdx)) acc = nullptr;
  const size_t ws = relu_grad_colsum_ws_bytes(B, K);
  *used = acc ? 3 : 2;
  if (ws && !ensure_ws(ws)) { ok = false; return true; }
  ok = cuda_ok(launch_relu_grad_colsum(bg->d, by->d, bdx->d, bdb->d, B, K, g.ws, g.ws_bytes, g.stream,
                                       acc ? acc->d : nullptr),
               "relu_grad + bias_grad");
  return true;
}

// bias_relu (x, b -> y) over whole rows, then bias_grad over y (column sums of
// the layer's output, the C1 forward).
static bool try_fused_bias_relu_colsum(const Disp& a, const Disp& b, bool& ok, int* used) {
  if (strcmp(a.name, "bias_relu") != 0 || a.nsrv < 2 || a.nuav < 1) return false;
  if (!a.srv[0] || !a.srv[1] || !a.uav[0]) return false;
  const uint64_t M = a.u[0], N = a.u[1];
  const uint64_t n = lim(M * N, a.gx);
  uint64_t B, K;
  if (N == 0 || n != M * N || !colsum_of(a, b, n, B, K) || B != M || K != N) return false;
  Buffer *bx = a.srv[0], *bb = a.srv[1], *by = a.uav[0], *bc = b.uav[0];
  if (bc == bx || bc == bb || bc == by || by == bb) return false;
  if (bx->count < n || by->count < n || bb->count < N) return false;
  const size_t ws = relu_grad_colsum_ws_bytes(B, K);
  *used = 2;
  if (ws && !ensure_ws(ws)) { ok = false; return true; }
  ok = cuda_ok(launch_bias_relu_colsum(bx->d, bb->d, by->d, bc->d, B, K, g.ws, g.ws_bytes, g.stream),
               "bias_relu + bias_grad");
  return true;
}

// ---------------------------------------------------------------------------
// BatchNorm statistics (shared by the reference name and dct_batchnorm_*)
// ---------------------------------------------------------------------------
static bool bn_stats(const Disp& d, const float* x, uint32_t N, uint32_t C, uint32_t S, float* mean, float* var,
                     float* rm, float* rv, bool training, float momentum, uint32_t c_eff) {
  if (!ensure_ws(bn_ws_bytes(N, C))) return false;
  double* ps = (double*)g.ws;
  double* chan = ps + (size_t)N * C * 2;
  cudaError_t e = launch_bn_plane_sums(x, nullptr, N, C, S, ps, g.stream);
  if (e == cudaSuccess) e = launch_bn_fold(ps, N, C, chan, g.stream);
  if (e != cudaSuccess) LAUNCH(e);
  double cnt = (double)N * S;
  LAUNCH(launch_bn_stats_final(chan, c_eff, cnt, mean, var, rm, rv, training, momentum, g.stream));
}

// ---------------------------------------------------------------------------
// broadcast binary from output shape + operand masks
// ---------------------------------------------------------------------------
static bool binary_from_masks(const Disp& d, int op, uint32_t ndim, uint32_t am, uint32_t bm, const uint32_t* shp,
                              const Buffer* A, const Buffer* B, Buffer* O) {
  int64_t shape[8], as[8], bs[8];
  uint64_t n = 1, na = 1, nb = 1;
  for (uint32_t i = 0; i < ndim; ++i) {
    shape[i] = shp[i];
    n *= shp[i];
    if (!((am >> i) & 1u)) na *= shp[i];
    if (!((bm >> i) & 1u)) nb *= shp[i];
  }
  int64_t sa = 1, sb = 1;
  for (int i = (int)ndim - 1; i >= 0; --i) {
    const bool ab = (am >> i) & 1u, bb = (bm >> i) & 1u;
    as[i] = ab ? 0 : sa;
    bs[i] = bb ? 0 : sb;
    if (!ab) sa *= shape[i];
    if (!bb) sb *= shape[i];
  }
  if (n == 0) return true;
  FITS(A, na, "a"); FITS(B, nb, "b"); FITS(O, n, "out");
  LAUNCH(launch_binary_bcast(op, A->d, B->d, O->d, (int)ndim, shape, as, bs, g.stream));
}

}  // namespace dct

using namespace dct;

// ===========================================================================
// exported C-ABI
// ===========================================================================
extern "C" {

DCT_API bool InitEngine() {
  LOCK;
  return init_engine();
}

DCT_API void GetGPUInfo(DctGPUInfo* out) {
  LOCK;
  if (!out) return;
  memset(out, 0, sizeof(*out));
  if (!ensure_init()) return;
  out->vendorId = 0x10DE;
  out->deviceId = 0;
  out->dedicatedVRAM = g.info.total_mem;
  out->sharedMemory = 0;
  out->isIntegrated = 0;
  snprintf(out->description, sizeof(out->description), "%s", g.name);
}

DCT_API bool CompileShader(const char* name, const wchar_t* path) {
  LOCK;
  (void)path;
  Shader* s = find_shader(name);
  if (!s) return false;       // no CUDA kernel behind this name (outside the hot path)
  s->compiled = true;
  return true;
}

DCT_API bool CompileShaderEx(const char* name, const wchar_t* path, const char* entry) {
  LOCK;
  (void)path; (void)entry;
  set_error(DCT_ERR_UNSUPPORTED, "CompileShaderEx(%s): HLSL source cannot run on CUDA", name ? name : "");
  return false;
}

DCT_API void* CreateBuffer(float* data, uint32_t count) {
  LOCK;
  return create_buffer(data, count);
}

DCT_API void AddRefBuffer(void* h) {
  LOCK;
  Buffer* b = buf_of(h);
  if (b) b->ref++;
  else if (h) set_error(DCT_ERR_HANDLE, "AddRefBuffer: unknown handle %p", h);
}

DCT_API void UpdateBuffer(void* h, float* data) {
  LOCK;
  Buffer* b = buf_of(h);
  if (!b || !data) {
    if (h && !b) set_error(DCT_ERR_HANDLE, "UpdateBuffer: unknown handle %p", h);
    return;
  }
  cudaPointerAttributes at{};
  const bool pinned = cudaPointerGetAttributes(&at, data) == cudaSuccess && at.type == cudaMemoryTypeHost;
  cudaGetLastError();
  cuda_ok(cudaMemcpyAsync(b->d, data, b->count * sizeof(float), cudaMemcpyHostToDevice, g.stream), "UpdateBuffer");
  if (pinned) rt_wait_stream("UpdateBuffer");            // the caller may reuse its memory on return
}

DCT_API void ReleaseBuffer(void* h) {
  LOCK;
  if (h) release_handle(h);
}

DCT_API void ReleaseBufferBatch(void** hs, uint32_t count) {
  LOCK;
  if (!hs) return;
  for (uint32_t i = 0; i < count; ++i)
    if (hs[i]) release_handle(hs[i]);
}

DCT_API void ReadBuffer(void* h, float* dst) {
  LOCK;
  Buffer* b = buf_of(h);
  if (!b || !dst) {
    if (h && !b) set_error(DCT_ERR_HANDLE, "ReadBuffer: unknown handle %p", h);
    return;
  }
  cuda_ok(cudaMemcpyAsync(dst, b->d, b->count * sizeof(float), cudaMemcpyDeviceToHost, g.stream), "ReadBuffer");
  rt_wait_stream("ReadBuffer");
}

DCT_API void ClearBuffer(void* h) {
  LOCK;
  Buffer* b = buf_of(h);
  if (!b) return;
  cuda_ok(cudaMemsetAsync(b->d, 0, b->count * sizeof(float), g.stream), "ClearBuffer");
}

DCT_API void FlushGPU() {
  LOCK;
  if (g.init) cudaStreamQuery(g.stream);                 // submission only, never waits
}

DCT_API void SyncGPU() {
  LOCK;
  if (g.init) rt_wait_stream("SyncGPU");
}

DCT_API void RunShader(const char* name, void** srvs, uint32_t nsrv, void** uavs, uint32_t nuav, uint32_t* threads,
                       void* cb, uint32_t cbsize) {
  LOCK;
  Shader* s = find_shader(name);
  if (!s || !(s->compiled || s->always)) {
    set_error(DCT_ERR_UNKNOWN_SHADER, "RunShader: '%s' is not a compiled kernel", name ? name : "");
    return;                                              // engine.cpp:397-399: silent return
  }
  dispatch(s, srvs, nsrv, uavs, nuav, threads, cb, cbsize);
}

DCT_API void RunShaderRaw(const char* name, void** srvs, uint32_t nsrv, void** uavs, uint32_t nuav,
                          uint32_t* threads, void* cb, uint32_t cbsize) {
  RunShader(name, srvs, nsrv, uavs, nuav, threads, cb, cbsize);
}

DCT_API void* RunShaderAlloc(const char* name, void** srvs, uint32_t nsrv, uint32_t out_count, uint32_t* threads,
                             void* cb, uint32_t cbsize) {
  LOCK;
  void* out = create_buffer(nullptr, out_count);
  if (!out) return nullptr;
  void* uavs[1] = {out};
  RunShader(name, srvs, nsrv, uavs, 1, threads, cb, cbsize);
  return out;
}

DCT_API void* RunShaderAlloc2(const char* name, void** srvs, uint32_t nsrv, uint32_t out_count, void* extra,
                              uint32_t* threads, void* cb, uint32_t cbsize) {
  LOCK;
  void* out = create_buffer(nullptr, out_count);
  if (!out) return nullptr;
  void* uavs[2] = {out, extra};
  RunShader(name, srvs, nsrv, uavs, 2, threads, cb, cbsize);
  return out;
}

// -- optimizers ---------------------------------------------------------------
static bool build_table(void** params, void** grads, uint32_t* sizes, uint32_t n, std::vector<MtTensor>& t,
                        bool need_params) {
  t.clear();
  for (uint32_t i = 0; i < n; ++i) {
    Buffer* w = params ? buf_of(params[i]) : nullptr;
    Buffer* gr = grads ? buf_of(grads[i]) : nullptr;
    if (!gr || (need_params && !w)) continue;            // engine.cpp:460 skips null pairs
    uint64_t cnt = sizes ? sizes[i] : gr->count;
    uint64_t cap = gr->count;
    if (w) cap = std::min(cap, w->count);
    if (cnt > cap) {
      set_error(DCT_ERR_SIZE, "optimizer: sizes[%u]=%llu exceeds the buffers (%llu)", i, (unsigned long long)cnt,
                (unsigned long long)cap);
      cnt = cap;
    }
    t.push_back(MtTensor{w ? w->d : nullptr, gr->d, nullptr, nullptr, cnt});
  }
  return true;
}

DCT_API void SGDBatch(void** params, void** grads, uint32_t* sizes, uint32_t n, float lr, float clip) {
  LOCK;
  if (!ensure_init() || n == 0) return;
  std::vector<MtTensor> t;
  build_table(params, grads, sizes, n, t, true);
  cuda_ok(launch_mt_sgd(t.data(), (int)t.size(), lr, clip, nullptr, g.stream), "SGDBatch");
}

DCT_API float SGDBatchClipped(void** params, void** grads, uint32_t* sizes, uint32_t n, float lr, float max_norm) {
  LOCK;
  if (!ensure_init() || n == 0) return 0.0f;
  std::vector<MtTensor> t;
  build_table(nullptr, grads, sizes, n, t, false);       // phase 1: every grad
  const uint64_t parts = mt_sumsq_blocks(t.data(), (int)t.size());
  if (!ensure_ws((parts + 8) * sizeof(double) + 64)) return 0.0f;
  double* part = (double*)g.ws;
  float* ns = (float*)((char*)g.ws + ((parts * sizeof(double) + 255) & ~size_t(255)));
  if (!cuda_ok(launch_mt_sumsq(t.data(), (int)t.size(), part, (int)parts, g.stream), "SGDBatchClipped(sumsq)")) return 0.0f;
  if (!cuda_ok(launch_norm_scale_from_parts(part, (int)parts, max_norm, ns, g.stream), "SGDBatchClipped(norm)")) return 0.0f;
  std::vector<MtTensor> t3;
  build_table(params, grads, sizes, n, t3, true);       // phase 3: param and grad present
  if (!cuda_ok(launch_mt_sgd(t3.data(), (int)t3.size(), lr, 0.0f, ns, g.stream), "SGDBatchClipped(sgd)")) return 0.0f;
  cuda_ok(cudaMemcpyAsync(g.host_small, ns, 2 * sizeof(float), cudaMemcpyDeviceToHost, g.stream), "SGDBatchClipped(D2H)");
  rt_wait_stream("SGDBatchClipped");
  return g.host_small[0];
}

// -- out-of-scope fused dense ops: exported so the reference binds --------------------
DCT_API void* MatMulAlloc(void*, void*, uint32_t, uint32_t, uint32_t, uint32_t) {
  LOCK;
  set_error(DCT_ERR_UNSUPPORTED, "MatMulAlloc: dense matmul is outside libdct_cuda's scope");
  return nullptr;
}
DCT_API void* ConvForwardFused(void*, void*, void*, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t,
                               uint32_t, uint32_t, uint32_t, uint32_t, void** pIm2col) {
  LOCK;
  if (pIm2col) *pIm2col = nullptr;
  set_error(DCT_ERR_UNSUPPORTED, "ConvForwardFused: convolution is outside libdct_cuda's scope");
  return nullptr;
}
DCT_API void ConvBackwardFused(void*, void*, void*, void*, void*, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t,
                               uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t,
                               void** pDF, void** pDB, void** pDI) {
  LOCK;
  if (pDF) *pDF = nullptr;
  if (pDB) *pDB = nullptr;
  if (pDI) *pDI = nullptr;
  set_error(DCT_ERR_UNSUPPORTED, "ConvBackwardFused: convolution is outside libdct_cuda's scope");
}

// -- max pooling (engine.cpp:880-929) ------------------------------------------------
// Forward: output and index buffers of batch*inC*outH*outW from the pool, the
// maxpool_forward kernel over every output, *pIndices = the index buffer.  The
// index buffer remembers the pooling geometry so that the backward pass can
// build dInput in one gather instead of a clear plus a scatter.
DCT_API void* MaxPoolForwardFused(void* x, uint32_t batch, uint32_t inC, uint32_t inH, uint32_t inW, uint32_t pool,
                                  uint32_t stride, void** pIndices) {
  LOCK;
  const char* W = "MaxPoolForwardFused";
  if (!ensure_init()) return nullptr;
  Buffer* bx = buf_of(x);
  if (!bx) { set_error(DCT_ERR_HANDLE, "%s: x is not a live buffer", W); return nullptr; }
  if (pool == 0 || stride == 0 || inH < pool || inW < pool) {
    set_error(DCT_ERR_ARG, "%s: pool %u / stride %u must be >= 1 and the pool must fit the %ux%u input", W, pool,
              stride, inH, inW);
    return nullptr;
  }
  const uint64_t bc = (uint64_t)batch * inC, outH = (inH - pool) / stride + 1, outW = (inW - pool) / stride + 1;
  const uint64_t nin = bc * inH * inW, nout = bc * outH * outW;
  if (nin > 0xFFFFFFFFull) { set_error(DCT_ERR_ARG, "%s: input past the 32-bit index space", W); return nullptr; }
  if (bx->count < nin) {
    set_error(DCT_ERR_SIZE, "%s: x holds %llu floats, the pooling reads %llu", W, (unsigned long long)bx->count,
              (unsigned long long)nin);
    return nullptr;
  }
  Buffer* out = create_buffer(nullptr, nout);
  if (!out) return nullptr;
  Buffer* idx = create_buffer(nullptr, nout);
  if (!idx) { release_internal(out); return nullptr; }
  const PoolShape gs{(uint32_t)bc, inH, inW, pool, stride, (uint32_t)outH, (uint32_t)outW};
  if (!cuda_ok(launch_maxpool_forward(bx->d, out->d, reinterpret_cast<uint32_t*>(idx->d), gs.outW, gs.outH, gs.bc, gs,
                                      g.stream), W)) {
    release_internal(out);
    release_internal(idx);
    return nullptr;
  }
  const uint32_t geom[7] = {gs.bc, gs.inH, gs.inW, gs.p, gs.s, gs.outH, gs.outW};
  memcpy(idx->pool_geom, geom, sizeof(geom));
  idx->has_pool_geom = true;
  if (pIndices) *pIndices = idx;
  else release_internal(idx);                    // nobody can reach it (the reference leaks it)
  return out;
}

// Backward: dInput of x_size floats = zeros plus dZ at each output's index,
// then the index buffer is released.  With the geometry recorded by the
// forward pass and windows that do not overlap, one gather kernel writes every
// element once; otherwise (or for an index buffer from elsewhere) the buffer
// is cleared and the outputs scattered, as the reference does.
DCT_API void* MaxPoolBackwardFused(void* grad_output, void* indices, uint32_t batch, uint32_t inC, uint32_t outH,
                                   uint32_t outW, uint32_t x_size) {
  LOCK;
  const char* W = "MaxPoolBackwardFused";
  if (!ensure_init()) return nullptr;
  Buffer* dx = create_buffer(nullptr, x_size);
  if (!dx) return nullptr;
  Buffer *bg = buf_of(grad_output), *bi = buf_of(indices);
  const uint64_t bc = (uint64_t)batch * inC, nout = bc * outH * outW;
  cudaError_t e = cudaSuccess;
  if (!bg || !bi) {
    set_error(DCT_ERR_HANDLE, "%s: grad_output or indices is not a live buffer", W);
    e = cudaMemsetAsync(dx->d, 0, (size_t)x_size * sizeof(float), g.stream);
  } else if (nout > 0xFFFFFFFFull || bg->count < nout || bi->count < nout) {
    set_error(DCT_ERR_SIZE, "%s: grad_output / indices hold fewer than batch*inC*outH*outW = %llu floats", W,
              (unsigned long long)nout);
    e = cudaMemsetAsync(dx->d, 0, (size_t)x_size * sizeof(float), g.stream);
  } else {
    const uint32_t* gm = bi->pool_geom;
    const PoolShape gs{gm[0], gm[1], gm[2], gm[3], gm[4], gm[5], gm[6]};
    const bool gather = bi->has_pool_geom && gs.bc == bc && gs.outH == outH && gs.outW == outW && gs.s >= gs.p &&
                        (uint64_t)gs.bc * gs.inH * gs.inW == x_size && device_flags() != nullptr;
    const uint32_t* ip = reinterpret_cast<const uint32_t*>(bi->d);
    if (gather) {
      e = launch_maxpool_backward_gather(bg->d, ip, dx->d, gs, device_flags(), g.stream);
    } else {
      e = cudaMemsetAsync(dx->d, 0, (size_t)x_size * sizeof(float), g.stream);
      if (e == cudaSuccess)
        e = launch_maxpool_scatter(bg->d, ip, dx->d, x_size, outW, outH, (uint32_t)bc, outH, outW, g.stream);
    }
  }
  cuda_ok(e, W);
  if (bi) release_handle(indices);               // engine.cpp:927: no longer needed after backward
  return dx;
}

// -- pool -------------------------------------------------------------------------
DCT_API void WarmPool(uint32_t* sizes, uint32_t n, uint32_t copies) {   // engine.cpp:617-635
  LOCK;
  if (!ensure_init() || !sizes) return;
  for (uint32_t i = 0; i < n; ++i) {
    const uint64_t count = sizes[i];
    if (count == 0) continue;
    auto& lst = g.pool[count];
    const size_t target = std::min<size_t>(copies, max_pool_for_size(count));
    while (lst.size() < target) {
      Buffer* b = create_buffer(nullptr, count);
      if (!b) break;
      release_internal(b);
      if (g.misses > 0) g.misses--;
    }
  }
}

DCT_API void GetPoolStats(uint64_t* hits, uint64_t* misses) {
  LOCK;
  if (hits) *hits = g.hits;
  if (misses) *misses = g.misses;
}

DCT_API void ResetPoolStats() {
  LOCK;
  g.hits = 0;
  g.misses = 0;
}

DCT_API uint64_t GetPoolMemory() {
  LOCK;
  return g.pool_bytes;
}

DCT_API void DrainPool() {
  LOCK;
  for (auto& kv : g.pool)
    for (Buffer* b : kv.second) destroy(b);
  g.pool.clear();
  g.pool_bytes = 0;
  if (g.init) {
    rt_wait_stream("DrainPool");
    cudaMemPool_t mp;
    if (cudaDeviceGetDefaultMemPool(&mp, g.info.device) == cudaSuccess) cudaMemPoolTrimTo(mp, 0);
  }
}

// -- graph replay ------------------------------------------------------------------
DCT_API void* ResolveShader(const char* name) {
  LOCK;
  Shader* s = find_shader(name);
  return (s && (s->compiled || s->always)) ? s : nullptr;
}

// RunSequence as one CUDA graph launch.  The reference replays the same
// command list every batch (ComputeGraph, nn_engine.py:2505-2771), so: the first
// call with a given list runs eagerly (and grows the scratch workspace as
// needed), the second identical call captures the stream into a graph, later
// identical calls launch that graph.  "Identical" compares the command bytes
// and, for every referenced buffer, its device pointer and size, so a handle
// that was released and reallocated never replays a graph into stale memory.
// A capture that fails (a command that errs, or would need a larger workspace)
// is discarded and the list runs eagerly.  DCT_SEQ_GRAPH=0 turns graphs off.
struct SeqGraph {
  std::vector<uint8_t> key;
  bool failed = false;               // this list could not be captured: stay eager
  cudaGraphExec_t exec = nullptr;
};
static SeqGraph g_seq;

static bool seq_key(const DctSeqCmd* cmds, uint32_t count, std::vector<uint8_t>& key) {
  key.assign(reinterpret_cast<const uint8_t*>(cmds), reinterpret_cast<const uint8_t*>(cmds + count));
  auto put = [&](const void* p, size_t n) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    key.insert(key.end(), b, b + n);
  };
  put(&g.ws, sizeof(g.ws));          // a graph bakes in the scratch workspace too
  put(&g.ws_bytes, sizeof(g.ws_bytes));
  for (uint32_t i = 0; i < count; ++i) {
    const DctSeqCmd& c = cmds[i];
    if (!c.shader) continue;
    if (!is_shader_ptr(c.shader)) return false;
    for (uint32_t v = 0; v < 12; ++v) {
      void* h = v < 8 ? (v < c.srvCount ? c.srvs[v] : nullptr) : (v - 8 < c.uavCount ? c.uavs[v - 8] : nullptr);
      if (!h) continue;
      Buffer* b = buf_of(h);
      if (!b) return false;
      put(&b->d, sizeof(b->d));
      put(&b->count, sizeof(b->count));
    }
  }
  return true;
}

static bool seq_run(DctSeqCmd* cmds, uint32_t count) {
  bool ok = true;
  auto disp_of = [](Disp& d, DctSeqCmd& c) {
    return make_disp(d, static_cast<Shader*>(c.shader), c.srvs, std::min<uint32_t>(c.srvCount, 8), c.uavs,
                     std::min<uint32_t>(c.uavCount, 4), c.threads, c.cbSize ? c.cbData : nullptr,
                     std::min<uint32_t>(c.cbSize, 64));
  };
  for (uint32_t i = 0; i < count; ++i) {
    DctSeqCmd& c = cmds[i];
    if (!c.shader) continue;
    if (!is_shader_ptr(c.shader)) {
      set_error(DCT_ERR_ARG, "RunSequence: command %u has a foreign shader pointer", i);
      ok = false;
      continue;
    }
    Shader* s = static_cast<Shader*>(c.shader);
    if (i + 1 < count && cmds[i + 1].shader && is_shader_ptr(cmds[i + 1].shader) && ensure_init()) {
      Disp a, b, cc;
      bool fused_ok = true;
      int used = 0;
      const int code0 = g.err_code;                  // commands that do not fuse leave no error behind
      const std::string msg0 = g.err;
      const bool have_c = i + 2 < count && cmds[i + 2].shader && is_shader_ptr(cmds[i + 2].shader);
      if (disp_of(a, c) && disp_of(b, cmds[i + 1])) {
        const Disp* pc = nullptr;
        if (have_c) {
          if (disp_of(cc, cmds[i + 2])) pc = &cc;
          else { g.err_code = code0; g.err = msg0; }   // that command reports its own error when it runs
        }
        if (try_fused_relu_bias_grad(a, b, pc, fused_ok, &used) || try_fused_bias_relu_colsum(a, b, fused_ok, &used)) {
          ok &= fused_ok;
          i += used - 1;
          continue;
        }
      }
      g.err_code = code0;
      g.err = msg0;
    }
    ok &= dispatch(s, c.srvs, std::min<uint32_t>(c.srvCount, 8), c.uavs, std::min<uint32_t>(c.uavCount, 4),
                   c.threads, c.cbSize ? c.cbData : nullptr, std::min<uint32_t>(c.cbSize, 64));
  }
  return ok;
}

static bool seq_capture(DctSeqCmd* cmds, uint32_t count) {
  if (cudaStreamBeginCapture(g.stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  const int code0 = g.err_code;
  const std::string msg0 = g.err;
  g_capturing = true;
  const bool ok = seq_run(cmds, count);
  g_capturing = false;
  cudaGraph_t graph = nullptr;
  const cudaError_t e = cudaStreamEndCapture(g.stream, &graph);
  cudaGraphExec_t exec = nullptr;
  bool good = ok && e == cudaSuccess && graph && cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
  if (graph) cudaGraphDestroy(graph);
  cudaGetLastError();
  if (!good) {                                       // the eager re-run reports its own errors
    g.err_code = code0;
    g.err = msg0;
    return false;
  }
  if (g_seq.exec) cudaGraphExecDestroy(g_seq.exec);
  g_seq.exec = exec;
  return true;
}

DCT_API void RunSequence(DctSeqCmd* cmds, uint32_t count) {
  LOCK;
  if (!cmds || !ensure_init()) return;
  const char* env = getenv("DCT_SEQ_GRAPH");
  std::vector<uint8_t> key;
  const bool cacheable = count > 0 && !(env && env[0] == '0') && seq_key(cmds, count, key);
  if (cacheable && key == g_seq.key && !g_seq.failed) {
    if (g_seq.exec || seq_capture(cmds, count)) {
      cuda_ok(cudaGraphLaunch(g_seq.exec, g.stream), "RunSequence(graph launch)");
      return;
    }
    g_seq.failed = true;
  }
  seq_run(cmds, count);
  if (cacheable && key != g_seq.key) {
    if (g_seq.exec) cudaGraphExecDestroy(g_seq.exec);
    g_seq.exec = nullptr;
    g_seq.failed = false;
    g_seq.key = std::move(key);
  }
}

DCT_API void RunSequenceWithSGD(DctSeqCmd* cmds, uint32_t count, void** params, void** grads, uint32_t* sizes,
                                uint32_t n, float lr, float clip) {
  LOCK;
  RunSequence(cmds, count);
  SGDBatch(params, grads, sizes, n, lr, clip);
}

// ===========================================================================
// extension entry points
// ===========================================================================
DCT_API const char* dct_last_error() {
  LOCK;
  return g.err.c_str();
}

DCT_API int dct_error_code() {
  LOCK;
  return g.err_code;
}

DCT_API void dct_clear_error() {
  LOCK;
  g.err_code = 0;
  g.err.clear();
}

DCT_API int dct_version() { return DCT_ABI_VERSION; }

DCT_API int dct_device() {
  LOCK;
  return ensure_init() ? g.info.device : -1;
}

DCT_API int dct_sm_count() {
  LOCK;
  return ensure_init() ? g.info.sm_count : 0;
}

DCT_API int dct_pci_bus_id(char* out, int len) {
  LOCK;
  if (!out || len <= 0 || !ensure_init()) return DCT_ERR_NO_DEVICE;
  return cuda_ok(cudaDeviceGetPCIBusId(out, len, g.info.device), "dct_pci_bus_id") ? 0 : DCT_ERR_CUDA;
}

DCT_API void* dct_stream() {
  LOCK;
  return ensure_init() ? (void*)g.stream : nullptr;
}

DCT_API int dct_synchronize() {
  LOCK;
  if (!ensure_init()) return DCT_ERR_NO_DEVICE;
  if (rt_wait_stream("dct_synchronize")) return 0;
  return g.err_code ? g.err_code : DCT_ERR_CUDA;
}

DCT_API int dct_timer_start() {
  LOCK;
  if (!ensure_init()) return DCT_ERR_NO_DEVICE;
  return cuda_ok(cudaEventRecord(g.ev0, g.stream), "dct_timer_start") ? 0 : DCT_ERR_CUDA;
}

DCT_API float dct_timer_stop_ms() {
  LOCK;
  if (!ensure_init()) return -1.0f;
  float ms = -1.0f;
  if (!cuda_ok(cudaEventRecord(g.ev1, g.stream), "dct_timer_stop")) return -1.0f;
  if (!rt_wait_stream("dct_timer_stop")) return -1.0f;
  if (!cuda_ok(cudaEventElapsedTime(&ms, g.ev0, g.ev1), "dct_timer_stop(elapsed)")) return -1.0f;
  if (!check_device_errors()) return -1.0f;
  return ms;
}

DCT_API void* dct_create_buffer(uint64_t count) {
  LOCK;
  return create_buffer(nullptr, count);
}

DCT_API void* dct_buffer_device_ptr(void* h) {
  LOCK;
  Buffer* b = buf_of(h);
  return b ? (void*)b->d : nullptr;
}

DCT_API uint64_t dct_buffer_count(void* h) {
  LOCK;
  Buffer* b = buf_of(h);
  return b ? b->count : 0;
}

DCT_API int dct_buffer_refcount(void* h) {
  LOCK;
  Buffer* b = buf_of(h);
  return b ? b->ref : 0;
}

DCT_API void* dct_wrap_device_ptr(void* dptr, uint64_t count) {
  LOCK;
  if (!ensure_init() || !dptr || count == 0) return nullptr;
  Buffer* b = new Buffer{kBufMagic, 1, count, static_cast<float*>(dptr), false};
  g.live.insert(b);
  return b;
}

DCT_API int dct_copy_h2d(void* h, const void* src, uint64_t offset_floats, uint64_t count) {
  LOCK;
  Buffer* b = buf_of(h);
  if (!b || !src) return DCT_ERR_HANDLE;
  if (offset_floats + count > b->count) return DCT_ERR_SIZE;
  return cuda_ok(cudaMemcpyAsync(b->d + offset_floats, src, count * 4, cudaMemcpyHostToDevice, g.stream), "dct_copy_h2d") ? 0 : DCT_ERR_CUDA;
}

DCT_API int dct_copy_d2h(void* h, void* dst, uint64_t offset_floats, uint64_t count) {
  LOCK;
  Buffer* b = buf_of(h);
  if (!b || !dst) return DCT_ERR_HANDLE;
  if (offset_floats + count > b->count) return DCT_ERR_SIZE;
  if (!cuda_ok(cudaMemcpyAsync(dst, b->d + offset_floats, count * 4, cudaMemcpyDeviceToHost, g.stream), "dct_copy_d2h")) return DCT_ERR_CUDA;
  return rt_wait_stream("dct_copy_d2h") ? 0 : (g.err_code ? g.err_code : DCT_ERR_CUDA);
}

DCT_API void* dct_host_alloc(uint64_t bytes) {
  LOCK;
  if (!ensure_init()) return nullptr;
  void* p = nullptr;
  return cuda_ok(cudaMallocHost(&p, bytes), "dct_host_alloc") ? p : nullptr;
}

DCT_API void dct_host_free(void* p) {
  LOCK;
  if (p) cudaFreeHost(p);
}

DCT_API int dct_fill_random(void* h, uint64_t seed, uint64_t offset, int dist, float a, float b) {
  LOCK;
  Buffer* x = buf_of(h);
  if (!x) return DCT_ERR_HANDLE;
  return cuda_ok(launch_fill_random(x->d, x->count, seed, offset, dist, a, b, g.stream), "dct_fill_random") ? 0 : DCT_ERR_CUDA;
}

DCT_API int dct_scatter(void* h, const int64_t* host_idx, const float* host_vals, uint64_t k) {
  LOCK;
  Buffer* x = buf_of(h);
  if (!x) return DCT_ERR_HANDLE;
  if (k == 0) return 0;
  for (uint64_t i = 0; i < k; ++i)
    if (host_idx[i] < 0 || (uint64_t)host_idx[i] >= x->count) return DCT_ERR_SIZE;
  void* dmem = nullptr;
  if (!cuda_ok(cudaMallocAsync(&dmem, k * 12, g.stream), "dct_scatter(alloc)")) return DCT_ERR_CUDA;
  int64_t* di = (int64_t*)dmem;
  float* dv = (float*)((char*)dmem + k * 8);
  cudaMemcpyAsync(di, host_idx, k * 8, cudaMemcpyHostToDevice, g.stream);
  cudaMemcpyAsync(dv, host_vals, k * 4, cudaMemcpyHostToDevice, g.stream);
  cudaError_t e = launch_scatter_values(x->d, di, dv, k, g.stream);
  cudaFreeAsync(dmem, g.stream);
  rt_wait_stream("dct_scatter");
  return cuda_ok(e, "dct_scatter") ? 0 : DCT_ERR_CUDA;
}

// --- NumPy-semantics ops ------------------------------------------------------------
static int run_ext(const char* name, void** srvs, uint32_t ns, void** uavs, uint32_t nu, const uint32_t* cb,
                   uint32_t cbwords) {
  Shader* s = find_shader(name);
  const uint32_t groups[3] = {0xffffffffu, 1, 1};
  dct_clear_error();
  const bool ok = dispatch(s, srvs, ns, uavs, nu, groups, cb, cbwords * 4);
  if (ok) return 0;
  return g.err_code ? g.err_code : DCT_ERR_ARG;
}

DCT_API int dct_unary(int op, void* x, void* y, uint64_t n, float alpha) {
  LOCK;
  if (n > 0xffffffffull) {
    Buffer* bx = buf_of(x); Buffer* by = buf_of(y);
    if (!bx || !by) return DCT_ERR_HANDLE;
    if (bx->count < n || by->count < n) return DCT_ERR_SIZE;
    return cuda_ok(launch_unary(op, bx->d, by->d, n, alpha, g.stream), "dct_unary") ? 0 : DCT_ERR_CUDA;
  }
  uint32_t alpha_bits;
  memcpy(&alpha_bits, &alpha, 4);
  const uint32_t cb[3] = {(uint32_t)op, (uint32_t)n, alpha_bits};
  void* s[1] = {x};
  void* u[1] = {y};
  return run_ext("dct_unary", s, 1, u, 1, cb, 3);
}

DCT_API int dct_binary(int op, void* a, const int64_t* a_shape, int a_ndim, void* b, const int64_t* b_shape,
                       int b_ndim, void* out) {
  LOCK;
  if (a_ndim < 0 || b_ndim < 0 || a_ndim > 8 || b_ndim > 8) return DCT_ERR_ARG;
  const int nd = std::max(a_ndim, b_ndim);
  uint32_t cb[12] = {0};
  cb[0] = (uint32_t)op;
  cb[1] = (uint32_t)nd;
  for (int i = 0; i < nd; ++i) {
    const int ia = i - (nd - a_ndim), ib = i - (nd - b_ndim);
    const int64_t ea = ia >= 0 ? a_shape[ia] : 1, eb = ib >= 0 ? b_shape[ib] : 1;
    if (ea != eb && ea != 1 && eb != 1) {
      set_error(DCT_ERR_ARG, "dct_binary: shapes do not broadcast at dim %d (%lld vs %lld)", i, (long long)ea,
                (long long)eb);
      return DCT_ERR_ARG;
    }
    const int64_t eo = ea == 1 ? eb : ea;
    if (eo > 0xffffffffll) return DCT_ERR_ARG;
    cb[4 + i] = (uint32_t)eo;
    if (ea == 1 && eo != 1) cb[2] |= 1u << i;
    if (eb == 1 && eo != 1) cb[3] |= 1u << i;
  }
  void* s[2] = {a, b};
  void* u[1] = {out};
  return run_ext("dct_binary", s, 2, u, 1, cb, 4 + nd);
}

// Right-align `t` against `g` (ndim = g_ndim), padding with 1s; false if t does
// not broadcast to g.
static bool align_target(const int64_t* g_shape, int g_ndim, const int64_t* t_shape, int t_ndim, int64_t* t_out,
                         const char* where) {
  if (g_ndim < 0 || g_ndim > 8 || t_ndim < 0 || t_ndim > g_ndim || (g_ndim && !g_shape) || (t_ndim && !t_shape)) {
    set_error(DCT_ERR_ARG, "%s: need 0 <= ndim(target) <= ndim(full) <= 8", where);
    return false;
  }
  for (int d = 0; d < g_ndim; ++d) {
    const int td = d - (g_ndim - t_ndim);
    t_out[d] = td >= 0 ? t_shape[td] : 1;
    if (g_shape[d] < 0 || !(t_out[d] == 1 || t_out[d] == g_shape[d])) {
      set_error(DCT_ERR_ARG, "%s: shape of the target does not broadcast to the full shape at dim %d", where, d);
      return false;
    }
  }
  return true;
}

DCT_API int dct_sum_to_shape(void* grad, const int64_t* g_shape, int g_ndim, const int64_t* t_shape, int t_ndim,
                             void* out) {
  LOCK;
  if (!ensure_init()) return DCT_ERR_NO_DEVICE;
  int64_t t[8];
  if (!align_target(g_shape, g_ndim, t_shape, t_ndim, t, "dct_sum_to_shape")) return DCT_ERR_ARG;
  Buffer *bg = buf_of(grad), *bo = buf_of(out);
  if (!bg || !bo) { set_error(DCT_ERR_HANDLE, "dct_sum_to_shape: not a live buffer"); return DCT_ERR_HANDLE; }
  uint64_t n = 1, tn = 1;
  for (int d = 0; d < g_ndim; ++d) { n *= (uint64_t)g_shape[d]; tn *= (uint64_t)t[d]; }
  if (bg->count < n || bo->count < tn) { set_error(DCT_ERR_SIZE, "dct_sum_to_shape: buffer too small"); return DCT_ERR_SIZE; }
  const size_t ws = sum_to_shape_ws_bytes(g_ndim, g_shape, t);
  if (ws && !ensure_ws(ws)) return DCT_ERR_CUDA;
  return cuda_ok(launch_sum_to_shape(bg->d, g_ndim, g_shape, t, bo->d, g.ws, g.ws_bytes, g.stream),
                 "dct_sum_to_shape") ? 0 : DCT_ERR_CUDA;
}

DCT_API int dct_bias_relu_backward(void* grad, void* out, void* dx, void* db, uint32_t rows, uint32_t cols) {
  LOCK;
  if (!ensure_init()) return DCT_ERR_NO_DEVICE;
  Buffer *bg = buf_of(grad), *by = buf_of(out), *bdx = buf_of(dx), *bdb = buf_of(db);
  if (!bg || !by || !bdx || !bdb) {
    set_error(DCT_ERR_HANDLE, "dct_bias_relu_backward: not a live buffer");
    return DCT_ERR_HANDLE;
  }
  const uint64_t n = (uint64_t)rows * cols;
  if (bg->count < n || by->count < n || bdx->count < n || bdb->count < cols) {
    set_error(DCT_ERR_SIZE, "dct_bias_relu_backward: a buffer holds fewer than %llu (or %u) floats",
              (unsigned long long)n, cols);
    return DCT_ERR_SIZE;
  }
  if (bdb == bg || bdb == by || bdb == bdx) {
    set_error(DCT_ERR_ARG, "dct_bias_relu_backward: db must not alias grad, out or dx");
    return DCT_ERR_ARG;
  }
  const size_t ws = relu_grad_colsum_ws_bytes(rows, cols);
  if (ws && !ensure_ws(ws)) return DCT_ERR_CUDA;
  return cuda_ok(launch_relu_grad_colsum(bg->d, by->d, bdx->d, bdb->d, rows, cols, g.ws, g.ws_bytes, g.stream),
                 "dct_bias_relu_backward") ? 0 : DCT_ERR_CUDA;
}

DCT_API int dct_broadcast_to(void* x, const int64_t* x_shape, int x_ndim, const int64_t* out_shape, int out_ndim,
                             void* out) {
  LOCK;
  if (!ensure_init()) return DCT_ERR_NO_DEVICE;
  int64_t xs[8];
  if (!align_target(out_shape, out_ndim, x_shape, x_ndim, xs, "dct_broadcast_to")) return DCT_ERR_ARG;
  Buffer *bx = buf_of(x), *bo = buf_of(out);
  if (!bx || !bo) { set_error(DCT_ERR_HANDLE, "dct_broadcast_to: not a live buffer"); return DCT_ERR_HANDLE; }
  int64_t str[8];
  uint64_t n = 1, xn = 1;
  int64_t s = 1;
  for (int d = out_ndim - 1; d >= 0; --d) {
    str[d] = xs[d] == 1 ? 0 : s;
    s *= xs[d];
  }
  for (int d = 0; d < out_ndim; ++d) { n *= (uint64_t)out_shape[d]; xn *= (uint64_t)xs[d]; }
  if (bx->count < xn || bo->count < n) { set_error(DCT_ERR_SIZE, "dct_broadcast_to: buffer too small"); return DCT_ERR_SIZE; }
  return cuda_ok(launch_binary_bcast(EW_FIRST, bx->d, bx->d, bo->d, out_ndim, out_shape, str, str, g.stream),
                 "dct_broadcast_to") ? 0 : DCT_ERR_CUDA;
}

DCT_API int dct_reduce(int op, void* x, uint64_t outer, uint64_t len, uint64_t inner, void* out, void* out_idx) {
  LOCK;
  if (outer > 0xffffffffull || len > 0xffffffffull || inner > 0xffffffffull) return DCT_ERR_ARG;
  const uint32_t cb[4] = {(uint32_t)op, (uint32_t)outer, (uint32_t)len, (uint32_t)inner};
  void* s[1] = {x};
  void* u[2] = {out, out_idx};
  return run_ext("dct_reduce", s, 1, u, out_idx ? 2 : 1, cb, 4);
}

DCT_API int dct_reduce_all(int op, void* x, uint64_t n, void* out, double* host_out64) {
  LOCK;
  Buffer* bx = buf_of(x);
  Buffer* bo = buf_of(out);
  if (!bx || !bo) return DCT_ERR_HANDLE;
  if (bx->count < n) return DCT_ERR_SIZE;
  if (n == 0 && (op == RED_MAX || op == RED_MIN)) {
    set_error(DCT_ERR_ARG, "dct_reduce_all: max/min of an empty vector has no identity");
    return DCT_ERR_ARG;
  }
  if (!ensure_ws(full_reduce_ws_bytes() + 256)) return DCT_ERR_CUDA;
  double* d64 = (double*)((char*)g.ws + full_reduce_ws_bytes());
  if (!cuda_ok(launch_full_reduce(op, bx->d, n, bo->d, d64, g.ws, g.stream), "dct_reduce_all")) return DCT_ERR_CUDA;
  if (host_out64) {
    if (!cuda_ok(cudaMemcpyAsync(g.host_small, d64, 8, cudaMemcpyDeviceToHost, g.stream), "dct_reduce_all(D2H)")) return DCT_ERR_CUDA;
    if (!rt_wait_stream("dct_reduce_all")) return g.err_code ? g.err_code : DCT_ERR_CUDA;
    memcpy(host_out64, g.host_small, 8);
  }
  return 0;
}

DCT_API int dct_softmax_ce(void* logits, void* labels, int labels_int32, uint32_t rows, uint32_t K, void* probs,
                           void* dlogits, void* loss, void* logprobs, float loss_div, float grad_div) {
  LOCK;
  uint32_t ld, gd;
  memcpy(&ld, &loss_div, 4);
  memcpy(&gd, &grad_div, 4);
  const uint32_t cb[5] = {rows, K, labels_int32 ? 1u : 0u, ld, gd};
  void* s[2] = {logits, labels};
  void* u[4] = {probs, dlogits, loss, logprobs};
  return run_ext("dct_softmax_ce", s, labels ? 2 : 1, u, 4, cb, 5);
}

DCT_API int dct_adam(void* w, void* m, void* v, void* grad, uint64_t n, float step_size, float beta1, float beta2,
                     float eps, float weight_decay, float clip) {
  LOCK;
  Buffer *bw = buf_of(w), *bm = buf_of(m), *bv = buf_of(v), *bg = buf_of(grad);
  if (!bw || !bm || !bv || !bg) return DCT_ERR_HANDLE;
  if (bw->count < n || bm->count < n || bv->count < n || bg->count < n) return DCT_ERR_SIZE;
  AdamParams p{step_size, beta1, beta2, eps, weight_decay, clip};
  return cuda_ok(launch_adam(bw->d, bm->d, bv->d, bg->d, n, p, g.stream), "dct_adam") ? 0 : DCT_ERR_CUDA;
}

DCT_API int dct_adam_batch(void** w, void** m, void** v, void** grads, const uint32_t* sizes, uint32_t n,
                           float step_size, float beta1, float beta2, float eps, float weight_decay, float clip) {
  LOCK;
  if (!ensure_init()) return DCT_ERR_NO_DEVICE;
  std::vector<MtTensor> t;
  for (uint32_t i = 0; i < n; ++i) {
    Buffer *bw = buf_of(w[i]), *bm = buf_of(m[i]), *bv = buf_of(v[i]), *bg = buf_of(grads[i]);
    if (!bw || !bg) continue;
    if (!bm || !bv) return DCT_ERR_HANDLE;
    uint64_t cnt = sizes ? sizes[i] : bw->count;
    if (cnt > std::min({bw->count, bm->count, bv->count, bg->count})) return DCT_ERR_SIZE;
    t.push_back(MtTensor{bw->d, bg->d, bm->d, bv->d, cnt});
  }
  AdamParams p{step_size, beta1, beta2, eps, weight_decay, clip};
  return cuda_ok(launch_mt_adam(t.data(), (int)t.size(), p, g.stream), "dct_adam_batch") ? 0 : DCT_ERR_CUDA;
}

DCT_API int dct_batchnorm_forward_train(void* x, void* gamma, void* beta, void* running_mean, void* running_var,
                                        void* batch_mean, void* batch_var, void* y, uint32_t N, uint32_t C,
                                        uint32_t S, float eps, float momentum) {
  LOCK;
  Buffer *bx = buf_of(x), *bg = buf_of(gamma), *bb = buf_of(beta), *rm = buf_of(running_mean),
         *rv = buf_of(running_var), *bm = buf_of(batch_mean), *bvv = buf_of(batch_var), *by = buf_of(y);
  if (!bx || !bg || !bb || !rm || !rv || !bm || !bvv || !by) return DCT_ERR_HANDLE;
  const uint64_t n = (uint64_t)N * C * S;
  if (bx->count < n || by->count < n || bg->count < C || bb->count < C || rm->count < C || rv->count < C ||
      bm->count < C || bvv->count < C)
    return DCT_ERR_SIZE;
  Disp d;
  memset(&d, 0, sizeof(d));
  d.name = "dct_batchnorm_forward_train";
  if (!bn_stats(d, bx->d, N, C, S, bm->d, bvv->d, rm->d, rv->d, true, momentum, C)) return g.err_code ? g.err_code : DCT_ERR_CUDA;
  return cuda_ok(launch_bn_forward(bx->d, bm->d, bvv->d, bg->d, bb->d, by->d, N, C, S, eps, n, g.stream),
                 "dct_batchnorm_forward_train") ? 0 : DCT_ERR_CUDA;
}

DCT_API int dct_batchnorm_backward(void* x, void* dy, void* batch_mean, void* batch_var, void* gamma, void* dgamma,
                                   void* dbeta, void* dx, uint32_t N, uint32_t C, uint32_t S, float eps) {
  LOCK;
  Buffer *bx = buf_of(x), *bd = buf_of(dy), *bm = buf_of(batch_mean), *bv = buf_of(batch_var), *bg = buf_of(gamma),
         *dg = buf_of(dgamma), *db = buf_of(dbeta), *bo = buf_of(dx);
  if (!bx || !bd || !bm || !bv || !bg || !dg || !db || !bo) return DCT_ERR_HANDLE;
  const uint64_t n = (uint64_t)N * C * S;
  if (bx->count < n || bd->count < n || bo->count < n) return DCT_ERR_SIZE;
  if (!ensure_ws(bn_ws_bytes(N, C))) return DCT_ERR_CUDA;
  double* ps = (double*)g.ws;
  double* chan = ps + (size_t)N * C * 2;
  cudaError_t e = launch_bn_plane_sums(bx->d, bd->d, N, C, S, ps, g.stream);
  if (e == cudaSuccess) e = launch_bn_fold(ps, N, C, chan, g.stream);
  if (e == cudaSuccess) e = launch_bn_bwd_final(chan, C, bm->d, bv->d, eps, dg->d, db->d, g.stream);
  if (e == cudaSuccess)
    e = launch_bn_backward_dx(bx->d, bd->d, bm->d, bv->d, bg->d, dg->d, db->d, bo->d, N, C, S, eps, n, g.stream);
  return cuda_ok(e, "dct_batchnorm_backward") ? 0 : DCT_ERR_CUDA;
}

}  // extern "C"
