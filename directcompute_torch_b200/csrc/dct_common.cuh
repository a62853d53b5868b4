// Shared device helpers for libdct_cuda (sm_100a).
//
// Every kernel of the library is memory-bound fp32 work: 128-bit vector
// loads/stores, streaming cache hints, float64 accumulation for every sum, and
// grids sized as a multiple of the SM count.  Nothing here uses tensor cores.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <math.h>

#include <utility>

#define DCT_DEV __device__ __forceinline__

namespace dct {

// ---------------------------------------------------------------------------
// launch geometry
// ---------------------------------------------------------------------------
struct DevInfo {
  int device = -1;
  int sm_count = 148;
  int max_threads_per_sm = 2048;
  size_t smem_optin = 227 * 1024;
  size_t total_mem = 0;
};
const DevInfo& dev_info();   // defined in runtime.cu
// device-visible error word (mapped host memory; null before InitEngine, then
// kernels skip the report).  Bits:
enum : uint32_t {
  DCT_DEVERR_WAIT_TIMEOUT = 1u,    // a bounded wait in a kernel ran out
  DCT_DEVERR_PEER_INVALID = 2u,    // a rank's shard of a sharded op was invalid
  DCT_DEVERR_PEER_WAIT = 4u,       // a peer's record did not arrive before the deadline
};
uint32_t* device_error_word();   // defined in runtime.cu
// Zeroed device words for kernels that raise a flag another kernel of the same
// stream consumes and clears (null before InitEngine).  Every kernel that
// sets one leaves it zero when the pair is done.
constexpr uint32_t kDeviceFlags = 64;
uint32_t* device_flags();        // defined in runtime.cu

// Blocks for a grid-stride kernel of `threads`-thread blocks covering `work`
// independent items: enough to fill every SM `waves` times, never more than
// the work needs.
inline unsigned grid_for(uint64_t work, int threads, int waves = 1) {
  const DevInfo& d = dev_info();
  uint64_t resident = (uint64_t)d.sm_count * (uint64_t)(d.max_threads_per_sm / threads) * waves;
  uint64_t need = (work + threads - 1) / threads;
  if (need < 1) need = 1;
  return (unsigned)(need < resident ? need : resident);
}

// ---------------------------------------------------------------------------
// programmatic dependent launch: a kernel launched with launch_pdl may start
// while the previous kernel on the stream finishes; it must call
// grid_dep_wait() before reading that kernel's results (a no-op when the
// kernel was launched the ordinary way)
// ---------------------------------------------------------------------------
DCT_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel of the stream, when launched with launch_pdl, be
// scheduled before this one ends; it still waits in grid_dep_wait for this
// grid to complete, so every kernel launched with launch_pdl calls
// grid_dep_wait before touching what earlier kernels wrote.
DCT_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// First statement of every kernel launched with launch_pdl: the next kernel may
// be scheduled now, and nothing here touches memory before the previous kernel
// of the stream has completed.  Both are no-ops for an ordinary launch.
DCT_DEV void pdl_entry() {
  grid_dep_launch();
  grid_dep_wait();
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// memory access
// ---------------------------------------------------------------------------
// Streaming (evict-first) 128-bit accesses: every large tensor here is touched
// exactly once per kernel, so it should not displace reusable lines in L2.
DCT_DEV float4 ld_stream4(const float* p) { return __ldcs(reinterpret_cast<const float4*>(p)); }
DCT_DEV void st_stream4(float* p, float4 v) { __stcs(reinterpret_cast<float4*>(p), v); }
DCT_DEV float ld_stream(const float* p) { return __ldcs(p); }
DCT_DEV void st_stream(float* p, float v) { __stcs(p, v); }
// Small operands reused by many threads (biases, broadcast rows): keep cached.
DCT_DEV float4 ld_keep4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
DCT_DEV float ld_keep(const float* p) { return __ldg(p); }

DCT_DEV bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned16_h(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// warp / block reductions (fixed shuffle order => run-to-run deterministic)
// ---------------------------------------------------------------------------
DCT_DEV double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  return v;  // lane 0 holds the total
}
DCT_DEV float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;  // every lane holds the total
}
DCT_DEV float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// (value, index) arg-reductions with NumPy's rule: NaN is the maximum (and the
// minimum), and among equal candidates the lowest index wins.
struct ValIdx {
  float v;
  int64_t i;
};
DCT_DEV bool better_max(float av, int64_t ai, float bv, int64_t bi) {
  bool an = isnan(av), bn = isnan(bv);
  if (an || bn) {
    if (an && bn) return ai < bi;
    return an;
  }
  if (av != bv) return av > bv;
  return ai < bi;
}
DCT_DEV bool better_min(float av, int64_t ai, float bv, int64_t bi) {
  bool an = isnan(av), bn = isnan(bv);
  if (an || bn) {
    if (an && bn) return ai < bi;
    return an;
  }
  if (av != bv) return av < bv;
  return ai < bi;
}
template <bool IS_MAX>
DCT_DEV bool better(float av, int64_t ai, float bv, int64_t bi) {
  return IS_MAX ? better_max(av, ai, bv, bi) : better_min(av, ai, bv, bi);
}
template <bool IS_MAX>
DCT_DEV void warp_argbest(float& v, int64_t& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, o);
    int64_t oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (better<IS_MAX>(ov, oi, v, i)) { v = ov; i = oi; }
  }
}

// This thread's share of a block's fold of n partials: p[t] + p[t + B] + ...
// (t = threadIdx.x, B = blockDim.x), added in that order.  Four loads are
// issued before their adds, so the partials' latency is paid once per four.
// (float partials are widened to double as they are added.)
template <typename T, typename N>
DCT_DEV double strided_sum(const T* p, N n) {
  double acc = 0.0;
  const N B = blockDim.x;
  N k = threadIdx.x;
  for (; k + 3 * B < n; k += 4 * B) {
    const T a0 = p[k], a1 = p[k + B], a2 = p[k + 2 * B], a3 = p[k + 3 * B];
    acc += (double)a0;
    acc += (double)a1;
    acc += (double)a2;
    acc += (double)a3;
  }
  for (; k < n; k += B) acc += (double)p[k];
  return acc;
}

// Sum a per-thread double across a block of blockDim.x threads (<= 1024) in a
// fixed order.  Returns the total in thread 0.  `sh` needs 32 doubles.
DCT_DEV double block_sum(double v, double* sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  double t = 0.0;
  if (wid == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    t = lane < nw ? sh[lane] : 0.0;
    t = warp_sum(t);
  }
  return t;
}

// ---------------------------------------------------------------------------
// fast unsigned division by a runtime-invariant divisor (round-up method of
// Granlund & Montgomery, "Division by invariant integers using multiplication",
// PLDI 1994): q = umulhi(n, m) + n >> s for n < 2^32.
// ---------------------------------------------------------------------------
struct FastDiv {
  uint32_t d = 1, m = 0, s = 0;
  FastDiv() = default;
  explicit FastDiv(uint32_t div) : d(div) {
    if (div == 1) { m = 0; s = 0; return; }
    uint32_t l = 0;
    while ((1ull << l) < div) ++l;               // l = ceil(log2(d))
    uint64_t mm = ((1ull << 32) * ((1ull << l) - div)) / div + 1;
    m = (uint32_t)mm;
    s = l - 1;
  }
  DCT_DEV uint32_t div(uint32_t n) const {
    if (d == 1) return n;
    uint32_t hi = __umulhi(n, m);
    return (hi + ((n - hi) >> 1)) >> s;
  }
};

}  // namespace dct
