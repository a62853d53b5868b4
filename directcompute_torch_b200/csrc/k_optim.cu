// Optimizer kernels of libdct_cuda (sm_100a).
//
// nn_sgd.hlsl:5-11, nn_sgd_clipped.hlsl:15-20 and nn_adam.hlsl:18-34, with the
// reference's per-parameter dispatch loops (engine.cpp:436-485 SGDBatch,
// engine.cpp:494-614 SGDBatchClipped, nn_engine.py:2217-2238 AdamW.step) folded
// into multi-tensor launches: one kernel walks a table of (param, grad, m, v, n)
// held in the kernel's parameter space, so a whole model steps in one launch.
//
// Arithmetic is the shaders' fp32 formula with every operation rounded
// separately (round-to-nearest intrinsics, IEEE sqrt and divide): results are
// bit-identical to the NumPy restatement.  Adam moves 28 bytes per element
// (read w, g, m, v; write w, m, v) with 128-bit streaming accesses.
#include "dct_common.cuh"
#include "kernels.h"

namespace dct {

namespace {

struct AdamK {
  float step, b1, b2, omb1, omb2, eps, wd, clip;
};

DCT_DEV float clampg(float g, float clip) {
  if (g > clip) g = clip;          // NaN passes through, like the shader
  if (g < -clip) g = -clip;
  return g;
}

DCT_DEV void adam1(float& w, float& m, float& v, float g, const AdamK& p) {
  g = clampg(g, p.clip);
  const float mt = __fadd_rn(__fmul_rn(p.b1, m), __fmul_rn(p.omb1, g));
  const float vt = __fadd_rn(__fmul_rn(p.b2, v), __fmul_rn(__fmul_rn(p.omb2, g), g));
  const float upd = __fdiv_rn(__fmul_rn(p.step, mt), __fadd_rn(__fsqrt_rn(vt), p.eps));
  w = __fsub_rn(__fsub_rn(w, __fmul_rn(p.wd, w)), upd);
  m = mt;
  v = vt;
}

DCT_DEV float sgd1(float w, float g, float lr, float clip) {
  return __fsub_rn(w, __fmul_rn(lr, clampg(g, clip)));
}

DCT_DEV float sgd_scaled1(float w, float g, float lr, float scale) {
  return __fsub_rn(w, __fmul_rn(__fmul_rn(lr, g), scale));
}

// Chunked schedule (one contiguous 16 KB slice of each array per block, all
// loads before any store): the block scheduler then walks the four streams in
// address order, which keeps DRAM pages open (see k_elementwise.cu).
constexpr int kOptU = 4;
constexpr uint64_t kOptChunk4 = 256ull * kOptU;

__global__ void __launch_bounds__(256) k_adam(float* __restrict__ w, float* __restrict__ m, float* __restrict__ v,
                                              const float* __restrict__ g, uint64_t n, AdamK p) {
  pdl_entry();
  const uint64_t n4 = n >> 2;
  const uint64_t base = (uint64_t)blockIdx.x * kOptChunk4 + threadIdx.x;
  float4 W[kOptU], M[kOptU], V[kOptU], G[kOptU];
#pragma unroll
  for (int k = 0; k < kOptU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i < n4) {
      W[k] = ld_stream4(w + 4 * i); M[k] = ld_stream4(m + 4 * i);
      V[k] = ld_stream4(v + 4 * i); G[k] = ld_stream4(g + 4 * i);
    }
  }
#pragma unroll
  for (int k = 0; k < kOptU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i < n4) {
      adam1(W[k].x, M[k].x, V[k].x, G[k].x, p); adam1(W[k].y, M[k].y, V[k].y, G[k].y, p);
      adam1(W[k].z, M[k].z, V[k].z, G[k].z, p); adam1(W[k].w, M[k].w, V[k].w, G[k].w, p);
      st_stream4(w + 4 * i, W[k]); st_stream4(m + 4 * i, M[k]); st_stream4(v + 4 * i, V[k]);
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const uint64_t t = 4 * n4 + threadIdx.x;
    float Wt = w[t], Mt = m[t], Vt = v[t];
    adam1(Wt, Mt, Vt, g[t], p);
    w[t] = Wt; m[t] = Mt; v[t] = Vt;
  }
}

__global__ void __launch_bounds__(256) k_adam_scalar(float* w, float* m, float* v, const float* g, uint64_t n, AdamK p) {
  pdl_entry();
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float W = w[i], M = m[i], V = v[i];
    adam1(W, M, V, g[i], p);
    w[i] = W; m[i] = M; v[i] = V;
  }
}

template <bool SCALED>
__global__ void __launch_bounds__(256) k_sgd(float* w, const float* __restrict__ g, uint64_t n, float lr, float clip,
                                             const float* ns) {
  pdl_entry();
  const float scale = SCALED ? ns[1] : 1.0f;
  const uint64_t n4 = n >> 2;
  const uint64_t base = (uint64_t)blockIdx.x * kOptChunk4 + threadIdx.x;
  float4 W[kOptU], G[kOptU];
#pragma unroll
  for (int k = 0; k < kOptU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i < n4) { W[k] = ld_stream4(w + 4 * i); G[k] = ld_stream4(g + 4 * i); }
  }
#pragma unroll
  for (int k = 0; k < kOptU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i >= n4) continue;
    float4 o = W[k];
    if (SCALED) {
      o.x = sgd_scaled1(o.x, G[k].x, lr, scale); o.y = sgd_scaled1(o.y, G[k].y, lr, scale);
      o.z = sgd_scaled1(o.z, G[k].z, lr, scale); o.w = sgd_scaled1(o.w, G[k].w, lr, scale);
    } else {
      o.x = sgd1(o.x, G[k].x, lr, clip); o.y = sgd1(o.y, G[k].y, lr, clip);
      o.z = sgd1(o.z, G[k].z, lr, clip); o.w = sgd1(o.w, G[k].w, lr, clip);
    }
    st_stream4(w + 4 * i, o);
  }
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const uint64_t t = 4 * n4 + threadIdx.x;
    w[t] = SCALED ? sgd_scaled1(w[t], g[t], lr, scale) : sgd1(w[t], g[t], lr, clip);
  }
}

template <bool SCALED>
__global__ void __launch_bounds__(256) k_sgd_scalar(float* w, const float* g, uint64_t n, float lr, float clip,
                                                    const float* ns) {
  pdl_entry();
  const float scale = SCALED ? ns[1] : 1.0f;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    w[i] = SCALED ? sgd_scaled1(w[i], g[i], lr, scale) : sgd1(w[i], g[i], lr, clip);
}

// ---------------------------------------------------------------------------
// multi-tensor apply
// ---------------------------------------------------------------------------
constexpr int kMtMax = 160;                     // tensors per launch (param space < 12 KB)
constexpr uint64_t kMtChunk = 256 * 4 * 8;      // elements per block

enum MtOp { MT_SGD = 0, MT_SGD_SCALED, MT_ADAM, MT_SUMSQ };

struct MtTable {
  int count;
  uint32_t block_start[kMtMax + 1];
  MtTensor t[kMtMax];
  AdamK adam;
  float lr, clip;
  const float* ns;
  double* partials;                              // MT_SUMSQ: one per block
  uint32_t part_base;
};

template <int OP>
__global__ void __launch_bounds__(256) k_mt(const __grid_constant__ MtTable tab) {
  pdl_entry();
  // locate this block's tensor (binary search over the block prefix)
  int lo = 0, hi = tab.count - 1;
  const uint32_t b = blockIdx.x;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tab.block_start[mid] <= b) lo = mid; else hi = mid - 1;
  }
  const MtTensor& T = tab.t[lo];
  const uint64_t c0 = (uint64_t)(b - tab.block_start[lo]) * kMtChunk;
  const uint64_t c1 = min(T.n, c0 + kMtChunk);
  double acc = 0.0;
  const float scale = (OP == MT_SGD_SCALED) ? tab.ns[1] : 1.0f;
  const bool vec = aligned16(T.w) && aligned16(T.g) && (OP != MT_ADAM || (aligned16(T.m) && aligned16(T.v)));
  const uint64_t v1 = vec ? c0 + ((c1 - c0) & ~3ull) : c0;
  for (uint64_t i = c0 + 4 * threadIdx.x; i < v1; i += 4 * blockDim.x) {
    if constexpr (OP == MT_SUMSQ) {
      const float4 G = ld_stream4(T.g + i);
      acc += (double)G.x * G.x + (double)G.y * G.y + (double)G.z * G.z + (double)G.w * G.w;
    } else if constexpr (OP == MT_ADAM) {
      float4 W = ld_stream4(T.w + i), M = ld_stream4(T.m + i), V = ld_stream4(T.v + i);
      const float4 G = ld_stream4(T.g + i);
      adam1(W.x, M.x, V.x, G.x, tab.adam); adam1(W.y, M.y, V.y, G.y, tab.adam);
      adam1(W.z, M.z, V.z, G.z, tab.adam); adam1(W.w, M.w, V.w, G.w, tab.adam);
      st_stream4(T.w + i, W); st_stream4(T.m + i, M); st_stream4(T.v + i, V);
    } else {
      float4 W = ld_stream4(T.w + i);
      const float4 G = ld_stream4(T.g + i);
      if (OP == MT_SGD) {
        W.x = sgd1(W.x, G.x, tab.lr, tab.clip); W.y = sgd1(W.y, G.y, tab.lr, tab.clip);
        W.z = sgd1(W.z, G.z, tab.lr, tab.clip); W.w = sgd1(W.w, G.w, tab.lr, tab.clip);
      } else {
        W.x = sgd_scaled1(W.x, G.x, tab.lr, scale); W.y = sgd_scaled1(W.y, G.y, tab.lr, scale);
        W.z = sgd_scaled1(W.z, G.z, tab.lr, scale); W.w = sgd_scaled1(W.w, G.w, tab.lr, scale);
      }
      st_stream4(T.w + i, W);
    }
  }
  for (uint64_t i = v1 + threadIdx.x; i < c1; i += blockDim.x) {
    if constexpr (OP == MT_SUMSQ) {
      const double d = (double)T.g[i];
      acc += d * d;
    } else if constexpr (OP == MT_ADAM) {
      float W = T.w[i], M = T.m[i], V = T.v[i];
      adam1(W, M, V, T.g[i], tab.adam);
      T.w[i] = W; T.m[i] = M; T.v[i] = V;
    } else if constexpr (OP == MT_SGD) {
      T.w[i] = sgd1(T.w[i], T.g[i], tab.lr, tab.clip);
    } else {
      T.w[i] = sgd_scaled1(T.w[i], T.g[i], tab.lr, scale);
    }
  }
  if constexpr (OP == MT_SUMSQ) {
    __shared__ double sh[32];
    const double t = block_sum(acc, sh);
    if (threadIdx.x == 0) tab.partials[tab.part_base + blockIdx.x] = t;
  }
}

AdamK to_k(const AdamParams& p) {
  AdamK k;
  k.step = p.step_size; k.b1 = p.beta1; k.b2 = p.beta2;
  k.omb1 = 1.0f - p.beta1;                     // fp32, as the shader's (1.0 - beta1)
  k.omb2 = 1.0f - p.beta2;
  k.eps = p.eps; k.wd = p.wd; k.clip = p.clip;
  return k;
}

// Fill `tab` with up to kMtMax non-empty tensors starting at *pos; returns blocks.
uint32_t fill_table(MtTable& tab, const MtTensor* t, int count, int* pos) {
  tab.count = 0;
  uint32_t blocks = 0;
  while (*pos < count && tab.count < kMtMax) {
    const MtTensor& x = t[*pos];
    ++*pos;
    if (x.n == 0 || !x.g) continue;
    const uint64_t nb = (x.n + kMtChunk - 1) / kMtChunk;
    if ((uint64_t)blocks + nb > 0x7fffffffull) { --*pos; break; }
    tab.block_start[tab.count] = blocks;
    tab.t[tab.count] = x;
    ++tab.count;
    blocks += (uint32_t)nb;
  }
  tab.block_start[tab.count] = blocks;
  return blocks;
}

template <int OP>
cudaError_t run_mt(const MtTensor* t, int count, MtTable& tab, cudaStream_t st) {
  int pos = 0;
  while (pos < count) {
    const uint32_t blocks = fill_table(tab, t, count, &pos);
    if (tab.count == 0 || blocks == 0) continue;
    launch_pdl(k_mt<OP>, dim3(blocks), dim3(256), 0, st, tab);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (OP == MT_SUMSQ) tab.part_base += blocks;
  }
  return cudaSuccess;
}

__global__ void k_norm_scale(const double* part, int n, float max_norm, float* ns) {
  pdl_entry();
  __shared__ double sh[32];
  const double t = block_sum(strided_sum(part, n), sh);
  if (threadIdx.x == 0) {
    const float norm = (float)sqrt(t);
    ns[0] = norm;
    ns[1] = norm > max_norm ? (float)((double)max_norm / ((double)norm + (double)1e-6f)) : 1.0f;
  }
}

}  // namespace

cudaError_t launch_adam(float* w, float* m, float* v, const float* g, uint64_t n, const AdamParams& p,
                        cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const AdamK k = to_k(p);
  const uint64_t blocks = ((n >> 2) + kOptChunk4 - 1) / kOptChunk4;
  if (aligned16_h(w) && aligned16_h(m) && aligned16_h(v) && aligned16_h(g) && blocks < (1ull << 31))
    launch_pdl(k_adam, dim3((unsigned)(blocks ? blocks : 1)), dim3(256), 0, st, w, m, v, g, n, k);
  else
    launch_pdl(k_adam_scalar, dim3(grid_for(n, 256)), dim3(256), 0, st, w, m, v, g, n, k);
  return cudaGetLastError();
}

template <bool SCALED>
static cudaError_t run_sgd(float* w, const float* g, uint64_t n, float lr, float clip, const float* ns,
                           cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const uint64_t blocks = ((n >> 2) + kOptChunk4 - 1) / kOptChunk4;
  if (aligned16_h(w) && aligned16_h(g) && blocks < (1ull << 31))
    launch_pdl(k_sgd<SCALED>, dim3((unsigned)(blocks ? blocks : 1)), dim3(256), 0, st, w, g, n, lr, clip, ns);
  else
    launch_pdl(k_sgd_scalar<SCALED>, dim3(grid_for(n, 256)), dim3(256), 0, st, w, g, n, lr, clip, ns);
  return cudaGetLastError();
}

cudaError_t launch_sgd(float* w, const float* g, uint64_t n, float lr, float clip, cudaStream_t st) {
  return run_sgd<false>(w, g, n, lr, clip, nullptr, st);
}

cudaError_t launch_sgd_clipped(float* w, const float* g, uint64_t n, float lr, const float* ns, cudaStream_t st) {
  return run_sgd<true>(w, g, n, lr, 0.0f, ns, st);
}

cudaError_t launch_mt_sgd(const MtTensor* t, int count, float lr, float clip, const float* ns, cudaStream_t st) {
  MtTable tab{};
  tab.lr = lr;
  tab.clip = clip;
  tab.ns = ns;
  return ns ? run_mt<MT_SGD_SCALED>(t, count, tab, st) : run_mt<MT_SGD>(t, count, tab, st);
}

cudaError_t launch_mt_adam(const MtTensor* t, int count, const AdamParams& p, cudaStream_t st) {
  MtTable tab{};
  tab.adam = to_k(p);
  return run_mt<MT_ADAM>(t, count, tab, st);
}

// number of partials launch_mt_sumsq writes for this tensor list
static uint64_t mt_blocks(const MtTensor* t, int count) {
  uint64_t b = 0;
  for (int i = 0; i < count; ++i)
    if (t[i].n && t[i].g) b += (t[i].n + kMtChunk - 1) / kMtChunk;
  return b;
}

cudaError_t launch_mt_sumsq(const MtTensor* t, int count, double* partials, int nparts, cudaStream_t st) {
  if ((uint64_t)nparts < mt_blocks(t, count)) return cudaErrorInvalidValue;
  MtTable tab{};
  tab.partials = partials;
  tab.part_base = 0;
  return run_mt<MT_SUMSQ>(t, count, tab, st);
}

uint64_t mt_sumsq_blocks(const MtTensor* t, int count) { return mt_blocks(t, count); }

cudaError_t launch_norm_scale_from_parts(const double* partials, int nparts, float max_norm, float* ns,
                                         cudaStream_t st) {
  launch_pdl(k_norm_scale, dim3(1), dim3(1024), 0, st, partials, nparts, max_norm, ns);
  return cudaGetLastError();
}

}  // namespace dct
