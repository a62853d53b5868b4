// BatchNorm (NCHW, training and eval) kernels of libdct_cuda (sm_100a).
//
// The reference runs one 256-thread group per CHANNEL that walks N*S elements
// with a divide and modulo per element (nn_batchnorm_mean_var.hlsl:19-60,
// nn_batchnorm_backward_reduce.hlsl:21-60) and two per-element apply shaders
// (nn_batchnorm_forward.hlsl:18-34, nn_batchnorm_backward_dx.hlsl:20-38).
//
// Here a warp owns one (n, c) plane of S contiguous floats, streams it with
// 128-bit loads and leaves two float64 plane sums; a fold launch adds the N
// plane sums of each channel in n order (deterministic; across GPUs the same
// per-channel sums are what the NCCL exchange combines); a finalize launch turns
// them into mean / biased var (+ the momentum update with the unbiased var) or
// dgamma / dbeta.  The apply kernels stream the flat array in 16 KB chunks per
// block and find each float4's channel with two fast divisions.
#include "dct_common.cuh"
#include "dct_fold.cuh"
#include "kernels.h"

namespace dct {

namespace {

DCT_DEV float rstd_of(float var, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));   // 1.0 / sqrt(v + eps)
}

// BWD == false: (sum x, sum x^2); BWD == true: (sum dy, sum dy*x)
template <bool BWD, bool VEC>
__global__ void __launch_bounds__(256) k_bn_plane_sums(const float* __restrict__ x, const float* __restrict__ dy,
                                                       uint64_t planes, uint32_t S, double* out) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const uint64_t gw = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint64_t nw = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  for (uint64_t pl = gw; pl < planes; pl += nw) {
    const float* px = x + pl * S;
    const float* pd = BWD ? dy + pl * S : nullptr;
    double a = 0.0, b = 0.0;
    if (VEC) {
      const uint32_t s4 = S >> 2;
      uint32_t i = lane;
      for (; i + 96 < s4; i += 128) {
        float4 vx[4], vd[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          vx[k] = ld_stream4(px + 4 * (i + 32 * k));
          if (BWD) vd[k] = ld_stream4(pd + 4 * (i + 32 * k));
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (BWD) {
            a += (double)vd[k].x + (double)vd[k].y + (double)vd[k].z + (double)vd[k].w;
            b += (double)vd[k].x * vx[k].x + (double)vd[k].y * vx[k].y + (double)vd[k].z * vx[k].z +
                 (double)vd[k].w * vx[k].w;
          } else {
            a += (double)vx[k].x + (double)vx[k].y + (double)vx[k].z + (double)vx[k].w;
            b += (double)vx[k].x * vx[k].x + (double)vx[k].y * vx[k].y + (double)vx[k].z * vx[k].z +
                 (double)vx[k].w * vx[k].w;
          }
        }
      }
      for (; i < s4; i += 32) {
        const float4 v = ld_stream4(px + 4 * i);
        if (BWD) {
          const float4 d = ld_stream4(pd + 4 * i);
          a += (double)d.x + (double)d.y + (double)d.z + (double)d.w;
          b += (double)d.x * v.x + (double)d.y * v.y + (double)d.z * v.z + (double)d.w * v.w;
        } else {
          a += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
          b += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
        }
      }
    } else {
      for (uint32_t i = lane; i < S; i += 32) {
        const double v = (double)px[i];
        if (BWD) { const double d = (double)pd[i]; a += d; b += d * v; }
        else { a += v; b += v * v; }
      }
    }
    a = warp_sum(a);
    b = warp_sum(b);
    if (lane == 0) { out[2 * pl] = a; out[2 * pl + 1] = b; }
  }
}

// chan[2c + j] = sum over n of ps[2 (n C + c) + j]: a warp per (c, j); lane l
// adds n = l, l + 32, ... in order, then a fixed shuffle tree (deterministic,
// and 32 loads in flight instead of one serial chain of N).
// Lane l's share of a channel's plane sums: q[l * step] + q[(l + 32) * step] + ...
// over n < N, added in that order with four loads issued ahead of their adds.
DCT_DEV double lane_plane_sum(const double* __restrict__ q, uint64_t step, uint32_t N, int lane) {
  double acc = 0.0;
  uint32_t n = lane;
  for (; n + 96 < N; n += 128) {
    const double a0 = q[n * step], a1 = q[(n + 32) * step], a2 = q[(n + 64) * step], a3 = q[(n + 96) * step];
    acc += a0;
    acc += a1;
    acc += a2;
    acc += a3;
  }
  for (; n < N; n += 32) acc += q[n * step];
  return acc;
}

__global__ void __launch_bounds__(256) k_bn_fold(const double* __restrict__ ps, uint32_t N, uint32_t C, double* chan) {
  pdl_entry();
  const uint32_t k = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;     // (c, j)
  const int lane = threadIdx.x & 31;
  if (k >= 2 * C) return;
  const uint32_t c = k >> 1, j = k & 1;
  double acc = lane_plane_sum(ps + 2 * (uint64_t)c + j, 2ull * C, N, lane);
  acc = warp_sum(acc);
  if (lane == 0) chan[k] = acc;
}

// The same fold for a sharded batch, in the same launch as the exchange over
// peer memory: lane 0 of the warp for sum k stores this rank's sum (record word
// k) into every peer's slot, then adds every rank's in rank order into out[k];
// block 0 also stores the header [count, valid, 2C, -] and writes out[2C], the
// global count (fold_sums).  The launch keeps every block resident, since each
// waits for the peers' puts.
__global__ void __launch_bounds__(256) k_bn_fold_xchg(const double* __restrict__ ps, uint32_t N, uint32_t C,
                                                      double* out, const __grid_constant__ PeerXfer p) {
  pdl_entry();
  bool gave_up = false;
  peer_put_header(p);
  const uint32_t nsum = 2 * C;
  const int lane = threadIdx.x & 31;
  const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
  for (uint32_t k = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; k < nsum; k += warps) {
    const uint32_t c = k >> 1, j = k & 1;
    double acc = lane_plane_sum(ps + 2 * (uint64_t)c + j, 2ull * C, N, lane);
    acc = warp_sum(acc);
    if (lane == 0) {
      peer_put_word(p, k, (unsigned long long)__double_as_longlong(acc));
      double tot = 0.0;
      for (int r = 0; r < p.world; ++r) {
        const double v = r == p.rank ? acc : peer_get_f64(p, r, k, gave_up);
        tot = r == 0 ? v : tot + v;
      }
      out[k] = tot;
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) fold_sums(PeerRecs{p, gave_up}, p.world, nsum, out, p.err, nsum);
  peer_sync(p, gave_up);
}

__global__ void k_bn_stats_final(const double* chan, uint32_t C, double cnt, float* mean, float* var, float* rm,
                                 float* rv, int training, float momentum, const double* cnt_dev) {
  pdl_entry();
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  if (cnt_dev) cnt = *cnt_dev;
  const double m = chan[2 * c] / cnt;
  const double v = fmax(0.0, chan[2 * c + 1] / cnt - m * m);
  mean[c] = (float)m;
  var[c] = (float)v;
  if (training) {
    const double mom = (double)momentum;
    const double unb = v * (cnt / fmax(1.0, cnt - 1.0));
    rm[c] = (float)((1.0 - mom) * (double)rm[c] + mom * m);
    rv[c] = (float)((1.0 - mom) * (double)rv[c] + mom * unb);
  }
}

__global__ void k_bn_bwd_final(const double* chan, uint32_t C, const float* mean, const float* var, float eps,
                               float* dgamma, float* dbeta) {
  pdl_entry();
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const double sdy = chan[2 * c], sdyx = chan[2 * c + 1];
  const double rstd = (double)rstd_of(var[c], eps);
  dgamma[c] = (float)((sdyx - (double)mean[c] * sdy) * rstd);
  dbeta[c] = (float)sdy;
}

// Apply kernels: chunked schedule over the flat NCHW array (one contiguous
// 16 KB slice per block, loads first); with S % 4 == 0 each float4 lies in one
// (n, c) plane, whose channel c = (i4 / (S/4)) % C comes from two fast
// divisions.  The per-channel constants are re-read through L1.  Elements at
// or beyond `limit` (the reference's groups*256 index space) are untouched.
constexpr int kBnU = 4;
constexpr uint64_t kBnChunk4 = 256ull * kBnU;

DCT_DEV float bn_fwd1(float v, float m, float r, float g, float b) {
  return __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, m), r), g), b);
}
DCT_DEV float bn_dx1(float xv, float d, float m, float r, float k1, float db, float dg, float mf) {
  const float xh = __fmul_rn(__fsub_rn(xv, m), r);
  return __fmul_rn(k1, __fsub_rn(d, __fdiv_rn(__fadd_rn(db, __fmul_rn(xh, dg)), mf)));
}

__global__ void __launch_bounds__(256) k_bn_forward_chunk(const float* __restrict__ x, const float* __restrict__ mean,
                                                          const float* __restrict__ var,
                                                          const float* __restrict__ gamma,
                                                          const float* __restrict__ beta, float* __restrict__ y,
                                                          uint32_t n4, FastDiv s4, FastDiv cdiv, float eps) {
  pdl_entry();
  const uint64_t base = (uint64_t)blockIdx.x * kBnChunk4 + threadIdx.x;
  float4 v[kBnU];
  uint32_t ch[kBnU];
#pragma unroll
  for (int k = 0; k < kBnU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i < n4) {
      v[k] = ld_stream4(x + 4 * i);
      const uint32_t pl = s4.div((uint32_t)i);
      ch[k] = pl - cdiv.div(pl) * cdiv.d;
    }
  }
#pragma unroll
  for (int k = 0; k < kBnU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i >= n4) continue;
    const uint32_t c = ch[k];
    const float m = ld_keep(mean + c), r = rstd_of(ld_keep(var + c), eps), g = ld_keep(gamma + c), b = ld_keep(beta + c);
    st_stream4(y + 4 * i, make_float4(bn_fwd1(v[k].x, m, r, g, b), bn_fwd1(v[k].y, m, r, g, b),
                                      bn_fwd1(v[k].z, m, r, g, b), bn_fwd1(v[k].w, m, r, g, b)));
  }
}

__global__ void __launch_bounds__(256) k_bn_dx_chunk(const float* __restrict__ x, const float* __restrict__ dy,
                                                     const float* __restrict__ mean, const float* __restrict__ var,
                                                     const float* __restrict__ gamma,
                                                     const float* __restrict__ dgamma,
                                                     const float* __restrict__ dbeta, float* __restrict__ dx,
                                                     uint32_t n4, FastDiv s4, FastDiv cdiv, float eps, float mf,
                                                     const double* __restrict__ cnt_dev) {
  pdl_entry();
  if (cnt_dev) mf = (float)*cnt_dev;
  const uint64_t base = (uint64_t)blockIdx.x * kBnChunk4 + threadIdx.x;
  float4 a[kBnU], d[kBnU];
  uint32_t ch[kBnU];
#pragma unroll
  for (int k = 0; k < kBnU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i < n4) {
      a[k] = ld_stream4(x + 4 * i);
      d[k] = ld_stream4(dy + 4 * i);
      const uint32_t pl = s4.div((uint32_t)i);
      ch[k] = pl - cdiv.div(pl) * cdiv.d;
    }
  }
#pragma unroll
  for (int k = 0; k < kBnU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i >= n4) continue;
    const uint32_t c = ch[k];
    const float m = ld_keep(mean + c), r = rstd_of(ld_keep(var + c), eps);
    const float k1 = __fmul_rn(ld_keep(gamma + c), r), dg = ld_keep(dgamma + c), db = ld_keep(dbeta + c);
    st_stream4(dx + 4 * i, make_float4(bn_dx1(a[k].x, d[k].x, m, r, k1, db, dg, mf),
                                       bn_dx1(a[k].y, d[k].y, m, r, k1, db, dg, mf),
                                       bn_dx1(a[k].z, d[k].z, m, r, k1, db, dg, mf),
                                       bn_dx1(a[k].w, d[k].w, m, r, k1, db, dg, mf)));
  }
}

// Scalar fallbacks (S % 4 != 0, unaligned, or > 2^34 elements): one warp per
// plane; elements >= limit untouched.
__global__ void __launch_bounds__(256) k_bn_forward(const float* __restrict__ x, const float* __restrict__ mean,
                                                    const float* __restrict__ var, const float* __restrict__ gamma,
                                                    const float* __restrict__ beta, float* __restrict__ y,
                                                    uint64_t planes, uint32_t C, uint32_t S, float eps,
                                                    uint64_t limit) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const uint64_t gw = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint64_t nw = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  for (uint64_t pl = gw; pl < planes; pl += nw) {
    const uint32_t c = (uint32_t)(pl % C);
    const float m = mean[c], r = rstd_of(var[c], eps), g = gamma[c], b = beta[c];
    const uint64_t base = pl * S;
    if (base >= limit) break;
    for (uint32_t i = lane; i < S; i += 32)
      if (base + i < limit) y[base + i] = bn_fwd1(x[base + i], m, r, g, b);
  }
}

__global__ void __launch_bounds__(256) k_bn_backward_dx(const float* __restrict__ x, const float* __restrict__ dy,
                                                        const float* __restrict__ mean, const float* __restrict__ var,
                                                        const float* __restrict__ gamma,
                                                        const float* __restrict__ dgamma,
                                                        const float* __restrict__ dbeta, float* __restrict__ dx,
                                                        uint64_t planes, uint32_t C, uint32_t S, float eps, float mf,
                                                        uint64_t limit, const double* __restrict__ cnt_dev) {
  pdl_entry();
  if (cnt_dev) mf = (float)*cnt_dev;
  const int lane = threadIdx.x & 31;
  const uint64_t gw = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint64_t nw = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  for (uint64_t pl = gw; pl < planes; pl += nw) {
    const uint32_t c = (uint32_t)(pl % C);
    const float m = mean[c], r = rstd_of(var[c], eps), dg = dgamma[c], db = dbeta[c];
    const float k1 = __fmul_rn(gamma[c], r);
    const uint64_t base = pl * S;
    if (base >= limit) break;
    for (uint32_t i = lane; i < S; i += 32)
      if (base + i < limit) dx[base + i] = bn_dx1(x[base + i], dy[base + i], m, r, k1, db, dg, mf);
  }
}

unsigned plane_blocks(uint64_t planes) {
  const DevInfo& d = dev_info();
  const uint64_t warps = planes;
  uint64_t blocks = (warps + 7) / 8;
  const uint64_t cap = (uint64_t)d.sm_count * (d.max_threads_per_sm / 256);
  return (unsigned)(blocks < cap ? (blocks ? blocks : 1) : cap);
}

}  // namespace

size_t bn_ws_bytes(uint32_t N, uint32_t C) {
  return ((size_t)N * C * 2 + (size_t)C * 2) * sizeof(double);
}

cudaError_t launch_bn_plane_sums(const float* x, const float* dy, uint32_t N, uint32_t C, uint32_t S,
                                 double* plane_sums, cudaStream_t st) {
  const uint64_t planes = (uint64_t)N * C;
  if (planes == 0) return cudaSuccess;
  const bool vec = (S % 4 == 0) && aligned16_h(x) && (!dy || aligned16_h(dy));
  const unsigned blocks = plane_blocks(planes);
  if (dy) {
    if (vec) launch_pdl(k_bn_plane_sums<true, true>, dim3(blocks), dim3(256), 0, st, x, dy, planes, S, plane_sums);
    else launch_pdl(k_bn_plane_sums<true, false>, dim3(blocks), dim3(256), 0, st, x, dy, planes, S, plane_sums);
  } else {
    if (vec) launch_pdl(k_bn_plane_sums<false, true>, dim3(blocks), dim3(256), 0, st, x, nullptr, planes, S, plane_sums);
    else launch_pdl(k_bn_plane_sums<false, false>, dim3(blocks), dim3(256), 0, st, x, nullptr, planes, S, plane_sums);
  }
  return cudaGetLastError();
}

cudaError_t launch_bn_fold(const double* plane_sums, uint32_t N, uint32_t C, double* chan, cudaStream_t st) {
  if (C == 0) return cudaSuccess;
  launch_pdl(k_bn_fold, dim3((unsigned)((2ull * C * 32 + 255) / 256)), dim3(256), 0, st, plane_sums, N, C, chan);
  return cudaGetLastError();
}

cudaError_t launch_bn_fold_xchg(const double* plane_sums, uint32_t N, uint32_t C, const PeerXfer& p, double* out,
                                cudaStream_t st) {
  if (C == 0) return cudaErrorInvalidValue;
  static int occ = 0;
  if (occ == 0) {
    int b = 0;
    const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_bn_fold_xchg, 256, 0);
    occ = (e == cudaSuccess && b > 0) ? b : 1;
    cudaGetLastError();
  }
  const uint64_t need = (2ull * C * 32 + 255) / 256, cap = (uint64_t)dev_info().sm_count * (uint64_t)occ;
  launch_pdl(k_bn_fold_xchg, dim3((unsigned)(need < cap ? need : cap)), dim3(256), 0, st, plane_sums, N, C, out, p);
  return cudaGetLastError();
}

cudaError_t launch_bn_stats_final(const double* chan, uint32_t C, double cnt, float* mean, float* var, float* rmean,
                                  float* rvar, bool training, float momentum, cudaStream_t st, const double* cnt_dev) {
  if (C == 0) return cudaSuccess;
  launch_pdl(k_bn_stats_final, dim3((C + 255) / 256), dim3(256), 0, st, chan, C, cnt, mean, var, rmean, rvar, training ? 1 : 0,
                                                      momentum, cnt_dev);
  return cudaGetLastError();
}

cudaError_t launch_bn_bwd_final(const double* chan, uint32_t C, const float* mean, const float* var, float eps,
                                float* dgamma, float* dbeta, cudaStream_t st) {
  if (C == 0) return cudaSuccess;
  launch_pdl(k_bn_bwd_final, dim3((C + 255) / 256), dim3(256), 0, st, chan, C, mean, var, eps, dgamma, dbeta);
  return cudaGetLastError();
}

cudaError_t launch_bn_forward(const float* x, const float* mean, const float* var, const float* gamma,
                              const float* beta, float* y, uint32_t N, uint32_t C, uint32_t S, float eps,
                              uint64_t limit, cudaStream_t st) {
  const uint64_t planes = (uint64_t)N * C;
  if (planes == 0 || S == 0) return cudaSuccess;
  const uint64_t total = planes * S;
  if (limit > total) limit = total;
  const bool vec = (S % 4 == 0) && (limit % 4 == 0) && limit / 4 < 0xffffffffull && aligned16_h(x) && aligned16_h(y);
  if (vec) {
    const uint32_t n4 = (uint32_t)(limit / 4);
    launch_pdl(k_bn_forward_chunk, dim3((unsigned)((n4 + kBnChunk4 - 1) / kBnChunk4)), dim3(256), 0, st, 
        x, mean, var, gamma, beta, y, n4, FastDiv(S / 4), FastDiv(C), eps);
  } else {
    launch_pdl(k_bn_forward, dim3(plane_blocks(planes)), dim3(256), 0, st, x, mean, var, gamma, beta, y, planes, C, S, eps, limit);
  }
  return cudaGetLastError();
}

cudaError_t launch_bn_backward_dx(const float* x, const float* dy, const float* mean, const float* var,
                                  const float* gamma, const float* dgamma, const float* dbeta, float* dx, uint32_t N,
                                  uint32_t C, uint32_t S, float eps, uint64_t limit, cudaStream_t st,
                                  const double* cnt_dev) {
  const uint64_t planes = (uint64_t)N * C;
  if (planes == 0 || S == 0) return cudaSuccess;
  const uint64_t total = planes * S;
  if (limit > total) limit = total;
  const float mf = (float)((uint32_t)(N * S));     // HLSL: (float)(N * S) in uint arithmetic
  const bool vec = (S % 4 == 0) && (limit % 4 == 0) && limit / 4 < 0xffffffffull && aligned16_h(x) &&
                   aligned16_h(dy) && aligned16_h(dx);
  if (vec) {
    const uint32_t n4 = (uint32_t)(limit / 4);
    launch_pdl(k_bn_dx_chunk, dim3((unsigned)((n4 + kBnChunk4 - 1) / kBnChunk4)), dim3(256), 0, st, 
        x, dy, mean, var, gamma, dgamma, dbeta, dx, n4, FastDiv(S / 4), FastDiv(C), eps, mf, cnt_dev);
  } else {
    launch_pdl(k_bn_backward_dx, dim3(plane_blocks(planes)), dim3(256), 0, st, x, dy, mean, var, gamma, dgamma, dbeta, dx, planes, C,
                                                            S, eps, mf, limit, cnt_dev);
  }
  return cudaGetLastError();
}

}  // namespace dct
