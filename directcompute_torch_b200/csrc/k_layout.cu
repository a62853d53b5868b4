// Layout kernels beside the hot path: nearest upsample and its gradient
// (nn_upsample.hlsl, nn_upsample_backward.hlsl), channel concat / slice
// (nn_concat_insert.hlsl, nn_slice.hlsl), max pooling (nn_maxpool_forward.hlsl,
// nn_maxpool_backward.hlsl, engine.cpp:880-929) and the conv output / gradient
// reshapes (nn_conv_reshape.hlsl, nn_conv_grad_reshape.hlsl,
// nn_conv_grad_reshape_relu.hlsl).
//
// Each is an HBM-bound copy, gather or scatter with a few flops per element.
// Index arithmetic is 32-bit like the HLSL's `uint` (the host refuses index
// spaces past 2^32) with FastDiv for the runtime divisors.  Every op has a
// 128-bit path for the shapes the reference produces (rows that are multiples
// of 4 floats, full coverage) and a scalar path for ragged shapes and partial
// group counts; both compute identical values.  The 128-bit paths use the
// chunked schedule of the elementwise kernels: block b owns units
// [b*256*U, (b+1)*256*U), each thread loads its U units (strided by the block
// size, so every instruction is coalesced) before it stores any.
#include "dct_common.cuh"
#include "kernels.h"

namespace dct {
namespace {

constexpr int kT = 256;
constexpr uint32_t kNoIndex = 0xFFFFFFFFu;        // maxpool: nothing beat the start value
constexpr float kPoolStart = -1e30f;              // nn_maxpool_forward.hlsl:27

DCT_DEV uint32_t gtid() { return blockIdx.x * blockDim.x + threadIdx.x; }
DCT_DEV uint32_t gstride() { return gridDim.x * blockDim.x; }

// ---------------------------------------------------------------------------
// nearest upsample by integer factors
// ---------------------------------------------------------------------------
struct UpGeom {
  FastDiv outW, outH, sH, sW;
  uint32_t inH, inW;
};

// Out[i] = X[(bc*inH + h/sH)*inW + w/sW] for i < n  (nn_upsample.hlsl:21-32)
__global__ void __launch_bounds__(kT) k_upsample(const float* __restrict__ x, float* __restrict__ y, uint32_t n,
                                                 UpGeom g) {
  pdl_entry();
  for (uint32_t i = gtid(); i < n; i += gstride()) {
    const uint32_t row = g.outW.div(i), w = i - row * g.outW.d;
    const uint32_t bc = g.outH.div(row), h = row - bc * g.outH.d;
    st_stream(y + i, __ldg(x + (bc * g.inH + g.sH.div(h)) * g.inW + g.sW.div(w)));
  }
}

// Output-major, four outputs of one row per unit (outW % 4 == 0, every output
// written), chunked.  SW = 1, 2, 4: the unit's inputs are one float4, one
// float2 or one float of the input row; SW = 0: any scale, four loads.  Input
// lines are re-read from L2 by the sH output rows they feed.
template <int SW>
__global__ void __launch_bounds__(kT) k_upsample_chunk(const float* __restrict__ x, float* __restrict__ y,
                                                       uint32_t nq, FastDiv outWq, UpGeom g) {
  pdl_entry();
  constexpr int U = 4;
  const uint32_t q0 = blockIdx.x * (kT * U) + threadIdx.x;
  float4 v[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const uint32_t q = q0 + k * kT;
    if (q >= nq) break;
    const uint32_t row = outWq.div(q);
    const uint32_t w0 = (q - row * outWq.d) * 4;
    const uint32_t bc = g.outH.div(row), h = row - bc * g.outH.d;
    const float* src = x + (bc * g.inH + g.sH.div(h)) * g.inW;
    if constexpr (SW == 1) {
      v[k] = __ldg(reinterpret_cast<const float4*>(src + w0));
    } else if constexpr (SW == 2) {
      const float2 a = __ldg(reinterpret_cast<const float2*>(src + w0 / 2));
      v[k] = make_float4(a.x, a.x, a.y, a.y);
    } else if constexpr (SW == 4) {
      const float a = __ldg(src + w0 / 4);
      v[k] = make_float4(a, a, a, a);
    } else {
      uint32_t wi = g.sW.div(w0), r = w0 - wi * g.sW.d;
      float t[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        t[c] = __ldg(src + wi);
        if (++r == g.sW.d) { r = 0; ++wi; }
      }
      v[k] = make_float4(t[0], t[1], t[2], t[3]);
    }
  }
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const uint32_t q = q0 + k * kT;
    if (q >= nq) break;
    st_stream4(y + 4 * (size_t)q, v[k]);
  }
}

struct UpBackGeom {
  FastDiv inW, inH;
  uint32_t outH, outW, sH, sW;
};

// DX[i] = sum of the sH x sW block of DY, rows outer / columns inner, skipping
// positions past outH / outW, accumulated in fp32 from 0.0f
// (nn_upsample_backward.hlsl:21-44)
__global__ void __launch_bounds__(kT) k_upsample_bwd(const float* __restrict__ dy, float* __restrict__ dx,
                                                     uint32_t n, UpBackGeom g) {
  pdl_entry();
  for (uint32_t i = gtid(); i < n; i += gstride()) {
    const uint32_t row = g.inW.div(i), w = i - row * g.inW.d;
    const uint32_t bc = g.inH.div(row), h = row - bc * g.inH.d;
    const uint32_t h0 = h * g.sH, w0 = w * g.sW;
    float sum = 0.0f;
    for (uint32_t sh = 0; sh < g.sH; ++sh) {
      const uint32_t ho = h0 + sh;
      if (ho >= g.outH) break;                       // every later row is past the edge too
      const float* r = dy + (bc * g.outH + ho) * g.outW;
      for (uint32_t sw = 0; sw < g.sW; ++sw) {
        const uint32_t wo = w0 + sw;
        if (wo >= g.outW) break;
        sum += ld_stream(r + wo);
      }
    }
    st_stream(dx + i, sum);
  }
}

// The 2x2 case with outH == 2*inH, outW == 2*inW, inW % 4 == 0: four inputs of
// one row per unit from two float4 pairs of DY, summed in the shader's order;
// chunked, two units per thread.
__global__ void __launch_bounds__(kT) k_upsample_bwd_2x2(const float* __restrict__ dy, float* __restrict__ dx,
                                                         uint32_t nq, FastDiv inWq, uint32_t inW) {
  pdl_entry();
  constexpr int U = 2;
  const uint32_t q0 = blockIdx.x * (kT * U) + threadIdx.x;
  float4 a0[U], a1[U], b0[U], b1[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const uint32_t q = q0 + k * kT;
    if (q >= nq) break;
    const uint32_t row = inWq.div(q);                // bc*inH + h
    const uint32_t w0 = (q - row * inWq.d) * 4;
    const float* r0 = dy + (size_t)(2 * row) * (2 * inW) + 2 * w0;
    const float* r1 = r0 + 2 * inW;
    a0[k] = ld_stream4(r0); a1[k] = ld_stream4(r0 + 4); b0[k] = ld_stream4(r1); b1[k] = ld_stream4(r1 + 4);
  }
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const uint32_t q = q0 + k * kT;
    if (q >= nq) break;
    float4 o;
    o.x = 0.0f; o.x += a0[k].x; o.x += a0[k].y; o.x += b0[k].x; o.x += b0[k].y;
    o.y = 0.0f; o.y += a0[k].z; o.y += a0[k].w; o.y += b0[k].z; o.y += b0[k].w;
    o.z = 0.0f; o.z += a1[k].x; o.z += a1[k].y; o.z += b1[k].x; o.z += b1[k].y;
    o.w = 0.0f; o.w += a1[k].z; o.w += a1[k].w; o.w += b1[k].z; o.w += b1[k].w;
    st_stream4(dx + 4 * (size_t)q, o);
  }
}

// ---------------------------------------------------------------------------
// channel concat / slice: rows of L = c_in*S floats at pitch c_out*S, offset c_off*S
// ---------------------------------------------------------------------------
// concat (nn_concat_insert.hlsl:18-26): dst[q*pitch + off + r] = src[i]
// slice  (nn_slice.hlsl:18-26):         dst[i] = src[q*pitch + off + r]   (i = q*L + r < n)
template <bool SLICE>
__global__ void __launch_bounds__(kT) k_channel_copy(const float* __restrict__ src, float* __restrict__ dst,
                                                     uint32_t n, FastDiv L, uint32_t pitch, uint32_t off) {
  pdl_entry();
  for (uint32_t i = gtid(); i < n; i += gstride()) {
    const uint32_t q = L.div(i), r = i - q * L.d;
    const uint32_t j = q * pitch + off + r;
    if (SLICE) st_stream(dst + i, ld_stream(src + j));
    else st_stream(dst + j, ld_stream(src + i));
  }
}
// the same with L, pitch, off and n multiples of 4: float4 units, chunked
template <bool SLICE>
__global__ void __launch_bounds__(kT) k_channel_copy4(const float* __restrict__ src, float* __restrict__ dst,
                                                      uint32_t nq, FastDiv Lq, uint32_t pitch, uint32_t off) {
  pdl_entry();
  constexpr int U = 4;
  const uint32_t q0 = blockIdx.x * (kT * U) + threadIdx.x;
  float4 v[U];
  size_t at[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const uint32_t q = q0 + k * kT;
    if (q >= nq) break;
    const uint32_t b = Lq.div(q), r = (q - b * Lq.d) * 4;
    const size_t j = (size_t)b * pitch + off + r, i = 4 * (size_t)q;
    v[k] = ld_stream4(src + (SLICE ? j : i));
    at[k] = SLICE ? i : j;
  }
#pragma unroll
  for (int k = 0; k < U; ++k) {
    if (q0 + k * kT >= nq) break;
    st_stream4(dst + at[k], v[k]);
  }
}

// ---------------------------------------------------------------------------
// max pooling
// ---------------------------------------------------------------------------
DCT_DEV void pool_take(float v, uint32_t k, float& best, uint32_t& bi) {
  if (v > best) { best = v; bi = k; }                // strict: the first maximum wins, NaN never
}

// covered outputs (bc < lb, oh < lh, ow < lw), flattened (nn_maxpool_forward.hlsl:22-51)
__global__ void __launch_bounds__(kT) k_maxpool_fwd(const float* __restrict__ x, float* __restrict__ out,
                                                    uint32_t* __restrict__ idx, uint32_t n, FastDiv lw, FastDiv lh,
                                                    PoolShape g) {
  pdl_entry();
  for (uint32_t i = gtid(); i < n; i += gstride()) {
    const uint32_t t = lw.div(i), ow = i - t * lw.d;
    const uint32_t bc = lh.div(t), oh = t - bc * lh.d;
    const uint32_t base = bc * (g.inH * g.inW);
    const uint32_t h0 = oh * g.s, w0 = ow * g.s;
    float best = kPoolStart;
    uint32_t bi = kNoIndex;
    for (uint32_t ph = 0; ph < g.p; ++ph) {
      const uint32_t ih = h0 + ph;
      if (ih >= g.inH) break;
      for (uint32_t pw = 0; pw < g.p; ++pw) {
        const uint32_t iw = w0 + pw;
        if (iw >= g.inW) break;
        const uint32_t k = base + ih * g.inW + iw;
        pool_take(__ldg(x + k), k, best, bi);
      }
    }
    const uint32_t o = bc * (g.outH * g.outW) + oh * g.outW + ow;
    out[o] = best;
    idx[o] = bi;
  }
}

// 2x2 windows, stride 2, every output, inW % 4 == 0: two outputs of one row
// per unit from one float4 of each of the window's two input rows; chunked.
__global__ void __launch_bounds__(kT) k_maxpool2x2(const float* __restrict__ x, float* __restrict__ out,
                                                   uint32_t* __restrict__ idx, uint32_t nq, FastDiv outWh,
                                                   FastDiv outH, uint32_t inH, uint32_t inW) {
  pdl_entry();
  constexpr int U = 4;
  const uint32_t q0 = blockIdx.x * (kT * U) + threadIdx.x;
  float4 a[U], b[U];
  uint32_t k0[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const uint32_t q = q0 + k * kT;
    if (q >= nq) break;
    const uint32_t row = outWh.div(q);               // bc*outH + oh
    const uint32_t c2 = q - row * outWh.d;
    const uint32_t bc = outH.div(row), oh = row - bc * outH.d;
    k0[k] = (bc * inH + 2 * oh) * inW + 4 * c2;
    a[k] = ld_stream4(x + k0[k]);
    b[k] = ld_stream4(x + k0[k] + inW);
  }
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const uint32_t q = q0 + k * kT;
    if (q >= nq) break;
    const uint32_t e = k0[k], f = e + inW;
    float m0 = kPoolStart, m1 = kPoolStart;
    uint32_t i0 = kNoIndex, i1 = kNoIndex;
    pool_take(a[k].x, e, m0, i0); pool_take(a[k].y, e + 1, m0, i0);
    pool_take(b[k].x, f, m0, i0); pool_take(b[k].y, f + 1, m0, i0);
    pool_take(a[k].z, e + 2, m1, i1); pool_take(a[k].w, e + 3, m1, i1);
    pool_take(b[k].z, f + 2, m1, i1); pool_take(b[k].w, f + 3, m1, i1);
    const size_t o = 2 * (size_t)q;                  // = row*outW + 2*c2
    *reinterpret_cast<float2*>(out + o) = make_float2(m0, m1);
    *reinterpret_cast<uint2*>(idx + o) = make_uint2(i0, i1);
  }
}

// dInput[idx[o]] = dZ[o] for covered outputs whose index is not 0xFFFFFFFF;
// indices past the buffer are dropped as D3D11 drops out-of-range UAV writes
// (nn_maxpool_backward.hlsl:18-24)
__global__ void __launch_bounds__(kT) k_maxpool_scatter(const float* __restrict__ dz, const uint32_t* __restrict__ idx,
                                                        float* __restrict__ d, uint64_t dcount, uint32_t n,
                                                        FastDiv lw, FastDiv lh, uint32_t outH, uint32_t outW,
                                                        bool full) {
  pdl_entry();
  for (uint32_t i = gtid(); i < n; i += gstride()) {
    uint32_t o = i;
    if (!full) {
      const uint32_t t = lw.div(i), ow = i - t * lw.d;
      const uint32_t bc = lh.div(t), oh = t - bc * lh.d;
      o = bc * (outH * outW) + oh * outW + ow;
    }
    const uint32_t k = idx[o];
    if (k != kNoIndex && k < dcount) d[k] = dz[o];
  }
}

// Is flat input index k inside window (bc, oh, ow)?
DCT_DEV bool in_window(uint32_t k, uint32_t bc, uint32_t oh, uint32_t ow, const FastDiv& inW, const PoolShape& g) {
  const uint32_t plane = g.inH * g.inW;
  const uint32_t kr = k - bc * plane;                // wraps past `plane` when k is in an earlier plane
  if (k < bc * plane || kr >= plane) return false;
  const uint32_t kh = inW.div(kr), kw = kr - kh * inW.d;
  return kh - oh * g.s < g.p && kw - ow * g.s < g.p && kh >= oh * g.s && kw >= ow * g.s;
}

// MaxPoolBackwardFused in one pass when windows do not overlap (s >= p): input
// element e of plane bc at (ih, iw) lies in at most one window o and becomes
// dZ[o] when idx[o] names it, else 0 -- the zeroed buffer plus scatter of
// engine.cpp:905-929, written once and coalesced.  An index outside its own
// window (the index buffer rewritten after the forward pass) sets *flag and is
// applied by k_maxpool_fixup.
__global__ void __launch_bounds__(kT) k_maxpool_gather(const float* __restrict__ dz, const uint32_t* __restrict__ idx,
                                                       float* __restrict__ d, uint32_t n, FastDiv inW, FastDiv inH,
                                                       FastDiv s, PoolShape g, uint32_t* flag) {
  pdl_entry();
  for (uint32_t e = gtid(); e < n; e += gstride()) {
    const uint32_t row = inW.div(e), iw = e - row * inW.d;
    const uint32_t bc = inH.div(row), ih = row - bc * inH.d;
    const uint32_t oh = s.div(ih), ow = s.div(iw);
    const uint32_t dh = ih - oh * s.d, dw = iw - ow * s.d;
    float v = 0.0f;
    if (oh < g.outH && ow < g.outW && dh < g.p && dw < g.p) {
      const uint32_t o = bc * (g.outH * g.outW) + oh * g.outW + ow;
      const uint32_t k = __ldg(idx + o);
      if (k == e) v = __ldg(dz + o);
      else if (dh == 0 && dw == 0 && k != kNoIndex && k < n && !in_window(k, bc, oh, ow, inW, g)) atomicOr(flag, 1u);
    }
    st_stream(d + e, v);
  }
}

// The same for 2x2 windows at stride 2 with inW % 4 == 0: four inputs of one
// row per unit from the (index, dZ) pairs of the two windows above them; chunked.
__global__ void __launch_bounds__(kT) k_maxpool_gather2x2(const float* __restrict__ dz,
                                                          const uint32_t* __restrict__ idx, float* __restrict__ d,
                                                          uint32_t nq, FastDiv inWq, FastDiv inH, FastDiv inW,
                                                          PoolShape g, uint32_t* flag) {
  pdl_entry();
  constexpr int U = 4;
  const uint32_t n = g.bc * g.inH * g.inW;
  const uint32_t q0 = blockIdx.x * (kT * U) + threadIdx.x;
  uint2 kk[U];
  float2 zz[U];
  bool top[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const uint32_t q = q0 + k * kT;
    kk[k] = make_uint2(kNoIndex, kNoIndex);
    zz[k] = make_float2(0.0f, 0.0f);
    top[k] = false;
    if (q >= nq) break;
    const uint32_t row = inWq.div(q), j = q - row * inWq.d;  // input row, float4 column
    const uint32_t bc = inH.div(row), ih = row - bc * inH.d;
    const uint32_t oh = ih >> 1;
    if (oh < g.outH) {
      const uint32_t o = bc * (g.outH * g.outW) + oh * g.outW + 2 * j;
      kk[k] = __ldg(reinterpret_cast<const uint2*>(idx + o));
      zz[k] = __ldg(reinterpret_cast<const float2*>(dz + o));
      top[k] = (ih & 1) == 0;                        // the windows' top rows check their indices
    }
  }
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const uint32_t q = q0 + k * kT;
    if (q >= nq) break;
    const uint32_t e0 = 4 * q;
    const uint2 kx = kk[k];
    const float2 z = zz[k];
    float4 v;
    v.x = kx.x == e0 ? z.x : 0.0f;
    v.y = kx.x == e0 + 1 ? z.x : 0.0f;
    v.z = kx.y == e0 + 2 ? z.y : 0.0f;
    v.w = kx.y == e0 + 3 ? z.y : 0.0f;
    if (top[k]) {
      const uint32_t k1 = e0 + inW.d;                // first element of the second window row
      const bool ok0 = kx.x == kNoIndex || kx.x >= n || kx.x == e0 || kx.x == e0 + 1 || kx.x == k1 || kx.x == k1 + 1;
      const bool ok1 = kx.y == kNoIndex || kx.y >= n || kx.y == e0 + 2 || kx.y == e0 + 3 || kx.y == k1 + 2 ||
                       kx.y == k1 + 3;
      if (!(ok0 && ok1)) atomicOr(flag, 1u);
    }
    st_stream4(d + (size_t)e0, v);
  }
}

// Applies indices that point outside their own window (only when the gather
// set *flag), then clears the flag.  One block: the flag is read by every
// thread before the barrier and cleared after it.
__global__ void __launch_bounds__(1024) k_maxpool_fixup(const float* __restrict__ dz, const uint32_t* __restrict__ idx,
                                                        float* __restrict__ d, uint32_t n, uint32_t nout, FastDiv outW,
                                                        FastDiv outH, FastDiv inW, PoolShape g, uint32_t* flag) {
  pdl_entry();
  if (*(volatile uint32_t*)flag == 0) return;
  for (uint32_t o = threadIdx.x; o < nout; o += blockDim.x) {
    const uint32_t k = idx[o];
    if (k == kNoIndex || k >= n) continue;
    const uint32_t r = outW.div(o), ow = o - r * outW.d;
    const uint32_t bc = outH.div(r), oh = r - bc * outH.d;
    if (!in_window(k, bc, oh, ow, inW, g)) d[k] = dz[o];
  }
  __syncthreads();
  if (threadIdx.x == 0) *flag = 0;
}

// ---------------------------------------------------------------------------
// conv output / gradient reshapes: rows of P = OH*OW pixels move between
// [OC][B][P] (the matmul layout) and [B][OC][P] (NCHW)
// ---------------------------------------------------------------------------
template <int ACT>
DCT_DEV float conv_act(float z) {                    // nn_conv_reshape.hlsl:22-24
  if constexpr (ACT == 1) return z > 0.0f ? z : 0.0f;    // max(0, z): NaN -> 0
  else if constexpr (ACT == 2) return tanhf(z);
  else return z;
}

// out[b, oc, px] = act(mm[oc, b*P + px] + bias[oc]) for covered (oc < loc, b*P+px < lbp)
template <int ACT>
__global__ void __launch_bounds__(kT) k_conv_reshape(const float* __restrict__ mm, const float* __restrict__ bias,
                                                     float* __restrict__ out, uint32_t n, FastDiv lbp, FastDiv P,
                                                     uint32_t OC, uint32_t BP) {
  pdl_entry();
  for (uint32_t i = gtid(); i < n; i += gstride()) {
    const uint32_t oc = lbp.div(i), bp = i - oc * lbp.d;
    const uint32_t b = P.div(bp), px = bp - b * P.d;
    st_stream(out + (b * OC + oc) * P.d + px, conv_act<ACT>(ld_stream(mm + oc * BP + bp) + __ldg(bias + oc)));
  }
}
// every output, P % 4 == 0: NCHW float4 units, chunked
template <int ACT>
__global__ void __launch_bounds__(kT) k_conv_reshape4(const float* __restrict__ mm, const float* __restrict__ bias,
                                                      float* __restrict__ out, uint32_t nq, FastDiv Pq, FastDiv OC,
                                                      uint32_t P, uint32_t BP) {
  pdl_entry();
  constexpr int U = 4;
  const uint32_t q0 = blockIdx.x * (kT * U) + threadIdx.x;
  float4 v[U];
  float bv[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const uint32_t q = q0 + k * kT;
    if (q >= nq) break;
    const uint32_t row = Pq.div(q), px = (q - row * Pq.d) * 4;
    const uint32_t b = OC.div(row), oc = row - b * OC.d;
    bv[k] = __ldg(bias + oc);
    v[k] = ld_stream4(mm + (size_t)oc * BP + (size_t)b * P + px);
  }
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const uint32_t q = q0 + k * kT;
    if (q >= nq) break;
    float4 w = v[k];
    w.x = conv_act<ACT>(w.x + bv[k]);
    w.y = conv_act<ACT>(w.y + bv[k]);
    w.z = conv_act<ACT>(w.z + bv[k]);
    w.w = conv_act<ACT>(w.w + bv[k]);
    st_stream4(out + 4 * (size_t)q, w);
  }
}

// out[oc, b*P + px] = dZ[b, oc, px], zeroed where fwd <= 0 (RELU)
// (nn_conv_grad_reshape.hlsl:24-27, nn_conv_grad_reshape_relu.hlsl:29-38)
template <bool RELU>
__global__ void __launch_bounds__(kT) k_conv_grad_reshape(const float* __restrict__ dz, const float* __restrict__ fwd,
                                                          float* __restrict__ out, uint32_t n, FastDiv lbp, FastDiv P,
                                                          uint32_t OC, uint32_t BP) {
  pdl_entry();
  for (uint32_t i = gtid(); i < n; i += gstride()) {
    const uint32_t oc = lbp.div(i), bp = i - oc * lbp.d;
    const uint32_t b = P.div(bp), px = bp - b * P.d;
    const uint32_t src = (b * OC + oc) * P.d + px;
    float gv = ld_stream(dz + src);
    if (RELU && ld_stream(fwd + src) <= 0.0f) gv = 0.0f;
    st_stream(out + oc * BP + bp, gv);
  }
}
template <bool RELU>
__global__ void __launch_bounds__(kT) k_conv_grad_reshape4(const float* __restrict__ dz, const float* __restrict__ fwd,
                                                           float* __restrict__ out, uint32_t nq, FastDiv BPq,
                                                           FastDiv Pq, uint32_t OC, uint32_t P) {
  pdl_entry();
  constexpr int U = 4;
  const uint32_t q0 = blockIdx.x * (kT * U) + threadIdx.x;
  float4 gv[U], f[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const uint32_t q = q0 + k * kT;
    if (q >= nq) break;
    const uint32_t oc = BPq.div(q), bq = q - oc * BPq.d;
    const uint32_t b = Pq.div(bq), pq = bq - b * Pq.d;
    const size_t src = ((size_t)b * OC + oc) * P + 4 * (size_t)pq;
    gv[k] = ld_stream4(dz + src);
    if (RELU) f[k] = ld_stream4(fwd + src);
  }
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const uint32_t q = q0 + k * kT;
    if (q >= nq) break;
    float4 g = gv[k];
    if (RELU) {
      if (f[k].x <= 0.0f) g.x = 0.0f;
      if (f[k].y <= 0.0f) g.y = 0.0f;
      if (f[k].z <= 0.0f) g.z = 0.0f;
      if (f[k].w <= 0.0f) g.w = 0.0f;
    }
    st_stream4(out + 4 * (size_t)q, g);
  }
}

template <typename K, typename... A>
cudaError_t go(K kernel, uint64_t work, cudaStream_t st, A... a) {
  return launch_pdl(kernel, dim3(grid_for(work, kT, 2)), dim3(kT), 0, st, a...);
}
// chunked kernels: one block per kT*U units
template <int U, typename K, typename... A>
cudaError_t chunked(K kernel, uint32_t units, cudaStream_t st, A... a) {
  return launch_pdl(kernel, dim3((units + kT * U - 1) / (kT * U)), dim3(kT), 0, st, a...);
}

}  // namespace

cudaError_t launch_upsample(const float* x, float* y, uint32_t n, uint32_t total, uint32_t inH, uint32_t inW,
                            uint32_t outH, uint32_t outW, uint32_t sH, uint32_t sW, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  UpGeom g{FastDiv(outW), FastDiv(outH), FastDiv(sH), FastDiv(sW), inH, inW};
  if (n == total && outW % 4 == 0 && aligned16_h(x) && aligned16_h(y)) {
    const uint32_t nq = n / 4;
    const FastDiv q(outW / 4);
    const unsigned grid = (nq + kT * 4 - 1) / (kT * 4);
    if (sW == 1 && inW % 4 == 0) launch_pdl(k_upsample_chunk<1>, dim3(grid), dim3(kT), 0, st, x, y, nq, q, g);
    else if (sW == 2 && inW % 2 == 0) launch_pdl(k_upsample_chunk<2>, dim3(grid), dim3(kT), 0, st, x, y, nq, q, g);
    else if (sW == 4) launch_pdl(k_upsample_chunk<4>, dim3(grid), dim3(kT), 0, st, x, y, nq, q, g);
    else launch_pdl(k_upsample_chunk<0>, dim3(grid), dim3(kT), 0, st, x, y, nq, q, g);
    return cudaGetLastError();
  }
  return go(k_upsample, n, st, x, y, n, g);
}

cudaError_t launch_upsample_backward(const float* dy, float* dx, uint32_t n, uint32_t total, uint32_t inH,
                                     uint32_t inW, uint32_t outH, uint32_t outW, uint32_t sH, uint32_t sW,
                                     cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  if (n == total && sH == 2 && sW == 2 && outH == 2 * inH && outW == 2 * inW && inW % 4 == 0 && aligned16_h(dy) &&
      aligned16_h(dx))
    return chunked<2>(k_upsample_bwd_2x2, n / 4, st, dy, dx, n / 4, FastDiv(inW / 4), inW);
  UpBackGeom g{FastDiv(inW), FastDiv(inH), outH, outW, sH, sW};
  return go(k_upsample_bwd, n, st, dy, dx, n, g);
}

cudaError_t launch_channel_copy(bool slice, const float* src, float* dst, uint32_t n, uint32_t L, uint32_t pitch,
                                uint32_t off, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const bool v4 = L % 4 == 0 && pitch % 4 == 0 && off % 4 == 0 && n % 4 == 0 && aligned16_h(src) && aligned16_h(dst);
  if (v4)
    return slice ? chunked<4>(k_channel_copy4<true>, n / 4, st, src, dst, n / 4, FastDiv(L / 4), pitch, off)
                 : chunked<4>(k_channel_copy4<false>, n / 4, st, src, dst, n / 4, FastDiv(L / 4), pitch, off);
  return slice ? go(k_channel_copy<true>, n, st, src, dst, n, FastDiv(L), pitch, off)
               : go(k_channel_copy<false>, n, st, src, dst, n, FastDiv(L), pitch, off);
}

cudaError_t launch_maxpool_forward(const float* x, float* out, uint32_t* idx, uint32_t lw, uint32_t lh, uint32_t lb,
                                   const PoolShape& g, cudaStream_t st) {
  const uint32_t n = lw * lh * lb;
  if (n == 0) return cudaSuccess;
  const bool full = lw == g.outW && lh == g.outH && lb == g.bc;
  if (full && g.p == 2 && g.s == 2 && g.inW % 4 == 0 && 2 * g.outW == g.inW && 2 * g.outH <= g.inH && aligned16_h(x))
    return chunked<4>(k_maxpool2x2, n / 2, st, x, out, idx, n / 2, FastDiv(g.outW / 2), FastDiv(g.outH), g.inH,
                      g.inW);
  return go(k_maxpool_fwd, n, st, x, out, idx, n, FastDiv(lw), FastDiv(lh), g);
}

cudaError_t launch_maxpool_scatter(const float* dz, const uint32_t* idx, float* d, uint64_t dcount, uint32_t lw,
                                   uint32_t lh, uint32_t lb, uint32_t outH, uint32_t outW, cudaStream_t st) {
  const uint32_t n = lw * lh * lb;
  if (n == 0) return cudaSuccess;
  const bool full = lw == outW && lh == outH;
  return go(k_maxpool_scatter, n, st, dz, idx, d, dcount, n, FastDiv(lw), FastDiv(lh), outH, outW, full);
}

cudaError_t launch_maxpool_backward_gather(const float* dz, const uint32_t* idx, float* d, const PoolShape& g,
                                           uint32_t* flag, cudaStream_t st) {
  const uint32_t n = g.bc * g.inH * g.inW, nout = g.bc * g.outH * g.outW;
  if (n == 0) return cudaSuccess;
  const FastDiv inW(g.inW);
  cudaError_t e;
  if (g.p == 2 && g.s == 2 && g.inW % 4 == 0 && 2 * g.outW == g.inW && aligned16_h(d))
    e = chunked<4>(k_maxpool_gather2x2, n / 4, st, dz, idx, d, n / 4, FastDiv(g.inW / 4), FastDiv(g.inH), inW, g,
                   flag);
  else
    e = go(k_maxpool_gather, n, st, dz, idx, d, n, inW, FastDiv(g.inH), FastDiv(g.s), g, flag);
  if (e != cudaSuccess || nout == 0) return e;
  launch_pdl(k_maxpool_fixup, dim3(1), dim3(1024), 0, st, dz, idx, d, n, nout, FastDiv(g.outW), FastDiv(g.outH), inW, g, flag);
  return cudaGetLastError();
}

cudaError_t launch_conv_reshape(const float* mm, const float* bias, float* out, uint32_t B, uint32_t OC, uint32_t P,
                                uint32_t lbp, uint32_t loc, uint32_t act, cudaStream_t st) {
  const uint32_t BP = B * P, n = lbp * loc;
  if (n == 0) return cudaSuccess;
  const int a = act == 1 ? 1 : act == 2 ? 2 : 0;
  if (lbp == BP && loc == OC && P % 4 == 0 && aligned16_h(mm) && aligned16_h(out)) {
    const FastDiv Pq(P / 4), fOC(OC);
    const uint32_t nq = n / 4;
    if (a == 1) return chunked<4>(k_conv_reshape4<1>, nq, st, mm, bias, out, nq, Pq, fOC, P, BP);
    if (a == 2) return chunked<4>(k_conv_reshape4<2>, nq, st, mm, bias, out, nq, Pq, fOC, P, BP);
    return chunked<4>(k_conv_reshape4<0>, nq, st, mm, bias, out, nq, Pq, fOC, P, BP);
  }
  const FastDiv fl(lbp), fP(P);
  if (a == 1) return go(k_conv_reshape<1>, n, st, mm, bias, out, n, fl, fP, OC, BP);
  if (a == 2) return go(k_conv_reshape<2>, n, st, mm, bias, out, n, fl, fP, OC, BP);
  return go(k_conv_reshape<0>, n, st, mm, bias, out, n, fl, fP, OC, BP);
}

cudaError_t launch_conv_grad_reshape(const float* dz, const float* fwd, float* out, uint32_t B, uint32_t OC,
                                     uint32_t P, uint32_t lbp, uint32_t loc, cudaStream_t st) {
  const uint32_t BP = B * P, n = lbp * loc;
  if (n == 0) return cudaSuccess;
  if (lbp == BP && loc == OC && P % 4 == 0 && aligned16_h(dz) && aligned16_h(out) && (!fwd || aligned16_h(fwd))) {
    const uint32_t nq = n / 4;
    if (fwd)
      return chunked<4>(k_conv_grad_reshape4<true>, nq, st, dz, fwd, out, nq, FastDiv(BP / 4), FastDiv(P / 4), OC, P);
    return chunked<4>(k_conv_grad_reshape4<false>, nq, st, dz, fwd, out, nq, FastDiv(BP / 4), FastDiv(P / 4), OC,
                               P);
  }
  if (fwd) return go(k_conv_grad_reshape<true>, n, st, dz, fwd, out, n, FastDiv(lbp), FastDiv(P), OC, BP);
  return go(k_conv_grad_reshape<false>, n, st, dz, fwd, out, n, FastDiv(lbp), FastDiv(P), OC, BP);
}

}  // namespace dct
