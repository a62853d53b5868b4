// Counter-based synthetic-data generator of libdct_cuda (sm_100a).
//
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy
// as 1, 2, 3", SC'11): 10 rounds of two 32x32->64 multiplies with the published
// multipliers and Weyl key increments.  Element i of a fill uses counter
// (i/4, offset) and key `seed`, so any slice of a tensor can be regenerated
// independently (sharded ranks fill their own rows).  Uniforms use the top 24
// bits (exact in fp32); normals use the Box-Muller transform.  The uniform
// stream is restated bit-for-bit on the host by oracle/rng.py.
#include "dct_common.cuh"
#include "kernels.h"

namespace dct {

namespace {

DCT_DEV uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += 0x9E3779B9u;
    k.y += 0xBB67AE85u;
  }
  return c;
}

DCT_DEV float u24(uint32_t x) { return (float)(x >> 8) * 5.9604644775390625e-08f; }  // [0, 1)

__global__ void __launch_bounds__(256) k_fill(float* y, uint64_t n, uint64_t seed, uint64_t offset, int dist,
                                              float lo, float hi) {
  pdl_entry();
  const uint2 key = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32));
  const uint64_t groups = (n + 3) / 4;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const bool vec = aligned16(y);
  for (uint64_t g = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; g < groups; g += stride) {
    const uint4 r = philox4x32_10(make_uint4((uint32_t)g, (uint32_t)(g >> 32), (uint32_t)offset,
                                             (uint32_t)(offset >> 32)), key);
    float v[4];
    if (dist == 0) {
      const float w = __fsub_rn(hi, lo);
      v[0] = __fadd_rn(__fmul_rn(u24(r.x), w), lo);
      v[1] = __fadd_rn(__fmul_rn(u24(r.y), w), lo);
      v[2] = __fadd_rn(__fmul_rn(u24(r.z), w), lo);
      v[3] = __fadd_rn(__fmul_rn(u24(r.w), w), lo);
    } else {
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const uint32_t a = p ? r.z : r.x, b = p ? r.w : r.y;
        const float u1 = (float)((a >> 8) + 1u) * 5.9604644775390625e-08f;   // (0, 1]
        const float u2 = u24(b);
        const float rad = sqrtf(-2.0f * logf(u1));
        float s, c;
        sincospif(2.0f * u2, &s, &c);
        v[2 * p] = __fmaf_rn(hi, rad * c, lo);
        v[2 * p + 1] = __fmaf_rn(hi, rad * s, lo);
      }
    }
    const uint64_t i = 4 * g;
    if (vec && i + 3 < n) {
      st_stream4(y + i, make_float4(v[0], v[1], v[2], v[3]));
    } else {
      for (int q = 0; q < 4; ++q)
        if (i + q < n) y[i + q] = v[q];
    }
  }
}

__global__ void k_scatter(float* x, const int64_t* idx, const float* vals, uint64_t k) {
  pdl_entry();
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < k; i += stride) x[idx[i]] = vals[i];
}

}  // namespace

cudaError_t launch_fill_random(float* y, uint64_t n, uint64_t seed, uint64_t offset, int dist, float lo, float hi,
                               cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  launch_pdl(k_fill, dim3(grid_for((n + 3) / 4, 256)), dim3(256), 0, st, y, n, seed, offset, dist, lo, hi);
  return cudaGetLastError();
}

cudaError_t launch_scatter_values(float* x, const int64_t* idx, const float* vals, uint64_t k, cudaStream_t st) {
  if (k == 0) return cudaSuccess;
  launch_pdl(k_scatter, dim3(grid_for(k, 256)), dim3(256), 0, st, x, idx, vals, k);
  return cudaGetLastError();
}

}  // namespace dct
