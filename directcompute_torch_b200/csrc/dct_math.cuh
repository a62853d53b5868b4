// Elementary functions of libdct_cuda written from the mathematics (no vendor
// math-library internals): the sigmoid, from Tang's table-driven exponential and
// a quotient corrected once by its exact remainder (see sigmoid_tab).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "dct_common.cuh"

namespace dct {

constexpr float kTwoM64 = 0x1p-64f;

// approximate reciprocal (the hardware's, about 1 ulp); only used where an
// exact-remainder correction follows
DCT_DEV float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// min that returns NaN if either operand is NaN (one instruction)
DCT_DEV float fmin_nanp(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// 2^(j/32) = hi + lo, j = 0..31: hi is the float nearest the value, lo the
// float nearest the rest; computed from the definition in 60-digit decimal
// arithmetic.  256 bytes.
static __device__ __align__(256) const float2 kExp2Tab[32] = {
    {0x1p+0f, 0.0f}, {0x1.059b0ep+0f, -0x1.9d4f52p-25f},
    {0x1.0b5586p+0f, 0x1.9f3122p-25f}, {0x1.11301ep+0f, -0x1.fdb496p-25f},
    {0x1.172b84p+0f, -0x1.c15742p-27f}, {0x1.1d4874p+0f, -0x1.d2e8cap-25f},
    {0x1.2387a6p+0f, 0x1.ceac48p-25f}, {0x1.29e9ep+0f, -0x1.5c0424p-25f},
    {0x1.306fep+0f, 0x1.4636e2p-25f}, {0x1.371a74p+0f, -0x1.18aac6p-25f},
    {0x1.3dea64p+0f, 0x1.824684p-25f}, {0x1.44e086p+0f, 0x1.8624b4p-30f},
    {0x1.4bfdaep+0f, -0x1.593abcp-25f}, {0x1.5342b6p+0f, -0x1.2c561p-25f},
    {0x1.5ab07ep+0f, -0x1.5bd5ecp-27f}, {0x1.6247ecp+0f, -0x1.f8b55p-25f},
    {0x1.6a09e6p+0f, 0x1.9fcef4p-26f}, {0x1.71f75ep+0f, 0x1.1d8beep-25f},
    {0x1.7a1148p+0f, -0x1.829fdp-25f}, {0x1.82589ap+0f, -0x1.accc7cp-26f},
    {0x1.8ace54p+0f, 0x1.15506ep-27f}, {0x1.93737cp+0f, -0x1.e64744p-25f},
    {0x1.9c4918p+0f, 0x1.51f848p-27f}, {0x1.a5503cp+0f, -0x1.b83b54p-25f},
    {0x1.ae89fap+0f, -0x1.a94b14p-26f}, {0x1.b7f77p+0f, -0x1.a09438p-25f},
    {0x1.c199bep+0f, -0x1.3d56b2p-27f}, {0x1.cb720ep+0f, -0x1.8837ccp-27f},
    {0x1.d5818ep+0f, -0x1.822dbcp-27f}, {0x1.dfc974p+0f, -0x1.908c94p-25f},
    {0x1.ea4afap+0f, 0x1.52486cp-27f}, {0x1.f50766p+0f, -0x1.246ebp-26f},
};

// sigmoid to within 1.5 ulp of the exact value over the whole float range (the
// ops' bar is 2 ulp), about 30 instructions and no branch.  `tab` is kExp2Tab
// or a copy of it (in shared memory for the streaming kernel).
//  * e = exp(-|x|) by Tang's table-driven method (ACM TOMS 15(2), 1989):
//    |x| is clamped to 104 (e^-104 rounds to 0; NaN stays NaN); k =
//    rint(-|x| * 32/ln2) by the 1.5*2^23 rounding trick; r = -|x| - k*ln2/32 with
//    ln2/32 split in two parts (the first has 12 significant bits, so k * part1
//    is exact for |k| < 2^13); exp(r) - 1 = r + r^2 (1/2 + r/6) on |r| <= ln2/64
//    (the omitted r^4/24 is below 2^-30.7, under 0.01 ulp); e = 2^(k>>5) * (T_hi + (T_hi p +
//    T_lo)), with the power of two applied as 2^(m+64) (exact: the product stays
//    normal) and then 2^-64 (one rounding, into the subnormals for |x| > 87.3).
//  * sigmoid = n / (1 + e), n = 1 for x >= 0 and e for x < 0: the denominator
//    kept exactly as s + t (Fast2Sum, Dekker 1971), q0 = n * rcp(s), and one
//    correction by the exact remainder n - q0 (s + t) (Markstein's scheme).
DCT_DEV float sigmoid_tab(float x, const float2* tab) {
  const float a = fmin_nanp(fabsf(x), 104.0f);
  const float kMagic = 12582912.0f;                    // 1.5 * 2^23
  const float y = __fmul_rn(-a, 0x1.715476p+5f);       // -|x| * 32/ln2
  const float kb = __fadd_rn(y, kMagic);               // integer part in the low mantissa bits
  const float kf = __fsub_rn(kb, kMagic);
  const int k = __float_as_int(kb) - __float_as_int(kMagic);     // in [-4802, 0] (NaN: any int)
  float r = __fmaf_rn(-kf, 0x1.62ep-6f, -a);           // exact
  r = __fmaf_rn(-kf, 0x1.0bfbe8p-20f, r);
  const float w = __fmaf_rn(r, 0x1.555556p-3f, 0.5f);  // 1/2 + r/6
  const float p = __fmaf_rn(w, __fmul_rn(r, r), r);    // exp(r) - 1
  const float2 t2 = tab[k & 31];
  const float ef = __fadd_rn(t2.x, __fmaf_rn(t2.x, p, t2.y));
  // ef * 2^(m + 64) * 2^-64, m = k >> 5 in [-151, 0]: 2^(m + 64) has exponent
  // field m + 191 in [40, 191]; multiplies (not exponent arithmetic) keep NaN
  const float sc = __int_as_float(((k >> 5) + 191) << 23);
  const float e = __fmul_rn(__fmul_rn(ef, sc), kTwoM64);
  const float s = __fadd_rn(1.0f, e);
  const float t = __fsub_rn(e, __fsub_rn(s, 1.0f));    // 1 + e = s + t exactly (1 >= e)
  const float n = x < 0.0f ? e : 1.0f;
  const float rc = rcp_approx(s);
  const float q0 = __fmul_rn(n, rc);
  float rho = __fmaf_rn(-q0, s, n);
  rho = __fmaf_rn(-q0, t, rho);
  return __fmaf_rn(rho, rc, q0);
}

DCT_DEV float sigmoid_acc(float x) { return sigmoid_tab(x, kExp2Tab); }

}  // namespace dct
