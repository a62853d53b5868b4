// Elementary functions of libdct_cuda written from the mathematics (no vendor
// math-library internals): the sigmoid, from Tang's table-driven exponential and
// a quotient corrected once by its remainder (see sigmoid_tab).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "dct_common.cuh"

namespace dct {

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

// 2^(j/32 - 64) = hi + lo, j = 0..31: hi is the float nearest the value, lo the
// float nearest the rest; computed from the definition in 60-digit decimal
// arithmetic and scaled by 2^-64 (exact: every entry stays a normal float), so
// that the sigmoid's final power of two is one multiply.  256 bytes.
static __device__ __align__(256) const float2 kExp2Tab[32] = {
    {0x1p-64f, 0.0f}, {0x1.059b0ep-64f, -0x1.9d4f52p-89f},
    {0x1.0b5586p-64f, 0x1.9f3122p-89f}, {0x1.11301ep-64f, -0x1.fdb496p-89f},
    {0x1.172b84p-64f, -0x1.c15742p-91f}, {0x1.1d4874p-64f, -0x1.d2e8cap-89f},
    {0x1.2387a6p-64f, 0x1.ceac48p-89f}, {0x1.29e9ep-64f, -0x1.5c0424p-89f},
    {0x1.306fep-64f, 0x1.4636e2p-89f}, {0x1.371a74p-64f, -0x1.18aac6p-89f},
    {0x1.3dea64p-64f, 0x1.824684p-89f}, {0x1.44e086p-64f, 0x1.8624b4p-94f},
    {0x1.4bfdaep-64f, -0x1.593abcp-89f}, {0x1.5342b6p-64f, -0x1.2c561p-89f},
    {0x1.5ab07ep-64f, -0x1.5bd5ecp-91f}, {0x1.6247ecp-64f, -0x1.f8b55p-89f},
    {0x1.6a09e6p-64f, 0x1.9fcef4p-90f}, {0x1.71f75ep-64f, 0x1.1d8beep-89f},
    {0x1.7a1148p-64f, -0x1.829fdp-89f}, {0x1.82589ap-64f, -0x1.accc7cp-90f},
    {0x1.8ace54p-64f, 0x1.15506ep-91f}, {0x1.93737cp-64f, -0x1.e64744p-89f},
    {0x1.9c4918p-64f, 0x1.51f848p-91f}, {0x1.a5503cp-64f, -0x1.b83b54p-89f},
    {0x1.ae89fap-64f, -0x1.a94b14p-90f}, {0x1.b7f77p-64f, -0x1.a09438p-89f},
    {0x1.c199bep-64f, -0x1.3d56b2p-91f}, {0x1.cb720ep-64f, -0x1.8837ccp-91f},
    {0x1.d5818ep-64f, -0x1.822dbcp-91f}, {0x1.dfc974p-64f, -0x1.908c94p-89f},
    {0x1.ea4afap-64f, 0x1.52486cp-91f}, {0x1.f50766p-64f, -0x1.246ebp-90f},
};

// sigmoid to within 1.5 ulp of the exact value over the whole float range (the
// ops' bar is 2 ulp), about 28 instructions and no branch.  `tab` is kExp2Tab
// or a copy of it (in shared memory for the streaming kernel).
//  * e = exp(-|x|) by Tang's table-driven method (ACM TOMS 15(2), 1989):
//    |x| is clamped to 104 (e^-104 rounds to 0; NaN stays NaN); k =
//    rint(-|x| * 32/ln2), rounded once by a fused multiply-add onto 1.5*2^23;
//    r = -|x| - k*ln2/32 with ln2/32 split in two parts (the first has 12
//    significant bits, so k * part1 is exact for |k| < 2^13); exp(r) - 1 =
//    r + r^2 (1/2 + r/6) on |r| <= ln2/64 (the omitted r^4/24 is below 2^-30.7,
//    under 0.01 ulp); e = 2^(k>>5) * (T_hi + (T_hi p + T_lo)).  The table holds
//    2^(j/32) * 2^-64, so the bracket is the same value scaled exactly by 2^-64
//    and one multiply by 2^(m+64) (a normal float) rounds it once, into the
//    subnormals for |x| > 87.3.
//  * sigmoid = n / (1 + e), n = 1 for x >= 0 and e for x < 0: q0 = n * rcp(1 + e),
//    then one correction by the remainder n - q0 (1 + e) (Markstein's scheme).
//    The remainder is (n - q0) - q0 e: q0 lies within a factor of two of n, so
//    n - q0 is exact (Sterbenz), and the fused multiply-add rounds the whole
//    remainder once.
DCT_DEV float sigmoid_tab(float x, const float2* tab) {
  const float a = fmin_nanp(fabsf(x), 104.0f);
  const float kMagic = 12582912.0f;                    // 1.5 * 2^23
  const float kb = __fmaf_rn(-a, 0x1.715476p+5f, kMagic);        // k = rint(-|x| * 32/ln2) in the low bits
  const float kf = __fsub_rn(kb, kMagic);
  const int k = __float_as_int(kb) - __float_as_int(kMagic);     // in [-4802, 0] (NaN: any int)
  float r = __fmaf_rn(-kf, 0x1.62ep-6f, -a);           // exact
  r = __fmaf_rn(-kf, 0x1.0bfbe8p-20f, r);
  const float w = __fmaf_rn(r, 0x1.555556p-3f, 0.5f);  // 1/2 + r/6
  const float p = __fmaf_rn(w, __fmul_rn(r, r), r);    // exp(r) - 1
  const float2 t2 = tab[k & 31];
  const float ef = __fadd_rn(t2.x, __fmaf_rn(t2.x, p, t2.y));    // 2^(j/32) e^r 2^-64
  // m = k >> 5 in [-151, 0]: 2^(m + 64) has exponent field m + 191 in [40, 191];
  // a multiply (not exponent arithmetic) keeps NaN
  const float sc = __int_as_float(((k >> 5) + 191) << 23);
  const float e = __fmul_rn(ef, sc);
  const float s = __fadd_rn(1.0f, e);
  const float n = x < 0.0f ? e : 1.0f;
  const float rc = rcp_approx(s);
  const float q0 = __fmul_rn(n, rc);
  const float rho = __fmaf_rn(-q0, e, __fsub_rn(n, q0));          // n - q0 (1 + e), rounded once
  return __fmaf_rn(rho, rc, q0);
}

DCT_DEV float sigmoid_acc(float x) { return sigmoid_tab(x, kExp2Tab); }

}  // namespace dct
