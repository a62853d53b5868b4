// Extended-precision elementary functions of libdct_cuda, written from the
// mathematics (no vendor math-library internals):
//
//  * exp of a non-positive argument as an unevaluated float-float sum
//    (hi + lo) * 2^k.  Argument reduction after Cody & Waite ("Software
//    Manual for the Elementary Functions", 1980): k = rint(a / ln 2),
//    r = -a - k ln 2 with ln 2 split into a float head and tail so the head
//    product is absorbed exactly by one fused multiply-add; exp(r) on
//    |r| <= ln2/2 by its Taylor series to degree 8 (truncation < 2^-32);
//    the sums 1 + r and the reduction are carried with the error-free
//    transformation of Dekker (1971, Fast2Sum).  The float-float result is
//    accurate to about 2^-28 relative before any final rounding.
//  * sigmoid(x) = 1 / (1 + e^-x) (x >= 0) or e^x / (1 + e^x) (x < 0), both
//    from e = exp(-|x|), with the denominator kept as float-float and the
//    quotient (approximate reciprocal times numerator) corrected once by its
//    exact remainder (one fused multiply-add, Markstein's scheme), so the
//    result is within about 0.6 ulp of the true value and the kernel has no
//    data-dependent branch.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "dct_common.cuh"

namespace dct {

// e^(-a) = (hi + lo) * 2^k for a >= 0 (NaN propagates; a > 104 gives 0).
DCT_DEV void exp_neg_ff(float a, float& hi, float& lo, int& k) {
  const float kInvLn2 = 1.4426950408889634f;
  const float kLn2Hi = 0.693147182464599609375f;      // float nearest ln 2
  const float kLn2Lo = -1.904654299957768e-09f;       // ln 2 - kLn2Hi
  const float x = -a;
  const float kf = rintf(__fmul_rn(x, kInvLn2));
  // r1 = x - k*ln2_hi is exact: one fused rounding of a value representable in 24 bits
  const float r1 = __fmaf_rn(-kf, kLn2Hi, x);
  // r = r1 - k*ln2_lo as (rh, rl); |k*ln2_lo| < 3e-7, so Fast2Sum's error is
  // below 2^-45 absolute even when |r1| is smaller than it
  const float t = __fmul_rn(kf, kLn2Lo);
  const float rh = __fsub_rn(r1, t);
  const float rl = __fsub_rn(__fsub_rn(r1, rh), t);
  // exp(r) - 1 - r = r^2 * P(r), P = sum_{n=2..8} r^(n-2)/n!  (|r| <= ln2/2: truncation < 2^-32)
  float p = 2.4801587301587302e-05f;                   // 1/8!
  p = __fmaf_rn(p, rh, 1.9841269841269841e-04f);       // 1/7!
  p = __fmaf_rn(p, rh, 1.3888888888888889e-03f);       // 1/6!
  p = __fmaf_rn(p, rh, 8.3333333333333333e-03f);       // 1/5!
  p = __fmaf_rn(p, rh, 4.1666666666666667e-02f);       // 1/4!
  p = __fmaf_rn(p, rh, 1.6666666666666667e-01f);       // 1/3!
  p = __fmaf_rn(p, rh, 0.5f);                          // 1/2!
  const float q = __fmul_rn(__fmul_rn(rh, rh), p);
  // 1 + rh + q as float-float: two Fast2Sums (|rh| >= |q|, 1 >= |rh + q|)
  const float u = __fadd_rn(rh, q);
  const float eu = __fsub_rn(q, __fsub_rn(u, rh));
  hi = __fadd_rn(1.0f, u);
  const float e2 = __fsub_rn(u, __fsub_rn(hi, 1.0f));
  lo = __fadd_rn(e2, __fadd_rn(eu, rl));
  k = (int)kf;
  if (a > 104.0f) { hi = 0.0f; lo = 0.0f; k = 0; }     // below every subnormal
}

// 2^k as a float for -126 <= k <= 127
DCT_DEV float pow2i(int k) { return __int_as_float((k + 127) << 23); }

// approximate reciprocal (the hardware's, about 1 ulp); only used where an
// exact-remainder correction follows
DCT_DEV float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// sigmoid for |x| > 87 (e^-|x| < 2^-125): 1 for x >= 0, else e^x rounded once
// into the subnormal range.  Rarely taken, so it may be slow.
DCT_DEV float sigmoid_tail(float x) {
  float h, l;
  int k;
  exp_neg_ff(fabsf(x), h, l, k);
  float eh, el;
  if (k >= -125) {
    const float sc = pow2i(k);
    eh = __fmul_rn(h, sc);                              // exact power-of-two scaling
    el = __fmul_rn(l, sc);
  } else {                                              // e below 2^-125: one rounding into the subnormals
    eh = __fmul_rn(__fmul_rn(__fadd_rn(h, l), pow2i(k + 64)), 5.42101086242752217e-20f);   // * 2^-64
    el = 0.0f;
  }
  // denominator 1 + e as (s, t): Fast2Sum, 1 >= e
  const float s = __fadd_rn(1.0f, eh);
  const float t = __fadd_rn(__fsub_rn(eh, __fsub_rn(s, 1.0f)), el);
  const bool neg = x < 0.0f;
  const float nh = neg ? eh : 1.0f;
  const float nl = neg ? el : 0.0f;
  // quotient (nh + nl) / (s + t): q0 from the approximate reciprocal, then one
  // correction by the exact remainder nh - q0*s (fused) -> error ~0.5 ulp
  const float r = rcp_approx(s);                        // s in [1, 2]
  const float q0 = __fmul_rn(nh, r);
  float rr = __fmaf_rn(-q0, s, nh);
  rr = __fadd_rn(rr, __fsub_rn(nl, __fmul_rn(q0, t)));
  return __fmaf_rn(rr, r, q0);
}

// sigmoid, <= 1 ulp, about 40 instructions on the common path.  e = e^-|x| is
// built directly as float-float: k = rint(-|x|/ln2) by the 1.5*2^23 rounding
// trick (no conversion unit), r = -|x| - k*ln2_hi exact by one fused
// multiply-add, exp(r) = 1 + r + r^2 P7(r) through two Fast2Sums, and the
// ln2 tail t = k*ln2_lo folded in as exp(r - t) = exp(r)(1 - t) (error t^2/2 <
// 2^-43); then the float-float quotient as in sigmoid_tail's final steps.
DCT_DEV float sigmoid_acc(float x) {
  const float a = fabsf(x);
  if (a > 87.0f) return sigmoid_tail(x);
  const float kMagic = 12582912.0f;                    // 1.5 * 2^23
  const float y = __fmul_rn(-a, 1.4426950408889634f);
  const float kb = __fadd_rn(y, kMagic);               // integer part in the low mantissa bits
  const float kf = __fsub_rn(kb, kMagic);
  const int k = __float_as_int(kb) - __float_as_int(kMagic);
  const float r = __fmaf_rn(-kf, 0.693147182464599609375f, -a);   // exact
  const float t = __fmul_rn(kf, -1.904654299957768e-09f);           // k * (ln2 - ln2_hi)
  float p = 1.9841269841269841e-04f;                   // 1/7!  (|r| <= ln2/2: truncation < 2^-27.5)
  p = __fmaf_rn(p, r, 1.3888888888888889e-03f);        // 1/6!
  p = __fmaf_rn(p, r, 8.3333333333333333e-03f);        // 1/5!
  p = __fmaf_rn(p, r, 4.1666666666666667e-02f);        // 1/4!
  p = __fmaf_rn(p, r, 1.6666666666666667e-01f);        // 1/3!
  p = __fmaf_rn(p, r, 0.5f);                           // 1/2!
  const float q = __fmul_rn(__fmul_rn(r, r), p);
  const float u = __fadd_rn(r, q);
  const float eu = __fsub_rn(q, __fsub_rn(u, r));
  const float hi = __fadd_rn(1.0f, u);
  const float e2 = __fsub_rn(u, __fsub_rn(hi, 1.0f));
  const float lo = __fadd_rn(e2, __fadd_rn(eu, __fmaf_rn(-t, r, -t)));
  const float sc = pow2i(k);                           // k >= -126 here
  const float eh = __fmul_rn(hi, sc), el = __fmul_rn(lo, sc);
  const float s = __fadd_rn(1.0f, eh);
  const float t2 = __fadd_rn(__fsub_rn(eh, __fsub_rn(s, 1.0f)), el);
  const bool neg = x < 0.0f;
  const float nh = neg ? eh : 1.0f;
  const float nl = neg ? el : 0.0f;
  const float rc = rcp_approx(s);
  const float q0 = __fmul_rn(nh, rc);
  float rr = __fmaf_rn(-q0, s, nh);
  rr = __fadd_rn(rr, __fmaf_rn(-q0, t2, nl));
  return __fmaf_rn(rr, rc, q0);
}

}  // namespace dct
