// a / b rounded to nearest, for many a over one b, without a full division per element.
//
// With r = RN(1/b) computed once (__frcp_rn), each quotient takes three rounded operations:
//   q0 = RN(a * r)          -- within one ulp of a / b
//   e  = RN(a - b * q0)     -- exact: the residual of a faithful quotient is representable (FMA)
//   q  = RN(q0 + e * r)
// This is Markstein's correction step (P. W. Markstein, "Computation of elementary functions on
// the IBM RISC System/6000 processor", IBM J. Res. Develop. 34(1), 1990, and "IA-64 and
// Elementary Functions", 2000): when r is the correctly rounded reciprocal and q0 a faithful
// quotient, q is the correctly rounded quotient, provided the quotient and the residual stay in
// the normal range. The library checks it against __fdiv_rn bit for bit on the GPU
// (flk_selftest_quotient).
#pragma once

namespace flk {

__device__ __forceinline__ float quotient_rn(float a, float b, float r) {
  const float q0 = __fmul_rn(a, r);
  const float e = __fmaf_rn(-b, q0, a);
  return __fmaf_rn(e, r, q0);
}

}  // namespace flk
