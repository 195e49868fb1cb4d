/*
 * colour_math.cuh — arithmetic shared by the colour kernels and their self-test (device code).
 *
 * Division by a per-launch constant d, correctly rounded, without a division instruction per
 * element: with r = RN(1/d) (the IEEE reciprocal) and q0 = RN(a * r), the remainder
 * e = a - q0 * d is exact in one FMA, and q1 = RN(q0 + e * r) is RN(a / d). This is Markstein's
 * correction step (P. Markstein, "Computation of elementary functions on the IBM RISC System/6000
 * processor", IBM J. Res. Dev. 34(1), 1990: a reciprocal within half an ulp and a quotient within
 * one ulp give the correctly rounded quotient after one correction), valid for finite a and d
 * away from overflow and underflow (it fails for |a| below ~2^-100, where the remainder
 * underflows). ajib_selftest_division checks it bit for bit against the IEEE division over every
 * float of magnitude in [2^-80, 2^18), which holds every dividend the post pass divides.
 */
#pragma once

#include <cuda_runtime.h>

namespace ajib {
namespace dev {

__device__ __forceinline__ float div_by(float a, float d, float r)
{
    const float q0 = __fmul_rn(a, r);
    const float e = __fmaf_rn(-q0, d, a);
    return __fmaf_rn(e, r, q0);
}

}  // namespace dev
}  // namespace ajib
