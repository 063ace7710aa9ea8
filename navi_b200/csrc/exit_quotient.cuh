// Correctly rounded quotient of a void cell's exit distance from a precomputed reciprocal
// (used by the grid trace kernel, checked by quotient_check.cu).
#pragma once

#include <cuda_runtime.h>

namespace tsdf {

// Divisors at or above this magnitude are divided with __fdiv_rn: their reciprocals are
// subnormal, outside the range where exit_quotient is exact.
constexpr float kQuotientMaxDivisor = 0x1p126f;

// RN(a / d) from r = RN(1 / d) and q0 = RN(a * r): one residual correction,
// RN(q0 + RN(a - q0 * d) * r) with both steps fused (Markstein's correction step:
// P. Markstein, IBM J. Res. Dev. 34(1), 1990; Muller et al., Handbook of Floating-Point
// Arithmetic, 2nd ed., section 4.7).  The fma computes the residual a - q0 * d exactly.
// The result equals __fdiv_rn(a, d) for every pair of binary32 significands (a, d in
// [1, 2), checked exhaustively by navi_check_exit_quotient).  Scaling a or d by a power
// of two scales r, q0, the residual and the quotient exactly while none of them leaves the
// normal range, so the equality holds for |d| < kQuotientMaxDivisor and |a| >= 2^-64; below
// that |a / d| < 1e-15, far under the 1e-4 floor the exit distance is clamped to, which any
// result of this formula then also meets.
__device__ __forceinline__ float exit_quotient(float a, float d, float r, float q0)
{
    return __fmaf_rn(__fmaf_rn(-q0, d, a), r, q0);
}

}  // namespace tsdf
