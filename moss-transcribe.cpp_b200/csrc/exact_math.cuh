// exp, sin and cos of the verify step, evaluated exactly as the CPU restatement
// of the path evaluates them: Cody-Waite range reduction and Taylor series in
// double, every operation rounded separately (this file is compiled with
// -fmad=false, so no product and sum are fused unless written as fma).
// Accuracy: the double result is within a few 1e-16 relative of the true
// value, so the returned float is the correctly rounded one except in rare
// near-tie cases.  Constants: ln 2 and pi/2 split into 32/33-bit leading parts
// so that n * part is exact for every reduction count that can occur.
#pragma once

namespace mtb {

constexpr double kLn2Hi = 0.6931471803691238;       // ln 2 to 32 bits
constexpr double kLn2Lo = 1.9082149292705877e-10;   // ln 2 - kLn2Hi
constexpr double kInvLn2 = 1.4426950408889634;
constexpr double kPio2_1 = 1.5707963267341256;      // pi/2 to 33 bits
constexpr double kPio2_2 = 6.077100506303966e-11;   // next 33 bits
constexpr double kPio2_3 = 2.0222662487959506e-21;  // remainder
constexpr double kTwoOverPi = 0.6366197723675814;

__device__ __forceinline__ float exact_expf(float x) {
    if (x != x) return x;
    if (x > 88.8f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    const double xd = (double)x;
    const double n = rint(xd * kInvLn2);
    const double r = (xd - n * kLn2Hi) - n * kLn2Lo;
    double p = 1.0 / 479001600.0;  // sum r^k / k!, k <= 12
    p = p * r + 1.0 / 39916800.0;
    p = p * r + 1.0 / 3628800.0;
    p = p * r + 1.0 / 362880.0;
    p = p * r + 1.0 / 40320.0;
    p = p * r + 1.0 / 5040.0;
    p = p * r + 1.0 / 720.0;
    p = p * r + 1.0 / 120.0;
    p = p * r + 1.0 / 24.0;
    p = p * r + 1.0 / 6.0;
    p = p * r + 0.5;
    p = p * r + 1.0;
    p = p * r + 1.0;
    return (float)ldexp(p, (int)n);
}

__device__ __forceinline__ void exact_sincosf(float x, float* s_out, float* c_out) {
    const double xd = (double)x;
    const double k = rint(xd * kTwoOverPi);
    const double r = ((xd - k * kPio2_1) - k * kPio2_2) - k * kPio2_3;
    const double r2 = r * r;
    double ps = -1.0 / 121645100408832000.0;  // sin r / r, to r^18
    ps = ps * r2 + 1.0 / 355687428096000.0;
    ps = ps * r2 - 1.0 / 1307674368000.0;
    ps = ps * r2 + 1.0 / 6227020800.0;
    ps = ps * r2 - 1.0 / 39916800.0;
    ps = ps * r2 + 1.0 / 362880.0;
    ps = ps * r2 - 1.0 / 5040.0;
    ps = ps * r2 + 1.0 / 120.0;
    ps = ps * r2 - 1.0 / 6.0;
    ps = ps * r2 + 1.0;
    const double sv = ps * r;
    double pc = 1.0 / 2432902008176640000.0;  // cos r, to r^20
    pc = pc * r2 - 1.0 / 6402373705728000.0;
    pc = pc * r2 + 1.0 / 20922789888000.0;
    pc = pc * r2 - 1.0 / 87178291200.0;
    pc = pc * r2 + 1.0 / 479001600.0;
    pc = pc * r2 - 1.0 / 3628800.0;
    pc = pc * r2 + 1.0 / 40320.0;
    pc = pc * r2 - 1.0 / 720.0;
    pc = pc * r2 + 1.0 / 24.0;
    pc = pc * r2 - 0.5;
    pc = pc * r2 + 1.0;
    const double cv = pc;
    const long long q = (((long long)k) % 4 + 4) % 4;
    double so, co;
    if (q == 0) { so = sv; co = cv; }
    else if (q == 1) { so = cv; co = -sv; }
    else if (q == 2) { so = -sv; co = -cv; }
    else { so = -cv; co = sv; }
    *s_out = (float)so;
    *c_out = (float)co;
}

}  // namespace mtb
