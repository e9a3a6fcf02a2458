// exp, sin and cos of the verify step, evaluated exactly as the CPU restatement
// of the path evaluates them (this file is compiled with -fmad=false, so no
// product and sum are fused unless written as fma).
// exp: float arithmetic throughout.  n = rint(x log2 e); Cody-Waite reduction
// r = x - n ln2 with ln2 split into a 16-bit head (0x3F317200) and a tail, each
// step one fmaf; e^r by the Taylor polynomial to r^7 in Horner form (fmaf per
// step, coefficients the floats nearest 1/k!); then exact scaling by 2^n (two
// factors below 2^-126, so a subnormal result is rounded once).  Within 1 ulp
// of the true value.
// sin/cos: Cody-Waite reduction by pi/2 and Taylor series in double, every
// operation rounded separately, so the returned float is the correctly rounded
// one except in rare near-tie cases.  Constants: pi/2 split into 33-bit
// leading parts so that k * part is exact for every reduction count that can
// occur.
#pragma once

namespace mtb {

constexpr double kPio2_1 = 1.5707963267341256;      // pi/2 to 33 bits
constexpr double kPio2_2 = 6.077100506303966e-11;   // next 33 bits
constexpr double kPio2_3 = 2.0222662487959506e-21;  // remainder
constexpr double kTwoOverPi = 0.6366197723675814;

__device__ __forceinline__ float exact_expf(float x) {
    // Branch-free: x is clamped for the arithmetic and the special cases are
    // selected at the end; 2^n is applied as (p * 2^a) * 2^b with
    // (a, b) = (n, 0), (1, 127) for n = 128, (n + 64, -64) for n < -126.
    const float xc = fminf(fmaxf(x, -103.972084f), 88.7228317f);
    // n = rint(xc * log2 e) by the 1.5 * 2^23 add (|n| <= 150: the sum's unit
    // in the last place is 1, so it rounds to nearest even), and its integer
    // value from the sum's low bits, with no conversion instructions.
    const float tm = __fadd_rn(__fmul_rn(xc, 1.44269502f), 12582912.0f);
    const float n = __fsub_rn(tm, 12582912.0f);
    float r = fmaf(n, -0.693145752f, xc);
    r = fmaf(n, -1.42860677e-6f, r);
    float p = 1.98412701e-4f;
    p = fmaf(p, r, 1.38888892e-3f);
    p = fmaf(p, r, 8.33333377e-3f);
    p = fmaf(p, r, 4.16666679e-2f);
    p = fmaf(p, r, 1.66666672e-1f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ni = (int)(__float_as_uint(tm) - 0x4B400000u);
    const int ea = ni > 127 ? 1 : (ni < -126 ? ni + 64 : ni);
    const int eb = ni > 127 ? 127 : (ni < -126 ? -64 : 0);
    const float y = __fmul_rn(__fmul_rn(p, __uint_as_float((unsigned)(ea + 127) << 23)),
                              __uint_as_float((unsigned)(eb + 127) << 23));
    return x != x ? x : (x > 88.7228317f ? INFINITY : (x < -103.972084f ? 0.0f : y));
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

// erf: the Maclaurin series erf x = (2 / sqrt pi) sum_n (-1)^n x^(2n+1) / (n! (2n+1))
// in double, every operation rounded separately: t_n = (t_(n-1) * -x^2) * (1 / n),
// s += t_n * (1 / (2n + 1)) from s = t_0 = x, until the added term is at most
// 2^-60 of the sum (at most 128 terms), then s * 2/sqrt(pi) rounded to float.
// |x| >= 4 gives +-1 (erf there rounds to +-1 in float).  The reciprocals are the
// correctly rounded doubles; the cancellation of the alternating series costs at
// most ~1e-10 absolute below |x| = 4, so the float result is the correctly rounded
// one except near ties.
struct ErfRcpTable {
    double v[258];  // v[k] = 1 / k, the correctly rounded double (v[0] unused)
};
constexpr ErfRcpTable make_erf_rcp_table() {
    ErfRcpTable t{};
    for (int k = 1; k < 258; ++k) t.v[k] = 1.0 / k;
    return t;
}
static __constant__ ErfRcpTable c_erf_rcp = make_erf_rcp_table();

__device__ __forceinline__ float exact_erff(float xf) {
    const double x = (double)xf;
    if (!(fabs(x) < 4.0)) return xf != xf ? xf : (xf > 0.0f ? 1.0f : -1.0f);
    const double mx2 = __dmul_rn(-x, x);
    double term = x, sum = x;
    for (int n = 1; n <= 128; ++n) {
        term = __dmul_rn(__dmul_rn(term, mx2), c_erf_rcp.v[n]);
        const double add = __dmul_rn(term, c_erf_rcp.v[2 * n + 1]);
        sum = __dadd_rn(sum, add);
        if (fabs(add) <= fabs(sum) * 8.673617379884035e-19) break;  // 2^-60
    }
    return (float)__dmul_rn(sum, 1.1283791670955126);  // 2 / sqrt(pi)
}

// GELU, erf form (ggml_vec_gelu_erf_f32): (0.5 x)(1 + erf(x / sqrt 2)).
__device__ __forceinline__ float exact_gelu_erf(float v) {
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, exact_erff(__fmul_rn(v, 0.707106781f))));
}

}  // namespace mtb
