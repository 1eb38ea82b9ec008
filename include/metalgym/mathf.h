// Project-owned single-precision transcendentals: sin, cos, exp, tanh, log.
//
// Why they exist: environment dynamics (cos/sin in the cart-pole step, the
// ray directions of the voxel camera), the categorical sampler (exp/log) and
// the Box-Muller draw must give the SAME float on the B200 and on the host
// CPU, so that GPU trajectories can be compared bit for bit with the
// reference environment code compiled as host C++. CUDA's and glibc's libm
// differ in the last bit on some inputs, so neither is used. Instead every
// function below is a fixed sequence of IEEE-754 double operations:
//   * only correctly rounded primitives are used (+, -, *, /, fma, rint,
//     floor, frexp, ldexp), and every product that feeds an addition is
//     written as an explicit fma(), so no compiler contraction setting can
//     change the result;
//   * range reduction is Cody-Waite with a three-part pi/2 (or two-part ln 2)
//     applied through fma, whose products are exact;
//   * the kernels are plain Taylor series (coefficients 1/n!, 1/(2n+1)),
//     evaluated by Horner's rule, truncated where the remainder is far below
//     one double ulp of the reduced argument's range;
//   * the double result is rounded once to float (round-to-nearest-even).
// Accuracy: the double result is within ~1e-15 relative of the true value
// for |x| < 2^20 (sin/cos) and the full float range (exp/log), so the float
// result is correctly rounded except in rare near-halfway cases. The exact
// float bits are what matter for parity, and those are identical on host and
// device because the operation sequence is identical.
#pragma once

#include <cmath>
#include "config.h"

namespace mg_math {

// pi/2 split into three doubles (pio2_1 + pio2_2 + pio2_3 ~ pi/2 to 160 bits).
constexpr double PIO2_1 = 0x1.921fb54442d18p+0;
constexpr double PIO2_2 = 0x1.1a62633145c07p-54;
constexpr double PIO2_3 = -0x1.f1976b7ed8fbcp-110;
constexpr double INV_PIO2 = 0x1.45f306dc9c883p-1;
// ln 2 split into two doubles.
constexpr double LN2_HI = 0x1.62e42fefa39efp-1;
constexpr double LN2_LO = 0x1.abc9e3b39803fp-56;
constexpr double INV_LN2 = 0x1.71547652b82fep+0;
constexpr double SQRT_HALF = 0.70710678118654752440;

// 1/n! for n = 2..16 (Taylor coefficients of sin, cos and exp).
constexpr double F2 = 0x1.0000000000000p-1;
constexpr double F3 = 0x1.5555555555555p-3;
constexpr double F4 = 0x1.5555555555555p-5;
constexpr double F5 = 0x1.1111111111111p-7;
constexpr double F6 = 0x1.6c16c16c16c17p-10;
constexpr double F7 = 0x1.a01a01a01a01ap-13;
constexpr double F8 = 0x1.a01a01a01a01ap-16;
constexpr double F9 = 0x1.71de3a556c734p-19;
constexpr double F10 = 0x1.27e4fb7789f5cp-22;
constexpr double F11 = 0x1.ae64567f544e4p-26;
constexpr double F12 = 0x1.1eed8eff8d898p-29;
constexpr double F13 = 0x1.6124613a86d09p-33;
constexpr double F14 = 0x1.93974a8c07c9dp-37;
constexpr double F15 = 0x1.ae7f3e733b81fp-41;
constexpr double F16 = 0x1.ae7f3e733b81fp-45;

// sin(r) and cos(r) for |r| <= pi/4 (+ a few ulps), z = r*r.
//   sin r = r + r z (-1/3! + z (1/5! - z (1/7! - ...)))   through r^15/15!
//   cos r = 1 + z (-1/2! + z (1/4! - z (1/6! - ...)))     through r^16/16!
MG_HD inline double sin_kernel(double r, double z) {
    double p = -F15;
    p = fma(p, z, F13);
    p = fma(p, z, -F11);
    p = fma(p, z, F9);
    p = fma(p, z, -F7);
    p = fma(p, z, F5);
    p = fma(p, z, -F3);
    return fma(r * z, p, r);
}
MG_HD inline double cos_kernel(double z) {
    double p = F16;
    p = fma(p, z, -F14);
    p = fma(p, z, F12);
    p = fma(p, z, -F10);
    p = fma(p, z, F8);
    p = fma(p, z, -F6);
    p = fma(p, z, F4);
    p = fma(p, z, -F2);
    return fma(z, p, 1.0);
}

// Shared core: reduces x to r in [-pi/4, pi/4] and quadrant n, then returns
// sin and cos of x (as doubles, before the final rounding).
MG_HD inline void sincos_core(float xf, double* s, double* c) {
    const double x = (double)xf;
    if (!(fabs(x) <= 1.0e300)) {  // NaN or infinity: NaN for both outputs
        *s = x - x;
        *c = x - x;
        return;
    }
    const double q = rint(x * INV_PIO2);
    double r = fma(-q, PIO2_1, x);
    r = fma(-q, PIO2_2, r);
    r = fma(-q, PIO2_3, r);
    // q mod 4 in {0,1,2,3}; every step is exact for any double q.
    const double qm = q - 4.0 * floor(q * 0.25);
    const int n = (int)qm;
    const double z = r * r;
    const double sr = sin_kernel(r, z);
    const double cr = cos_kernel(z);
    switch (n & 3) {
        case 0: *s = sr; *c = cr; break;
        case 1: *s = cr; *c = -sr; break;
        case 2: *s = -sr; *c = -cr; break;
        default: *s = -cr; *c = sr; break;
    }
}

}  // namespace mg_math

MG_HD inline float mg_sinf(float x) {
    double s, c;
    mg_math::sincos_core(x, &s, &c);
    return (float)s;
}
MG_HD inline float mg_cosf(float x) {
    double s, c;
    mg_math::sincos_core(x, &s, &c);
    return (float)c;
}
MG_HD inline void mg_sincosf(float x, float* s, float* c) {
    double sd, cd;
    mg_math::sincos_core(x, &sd, &cd);
    *s = (float)sd;
    *c = (float)cd;
}

// e^x: x = k ln2 + r, |r| <= ln2/2, e^r by Taylor through r^14/14!.
MG_HD inline float mg_expf(float xf) {
    using namespace mg_math;
    if (xf != xf) return xf;
    double x = (double)xf;
    if (x > 130.0) x = 130.0;    // result rounds to +inf in float either way
    if (x < -160.0) x = -160.0;  // result rounds to +0 in float either way
    const double k = rint(x * INV_LN2);
    double r = fma(-k, LN2_HI, x);
    r = fma(-k, LN2_LO, r);
    double p = F14;
    p = fma(p, r, F13);
    p = fma(p, r, F12);
    p = fma(p, r, F11);
    p = fma(p, r, F10);
    p = fma(p, r, F9);
    p = fma(p, r, F8);
    p = fma(p, r, F7);
    p = fma(p, r, F6);
    p = fma(p, r, F5);
    p = fma(p, r, F4);
    p = fma(p, r, F3);
    p = fma(p, r, F2);
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
    return (float)ldexp(p, (int)k);
}

// tanh x = sign(x) E / (E + 2) with E = e^(2|x|) - 1, which has no
// cancellation for small |x|: 2|x| = k ln2 + r, |r| <= ln2/2, e^r - 1 = r (1 +
// r/2! + ... + r^13/14!) by Taylor, E = 2^k (e^r - 1) + (2^k - 1). Beyond
// |x| = 20, tanh x rounds to +-1 in float.
MG_HD inline float mg_tanhf(float xf) {
    using namespace mg_math;
    if (xf != xf || xf == 0.0f) return xf;  // NaN, and +-0 keeps its sign
    const double ax = xf < 0.0f ? -(double)xf : (double)xf;
    if (ax > 20.0) return xf < 0.0f ? -1.0f : 1.0f;
    const double y = 2.0 * ax;
    const double k = rint(y * INV_LN2);
    double r = fma(-k, LN2_HI, y);
    r = fma(-k, LN2_LO, r);
    double p = F14;
    p = fma(p, r, F13);
    p = fma(p, r, F12);
    p = fma(p, r, F11);
    p = fma(p, r, F10);
    p = fma(p, r, F9);
    p = fma(p, r, F8);
    p = fma(p, r, F7);
    p = fma(p, r, F6);
    p = fma(p, r, F5);
    p = fma(p, r, F4);
    p = fma(p, r, F3);
    p = fma(p, r, F2);
    p = fma(p, r, 1.0);
    const double em1 = p * r;  // e^r - 1
    const double sk = ldexp(1.0, (int)k);
    const double e = fma(sk, em1, sk - 1.0);
    const double t = e / (e + 2.0);
    return (float)(xf < 0.0f ? -t : t);
}

// ln x: x = 2^e m with m in [sqrt(1/2), sqrt(2)), s = (m-1)/(m+1),
// ln m = 2 s (1 + s^2/3 + s^4/5 + ... + s^20/21).
MG_HD inline float mg_logf(float xf) {
    using namespace mg_math;
    if (xf != xf) return xf;
    if (xf < 0.0f) return (xf - xf) / (xf - xf);  // NaN
    if (xf == 0.0f) return -1.0f / 0.0f;          // -inf
    if (xf == 1.0f / 0.0f) return xf;             // +inf
    int e = 0;
    double m = frexp((double)xf, &e);  // m in [0.5, 1)
    if (m < SQRT_HALF) {
        m = m * 2.0;
        e = e - 1;
    }
    const double f = m - 1.0;
    const double s = f / (m + 1.0);
    const double z = s * s;
    double p = 1.0 / 21.0;
    p = fma(p, z, 1.0 / 19.0);
    p = fma(p, z, 1.0 / 17.0);
    p = fma(p, z, 1.0 / 15.0);
    p = fma(p, z, 1.0 / 13.0);
    p = fma(p, z, 1.0 / 11.0);
    p = fma(p, z, 1.0 / 9.0);
    p = fma(p, z, 1.0 / 7.0);
    p = fma(p, z, 1.0 / 5.0);
    p = fma(p, z, 1.0 / 3.0);
    p = fma(p, z, 1.0);
    const double lm = (2.0 * s) * p;
    const double ed = (double)e;
    return (float)fma(ed, LN2_HI, fma(ed, LN2_LO, lm));
}
