// cuju-b200: the transcendental functions of glibc 2.39 (x86-64, FMA build), bit for bit on the
// device. GRF's results depend on glibc's exact outputs, so each function restates the published
// algorithm that glibc runs, with the same constants, the same operation order and the same fused
// steps (an explicit `fma` wherever glibc's FMA build contracts, nothing else fused):
//   lm_sinf / lm_cosf / lm_sincosf  Arm Optimized Routines v21.02 sinf.c, cosf.c, sincosf.h
//   lm_powf                         Arm Optimized Routines v21.02 powf.c (+ exp2f/log2 data)
//   lm_acosf / lm_atanf / lm_atan2f FreeBSD msun e_acosf.c, s_atanf.c, e_atan2f.c
//   lm_asinf                        glibc sysdeps/ieee754/flt-32/e_asinf.c
//   lm_sin / lm_cos                 glibc dbl-64 s_sin.c + branred.c (IBM Accurate Math Library)
//   lm_acos                         glibc dbl-64 e_asin.c (__ieee754_acos)
//   lm_pow                          Arm Optimized Routines v21.02 pow.c
// The reference carries ports of the same code: cuju include/cuju/libm/*.h. CUDA's own math
// functions are never used for these, since they round differently.
#pragma once

#include "common.cuh"

#if defined(__CUDACC__)
#define CB_TABLE_U64(name, n, ...)                              \
    static const uint64_t name##_h[n] = __VA_ARGS__;            \
    static __device__ const uint64_t name##_d[n] = __VA_ARGS__;
#else
#define CB_TABLE_U64(name, n, ...) static const uint64_t name##_h[n] = __VA_ARGS__;
#endif
#if CB_DEVICE_PASS
#define CB_TAB(name) (name##_d)
#else
#define CB_TAB(name) (name##_h)
#endif

namespace cb {
namespace lm {
#include "libm_tables.inc"

CB_HD double tabd(const uint64_t *t, int i) { return u2d(t[i]); }

// ============================================================================================
// Float sine and cosine: Arm Optimized Routines sinf/cosf.
struct SinCosF {
    float s, c;
};
struct SCPoly {
    double c0, c1, c2, c3, c4;  // cosine terms
    double s1, s2, s3;          // sine terms
};
CB_HD SCPoly sc_poly(bool negated) {
    SCPoly p;
    const double k = negated ? -1.0 : 1.0;
    p.c0 = k * 0x1p0;
    p.c1 = k * -0x1.ffffffd0c621cp-2;
    p.c2 = k * 0x1.55553e1068f19p-5;
    p.c3 = k * -0x1.6c087e89a359dp-10;
    p.c4 = k * 0x1.99343027bf8c3p-16;
    p.s1 = -0x1.555545995a603p-3;
    p.s2 = 0x1.1107605230bc4p-7;
    p.s3 = -0x1.994eb3774cf24p-13;
    return p;
}
CB_HD uint32_t top12f(float v) { return (f2u(v) >> 20) & 0x7ff; }
constexpr double kHalfPiInvScaled = 0x1.45F306DC9C883p+23;  // 2^24 * 2/pi
constexpr double kHalfPiD = 0x1.921FB54442D18p0;
CB_HD double sign4(int q) { return (q == 1 || q == 2) ? -1.0 : 1.0; }

// |x| < 120: nearest multiple n of pi/2, remainder x - n*pi/2 in one fused step.
CB_HD double sc_reduce_small(double x, int *q) {
    double r = x * kHalfPiInvScaled;
    int n = ((int32_t)r + 0x800000) >> 24;
    *q = n;
    return fma(-(double)n, kHalfPiD, x);
}

// Large finite |x| (>= 120): Payne-Hanek style with 4/pi bits in overlapping 32-bit words.
CB_HDNI double sc_reduce_large(uint32_t xi, int *q) {
    // 4/pi in words that start 8 bits apart (Arm Optimized Routines __inv_pio4).
    const uint32_t kInvPio4[24] = {
        0xa2,       0xa2f9,     0xa2f983,   0xa2f9836e, 0xf9836e4e, 0x836e4e44,
        0x6e4e4415, 0x4e441529, 0x441529fc, 0x1529fc27, 0x29fc2757, 0xfc2757d1,
        0x2757d1f5, 0x57d1f534, 0xd1f534dd, 0xf534ddc0, 0x34ddc0db, 0xddc0db62,
        0xc0db6295, 0xdb629599, 0x6295993c, 0x95993c43, 0x993c4390, 0x3c439041};
    const uint32_t *arr = &kInvPio4[(xi >> 26) & 15];
    int shift = (xi >> 23) & 7;
    uint64_t n, r0, r1, r2;
    xi = (xi & 0xffffff) | 0x800000;
    xi <<= shift;
    r0 = (uint32_t)(xi * arr[0]);
    r1 = (uint64_t)xi * arr[4];
    r2 = (uint64_t)xi * arr[8];
    r0 = (r2 >> 32) | (r0 << 32);
    r0 += r1;
    n = (r0 + (1ULL << 61)) >> 62;
    r0 -= n << 62;
    double x = (double)(int64_t)r0;
    *q = (int)n;
    return x * 0x1.921FB54442D18p-62;
}

// Even quadrant: sine polynomial; odd: cosine polynomial.
CB_HD float sc_eval(double x, double x2, const SCPoly &p, int n) {
    if ((n & 1) == 0) {
        double x3 = x * x2;
        double s1 = fma(x2, p.s3, p.s2);
        double x7 = x3 * x2;
        double s = fma(x3, p.s1, x);
        return (float)fma(x7, s1, s);
    }
    double x4 = x2 * x2;
    double c2 = fma(x2, p.c4, p.c3);
    double c1 = fma(x2, p.c1, p.c0);
    double x6 = x4 * x2;
    double c = fma(x4, p.c2, c1);
    return (float)fma(x6, c2, c);
}

// Classifies the argument; returns 0 tiny, 1 small, 2 reduced, 3 invalid and fills the reduction.
CB_HD int sc_classify(float xf, double &r, int &q, bool &neg_table, double &sgn) {
    const uint32_t t = top12f(xf);
    r = xf;
    if (t < top12f((float)0x1.921FB54442D18p-1)) {
        if (t < top12f(0x1p-12f)) return 0;
        return 1;
    }
    if (t < top12f(120.0f)) {
        r = sc_reduce_small(r, &q);
        sgn = sign4(q & 3);
        neg_table = (q & 2) != 0;
        return 2;
    }
    if (t < top12f(INFINITY)) {
        uint32_t xi = f2u(xf);
        int s = xi >> 31;
        r = sc_reduce_large(xi, &q);
        sgn = sign4((q + s) & 3);
        neg_table = ((q + s) & 2) != 0;
        return 2;
    }
    return 3;
}

CB_HDNI float lm_sinf(float x) {
    double r, sgn = 1;
    int q = 0;
    bool neg = false;
    switch (sc_classify(x, r, q, neg, sgn)) {
        case 0: return x;
        case 1: return sc_eval(r, r * r, sc_poly(false), 0);
        case 2: return sc_eval(r * sgn, r * r, sc_poly(neg), q);
        default: return (x - x) / (x - x);
    }
}
CB_HDNI float lm_cosf(float x) {
    double r, sgn = 1;
    int q = 0;
    bool neg = false;
    switch (sc_classify(x, r, q, neg, sgn)) {
        case 0: return 1.0f;
        case 1: return sc_eval(r, r * r, sc_poly(false), 1);
        case 2: return sc_eval(r * sgn, r * r, sc_poly(neg), q ^ 1);
        default: return (x - x) / (x - x);
    }
}
// Both from one reduction; each result equals lm_sinf / lm_cosf bit for bit.
CB_HDNI SinCosF lm_sincosf(float x) {
    double r, sgn = 1;
    int q = 0;
    bool neg = false;
    switch (sc_classify(x, r, q, neg, sgn)) {
        case 0: return SinCosF{x, 1.0f};
        case 1: {
            const SCPoly p = sc_poly(false);
            double x2 = r * r;
            return SinCosF{sc_eval(r, x2, p, 0), sc_eval(r, x2, p, 1)};
        }
        case 2: {
            const SCPoly p = sc_poly(neg);
            double rs = r * sgn, x2 = r * r;
            return SinCosF{sc_eval(rs, x2, p, q), sc_eval(rs, x2, p, q ^ 1)};
        }
        default: {
            float nan = (x - x) / (x - x);
            return SinCosF{nan, nan};
        }
    }
}

// ============================================================================================
// Float power: Arm Optimized Routines powf.
CB_HD double powf_log2(uint32_t ix) {
    const uint32_t kOff = 0x3f330000;
    uint32_t tmp = ix - kOff;
    int i = (tmp >> (23 - 4)) % 16;
    uint32_t top = tmp & 0xff800000;
    uint32_t iz = ix - top;
    int k = (int32_t)top >> 23;
    double invc = tabd(CB_TAB(kPowfLog2Tab), 2 * i), logc = tabd(CB_TAB(kPowfLog2Tab), 2 * i + 1);
    double z = (double)u2f(iz);
    double r = fma(z, invc, -1.0);
    double y0 = logc + (double)k;
    double r2 = r * r;
    double y = fma(0x1.27616c9496e0bp-2, r, -0x1.71969a075c67ap-2);
    double p = fma(0x1.ec70a6ca7baddp-2, r, -0x1.7154748bef6c8p-1);
    double r4 = r2 * r2;
    double q = fma(0x1.71547652ab82bp0, r, y0);
    q = fma(p, r2, q);
    y = fma(y, r4, q);
    return y;
}
CB_HD float powf_exp2(double xd, uint32_t sign_bias) {
    const double kShift = 0x1.8p+52 / 32;
    double kd = xd + kShift;
    uint64_t ki = d2u(kd);
    kd -= kShift;
    double r = xd - kd;
    uint64_t t = CB_TAB(kPowfExp2Tab)[ki % 32];
    uint64_t ski = ki + sign_bias;
    t += ski << (52 - 5);
    double s = u2d(t);
    double z = fma(0x1.c6af84b912394p-5, r, 0x1.ebfce50fac4f3p-3);
    double r2 = r * r;
    double y = fma(0x1.62e42ff0c52d6p-1, r, 1.0);
    y = fma(z, r2, y);
    y = y * s;
    return (float)y;
}
CB_HD int powf_checkint(uint32_t iy) {
    int e = iy >> 23 & 0xff;
    if (e < 0x7f) return 0;
    if (e > 0x7f + 23) return 2;
    if (iy & ((1 << (0x7f + 23 - e)) - 1)) return 0;
    if (iy & (1 << (0x7f + 23 - e))) return 1;
    return 2;
}
CB_HD int zeroinfnan_f(uint32_t ix) { return 2 * ix - 1 >= 2u * 0x7f800000 - 1; }
CB_HD int is_snan_f(float v) { uint32_t b = f2u(v); return 2 * (b ^ 0x00400000) > 2u * 0x7fc00000; }
CB_HD float xflow_f(uint32_t sign, float y) { return (sign ? -y : y) * y; }

CB_HDNI float lm_powf(float x, float y) {
    uint32_t sign_bias = 0;
    uint32_t ix = f2u(x), iy = f2u(y);
    if (ix - 0x00800000 >= 0x7f800000 - 0x00800000 || zeroinfnan_f(iy)) {
        if (zeroinfnan_f(iy)) {
            if (2 * iy == 0) return is_snan_f(x) ? x + y : 1.0f;
            if (ix == 0x3f800000) return is_snan_f(y) ? x + y : 1.0f;
            if (2 * ix > 2u * 0x7f800000 || 2 * iy > 2u * 0x7f800000) return x + y;
            if (2 * ix == 2 * 0x3f800000) return 1.0f;
            if ((2 * ix < 2 * 0x3f800000) == !(iy & 0x80000000)) return 0.0f;
            return y * y;
        }
        if (zeroinfnan_f(ix)) {
            float x2 = x * x;
            if (ix & 0x80000000 && powf_checkint(iy) == 1) {
                x2 = -x2;
                sign_bias = 1;
            }
            if (2 * ix == 0 && iy & 0x80000000) {
                float zero = 0.0f;
                return (sign_bias ? -1.0f : 1.0f) / zero;
            }
            return iy & 0x80000000 ? 1 / x2 : x2;
        }
        if (ix & 0x80000000) {
            int yint = powf_checkint(iy);
            if (yint == 0) return (x - x) / (x - x);
            if (yint == 1) sign_bias = 1 << (5 + 11);
            ix &= 0x7fffffff;
        }
        if (ix < 0x00800000) {
            ix = f2u(x * 0x1p23f);
            ix &= 0x7fffffff;
            ix -= 23 << 23;
        }
    }
    double logx = powf_log2(ix);
    double ylogx = (double)y * logx;
    if ((d2u(ylogx) >> 47 & 0xffff) >= d2u(126.0) >> 47) {
        if (ylogx > 0x1.fffffffd1d571p+6) return xflow_f(sign_bias, 0x1p97f);
        if (ylogx <= -150.0) return xflow_f(sign_bias, 0x1p-95f);
        if (ylogx < -149.0) return xflow_f(sign_bias, 0x1.4p-75f);
    }
    return powf_exp2(ylogx, sign_bias);
}
// powf for a positive exponent that is not an odd integer; 0 and 1 bases short-cut to the same
// results powf gives.
CB_HD float lm_powf_pos(float x, float y) {
    if (x == 0.0f) return 0.0f;
    if (x == 1.0f) return 1.0f;
    return lm_powf(x, y);
}

// ============================================================================================
// Float inverse trigonometric functions: FreeBSD msun (glibc runs the same code for these).
CB_HD int32_t fword(float v) { return (int32_t)f2u(v); }
CB_HD float ffromword(int32_t w) { return u2f((uint32_t)w); }

CB_HD float acosf_ratio(float z) {
    const float pS0 = (float)1.6666667163e-01, pS1 = (float)-3.2556581497e-01,
                pS2 = (float)2.0121252537e-01, pS3 = (float)-4.0055535734e-02,
                pS4 = (float)7.9153501429e-04, pS5 = (float)3.4793309169e-05,
                qS1 = (float)-2.4033949375e+00, qS2 = (float)2.0209457874e+00,
                qS3 = (float)-6.8828397989e-01, qS4 = (float)7.7038154006e-02;
    float p = z * (pS0 + z * (pS1 + z * (pS2 + z * (pS3 + z * (pS4 + z * pS5)))));
    float q = (float)1.0 + z * (qS1 + z * (qS2 + z * (qS3 + z * qS4)));
    return p / q;
}

CB_HDNI float lm_acosf(float x) {
    const float pi = (float)3.1415925026e+00, pio2_hi = (float)1.5707962513e+00,
                pio2_lo = (float)7.5497894159e-08;
    int32_t hx = fword(x), ix = hx & 0x7fffffff;
    if (ix == 0x3f800000) {
        if (hx > 0) return 0.0;
        return pi + (float)2.0 * pio2_lo;
    }
    if (ix > 0x3f800000) return (x - x) / (x - x);
    if (ix < 0x3f000000) {
        if (ix <= 0x32800000) return pio2_hi + pio2_lo;
        float z = x * x;
        float r = acosf_ratio(z);
        return pio2_hi - (x - (pio2_lo - x * r));
    }
    if (hx < 0) {
        float z = ((float)1.0 + x) * (float)0.5;
        // FreeBSD evaluates p and q before s = sqrtf(z), r = p/q afterwards; the values do not
        // depend on that order.
        float s = sqrtf(z);
        float r = acosf_ratio(z);
        float w = r * s - pio2_lo;
        return pi - (float)2.0 * (s + w);
    }
    float z = ((float)1.0 - x) * (float)0.5;
    float s = sqrtf(z);
    float df = ffromword(fword(s) & 0xfffff000);
    float c = (z - df * df) / (s + df);
    float r = acosf_ratio(z);
    float w = r * s + c;
    return (float)2.0 * (df + w);
}

CB_HDNI float lm_asinf(float x) {
    const float one = 1.0f, huge = 1.000e+30f, pio2_hi = 1.57079637050628662109375f,
                pio2_lo = -4.37113900018624283e-8f, pio4_hi = 0.785398185253143310546875f,
                p0 = 1.666675248e-1f, p1 = 7.495297643e-2f, p2 = 4.547037598e-2f,
                p3 = 2.417951451e-2f, p4 = 4.216630880e-2f;
    int32_t hx = fword(x), ix = hx & 0x7fffffff;
    if (ix == 0x3f800000) return x * pio2_hi + x * pio2_lo;
    if (ix > 0x3f800000) return (x - x) / (x - x);
    if (ix < 0x3f000000) {
        if (ix < 0x32000000) {
            if (huge + x > one) return x;
        } else {
            float t = x * x;
            float w = t * (p0 + t * (p1 + t * (p2 + t * (p3 + t * p4))));
            return x + x * w;
        }
    }
    float w = one - fabsf(x);
    float t = w * 0.5f;
    float p = t * (p0 + t * (p1 + t * (p2 + t * (p3 + t * p4))));
    float s = sqrtf(t);
    if (ix >= 0x3F79999A) {
        t = pio2_hi - (2.0f * (s + s * p) - pio2_lo);
    } else {
        w = ffromword(fword(s) & 0xfffff000);
        float c = (t - w * w) / (s + w);
        float r = p;
        p = 2.0f * s * r - (pio2_lo - 2.0f * c);
        float q = pio4_hi - 2.0f * w;
        t = pio4_hi - (p - q);
    }
    return hx > 0 ? t : -t;
}

CB_HDNI float lm_atanf(float x) {
    const float atanhi[4] = {(float)4.6364760399e-01, (float)7.8539812565e-01,
                             (float)9.8279368877e-01, (float)1.5707962513e+00};
    const float atanlo[4] = {(float)5.0121582440e-09, (float)3.7748947079e-08,
                             (float)3.4473217170e-08, (float)7.5497894159e-08};
    const float aT[11] = {(float)3.3333334327e-01,  (float)-2.0000000298e-01,
                          (float)1.4285714924e-01,  (float)-1.1111110449e-01,
                          (float)9.0908870101e-02,  (float)-7.6918758452e-02,
                          (float)6.6610731184e-02,  (float)-5.8335702866e-02,
                          (float)4.9768779427e-02,  (float)-3.6531571299e-02,
                          (float)1.6285819933e-02};
    const float one = 1.0f, huge = 1.0e30f;
    int32_t hx = fword(x), ix = hx & 0x7fffffff, id;
    if (ix >= 0x4c000000) {
        if (ix > 0x7f800000) return x + x;
        if (hx > 0) return atanhi[3] + atanlo[3];
        return -atanhi[3] - atanlo[3];
    }
    if (ix < 0x3ee00000) {
        if (ix < 0x31000000) {
            if (huge + x > one) return x;
        }
        id = -1;
    } else {
        x = fabsf(x);
        if (ix < 0x3f980000) {
            if (ix < 0x3f300000) {
                id = 0;
                x = ((float)2.0 * x - one) / ((float)2.0 + x);
            } else {
                id = 1;
                x = (x - one) / (x + one);
            }
        } else if (ix < 0x401c0000) {
            id = 2;
            x = (x - (float)1.5) / (one + (float)1.5 * x);
        } else {
            id = 3;
            x = -(float)1.0 / x;
        }
    }
    float z = x * x;
    float w = z * z;
    float s1 = z * (aT[0] + w * (aT[2] + w * (aT[4] + w * (aT[6] + w * (aT[8] + w * aT[10])))));
    float s2 = w * (aT[1] + w * (aT[3] + w * (aT[5] + w * (aT[7] + w * aT[9]))));
    if (id < 0) return x - x * (s1 + s2);
    z = atanhi[id] - ((x * (s1 + s2) - atanlo[id]) - x);
    return hx < 0 ? -z : z;
}

CB_HDNI float lm_atan2f(float y, float x) {
    const float tiny = 1.0e-30f, zero = 0.0f, pi_o_4 = (float)7.8539818525e-01,
                pi_o_2 = (float)1.5707963705e+00, pi = (float)3.1415927410e+00,
                pi_lo = (float)-8.7422776573e-08;
    int32_t hx = fword(x), hy = fword(y);
    int32_t ix = hx & 0x7fffffff, iy = hy & 0x7fffffff;
    if (ix > 0x7f800000 || iy > 0x7f800000) return x + y;
    if (hx == 0x3f800000) return lm_atanf(y);
    int32_t m = ((hy >> 31) & 1) | ((hx >> 30) & 2);
    if (iy == 0) {
        switch (m) {
            case 0:
            case 1: return y;
            case 2: return pi + tiny;
            default: return -pi - tiny;
        }
    }
    if (ix == 0) return hy < 0 ? -pi_o_2 - tiny : pi_o_2 + tiny;
    if (ix == 0x7f800000) {
        if (iy == 0x7f800000) {
            switch (m) {
                case 0: return pi_o_4 + tiny;
                case 1: return -pi_o_4 - tiny;
                case 2: return (float)3.0 * pi_o_4 + tiny;
                default: return (float)-3.0 * pi_o_4 - tiny;
            }
        }
        switch (m) {
            case 0: return zero;
            case 1: return -zero;
            case 2: return pi + tiny;
            default: return -pi - tiny;
        }
    }
    if (iy == 0x7f800000) return hy < 0 ? -pi_o_2 - tiny : pi_o_2 + tiny;
    int32_t k = (iy - ix) >> 23;
    float z;
    if (k > 60)
        z = pi_o_2 + (float)0.5 * pi_lo;
    else if (hx < 0 && k < -60)
        z = 0.0;
    else
        z = lm_atanf(fabsf(y / x));
    switch (m) {
        case 0: return z;
        case 1: return ffromword(fword(z) ^ (int32_t)0x80000000);
        case 2: return pi - (z - pi_lo);
        default: return (z - pi_lo) - pi;
    }
}

// ============================================================================================
// Double sine / cosine: glibc's IBM Accurate Mathematical Library (s_sin.c, branred.c).
constexpr double kSinT1 = -0x1.5555555555555p-3, kSinT2 = 0x1.1111111110ECEp-7,
                 kSinT3 = -0x1.A01A019DB08B8p-13, kSinT4 = 0x1.71DE27B9A7ED9p-19,
                 kSinT5 = -0x1.ADDFFC2FCDF59p-26;
constexpr double kBig = 0x1.8000000000000p45;  // rounds |x| to 1/128 and exposes the index
constexpr double kHp0 = 0x1.921FB54442D18p0, kHp1 = 0x1.1A62633145C07p-54;
constexpr double kMp1 = 0x1.921FB58000000p0, kMp2 = -0x1.DDE973C000000p-27,
                 kPp3 = -0x1.CB3B398000000p-55, kPp4 = -0x1.d747f23e32ed7p-83;
constexpr double kHpInv = 0x1.45F306DC9C883p-1, kToInt = 0x1.8000000000000p52;
constexpr double kSn3 = -0x1.5555555555515p-3, kSn5 = 0x1.11110e829872fp-7;
constexpr double kCs2 = 0x1.0000000000000p-1, kCs4 = -0x1.5555555555535p-5,
                 kCs6 = 0x1.6c16bedd9e239p-10;

CB_HD int sctab_index(double u) { return (int)(uint32_t)d2u(u) << 2; }

// cos(x + dx), |x| <= 0.855469 (glibc do_cos)
CB_HD double dcos_core(double x, double dx) {
    const uint64_t *T = CB_TAB(kSinCosTab);
    if (x < 0) dx = -dx;
    double u = kBig + fabs(x);
    x = fabs(x) - (u - kBig) + dx;
    double xx = x * x;
    double s = fma(x * xx, fma(xx, kSn5, kSn3), x);
    double c = xx * fma(xx, fma(xx, kCs6, kCs4), kCs2);
    int k = sctab_index(u);
    double sn = tabd(T, k), ssn = tabd(T, k + 1), cs = tabd(T, k + 2), ccs = tabd(T, k + 3);
    double cor = fma(-s, sn, fma(-c, cs, fma(-s, ssn, ccs)));
    return cs + cor;
}
// sin(x + dx), |x| <= 0.855469 (glibc do_sin)
CB_HD double dsin_core(double x, double dx) {
    double x0 = x;
    if (fabs(x) < 0.126) {
        double xx = x * x;
        double t = fma(xx, fma(xx, fma(xx, fma(xx, kSinT5, kSinT4), kSinT3), kSinT2), kSinT1);
        double cor = fma(xx, fma(t, x, -(0.5 * dx)), dx);
        return x + cor;
    }
    const uint64_t *T = CB_TAB(kSinCosTab);
    if (x <= 0) dx = -dx;
    double u = kBig + fabs(x);
    x = fabs(x) - (u - kBig);
    double xx = x * x;
    double s = x + fma(x * xx, fma(xx, kSn5, kSn3), dx);
    double c = fma(x, dx, xx * fma(xx, fma(xx, kCs6, kCs4), kCs2));
    int k = sctab_index(u);
    double sn = tabd(T, k), ssn = tabd(T, k + 1), cs = tabd(T, k + 2), ccs = tabd(T, k + 3);
    double cor = fma(s, cs, fma(-c, sn, fma(s, ccs, ssn)));
    return copysign(sn + cor, x0);
}
// |x| < 105414350 (glibc reduce_sincos)
CB_HD int dreduce(double x, double *a, double *da) {
    double t = fma(x, kHpInv, kToInt);
    double xn = t - kToInt;
    double y = fma(-xn, kMp2, fma(-xn, kMp1, x));
    int n = (int)(uint32_t)d2u(t) & 3;
    double b = fma(-xn, kPp3, y);
    double db = fma(-xn, kPp3, y - b);
    double r = fma(-xn, kPp4, b);
    db = db + fma(-xn, kPp4, b - r);
    *a = r;
    *da = db;
    return n;
}
CB_HD double dsincos_quadrant(double a, double da, int n) {
    double r = (n & 1) ? dcos_core(a, da) : dsin_core(a, da);
    return (n & 2) ? -r : r;
}
// glibc branred.c, one half of the split argument; built without FMA.
CB_HD void branred_part(double x, double *f, double *ft, double *s_out) {
    const uint64_t *toverp = CB_TAB(kTwoOverPi24);
    const double t576 = 0x1p576, tm24 = 0x1p-24, big = 0x1.8p52, big1 = 0x1.8p54;
    double r[6], b, bb, s = 0, t;
    int k = (int)((d2u(x) >> 52) & 2047);
    k = (k - 450) / 24;
    if (k < 0) k = 0;
    double gor = u2d(d2u(t576) - ((uint64_t)(k * 24) << 52));
    for (int i = 0; i < 6; i++) {
        r[i] = x * tabd(toverp, k + i) * gor;
        gor *= tm24;
    }
    for (int i = 0; i < 3; i++) {
        b = (r[i] + big) - big;
        s += b;
        r[i] -= b;
    }
    t = 0;
    for (int i = 0; i < 6; i++) t += r[5 - i];
    bb = (((((r[0] - t) + r[1]) + r[2]) + r[3]) + r[4]) + r[5];
    b = (t + big) - big;
    s += b;
    t -= b;
    b = t + bb;
    bb = (t - b) + bb;
    double sb = (s + big1) - big1;
    s -= sb;
    *f = b;
    *ft = bb;
    *s_out = s;
}
CB_HDNI int branred(double x, double *a, double *aa) {
    const double tm600 = 0x1p-600, split = 134217729.0;
    const double hp0 = 0x1.921FB54442D18p0, hp1 = 0x1.1A62633145C07p-54;
    const double mp1 = 0x1.921FB58000000p0, mp2 = -0x1.DDE9740000000p-27;
    double b, bb, sum, s1, s2, b1, bb1, b2, bb2, x1, x2, t1, t2, t;
    x *= tm600;
    t = x * split;
    x1 = t - (t - x);
    x2 = x - x1;
    branred_part(x1, &b1, &bb1, &s1);
    branred_part(x2, &b2, &bb2, &s2);
    sum = s1 + s2;
    b = b1 + b2;
    bb = (fabs(b1) > fabs(b2)) ? (b1 - b) + b2 : (b2 - b) + b1;
    if (b > 0.5) {
        b -= 1.0;
        sum += 1.0;
    } else if (b < -0.5) {
        b += 1.0;
        sum -= 1.0;
    }
    s1 = b + ((bb + bb1) + bb2);
    s2 = ((b - s1) + bb) + (bb1 + bb2);
    b = s1 * split;
    t1 = b - (b - s1);
    t2 = s1 - t1;
    b = s1 * hp0;
    bb = (((t1 * mp1 - b) + t1 * mp2) + t2 * mp1) + ((t2 * mp2 + s1 * hp1) + s2 * hp0);
    s1 = b + bb;
    t = (b - s1) + bb;
    *a = s1;
    *aa = t;
    return ((int)sum) & 3;
}
CB_HDNI double lm_sin(double x) {
    int32_t k = (int32_t)(d2u(x) >> 32) & 0x7fffffff;
    if (k < 0x3e500000) return x;
    if (k < 0x3feb6000) return dsin_core(x, 0);
    if (k < 0x400368fd) {
        double t = kHp0 - fabs(x);
        return copysign(dcos_core(t, kHp1), x);
    }
    double a, da;
    if (k < 0x419921FB) {
        int n = dreduce(x, &a, &da);
        return dsincos_quadrant(a, da, n);
    }
    if (k < 0x7ff00000) {
        int n = branred(x, &a, &da);
        return dsincos_quadrant(a, da, n);
    }
    return x / x;
}
CB_HDNI double lm_cos(double x) {
    int32_t k = (int32_t)(d2u(x) >> 32) & 0x7fffffff;
    if (k < 0x3e400000) return 1.0;
    if (k < 0x3feb6000) return dcos_core(x, 0);
    if (k < 0x400368fd) {
        double y = kHp0 - fabs(x);
        double a = y + kHp1;
        double da = (y - a) + kHp1;
        return dsin_core(a, da);
    }
    double a, da;
    if (k < 0x419921FB) {
        int n = dreduce(x, &a, &da);
        return dsincos_quadrant(a, da, n + 1);
    }
    if (k < 0x7ff00000) {
        int n = branred(x, &a, &da);
        return dsincos_quadrant(a, da, n + 1);
    }
    return x / x;
}

// ============================================================================================
// Double arc cosine: glibc e_asin.c __ieee754_acos (IBM).
constexpr double kAsinP1 = 0x1.55555555554f9p-3, kAsinP2 = 0x1.333333336127dp-4,
                 kAsinP3 = 0x1.6db6dae42c0e4p-5, kAsinP4 = 0x1.f1c7e04f4ad99p-6,
                 kAsinP5 = 0x1.6e442c822d419p-6, kAsinP6 = 0x1.292d80f453c72p-6;
constexpr double kRt0 = 0x1.fffffffecc1ddp-1, kRt1 = 0x1.fffffff757304p-2,
                 kRt2 = 0x1.800496769c91ap-2, kRt3 = 0x1.4006318d1dab9p-2;

CB_HD double asin_series(double z) {
    return fma(fma(fma(fma(fma(z, kAsinP6, kAsinP5), z, kAsinP4), z, kAsinP3), z, kAsinP2), z,
               kAsinP1);
}
// Table branch: Taylor expansion around a tabulated point; `deg` is the last term offset.
CB_HD double acos_tab(int n, int deg, double x, int32_t hx) {
    const uint64_t *T = CB_TAB(kAsinTab);
    double y = hx > 0 ? x - tabd(T, n) : -x - tabd(T, n);
    double acc = tabd(T, n + deg);
    for (int j = deg - 1; j >= 2; j--) acc = fma(acc, y, tabd(T, n + j));
    double res1 = fma(y * y, acc, tabd(T, n + deg + 1));
    double lo = fma(tabd(T, n + 1), y, res1);
    double hi = hx > 0 ? (kHp0 - tabd(T, n + deg + 2)) : (kHp0 + tabd(T, n + deg + 2));
    lo = hx > 0 ? (kHp1 - lo) : (kHp1 + lo);
    return hi + lo;
}
CB_HDNI double lm_acos(double x) {
    uint64_t bits = d2u(x);
    int32_t hx = (int32_t)(bits >> 32);
    int32_t k = hx & 0x7fffffff;
    if (k < 0x3c880000) return kHp0;
    if (k < 0x3fc00000) {
        double x2 = x * x;
        double r = kHp0 - x;
        double cor = fma(-asin_series(x2), x * x2, ((kHp0 - r) - x) + kHp1);
        return r + cor;
    }
    if (k < 0x3fe00000) {
        int n = (k < 0x3fd00000) ? 11 * ((k & 0x000fffff) >> 15) : 11 * ((k & 0x000fffff) >> 14) + 352;
        return acos_tab(n, 6, x, hx);
    }
    if (k < 0x3fe80000) return acos_tab(1056 + ((k & 0x000fe000) >> 11) * 3, 7, x, hx);
    if (k < 0x3fed8000) return acos_tab(992 + ((k & 0x000fe000) >> 13) * 13, 8, x, hx);
    if (k < 0x3fee8000) return acos_tab(884 + ((k & 0x000fe000) >> 13) * 14, 9, x, hx);
    if (k < 0x3fef0000) return acos_tab(768 + ((k & 0x000fe000) >> 13) * 15, 10, x, hx);
    if (k < 0x3ff00000) {
        double z = 0.5 * (hx > 0 ? (1.0 - x) : (1.0 + x));
        int32_t kz = (int32_t)(d2u(z) >> 32);
        double t = tabd(CB_TAB(kRsqrtSeed), (kz & 0x001fffff) >> 14) *
                   tabd(CB_TAB(kPow2Tab), 511 - (kz >> 21));
        double r = fma(-(t * t), z, 1.0);
        t = t * fma(fma(fma(r, kRt3, kRt2), r, kRt1), r, kRt0);
        double c = t * z;
        double refine = fma(-(t * 0.5), c, 1.5);
        const double split = 134217728.0;
        double w = fma(-c, split, fma(c, split, c));
        double cc = fma(-w, w, z) / fma(refine, c, w);
        double p = asin_series(z) * z;
        double prod = p * (w + cc);
        if (hx < 0) {
            double cor = (kHp1 - cc) - prod;
            double dd = kHp0 - w;
            double res = dd + cor;
            return res + res;
        }
        double cor = cc + prod;
        double res = w + cor;
        return res + res;
    }
    if (k == 0x3ff00000 && (uint32_t)bits == 0) return hx > 0 ? 0 : 2.0 * kHp0;
    return (x - x) / (x - x);
}

// ============================================================================================
// Double power: Arm Optimized Routines pow.c.
constexpr double kLn2Hi = 0x1.62e42fefa3800p-1, kLn2Lo = 0x1.ef35793c76730p-45;
constexpr double kInvLn2N = 0x1.71547652b82fep0 * 128;
constexpr double kNegLn2HiN = -0x1.62e42fefa0000p-8, kNegLn2LoN = -0x1.cf79abc9e3b3ap-47;
constexpr double kExpShift = 0x1.8p52;

CB_HD uint32_t top12d(double v) { return (uint32_t)(d2u(v) >> 52); }

CB_HD double pow_log(uint64_t ix, double *tail) {
    const uint64_t *T = CB_TAB(kPowLogTab);
    // log(1+r) polynomial after the linear term, evaluation scale factors folded in.
    const double A0 = -0x1p-1, A1 = 0x1.555555555556p-2 * -2, A2 = -0x1.0000000000006p-2 * -2,
                 A3 = 0x1.999999959554ep-3 * 4, A4 = -0x1.555555529a47ap-3 * 4,
                 A5 = 0x1.2495b9b4845e9p-3 * -8, A6 = -0x1.0002b8b263fc3p-3 * -8;
    const uint64_t kOff = 0x3fe6955500000000ull;
    uint64_t tmp = ix - kOff;
    int i = (int)((tmp >> (52 - 7)) % 128);
    int k = (int)((int64_t)tmp >> 52);
    uint64_t iz = ix - (tmp & 0xfffull << 52);
    double z = u2d(iz);
    double kd = (double)k;
    double invc = tabd(T, 3 * i), logc = tabd(T, 3 * i + 1), logctail = tabd(T, 3 * i + 2);
    double r = fma(z, invc, -1.0);
    double t1 = fma(kd, kLn2Hi, logc);
    double t2 = t1 + r;
    double lo1 = fma(kd, kLn2Lo, logctail);
    double lo2 = t1 - t2 + r;
    double ar = A0 * r;
    double ar2 = r * ar;
    double ar3 = r * ar2;
    double hi = t2 + ar2;
    double lo3 = fma(ar, r, -ar2);
    double lo4 = t2 - hi + ar2;
    double p56 = fma(r, A6, A5);
    double p34 = fma(ar2, p56, fma(r, A4, A3));
    double p12 = fma(ar2, p34, fma(r, A2, A1));
    double lo = fma(ar3, p12, lo1 + lo2 + lo3 + lo4);
    double y = hi + lo;
    *tail = hi - y + lo;
    return y;
}
CB_HD double pow_oflow(uint32_t s) { double v = s ? -0x1p769 : 0x1p769; return v * 0x1p769; }
CB_HD double pow_uflow(uint32_t s) { double v = s ? -0x1p-767 : 0x1p-767; return v * 0x1p-767; }
CB_HDNI double pow_special(double tmp, uint64_t sbits, uint64_t ki) {
    double scale, y;
    if ((ki & 0x80000000) == 0) {
        sbits -= 1009ull << 52;
        scale = u2d(sbits);
        return 0x1p1009 * fma(scale, tmp, scale);
    }
    sbits += 1022ull << 52;
    scale = u2d(sbits);
    double st = scale * tmp;
    y = scale + st;
    if (fabs(y) < 1.0) {
        double hi, lo, one = 1.0;
        if (y < 0.0) one = -1.0;
        lo = scale - y + st;
        hi = one + y;
        lo = one - hi + y + lo;
        y = (hi + lo) - one;
        if (y == 0.0) y = u2d(sbits & 0x8000000000000000ull);
    }
    return 0x1p-1022 * y;
}
CB_HD double pow_exp(double x, double xtail, uint32_t sign_bias) {
    const uint64_t *T = CB_TAB(kPowExpTab);
    const double C2 = 0x1.ffffffffffdbdp-2, C3 = 0x1.555555555543cp-3, C4 = 0x1.55555cf172b91p-5,
                 C5 = 0x1.1111167a4d017p-7;
    uint32_t abstop = top12d(x) & 0x7ff;
    if (abstop - top12d(0x1p-54) >= top12d(512.0) - top12d(0x1p-54)) {
        if (abstop - top12d(0x1p-54) >= 0x80000000) {
            double one = 1.0 + x;
            return sign_bias ? -one : one;
        }
        if (abstop >= top12d(1024.0)) {
            if (d2u(x) >> 63) return pow_uflow(sign_bias);
            return pow_oflow(sign_bias);
        }
        abstop = 0;
    }
    double kd = fma(kInvLn2N, x, kExpShift);
    uint64_t ki = d2u(kd);
    kd -= kExpShift;
    double r = fma(kd, kNegLn2LoN, fma(kd, kNegLn2HiN, x));
    r += xtail;
    uint64_t idx = 2 * (ki % 128);
    uint64_t top = (ki + sign_bias) << (52 - 7);
    double tail = u2d(T[idx]);
    uint64_t sbits = T[idx + 1] + top;
    double r2 = r * r;
    double tmp = fma(fma(r, C5, C4), r2 * r2, fma(fma(r, C3, C2), r2, tail + r));
    if (abstop == 0) return pow_special(tmp, sbits, ki);
    double scale = u2d(sbits);
    return fma(scale, tmp, scale);
}
CB_HD int pow_checkint(uint64_t iy) {
    int e = iy >> 52 & 0x7ff;
    if (e < 0x3ff) return 0;
    if (e > 0x3ff + 52) return 2;
    if (iy & ((1ull << (0x3ff + 52 - e)) - 1)) return 0;
    if (iy & (1ull << (0x3ff + 52 - e))) return 1;
    return 2;
}
CB_HD int zeroinfnan_d(uint64_t i) { return 2 * i - 1 >= 2 * d2u(INFINITY) - 1; }
CB_HD bool is_snan_d(double v) {
    uint64_t b = d2u(v);
    return 2 * (b ^ 0x0008000000000000ull) > 2 * 0x7ff8000000000000ull;
}
CB_HDNI double lm_pow(double x, double y) {
    uint32_t sign_bias = 0;
    uint64_t ix = d2u(x), iy = d2u(y);
    uint32_t topx = top12d(x), topy = top12d(y);
    if (topx - 0x001 >= 0x7ff - 0x001 || (topy & 0x7ff) - 0x3be >= 0x43e - 0x3be) {
        if (zeroinfnan_d(iy)) {
            if (2 * iy == 0) return is_snan_d(x) ? x + y : 1.0;
            if (ix == d2u(1.0)) return is_snan_d(y) ? x + y : 1.0;
            if (2 * ix > 2 * d2u(INFINITY) || 2 * iy > 2 * d2u(INFINITY)) return x + y;
            if (2 * ix == 2 * d2u(1.0)) return 1.0;
            if ((2 * ix < 2 * d2u(1.0)) == !(iy >> 63)) return 0.0;
            return y * y;
        }
        if (zeroinfnan_d(ix)) {
            double x2 = x * x;
            if (ix >> 63 && pow_checkint(iy) == 1) x2 = -x2;
            return iy >> 63 ? 1 / x2 : x2;
        }
        if (ix >> 63) {
            int yint = pow_checkint(iy);
            if (yint == 0) return (x - x) / (x - x);
            if (yint == 1) sign_bias = 0x800 << 7;
            ix &= 0x7fffffffffffffffull;
            topx &= 0x7ff;
        }
        if ((topy & 0x7ff) - 0x3be >= 0x43e - 0x3be) {
            if (ix == d2u(1.0)) return 1.0;
            if ((topy & 0x7ff) < 0x3be) return ix > d2u(1.0) ? 1.0 + y : 1.0 - y;
            return (ix > d2u(1.0)) == (topy < 0x800) ? pow_oflow(0) : pow_uflow(0);
        }
        if (topx == 0) {
            ix = d2u(x * 0x1p52);
            ix &= 0x7fffffffffffffffull;
            ix -= 52ull << 52;
        }
    }
    double lo;
    double hi = pow_log(ix, &lo);
    double ehi = y * hi;
    double elo = fma(y, lo, fma(y, hi, -ehi));
    return pow_exp(ehi, elo, sign_bias);
}

}  // namespace lm
}  // namespace cb
