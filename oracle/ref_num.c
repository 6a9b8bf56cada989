/*
 * oracle/ref_num.c -- det-num restated in C (TEST INFRASTRUCTURE, see ref.h).
 *
 * Follows crates/det-num/src/{reduce,math,round,f16,hash,canary}.rs and the
 * vendored libm files under crates/det-num/src/vendored_libm/ (rust-lang/libm
 * 0.2.16, itself from FreeBSD msun).  The transcendental routines below are
 * restatements of the published fdlibm algorithms; their notices follow.
 *
 * ====================================================
 * Copyright (C) 1993 by Sun Microsystems, Inc. All rights reserved.
 *
 * Developed at SunPro, a Sun Microsystems, Inc. business.
 * Permission to use, copy, modify, and distribute this
 * software is freely granted, provided that this notice
 * is preserved.
 * ====================================================
 * Copyright (C) 2004 by Sun Microsystems, Inc. All rights reserved.
 *
 * Permission to use, copy, modify, and distribute this
 * software is freely granted, provided that this notice
 * is preserved.
 * ====================================================
 * expf: conversion to float by Ian Lance Taylor, Cygnus Support.
 */
#include "ref.h"
#include "ref_internal.h"

#include <math.h>
#include <string.h>

/* ---- reduce.rs:2-38: 8-lane interleaved accumulation, fixed combine tree */
static float finish_8lane(const float a[8]) {
    return ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
}

float ref_dot_f32(const float* x, const float* y, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (size_t i = 0; i < n; i++) acc[i & 7] += x[i] * y[i];
    return finish_8lane(acc);
}

/* sum_f32_ref (det-num reduce.rs:14-23): 8 lane chains, fixed combine tree */
float ref_sum_f32(const float* x, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (size_t i = 0; i < n; i++) acc[i & 7] += x[i];
    return finish_8lane(acc);
}

/* sum_squares_f32_ref (det-num reduce.rs:25-38) */
float ref_sum_squares_f32(const float* x, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (size_t i = 0; i < n; i++) acc[i & 7] += x[i] * x[i];
    return finish_8lane(acc);
}

/* ---- vendored_libm.rs:94-119 scalbn_f32 ------------------------------- */
static float scalbnf_ref(float x, int n) {
    const float x1p127 = u2f(0x7f000000u);
    const float x1p_126 = u2f(0x00800000u);
    if (n > 127) {
        x *= x1p127;
        n -= 127;
        if (n > 127) {
            x *= x1p127;
            n -= 127;
            if (n > 127) n = 127;
        }
    } else if (n < -126) {
        x *= x1p_126;
        n += 126;
        if (n < -126) {
            x *= x1p_126;
            n += 126;
            if (n < -126) n = -126;
        }
    }
    return x * u2f((uint32_t)(0x7f + n) << 23);
}

/* ---- vendored_libm/expf.rs:33-106 (FreeBSD e_expf.c) ------------------- */
float ref_expf(float x) {
    static const float HALF[2] = {0.5f, -0.5f};
    const float LN2_HI = u2f(0x3f317200u);
    const float LN2_LO = u2f(0x35bfbe8eu);
    const float INV_LN2 = u2f(0x3fb8aa3bu);
    const float P1 = 1.6666625440e-1f;
    const float P2 = -2.7667332906e-3f;
    const float x1p127 = u2f(0x7f000000u);

    uint32_t hx = f2u(x);
    int sign = (int)(hx >> 31);
    hx &= 0x7fffffffu;
    if (hx >= 0x42aeac50u) {
        if (hx > 0x7f800000u) return x; /* NaN */
        if (hx >= 0x42b17218u && !sign) return x * x1p127; /* overflow */
        if (sign && hx >= 0x42cff1b5u) return 0.0f;         /* underflow */
    }
    int k;
    float hi, lo;
    if (hx > 0x3eb17218u) {
        if (hx > 0x3f851592u)
            k = f32_as_i32(INV_LN2 * x + HALF[sign]);
        else
            k = 1 - sign - sign;
        float kf = (float)k;
        hi = x - kf * LN2_HI;
        lo = kf * LN2_LO;
        x = hi - lo;
    } else if (hx > 0x39000000u) {
        k = 0;
        hi = x;
        lo = 0.0f;
    } else {
        return 1.0f + x;
    }
    float xx = x * x;
    float c = x - xx * (P1 + xx * P2);
    float y = 1.0f + (x * c / (2.0f - c) - lo + hi);
    return k == 0 ? y : scalbnf_ref(y, k);
}

void ref_expf_batch(const float* x, float* y, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] = ref_expf(x[i]);
}

/* math.rs:30-34 */
float ref_silu(float x) {
    float t = ref_expf(-x);
    float d = 1.0f + t;
    return x / d;
}

/* ---- vendored_libm.rs scalbn_f64 ---------------------------------------- */
static double scalbn_ref(double x, int n) {
    const double x1p1023 = u2d(0x7fe0000000000000ull);
    const double x1p_1022 = u2d(0x0010000000000000ull);
    if (n > 1023) {
        x *= x1p1023;
        n -= 1023;
        if (n > 1023) {
            x *= x1p1023;
            n -= 1023;
            if (n > 1023) n = 1023;
        }
    } else if (n < -1022) {
        x *= x1p_1022;
        n += 1022;
        if (n < -1022) {
            x *= x1p_1022;
            n += 1022;
            if (n < -1022) n = -1022;
        }
    }
    return x * u2d((uint64_t)(0x3ff + n) << 52);
}

/* ---- vendored_libm/exp.rs (FreeBSD e_exp.c) ------------------------------ */
double ref_exp_f64(double x) {
    static const double HALF[2] = {0.5, -0.5};
    const double LN2HI = 6.93147180369123816490e-01;
    const double LN2LO = 1.90821492927058770002e-10;
    const double INVLN2 = 1.44269504088896338700e+00;
    const double P1 = 1.66666666666666019037e-01;
    const double P2 = -2.77777777770155933842e-03;
    const double P3 = 6.61375632143793436117e-05;
    const double P4 = -1.65339022054652515390e-06;
    const double P5 = 4.13813679705723846039e-08;
    const double x1p1023 = u2d(0x7fe0000000000000ull);

    uint32_t hx = (uint32_t)(d2u(x) >> 32);
    int sign = (int)(hx >> 31);
    hx &= 0x7fffffffu;
    if (hx >= 0x4086232bu) {
        if (x != x) return x;
        if (x > 709.782712893383973096) return x * x1p1023;
        if (x < -708.39641853226410622) {
            if (x < -745.13321910194110842) return 0.0;
        }
    }
    int k;
    double hi, lo;
    if (hx > 0x3fd62e42u) {
        if (hx >= 0x3ff0a2b2u)
            k = f64_as_i32(INVLN2 * x + HALF[sign]);
        else
            k = 1 - sign - sign;
        hi = x - (double)k * LN2HI;
        lo = (double)k * LN2LO;
        x = hi - lo;
    } else if (hx > 0x3e300000u) {
        k = 0;
        hi = x;
        lo = 0.0;
    } else {
        return 1.0 + x;
    }
    double xx = x * x;
    double c = x - xx * (P1 + xx * (P2 + xx * (P3 + xx * (P4 + xx * P5))));
    double y = 1.0 + (x * c / (2.0 - c) - lo + hi);
    return k == 0 ? y : scalbn_ref(y, k);
}

/* ---- vendored_libm/log.rs (FreeBSD e_log.c) ------------------------------- */
double ref_ln_f64(double x) {
    const double LN2_HI = 6.93147180369123816490e-01;
    const double LN2_LO = 1.90821492927058770002e-10;
    const double LG1 = 6.666666666666735130e-01;
    const double LG2 = 3.999999999940941908e-01;
    const double LG3 = 2.857142874366239149e-01;
    const double LG4 = 2.222219843214978396e-01;
    const double LG5 = 1.818357216161805012e-01;
    const double LG6 = 1.531383769920937332e-01;
    const double LG7 = 1.479819860511658591e-01;
    const double x1p54 = u2d(0x4350000000000000ull);

    uint64_t ui = d2u(x);
    uint32_t hx = (uint32_t)(ui >> 32);
    int k = 0;
    if (hx < 0x00100000u || (hx >> 31) != 0) {
        if ((ui << 1) == 0) return -1.0 / (x * x);
        if ((hx >> 31) != 0) return (x - x) / 0.0;
        k -= 54;
        x *= x1p54;
        ui = d2u(x);
        hx = (uint32_t)(ui >> 32);
    } else if (hx >= 0x7ff00000u) {
        return x;
    } else if (hx == 0x3ff00000u && (ui << 32) == 0) {
        return 0.0;
    }
    hx += 0x3ff00000u - 0x3fe6a09eu;
    k += (int)(hx >> 20) - 0x3ff;
    hx = (hx & 0x000fffffu) + 0x3fe6a09eu;
    ui = ((uint64_t)hx << 32) | (ui & 0xffffffffull);
    x = u2d(ui);

    double f = x - 1.0;
    double hfsq = 0.5 * f * f;
    double s = f / (2.0 + f);
    double z = s * s;
    double w = z * z;
    double t1 = w * (LG2 + w * (LG4 + w * LG6));
    double t2 = z * (LG1 + w * (LG3 + w * (LG5 + w * LG7)));
    double r = t2 + t1;
    double dk = (double)k;
    return s * (hfsq + r) + dk * LN2_LO - hfsq + f + dk * LN2_HI;
}

/* ---- vendored_libm/k_sin.rs, k_cos.rs ------------------------------------ */
static double k_sin(double x, double y, int iy) {
    const double S1 = -1.66666666666666324348e-01;
    const double S2 = 8.33333333332248946124e-03;
    const double S3 = -1.98412698298579493134e-04;
    const double S4 = 2.75573137070700676789e-06;
    const double S5 = -2.50507602534068634195e-08;
    const double S6 = 1.58969099521155010221e-10;
    double z = x * x;
    double w = z * z;
    double r = S2 + z * (S3 + z * S4) + z * w * (S5 + z * S6);
    double v = z * x;
    if (iy == 0) return x + v * (S1 + z * r);
    return x - ((z * (0.5 * y - v * r) - y) - v * S1);
}

/* k_cos (det-num vendored_libm/k_cos.rs:54) */
static double k_cos(double x, double y) {
    const double C1 = 4.16666666666666019037e-02;
    const double C2 = -1.38888888888741095749e-03;
    const double C3 = 2.48015872894767294178e-05;
    const double C4 = -2.75573143513906633035e-07;
    const double C5 = 2.08757232129817482790e-09;
    const double C6 = -1.13596475577881948265e-11;
    double z = x * x;
    double w = z * z;
    double r = z * (C1 + z * (C2 + z * C3)) + w * w * (C4 + z * (C5 + z * C6));
    double hz = 0.5 * z;
    w = 1.0 - hz;
    return w + (((1.0 - w) - hz) + (z * r - x * y));
}

/* ---- vendored_libm/rem_pio2.rs (FreeBSD e_rem_pio2.c) -------------------
 * Only the |x| < 2^20*(pi/2) branches are restated.  Larger arguments would
 * need rem_pio2_large (k_rem_pio2.c); the only caller on this path is the
 * RoPE table, whose phase is pos * omega <= pos < context length, so such
 * inputs are rejected by ref_rope_tables before they get here. */
static int rem_pio2(double x, double* y0, double* y1, int* large) {
    const double EPS = 2.2204460492503131e-16;
    const double TO_INT = 1.5 / EPS;
    const double INV_PIO2 = 6.36619772367581382433e-01;
    const double PIO2_1 = 1.57079632673412561417e+00;
    const double PIO2_1T = 6.07710050650619224932e-11;
    const double PIO2_2 = 6.07710050630396597660e-11;
    const double PIO2_2T = 2.02226624879595063154e-21;
    const double PIO2_3 = 2.02226624871116645580e-21;
    const double PIO2_3T = 8.47842766036889956997e-32;

    int sign = (int)(d2u(x) >> 63);
    uint32_t ix = (uint32_t)(d2u(x) >> 32) & 0x7fffffffu;
    *large = 0;

    if (ix <= 0x400f6a7au) {
        if ((ix & 0xfffffu) == 0x921fbu) goto medium;
        if (ix <= 0x4002d97cu) {
            if (sign == 0) {
                double z = x - PIO2_1;
                *y0 = z - PIO2_1T;
                *y1 = (z - *y0) - PIO2_1T;
                return 1;
            } else {
                double z = x + PIO2_1;
                *y0 = z + PIO2_1T;
                *y1 = (z - *y0) + PIO2_1T;
                return -1;
            }
        } else if (sign == 0) {
            double z = x - 2.0 * PIO2_1;
            *y0 = z - 2.0 * PIO2_1T;
            *y1 = (z - *y0) - 2.0 * PIO2_1T;
            return 2;
        } else {
            double z = x + 2.0 * PIO2_1;
            *y0 = z + 2.0 * PIO2_1T;
            *y1 = (z - *y0) + 2.0 * PIO2_1T;
            return -2;
        }
    }
    if (ix <= 0x401c463bu) {
        if (ix <= 0x4015fdbcu) {
            if (ix == 0x4012d97cu) goto medium;
            if (sign == 0) {
                double z = x - 3.0 * PIO2_1;
                *y0 = z - 3.0 * PIO2_1T;
                *y1 = (z - *y0) - 3.0 * PIO2_1T;
                return 3;
            } else {
                double z = x + 3.0 * PIO2_1;
                *y0 = z + 3.0 * PIO2_1T;
                *y1 = (z - *y0) + 3.0 * PIO2_1T;
                return -3;
            }
        } else {
            if (ix == 0x401921fbu) goto medium;
            if (sign == 0) {
                double z = x - 4.0 * PIO2_1;
                *y0 = z - 4.0 * PIO2_1T;
                *y1 = (z - *y0) - 4.0 * PIO2_1T;
                return 4;
            } else {
                double z = x + 4.0 * PIO2_1;
                *y0 = z + 4.0 * PIO2_1T;
                *y1 = (z - *y0) + 4.0 * PIO2_1T;
                return -4;
            }
        }
    }
    if (ix < 0x413921fbu) goto medium;
    if (ix >= 0x7ff00000u) {
        *y0 = x - x;
        *y1 = *y0;
        return 0;
    }
    *large = 1;
    *y0 = 0.0;
    *y1 = 0.0;
    return 0;

medium: {
    double tmp = x * INV_PIO2 + TO_INT;
    double f_n = tmp - TO_INT;
    int n = f64_as_i32(f_n);
    double r = x - f_n * PIO2_1;
    double w = f_n * PIO2_1T;
    double yy0 = r - w;
    int ey = (int)(d2u(yy0) >> 52) & 0x7ff;
    int ex = (int)(ix >> 20);
    if (ex - ey > 16) {
        double t = r;
        w = f_n * PIO2_2;
        r = t - w;
        w = f_n * PIO2_2T - ((t - r) - w);
        yy0 = r - w;
        ey = (int)(d2u(yy0) >> 52) & 0x7ff;
        if (ex - ey > 49) {
            t = r;
            w = f_n * PIO2_3;
            r = t - w;
            w = f_n * PIO2_3T - ((t - r) - w);
            yy0 = r - w;
        }
    }
    *y0 = yy0;
    *y1 = (r - yy0) - w;
    return n;
}
}

/* ---- vendored_libm/sin.rs, cos.rs ---------------------------------------- */
double ref_sin_f64(double x) {
    const double x1p120 = u2d(0x4770000000000000ull);
    (void)x1p120;
    uint32_t ix = (uint32_t)(d2u(x) >> 32) & 0x7fffffffu;
    if (ix <= 0x3fe921fbu) {
        if (ix < 0x3e500000u) return x;
        return k_sin(x, 0.0, 0);
    }
    if (ix >= 0x7ff00000u) return x - x;
    double y0, y1;
    int large;
    int n = rem_pio2(x, &y0, &y1, &large);
    if (large) return NAN; /* out of this restatement's domain, see rem_pio2 */
    switch (n & 3) {
        case 0: return k_sin(y0, y1, 1);
        case 1: return k_cos(y0, y1);
        case 2: return -k_sin(y0, y1, 1);
        default: return -k_cos(y0, y1);
    }
}

/* cos (det-num vendored_libm/cos.rs:48) */
double ref_cos_f64(double x) {
    uint32_t ix = (uint32_t)(d2u(x) >> 32) & 0x7fffffffu;
    if (ix <= 0x3fe921fbu) {
        if (ix < 0x3e46a09eu) {
            if (f64_as_i32(x) == 0) return 1.0;
        }
        return k_cos(x, 0.0);
    }
    if (ix >= 0x7ff00000u) return x - x;
    double y0, y1;
    int large;
    int n = rem_pio2(x, &y0, &y1, &large);
    if (large) return NAN;
    switch (n & 3) {
        case 0: return k_cos(y0, y1);
        case 1: return -k_sin(y0, y1, 1);
        case 2: return -k_cos(y0, y1);
        default: return k_sin(y0, y1, 1);
    }
}

/* ---- f16.rs:6-34 ------------------------------------------------------------ */
float ref_f16_to_f32(uint16_t bits) {
    uint32_t sign = ((uint32_t)bits & 0x8000u) << 16;
    uint32_t exp = (bits >> 10) & 0x1f;
    uint32_t frac = bits & 0x03ffu;
    uint32_t out;
    if (exp == 0) {
        if (frac == 0) {
            out = sign;
        } else {
            uint32_t f = frac;
            int e = -14;
            while ((f & 0x0400u) == 0) {
                f <<= 1;
                e -= 1;
            }
            f &= 0x03ffu;
            out = sign | ((uint32_t)(e + 127) << 23) | (f << 13);
        }
    } else if (exp == 0x1f) {
        out = sign | 0x7f800000u | (frac << 13);
    } else {
        out = sign | ((uint32_t)((int)exp - 15 + 127) << 23) | (frac << 13);
    }
    return u2f(out);
}

/* ---- round.rs:2-20 -------------------------------------------------------- */
int32_t ref_round_ties_even_i32(float x) {
    if (!isfinite(x)) return f32_as_i32(x);
    if (!(x >= -8388608.0f && x < 8388608.0f)) return f32_as_i32(x);
    int32_t t = f32_as_i32(x);
    float frac = x - (float)t;
    if (frac > 0.5f || (frac == 0.5f && (t & 1) != 0)) return t + 1;
    if (frac < -0.5f || (frac == -0.5f && (t & 1) != 0)) return t - 1;
    return t;
}

/* ---- hash.rs: SHA-256 (FIPS 180-4) ----------------------------------------- */
static const uint32_t SHA_K[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

static inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

/* Sha256::compress (det-num hash.rs:78): FIPS 180-4 block function */
static void sha_compress(uint32_t st[8], const uint8_t blk[64]) {
    uint32_t w[64];
    for (int i = 0; i < 16; i++)
        w[i] = ((uint32_t)blk[4 * i] << 24) | ((uint32_t)blk[4 * i + 1] << 16) |
               ((uint32_t)blk[4 * i + 2] << 8) | (uint32_t)blk[4 * i + 3];
    for (int i = 16; i < 64; i++) {
        uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
        uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
        w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = st[0], b = st[1], c = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
    for (int i = 0; i < 64; i++) {
        uint32_t s1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
        uint32_t ch = (e & f) ^ (~e & g);
        uint32_t t1 = h + s1 + ch + SHA_K[i] + w[i];
        uint32_t s0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
        uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
        uint32_t t2 = s0 + mj;
        h = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    st[0] += a; st[1] += b; st[2] += c; st[3] += d;
    st[4] += e; st[5] += f; st[6] += g; st[7] += h;
}

void ref_sha256_init(ref_sha256_ctx* c) {
    static const uint32_t iv[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                                   0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    memcpy(c->state, iv, sizeof iv);
    c->len = 0;
    c->buf_len = 0;
}

void ref_sha256_update(ref_sha256_ctx* c, const uint8_t* in, size_t n) {
    c->len += n;
    if (c->buf_len) {
        size_t k = 64 - c->buf_len < n ? 64 - c->buf_len : n;
        memcpy(c->buf + c->buf_len, in, k);
        c->buf_len += k;
        in += k;
        n -= k;
        if (c->buf_len == 64) {
            sha_compress(c->state, c->buf);
            c->buf_len = 0;
        }
    }
    while (n >= 64) {
        sha_compress(c->state, in);
        in += 64;
        n -= 64;
    }
    if (n) {
        memcpy(c->buf, in, n);
        c->buf_len = n;
    }
}

void ref_sha256_final(ref_sha256_ctx* c, uint8_t out[32]) {
    uint64_t bits = c->len * 8;
    c->buf[c->buf_len++] = 0x80;
    if (c->buf_len > 56) {
        memset(c->buf + c->buf_len, 0, 64 - c->buf_len);
        sha_compress(c->state, c->buf);
        c->buf_len = 0;
    }
    memset(c->buf + c->buf_len, 0, 56 - c->buf_len);
    for (int i = 0; i < 8; i++) c->buf[56 + i] = (uint8_t)(bits >> (56 - 8 * i));
    sha_compress(c->state, c->buf);
    for (int i = 0; i < 8; i++) {
        out[4 * i] = (uint8_t)(c->state[i] >> 24);
        out[4 * i + 1] = (uint8_t)(c->state[i] >> 16);
        out[4 * i + 2] = (uint8_t)(c->state[i] >> 8);
        out[4 * i + 3] = (uint8_t)c->state[i];
    }
}

void ref_sha256(const uint8_t* data, size_t len, uint8_t out[32]) {
    ref_sha256_ctx c;
    ref_sha256_init(&c);
    ref_sha256_update(&c, data, len);
    ref_sha256_final(&c, out);
}

void sha_update_f32(ref_sha256_ctx* c, float v) {
    uint32_t b = f2u(v);
    uint8_t le[4] = {(uint8_t)b, (uint8_t)(b >> 8), (uint8_t)(b >> 16), (uint8_t)(b >> 24)};
    ref_sha256_update(c, le, 4);
}

/* ---- canary.rs:26-53 ------------------------------------------------------- */
void ref_canary_hash(uint8_t out[32]) {
    float x[9] = {u2f(1), u2f(2), -0.0f, 1.0f, -2.5f, 3.25f, 1024.0f, -4096.0f, 0.125f};
    float y[9] = {2.0f, -3.0f, 4.0f, 0.5f, -8.0f, 16.0f, -0.25f, 0.03125f, -64.0f};
    float v[6];
    v[0] = ref_dot_f32(x, y, 9);
    v[1] = ref_expf(-1.0f);
    v[2] = ref_expf(0.0f);
    v[3] = ref_f16_to_f32(0x3555);
    v[4] = (float)ref_round_ties_even_i32(2.5f);
    v[5] = u2f(1) + u2f(1);
    ref_sha256_ctx c;
    ref_sha256_init(&c);
    for (int i = 0; i < 6; i++) sha_update_f32(&c, v[i]);
    ref_sha256_final(&c, out);
}
