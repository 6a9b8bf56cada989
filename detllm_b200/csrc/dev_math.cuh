// dev_math.cuh -- device numerics that reproduce det-num bit for bit.
//
// Every f32/f64 operation is an explicitly rounded intrinsic (__fadd_rn,
// __fmul_rn, __fdiv_rn, __fsqrt_rn, __dadd_rn, ...), which the compiler never
// contracts into FMA; the library is also built with --fmad=false and
// -ftz=false so subnormals behave as IEEE-754 requires.
//
// The transcendental routines restate det-num's vendored fdlibm code
// (crates/det-num/src/vendored_libm/, rust-lang/libm 0.2.16 from FreeBSD
// msun); they are not CUDA's math library.
//
// ====================================================
// Copyright (C) 1993 by Sun Microsystems, Inc. All rights reserved.
//
// Developed at SunPro, a Sun Microsystems, Inc. business.
// Permission to use, copy, modify, and distribute this
// software is freely granted, provided that this notice
// is preserved.
// ====================================================
// Copyright (C) 2004 by Sun Microsystems, Inc. All rights reserved.
//
// Permission to use, copy, modify, and distribute this
// software is freely granted, provided that this notice
// is preserved.
// ====================================================
// expf: conversion to float by Ian Lance Taylor, Cygnus Support.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#define DI __device__ __forceinline__

namespace det {

DI float fadd(float a, float b) { return __fadd_rn(a, b); }
DI float fsub(float a, float b) { return __fsub_rn(a, b); }
DI float fmul(float a, float b) { return __fmul_rn(a, b); }
DI float fdiv(float a, float b) { return __fdiv_rn(a, b); }
DI double dadd(double a, double b) { return __dadd_rn(a, b); }
DI double dsub(double a, double b) { return __dsub_rn(a, b); }
DI double dmul(double a, double b) { return __dmul_rn(a, b); }
DI double ddiv(double a, double b) { return __ddiv_rn(a, b); }

DI bool finite(float x) { return (__float_as_uint(x) & 0x7f800000u) != 0x7f800000u; }

// f16 bits -> f32 (det-num f16.rs:6-34): the conversion is exact for every
// finite f16; non-finite scales are rejected when the model is loaded.
DI float f16_bits_to_f32(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// Rust `f32 as i32` for the finite, in-range arguments on this path.
DI int f32_to_i32_trunc(float x) { return __float2int_rz(x); }

// ---- expf: det-num vendored_libm/expf.rs:33-106 ---------------------------
DI float scalbnf(float x, int n) {  // vendored_libm.rs:94-119
  const float x1p127 = __uint_as_float(0x7f000000u);
  const float x1p_126 = __uint_as_float(0x00800000u);
  if (n > 127) {
    x = fmul(x, x1p127);
    n -= 127;
    if (n > 127) {
      x = fmul(x, x1p127);
      n -= 127;
      if (n > 127) n = 127;
    }
  } else if (n < -126) {
    x = fmul(x, x1p_126);
    n += 126;
    if (n < -126) {
      x = fmul(x, x1p_126);
      n += 126;
      if (n < -126) n = -126;
    }
  }
  return fmul(x, __uint_as_float((uint32_t)(0x7f + n) << 23));
}

DI float expf_det(float x) {
  const float LN2_HI = __uint_as_float(0x3f317200u);
  const float LN2_LO = __uint_as_float(0x35bfbe8eu);
  const float INV_LN2 = __uint_as_float(0x3fb8aa3bu);
  const float P1 = 1.6666625440e-1f;
  const float P2 = -2.7667332906e-3f;
  const float x1p127 = __uint_as_float(0x7f000000u);
  uint32_t hx = __float_as_uint(x);
  const int sign = (int)(hx >> 31);
  hx &= 0x7fffffffu;
  if (hx >= 0x42aeac50u) {
    if (hx > 0x7f800000u) return x;
    if (hx >= 0x42b17218u && !sign) return fmul(x, x1p127);
    if (sign && hx >= 0x42cff1b5u) return 0.0f;
  }
  int k;
  float hi, lo;
  if (hx > 0x3eb17218u) {
    if (hx > 0x3f851592u)
      k = f32_to_i32_trunc(fadd(fmul(INV_LN2, x), sign ? -0.5f : 0.5f));
    else
      k = 1 - sign - sign;
    const float kf = __int2float_rn(k);
    hi = fsub(x, fmul(kf, LN2_HI));
    lo = fmul(kf, LN2_LO);
    x = fsub(hi, lo);
  } else if (hx > 0x39000000u) {
    k = 0;
    hi = x;
    lo = 0.0f;
  } else {
    return fadd(1.0f, x);
  }
  const float xx = fmul(x, x);
  const float c = fsub(x, fmul(xx, fadd(P1, fmul(xx, P2))));
  const float y = fadd(1.0f, fadd(fsub(fdiv(fmul(x, c), fsub(2.0f, c)), lo), hi));
  return k == 0 ? y : scalbnf(y, k);
}

// silu_f32 (det-num math.rs:30-34)
DI float silu_det(float x) {
  const float t = expf_det(-x);
  const float d = fadd(1.0f, t);
  return fdiv(x, d);
}

// ---- f64 routines for the RoPE table (det-model lib.rs:813-846) ----------
DI double scalbn_d(double x, int n) {  // vendored_libm.rs scalbn_f64
  const double x1p1023 = __longlong_as_double(0x7fe0000000000000ll);
  const double x1p_1022 = __longlong_as_double(0x0010000000000000ll);
  if (n > 1023) {
    x = dmul(x, x1p1023);
    n -= 1023;
    if (n > 1023) {
      x = dmul(x, x1p1023);
      n -= 1023;
      if (n > 1023) n = 1023;
    }
  } else if (n < -1022) {
    x = dmul(x, x1p_1022);
    n += 1022;
    if (n < -1022) {
      x = dmul(x, x1p_1022);
      n += 1022;
      if (n < -1022) n = -1022;
    }
  }
  return dmul(x, __longlong_as_double((long long)((uint64_t)(0x3ff + n) << 52)));
}

DI uint32_t hi_word(double x) { return (uint32_t)((uint64_t)__double_as_longlong(x) >> 32); }

// vendored_libm/exp.rs
DI double exp_det(double x) {
  const double LN2HI = 6.93147180369123816490e-01, LN2LO = 1.90821492927058770002e-10;
  const double INVLN2 = 1.44269504088896338700e+00;
  const double P1 = 1.66666666666666019037e-01, P2 = -2.77777777770155933842e-03;
  const double P3 = 6.61375632143793436117e-05, P4 = -1.65339022054652515390e-06;
  const double P5 = 4.13813679705723846039e-08;
  const double x1p1023 = __longlong_as_double(0x7fe0000000000000ll);
  uint32_t hx = hi_word(x);
  const int sign = (int)(hx >> 31);
  hx &= 0x7fffffffu;
  if (hx >= 0x4086232bu) {
    if (x != x) return x;
    if (x > 709.782712893383973096) return dmul(x, x1p1023);
    if (x < -708.39641853226410622 && x < -745.13321910194110842) return 0.0;
  }
  int k;
  double hi, lo;
  if (hx > 0x3fd62e42u) {
    if (hx >= 0x3ff0a2b2u)
      k = __double2int_rz(dadd(dmul(INVLN2, x), sign ? -0.5 : 0.5));
    else
      k = 1 - sign - sign;
    const double kd = (double)k;
    hi = dsub(x, dmul(kd, LN2HI));
    lo = dmul(kd, LN2LO);
    x = dsub(hi, lo);
  } else if (hx > 0x3e300000u) {
    k = 0;
    hi = x;
    lo = 0.0;
  } else {
    return dadd(1.0, x);
  }
  const double xx = dmul(x, x);
  const double poly = dadd(P1, dmul(xx, dadd(P2, dmul(xx, dadd(P3, dmul(xx, dadd(P4, dmul(xx, P5))))))));
  const double c = dsub(x, dmul(xx, poly));
  const double y = dadd(1.0, dadd(dsub(ddiv(dmul(x, c), dsub(2.0, c)), lo), hi));
  return k == 0 ? y : scalbn_d(y, k);
}

// vendored_libm/log.rs
DI double log_det(double x) {
  const double LN2_HI = 6.93147180369123816490e-01, LN2_LO = 1.90821492927058770002e-10;
  const double LG1 = 6.666666666666735130e-01, LG2 = 3.999999999940941908e-01;
  const double LG3 = 2.857142874366239149e-01, LG4 = 2.222219843214978396e-01;
  const double LG5 = 1.818357216161805012e-01, LG6 = 1.531383769920937332e-01;
  const double LG7 = 1.479819860511658591e-01;
  const double x1p54 = __longlong_as_double(0x4350000000000000ll);
  uint64_t ui = (uint64_t)__double_as_longlong(x);
  uint32_t hx = (uint32_t)(ui >> 32);
  int k = 0;
  if (hx < 0x00100000u || (hx >> 31) != 0) {
    if ((ui << 1) == 0) return ddiv(-1.0, dmul(x, x));
    if ((hx >> 31) != 0) return ddiv(dsub(x, x), 0.0);
    k -= 54;
    x = dmul(x, x1p54);
    ui = (uint64_t)__double_as_longlong(x);
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
  x = __longlong_as_double((long long)ui);
  const double f = dsub(x, 1.0);
  const double hfsq = dmul(dmul(0.5, f), f);
  const double s = ddiv(f, dadd(2.0, f));
  const double z = dmul(s, s);
  const double w = dmul(z, z);
  const double t1 = dmul(w, dadd(LG2, dmul(w, dadd(LG4, dmul(w, LG6)))));
  const double t2 = dmul(z, dadd(LG1, dmul(w, dadd(LG3, dmul(w, dadd(LG5, dmul(w, LG7)))))));
  const double r = dadd(t2, t1);
  const double dk = (double)k;
  // s*(hfsq+r) + dk*LN2_LO - hfsq + f + dk*LN2_HI, left to right
  return dadd(dadd(dsub(dadd(dmul(s, dadd(hfsq, r)), dmul(dk, LN2_LO)), hfsq), f), dmul(dk, LN2_HI));
}

// vendored_libm/k_sin.rs
DI double k_sin(double x, double y, int iy) {
  const double S1 = -1.66666666666666324348e-01, S2 = 8.33333333332248946124e-03;
  const double S3 = -1.98412698298579493134e-04, S4 = 2.75573137070700676789e-06;
  const double S5 = -2.50507602534068634195e-08, S6 = 1.58969099521155010221e-10;
  const double z = dmul(x, x);
  const double w = dmul(z, z);
  const double r = dadd(dadd(S2, dmul(z, dadd(S3, dmul(z, S4)))), dmul(dmul(z, w), dadd(S5, dmul(z, S6))));
  const double v = dmul(z, x);
  if (iy == 0) return dadd(x, dmul(v, dadd(S1, dmul(z, r))));
  return dsub(x, dsub(dsub(dmul(z, dsub(dmul(0.5, y), dmul(v, r))), y), dmul(v, S1)));
}

// vendored_libm/k_cos.rs
DI double k_cos(double x, double y) {
  const double C1 = 4.16666666666666019037e-02, C2 = -1.38888888888741095749e-03;
  const double C3 = 2.48015872894767294178e-05, C4 = -2.75573143513906633035e-07;
  const double C5 = 2.08757232129817482790e-09, C6 = -1.13596475577881948265e-11;
  const double z = dmul(x, x);
  double w = dmul(z, z);
  const double r = dadd(dmul(z, dadd(C1, dmul(z, dadd(C2, dmul(z, C3))))),
                        dmul(dmul(w, w), dadd(C4, dmul(z, dadd(C5, dmul(z, C6))))));
  const double hz = dmul(0.5, z);
  w = dsub(1.0, hz);
  return dadd(w, dadd(dsub(dsub(1.0, w), hz), dsub(dmul(z, r), dmul(x, y))));
}

// vendored_libm/rem_pio2.rs for |x| < 2^20*pi/2 (the RoPE phase pos*omega is
// below the context length, which the host caps at 2^20).  Returns n, y0, y1.
DI int rem_pio2(double x, double& y0, double& y1) {
  const double TO_INT = 1.5 / 2.2204460492503131e-16;
  const double INV_PIO2 = 6.36619772367581382433e-01;
  const double PIO2_1 = 1.57079632673412561417e+00, PIO2_1T = 6.07710050650619224932e-11;
  const double PIO2_2 = 6.07710050630396597660e-11, PIO2_2T = 2.02226624879595063154e-21;
  const double PIO2_3 = 2.02226624871116645580e-21, PIO2_3T = 8.47842766036889956997e-32;
  const int sign = (int)((uint64_t)__double_as_longlong(x) >> 63);
  const uint32_t ix = hi_word(x) & 0x7fffffffu;
  bool medium = false;
  int n = 0;
  double m = 0.0;
  if (ix <= 0x400f6a7au) {
    if ((ix & 0xfffffu) == 0x921fbu) {
      medium = true;
    } else if (ix <= 0x4002d97cu) {
      n = sign ? -1 : 1;
      m = 1.0;
    } else {
      n = sign ? -2 : 2;
      m = 2.0;
    }
  } else if (ix <= 0x401c463bu) {
    if (ix <= 0x4015fdbcu) {
      if (ix == 0x4012d97cu) medium = true;
      else { n = sign ? -3 : 3; m = 3.0; }
    } else {
      if (ix == 0x401921fbu) medium = true;
      else { n = sign ? -4 : 4; m = 4.0; }
    }
  } else {
    medium = true;
  }
  if (!medium) {
    // z = x -/+ m*PIO2_1; y0 = z -/+ m*PIO2_1T; y1 = (z - y0) -/+ m*PIO2_1T
    const double a = dmul(m, PIO2_1), b = dmul(m, PIO2_1T);
    if (!sign) {
      const double z = dsub(x, a);
      y0 = dsub(z, b);
      y1 = dsub(dsub(z, y0), b);
    } else {
      const double z = dadd(x, a);
      y0 = dadd(z, b);
      y1 = dadd(dsub(z, y0), b);
    }
    return n;
  }
  const double tmp = dadd(dmul(x, INV_PIO2), TO_INT);
  const double f_n = dsub(tmp, TO_INT);
  n = __double2int_rz(f_n);
  double r = dsub(x, dmul(f_n, PIO2_1));
  double w = dmul(f_n, PIO2_1T);
  double yy = dsub(r, w);
  int ey = (int)(((uint64_t)__double_as_longlong(yy) >> 52) & 0x7ff);
  const int ex = (int)(ix >> 20);
  if (ex - ey > 16) {
    double t = r;
    w = dmul(f_n, PIO2_2);
    r = dsub(t, w);
    w = dsub(dmul(f_n, PIO2_2T), dsub(dsub(t, r), w));
    yy = dsub(r, w);
    ey = (int)(((uint64_t)__double_as_longlong(yy) >> 52) & 0x7ff);
    if (ex - ey > 49) {
      t = r;
      w = dmul(f_n, PIO2_3);
      r = dsub(t, w);
      w = dsub(dmul(f_n, PIO2_3T), dsub(dsub(t, r), w));
      yy = dsub(r, w);
    }
  }
  y0 = yy;
  y1 = dsub(dsub(r, yy), w);
  return n;
}

// vendored_libm/sin.rs and cos.rs (finite arguments)
DI double sin_det(double x) {
  const uint32_t ix = hi_word(x) & 0x7fffffffu;
  if (ix <= 0x3fe921fbu) {
    if (ix < 0x3e500000u) return x;
    return k_sin(x, 0.0, 0);
  }
  double y0, y1;
  const int n = rem_pio2(x, y0, y1);
  switch (n & 3) {
    case 0: return k_sin(y0, y1, 1);
    case 1: return k_cos(y0, y1);
    case 2: return -k_sin(y0, y1, 1);
    default: return -k_cos(y0, y1);
  }
}

DI double cos_det(double x) {
  const uint32_t ix = hi_word(x) & 0x7fffffffu;
  if (ix <= 0x3fe921fbu) {
    if (ix < 0x3e46a09eu && __double2int_rz(x) == 0) return 1.0;
    return k_cos(x, 0.0);
  }
  double y0, y1;
  const int n = rem_pio2(x, y0, y1);
  switch (n & 3) {
    case 0: return k_cos(y0, y1);
    case 1: return -k_sin(y0, y1, 1);
    case 2: return -k_cos(y0, y1);
    default: return k_sin(y0, y1, 1);
  }
}

// finish_8lane (det-num reduce.rs:36-38)
DI float finish8(const float a[8]) {
  return fadd(fadd(fadd(a[0], a[1]), fadd(a[2], a[3])), fadd(fadd(a[4], a[5]), fadd(a[6], a[7])));
}

// get_scale_min_k4 of a Q4_K super-block's 12 scale bytes: the 6-bit scale
// and min of sub-block idx (det-quant lib.rs:506-518)
DI void q4k_scale_min(const uint8_t* s, int idx, int& sc, int& mn) {
  if (idx < 4) {
    sc = s[idx] & 0x3f;
    mn = s[idx + 4] & 0x3f;
  } else {
    sc = (s[idx + 4] & 0x0f) | ((s[idx - 4] >> 6) << 4);
    mn = (s[idx + 4] >> 4) | ((s[idx] >> 6) << 4);
  }
}

// q6_k_quant: the signed 6-bit value of element `index` (0..255) of a Q6_K
// block body (ql[128] | qh[64] | scales[16]) (det-quant lib.rs:536-556)
DI int q6k_quant(const uint8_t* body, int index) {
  const int half = index >> 7, within = index & 127, l = within & 31, part = within >> 5;
  const uint8_t* ql = body;
  const uint8_t* qh = body + 128;
  int v, shift;
  switch (part) {
    case 0: v = ql[half * 64 + l] & 0x0f; shift = 0; break;
    case 1: v = ql[half * 64 + l + 32] & 0x0f; shift = 2; break;
    case 2: v = ql[half * 64 + l] >> 4; shift = 4; break;
    default: v = ql[half * 64 + l + 32] >> 4; shift = 6; break;
  }
  const int high = ((qh[half * 32 + l] >> shift) & 0x03) << 4;
  return (v | high) - 32;
}


// ---- programmatic dependent launch -----------------------------------------
// Kernels are launched with programmatic stream serialization, so a kernel
// may start while its predecessor in the stream is still running.
// pdl_wait() blocks until the predecessor grid has completed and its memory
// writes are visible (it returns at once for a plain launch); every kernel
// calls it before it reads or writes anything another kernel touches.
// pdl_trigger() then lets the successor begin launching.  Only reads of
// constant data (weights) may come before pdl_wait().
DI void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
DI void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
DI void pdl_enter() {
  pdl_wait();
  pdl_trigger();
}

// ---- Q8A activation layout ---------------------------------------------------
// Quantised activations of T positions x K elements are stored block-major
// in groups of 64 positions: for group G and block b, 64 consecutive 32-byte
// position blocks, then the next block.  Within a position block the two
// 16-byte halves are swapped for positions with bit 2 set, which makes the
// tensor-core B-fragment reads from shared memory bank-conflict free.  One
// (group, block) slab is 2 KiB of quants and 256 B of f32 scales, so a GEMM
// stage is a few contiguous bulk copies.  The 64 scales of a slab are
// permuted within each half of 32 positions: position 8j + 2u + e sits at
// 8u + 2j + e, so the tensor-core lane with column pair u reads the scales
// of its positions (8j + 2u, +1), j = 0..3, as 8 contiguous floats.
constexpr int Q8A_GROUP = 64;
DI size_t q8a_slot(int nb, int t, int b) { return ((size_t)(t >> 6) * nb + b) * Q8A_GROUP + (t & 63); }
DI int q8a_sperm(int p) { return (p & 32) | (((p >> 1) & 3) << 3) | (((p >> 3) & 3) << 1) | (p & 1); }
// index of the scale of block b of position t
DI size_t q8a_dslot(int nb, int t, int b) {
  return ((size_t)(t >> 6) * nb + b) * Q8A_GROUP + q8a_sperm(t & 63);
}
DI int q8a_swz(int t) { return ((t >> 2) & 1) << 4; }
// byte of element i (0..31) of block b of position t
DI size_t q8a_elem(int nb, int t, int b, int i) { return q8a_slot(nb, t, b) * 32 + (size_t)(i ^ q8a_swz(t)); }

// Exact int32 -> f32 for |v| < 2^22 via the 1.5*2^23 bias: the bits of
// (0x4B400000 + v) read as f32 equal 12582912 + v exactly.
DI float exact_small_int_to_f32(int v) { return __fsub_rn(__int_as_float(0x4B400000 + v), 12582912.0f); }

}  // namespace det
