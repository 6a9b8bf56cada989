/*
 * oracle/ref_internal.h -- shared helpers of the CPU oracle (TEST
 * INFRASTRUCTURE, see ref.h): bit casts and Rust `as` conversion semantics.
 */
#ifndef DETLLM_ORACLE_REF_INTERNAL_H
#define DETLLM_ORACLE_REF_INTERNAL_H

#include <stdint.h>
#include <string.h>

#include "ref.h"

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint64_t d2u(double f) { uint64_t u; memcpy(&u, &f, 8); return u; }
static inline double u2d(uint64_t u) { double f; memcpy(&f, &u, 8); return f; }
static inline int isfinite_f(float x) { return (f2u(x) & 0x7f800000u) != 0x7f800000u; }

/* Rust `f32 as i32`: truncate toward zero, saturate, NaN -> 0. */
static inline int32_t f32_as_i32(float x) {
    if (x != x) return 0;
    if (x >= 2147483648.0f) return INT32_MAX;
    if (x < -2147483648.0f) return INT32_MIN;
    return (int32_t)x;
}
/* Rust `f32 as u32`. */
static inline uint32_t f32_as_u32(float x) {
    if (x != x) return 0;
    if (x >= 4294967296.0f) return UINT32_MAX;
    if (x <= -1.0f) return 0;
    return (uint32_t)x;
}
/* Rust `f64 as i32`. */
static inline int32_t f64_as_i32(double x) {
    if (x != x) return 0;
    if (x >= 2147483648.0) return INT32_MAX;
    if (x <= -2147483649.0) return INT32_MIN;
    return (int32_t)x;
}

void sha_update_f32(ref_sha256_ctx* c, float v);

/* thread pool (ref_model.c): runs fn(ctx, begin, end) over [0, n) split into
 * contiguous chunks of ceil(n / threads), like det-model lib.rs:291-321. */
typedef void (*ref_range_fn)(void* ctx, size_t begin, size_t end);
void ref_parallel_for(size_t n, ref_range_fn fn, void* ctx);
int ref_thread_count(void);

#endif
