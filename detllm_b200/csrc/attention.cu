// attention.cu -- causal GQA attention for a chunk of T positions, exact to
// the reference's f32 arithmetic, in three tiled kernels.
//
// Reference: attention_one_head and its helpers (crates/det-model/src/
// lib.rs:2298-2418).  For a query at position p (score_len = p + 1):
//   s_j  = dot_f32_ref(q, k_j) * scale              (8 interleaved lanes, then
//                                                    the fixed combine tree)
//   e_j  = exp_f32(max(s_j - max_j s_j, -88)),  z = sum_f32_ref(e)
//   p_j  = e_j / z
//   o[d] = sum over j = 0, 1, ... of p_j * v_j[d]   (one ordered chain per d)
// and score_len == 1 copies v_0.  No step may be reassociated, so every
// product and sum here is a separately rounded f32 operation on the CUDA
// cores; what the kernels change is only which thread does which chain and
// how operands reach it:
//
//   attn_scores   one CTA per (64-key tile, block of queries, KV head):
//                 the 64 query-head rows of a GQA group block share each K
//                 tile in shared memory; a thread owns a 4 x 4 tile of dots
//                 and runs their eight lane chains one lane at a time
//                 (lane-major operand layout), combining finished lanes in
//                 the reference's tree order, so 16 dots need ~64 registers.
//   attn_softmax  one warp per (position, head) row: max, e_j, the eight
//                 ordered z chains, p_j = e_j / z, written back in place.
//   attn_pv       one CTA per (block of query-head rows, KV head): P and V
//                 tiles staged in shared memory, a thread owns 4 rows x 4
//                 dims = 16 independent ordered chains over j.
//
// Rows of different queries in one CTA have different score lengths; the
// PV chains of shorter rows see p = 0 for the extra keys, and adding
// 0 * v (v finite, the chain never -0) leaves an f32 sum unchanged.
#include <atomic>
#include <cuda_runtime.h>

#include <algorithm>

#include "dev_math.cuh"
#include "internal.h"

namespace det {
namespace {

DI unsigned long long pk2(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
// two separately rounded products (packed IEEE multiply)
DI float2 mul2(float a0, float a1, float b0, float b1) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pk2(a0, a1)), "l"(pk2(b0, b1)));
  float2 o;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(o.x), "=f"(o.y) : "l"(r));
  return o;
}
// acc + p for two pairs, each rounded once: written as fma(p, one, acc) with
// `one` == 1.0 a kernel argument, because a packed add fed by a packed
// multiply is contracted into a fused multiply-add by the code generator
DI float2 add_by_fma2(float2 p, float one, float2 acc) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(pk2(p.x, p.y)), "l"(pk2(one, one)), "l"(pk2(acc.x, acc.y)));  // exact: p * 1
  float2 o;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(o.x), "=f"(o.y) : "l"(r));
  return o;
}

// ---- scores -------------------------------------------------------------------
constexpr int QK_ROWS = 64;  // query-head rows per CTA
constexpr int QK_KEYS = 64;  // keys per CTA
constexpr int QK_THREADS = 256;

// lane-major position of element d within a row of HD floats: the HD/8
// elements of lane l (d = 8i + l) are contiguous
template <int HD>
DI int lm(int d) {
  return (d & 7) * (HD / 8) + (d >> 3);
}

// Shared-memory operands: QK_ROWS query-head rows and QK_KEYS key rows of
// HD + 4 floats (padded stride), each row lane-major (element d at lm(d)),
// so the HD / 8 elements of one lane chain are contiguous.  A thread owns
// the dots of rows mt + 16r and keys jt + 16c (r, c < 4) and runs their
// eight lane chains one lane at a time: a 16-byte load of a row and of a key
// gives four consecutive elements of the same chain, a packed multiply
// forms two products at a time, and the chain adds them in order one by one.
template <int HD>
__global__ void __launch_bounds__(QK_THREADS, 3) attn_scores_kernel(const float* __restrict__ q,
                                                                 const float* __restrict__ kc, const int* pos0p,
                                                                 int T, int n_head, int gsz, int qb, int n_ctx,
                                                                 int s_ld, float scale, float* __restrict__ S,
                                                                 uint32_t* err) {
  pdl_enter();
  constexpr int RS = HD + 4;  // padded row stride (floats): conflict-free strided rows
  constexpr int PER = HD / 8; // elements per lane chain
  extern __shared__ float4 qk_smem[];
  float* qs = reinterpret_cast<float*>(qk_smem);  // [QK_ROWS][RS]
  float* ks = qs + QK_ROWS * RS;                  // [QK_KEYS][RS]
  const int pos0 = *pos0p;
  const int j0 = blockIdx.x * QK_KEYS;
  const int t0 = blockIdx.y * qb;
  const int kvh = blockIdx.z;
  const int tq = min(qb, T - t0);  // queries in this block
  const int jmax = pos0 + t0 + tq;  // longest score row of the block
  if (j0 >= jmax) return;
  const int tid = threadIdx.x;
  const int rows = tq * gsz;

  // stage Q rows (m = qi * gsz + hh) and K rows j0.. in lane-major order
  for (int i = tid; i < QK_ROWS * (HD / 4); i += QK_THREADS) {
    const int m = i / (HD / 4), d4 = (i - m * (HD / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (m < rows) {
      const int qi = m / gsz, hh = m - qi * gsz;
      v = *reinterpret_cast<const float4*>(q + ((size_t)(t0 + qi) * n_head + kvh * gsz + hh) * HD + d4);
      if (!finite(v.x) || !finite(v.y) || !finite(v.z) || !finite(v.w)) atomicOr(err, ERRF_NONFINITE);
    }
    float* r = qs + m * RS;
    r[lm<HD>(d4)] = v.x;
    r[lm<HD>(d4 + 1)] = v.y;
    r[lm<HD>(d4 + 2)] = v.z;
    r[lm<HD>(d4 + 3)] = v.w;
  }
  for (int i = tid; i < QK_KEYS * (HD / 4); i += QK_THREADS) {
    const int jj = i / (HD / 4), d4 = (i - jj * (HD / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (j0 + jj < jmax) {
      v = *reinterpret_cast<const float4*>(kc + ((size_t)kvh * n_ctx + j0 + jj) * HD + d4);
      if (!finite(v.x) || !finite(v.y) || !finite(v.z) || !finite(v.w)) atomicOr(err, ERRF_NONFINITE);
    }
    float* r = ks + jj * RS;
    r[lm<HD>(d4)] = v.x;
    r[lm<HD>(d4 + 1)] = v.y;
    r[lm<HD>(d4 + 2)] = v.z;
    r[lm<HD>(d4 + 3)] = v.w;
  }
  __syncthreads();

  // thread tile: rows mt + 16r, keys jt + 16c
  const int warp = tid >> 5, lane = tid & 31;
  const int mt = 2 * warp + (lane >> 4), jt = lane & 15;
  float t01[4][4], t03[4][4], t45[4][4], a[4][4], b[4][4];

  // one lane chain for the 16 dots: acc[r][c] = sum over i of q[8i+l] k[8i+l]
  auto chain = [&](int l, float (&acc)[4][4]) {
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int c = 0; c < 4; c++) acc[r][c] = 0.0f;
#pragma unroll
    for (int i = 0; i < PER; i += 4) {
      float4 qv[4], kv[4];
#pragma unroll
      for (int r = 0; r < 4; r++) qv[r] = *reinterpret_cast<const float4*>(qs + (mt + 16 * r) * RS + l * PER + i);
#pragma unroll
      for (int c = 0; c < 4; c++) kv[c] = *reinterpret_cast<const float4*>(ks + (jt + 16 * c) * RS + l * PER + i);
#pragma unroll
      for (int r = 0; r < 4; r++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const float2 p01 = mul2(qv[r].x, qv[r].y, kv[c].x, kv[c].y);
          const float2 p23 = mul2(qv[r].z, qv[r].w, kv[c].z, kv[c].w);
          float s = acc[r][c];
          s = fadd(s, p01.x);
          s = fadd(s, p01.y);
          s = fadd(s, p23.x);
          s = fadd(s, p23.y);
          acc[r][c] = s;
        }
    }
  };
  auto add_into = [&](float (&dst)[4][4], const float (&x)[4][4], const float (&y)[4][4]) {
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int c = 0; c < 4; c++) dst[r][c] = fadd(x[r][c], y[r][c]);
  };
  // finish_8lane: ((l0 + l1) + (l2 + l3)) + ((l4 + l5) + (l6 + l7))
  chain(0, a);
  chain(1, b);
  add_into(t01, a, b);
  chain(2, a);
  chain(3, b);
  add_into(a, a, b);
  add_into(t03, t01, a);
  chain(4, a);
  chain(5, b);
  add_into(t45, a, b);
  chain(6, a);
  chain(7, b);
  add_into(a, a, b);
  add_into(a, t45, a);
  add_into(a, t03, a);

#pragma unroll
  for (int r = 0; r < 4; r++) {
    const int m = mt + 16 * r;
    if (m >= rows) continue;
    const int qi = m / gsz, hh = m - qi * gsz;
    const int t = t0 + qi;
    const int len = pos0 + t + 1;
    if (len == 1) continue;  // score_len == 1 copies v_0 (no scores)
    float* srow = S + ((size_t)t * n_head + kvh * gsz + hh) * s_ld;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int j = j0 + jt + 16 * c;
      if (j < len) {
        const float s = fmul(a[r][c], scale);
        if (!finite(s)) atomicOr(err, ERRF_NONFINITE);
        srow[j] = s;
      }
    }
  }
}

// ---- softmax: one warp per row ---------------------------------------------------
// The row is staged in shared memory (when it fits) so the eight ordered z
// chains read on-chip.  p_j is written back in place, and the row is zeroed
// from its score length up to the end of the 32-key tile that the PV kernel
// reads past it (at most 31 keys further).
constexpr int SM_SMEM_FLOATS = 12288;  // largest staged row set per CTA

template <bool STAGED>
__global__ void attn_softmax_kernel(float* __restrict__ S, const int* pos0p, int T, int n_head, int s_ld, int rpc,
                                    uint32_t* err) {
  pdl_enter();
  extern __shared__ float sm_rows[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * rpc + warp;
  if (row >= T * n_head) return;
  const int t = row / n_head;
  const int len = *pos0p + t + 1;
  if (len == 1) return;
  float* s = S + (size_t)row * s_ld;
  float* b = STAGED ? sm_rows + (size_t)warp * s_ld : s;
  float mx = -INFINITY;
  for (int j = lane; j < len; j += 32) {
    const float v = s[j];
    if (STAGED) b[j] = v;
    mx = fmaxf(mx, v);
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  for (int j = lane; j < len; j += 32) {
    const float d = fsub(b[j], mx);
    b[j] = expf_det(d > -88.0f ? d : -88.0f);
  }
  __syncwarp();
  // sum_f32_ref: lane l < 8 runs the ordered chain over j = l, l + 8, ...
  float acc = 0.0f;
  if (lane < 8) {
    int j = lane;
    for (; j + 56 < len; j += 64) {
      float e[8];
#pragma unroll
      for (int k = 0; k < 8; k++) e[k] = b[j + 8 * k];
#pragma unroll
      for (int k = 0; k < 8; k++) acc = fadd(acc, e[k]);
    }
    for (; j < len; j += 8) acc = fadd(acc, b[j]);
  }
  float l8[8];
#pragma unroll
  for (int k = 0; k < 8; k++) l8[k] = __shfl_sync(0xffffffffu, acc, k);
  const float z = finish8(l8);
  if (!finite(z) || z == 0.0f) {
    if (lane == 0) atomicOr(err, ERRF_NONFINITE);
    return;
  }
  for (int j = lane; j < len; j += 32) {
    const float p = fdiv(b[j], z);
    if (!finite(p)) atomicOr(err, ERRF_NONFINITE);
    s[j] = p;
  }
  const int zend = min(s_ld, (len + 31 + 31) & ~31);
  for (int j = len + lane; j < zend; j += 32) s[j] = 0.0f;
}

// Long rows (a window of thousands of keys): the staged kernel would hold a
// whole row in shared memory per warp and keep the SM nearly empty.  Here a
// warp owns a row in global memory (L2): a max pass, then blocks of 256
// elements in which lane l computes e_j for j = base + 32k + 8(l >> 3) +
// (l & 7), k < 8, and writes it back in place; lane c < 8 runs the ordered
// z chain of class c (j = c, c + 8, ...) by taking the class's values from
// lanes c + 8, c + 16, c + 24 with shuffles, in increasing j; then
// p_j = e_j / z in place and zeros to the end of the PV tile.  Elements past
// the row add +0 to a chain, which leaves it unchanged.
constexpr int SL_WARPS = 8;

__global__ void __launch_bounds__(SL_WARPS * 32) attn_softmax_long_kernel(float* __restrict__ S, const int* pos0p,
                                                                          int T, int n_head, int s_ld, uint32_t* err) {
  pdl_enter();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * SL_WARPS + warp;
  if (row >= T * n_head) return;
  const int t = row / n_head;
  const int len = *pos0p + t + 1;
  if (len == 1) return;
  float* s = S + (size_t)row * s_ld;
  // max (order-free); rows start 128-byte aligned (s_ld is a multiple of 32)
  float mx = -INFINITY;
  const int n4 = len >> 2;
  const float4* s4 = reinterpret_cast<const float4*>(s);
#pragma unroll 4
  for (int i = lane; i < n4; i += 32) {
    const float4 v = s4[i];
    mx = fmaxf(fmaxf(mx, v.x), fmaxf(fmaxf(v.y, v.z), v.w));
  }
  for (int j = 4 * n4 + lane; j < len; j += 32) mx = fmaxf(mx, s[j]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  // e_j in place, and the eight ordered z chains (sum_f32_ref)
  // (lane = 8 (lane >> 3) + (lane & 7): element base + 32 k + lane is of
  // class lane & 7; the loads of a block are issued before any store)
  float acc = 0.0f;
  for (int base = 0; base < len; base += 256) {
    float e[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int j = base + 32 * k + lane;
      e[k] = j < len ? s[j] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int j = base + 32 * k + lane;
      if (j < len) {
        const float d = fsub(e[k], mx);
        e[k] = expf_det(d > -88.0f ? d : -88.0f);
      }
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int j = base + 32 * k + lane;
      if (j < len) s[j] = e[k];
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const float e1 = __shfl_down_sync(0xffffffffu, e[k], 8);
      const float e2 = __shfl_down_sync(0xffffffffu, e[k], 16);
      const float e3 = __shfl_down_sync(0xffffffffu, e[k], 24);
      acc = fadd(acc, e[k]);
      acc = fadd(acc, e1);
      acc = fadd(acc, e2);
      acc = fadd(acc, e3);
    }
  }
  float l8[8];
#pragma unroll
  for (int k = 0; k < 8; k++) l8[k] = __shfl_sync(0xffffffffu, acc, k);
  const float z = finish8(l8);
  if (!finite(z) || z == 0.0f) {
    if (lane == 0) atomicOr(err, ERRF_NONFINITE);
    return;
  }
  __syncwarp();  // every lane's e_j stores precede the reads below
  bool bad = false;
  for (int base = 0; base < len; base += 256) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int j = base + 32 * k + lane;
      v[k] = j < len ? s[j] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int j = base + 32 * k + lane;
      if (j < len) {
        const float p = fdiv(v[k], z);
        bad |= !finite(p);
        s[j] = p;
      }
    }
  }
  if (bad) atomicOr(err, ERRF_NONFINITE);
  const int zend = min(s_ld, (len + 31 + 31) & ~31);
  for (int j = len + lane; j < zend; j += 32) s[j] = 0.0f;
}

// ---- P x V ----------------------------------------------------------------------
// P and V tiles of PV_KEYS keys are double-buffered in shared memory with
// cp.async; P stays row-major, so one 16-byte load gives 4 keys of a row.
constexpr int PV_ROWS = 32;  // query-head rows per CTA
constexpr int PV_KEYS = 32;  // keys per staged tile
constexpr int PV_PS = PV_KEYS + 4;  // padded P row (floats)

DI void cp_async16(void* sdst, const void* gsrc) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(sdst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gsrc) : "memory");
}
DI void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
DI void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

template <int HD>
__global__ void __launch_bounds__((PV_ROWS / 4) * (HD / 4)) attn_pv_kernel(const float* __restrict__ P,
                                                                           const float* __restrict__ vc,
                                                                           const int* pos0p, int T, int n_head,
                                                                           int gsz, int qb, int n_ctx, int s_ld,
                                                                           float one, float* __restrict__ out,
                                                                           uint32_t* err) {
  pdl_enter();
  constexpr int NT = (PV_ROWS / 4) * (HD / 4);
  __shared__ __align__(16) float ps[2][PV_ROWS][PV_PS];
  __shared__ __align__(16) float vs[2][PV_KEYS][HD];
  const int pos0 = *pos0p;
  const int t0 = blockIdx.x * qb;
  const int kvh = blockIdx.y;
  const int tq = min(qb, T - t0);
  const int rows = tq * gsz;
  const int jmax = pos0 + t0 + tq;  // longest score row of the block
  const int tid = threadIdx.x;
  const int mt = tid / (HD / 4), dt = tid - mt * (HD / 4);
  const float* vb = vc + (size_t)kvh * n_ctx * HD;

  // tile k -> buffer k & 1: P rows (zero past each row's length, written by
  // the softmax), V rows below jmax (zeros above, never read from memory)
  auto load_tile = [&](int k) {
    const int jc = k * PV_KEYS, bf = k & 1;
    for (int i = tid; i < PV_ROWS * (PV_KEYS / 4); i += NT) {
      const int m = i / (PV_KEYS / 4), c4 = (i - m * (PV_KEYS / 4)) * 4;
      if (m < rows) {
        const int qi = m / gsz, hh = m - qi * gsz;
        cp_async16(&ps[bf][m][c4], P + ((size_t)(t0 + qi) * n_head + kvh * gsz + hh) * s_ld + jc + c4);
      }
    }
    for (int i = tid; i < PV_KEYS * (HD / 4); i += NT) {
      const int jj = i / (HD / 4), d4 = (i - jj * (HD / 4)) * 4;
      if (jc + jj < jmax)
        cp_async16(&vs[bf][jj][d4], vb + (size_t)(jc + jj) * HD + d4);
      else
        *reinterpret_cast<float4*>(&vs[bf][jj][d4]) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    cp_async_commit();
  };

  float2 o[4][2];  // rows mt*4 + r, dims (dt*4, +1) and (dt*4 + 2, +3)
#pragma unroll
  for (int r = 0; r < 4; r++) o[r][0] = o[r][1] = make_float2(0.f, 0.f);

  const int ntile = (jmax + PV_KEYS - 1) / PV_KEYS;
  load_tile(0);
  for (int k = 0; k < ntile; k++) {
    if (k + 1 < ntile) {
      load_tile(k + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // tile k visible to every thread
    const int bf = k & 1;
#pragma unroll 2
    for (int jj = 0; jj < PV_KEYS; jj += 4) {
      float4 p4[4], v4[4];
#pragma unroll
      for (int r = 0; r < 4; r++) p4[r] = *reinterpret_cast<const float4*>(&ps[bf][mt * 4 + r][jj]);
#pragma unroll
      for (int c = 0; c < 4; c++) v4[c] = *reinterpret_cast<const float4*>(&vs[bf][jj + c][dt * 4]);
#pragma unroll
      for (int c = 0; c < 4; c++) {
#pragma unroll
        for (int r = 0; r < 4; r++) {
          const float pr = c == 0 ? p4[r].x : c == 1 ? p4[r].y : c == 2 ? p4[r].z : p4[r].w;
          o[r][0] = add_by_fma2(mul2(pr, pr, v4[c].x, v4[c].y), one, o[r][0]);
          o[r][1] = add_by_fma2(mul2(pr, pr, v4[c].z, v4[c].w), one, o[r][1]);
        }
      }
    }
    __syncthreads();  // buffer k & 1 free for tile k + 2
  }
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const int m = mt * 4 + r;
    if (m >= rows) continue;
    const int qi = m / gsz, hh = m - qi * gsz;
    const int t = t0 + qi;
    float* ob = out + ((size_t)t * n_head + kvh * gsz + hh) * HD + dt * 4;
    float4 v;
    if (pos0 + t == 0) {  // score_len == 1 copies v_0 (lib.rs:2319-2322)
      v = *reinterpret_cast<const float4*>(vb + dt * 4);
    } else {
      // a non-finite value of V below jmax reaches this row or the block's
      // longest row (whose p_j are all > 0), as in the reference's check
      v = make_float4(o[r][0].x, o[r][0].y, o[r][1].x, o[r][1].y);
      if (!finite(v.x) || !finite(v.y) || !finite(v.z) || !finite(v.w)) atomicOr(err, ERRF_NONFINITE);
    }
    *reinterpret_cast<float4*>(ob) = v;
  }
}

// score rows are padded to whole 32-key tiles (16-byte aligned, and the PV
// kernel's last tile stays inside the row)
int score_ld(int n_ctx) { return (n_ctx + 31) & ~31; }

// ---- decode (T <= 8): one CTA per softmax row, one thread per PV chain -----------
// With a handful of query rows the per-row kernels above leave most of the
// GPU idle.  The softmax gives each (position, head) row a CTA: exps by all
// threads into shared memory, the eight ordered Z chains by eight threads,
// p = e / Z by all.  PV gives each (KV head, 8 dims, position) a CTA with one
// ordered chain o[d] += p_j v_j[d] per thread, over 64-key tiles of P and V
// staged with cp.async, PD_STAGES tiles in flight (a tile's 64 adds are far
// shorter than a load from HBM); as in the chunked path the rows are zero
// past their length, so whole tiles are summed exactly.
constexpr int SD_THREADS = 256;
constexpr int PD_KEYS = 64;
constexpr int PD_DIMS = 8;
constexpr int PD_STAGES = 4;
DI int pd_ps_floats(int gsz) { return PD_STAGES * gsz * PD_KEYS; }
inline size_t pd_smem_bytes(int gsz) { return (size_t)PD_STAGES * (gsz * PD_KEYS + PD_KEYS * PD_DIMS) * sizeof(float); }

__global__ void __launch_bounds__(SD_THREADS) attn_softmax_row_kernel(float* __restrict__ S, const int* pos0p,
                                                                     int n_head, int s_ld, uint32_t* err) {
  pdl_enter();
  extern __shared__ float sm_row[];  // [s_ld]
  __shared__ float red[SD_THREADS / 32];
  __shared__ float lanes[8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.x;
  const int t = row / n_head;
  const int len = *pos0p + t + 1;
  if (len == 1) return;
  float* s = S + (size_t)row * s_ld;
  float mx = -INFINITY;
  for (int j = tid; j < len; j += SD_THREADS) {
    const float v = s[j];
    sm_row[j] = v;
    mx = fmaxf(mx, v);
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < SD_THREADS / 32; w++) mx = fmaxf(mx, red[w]);
  for (int j = tid; j < len; j += SD_THREADS) {
    const float d = fsub(sm_row[j], mx);
    sm_row[j] = expf_det(d > -88.0f ? d : -88.0f);
  }
  __syncthreads();
  if (tid < 8) {  // sum_f32_ref: the ordered chain of lane tid
    float acc = 0.0f;
    int j = tid;
    for (; j + 56 < len; j += 64) {
      float e[8];
#pragma unroll
      for (int k = 0; k < 8; k++) e[k] = sm_row[j + 8 * k];
#pragma unroll
      for (int k = 0; k < 8; k++) acc = fadd(acc, e[k]);
    }
    for (; j < len; j += 8) acc = fadd(acc, sm_row[j]);
    lanes[tid] = acc;
  }
  __syncthreads();
  const float z = finish8(lanes);
  if (!finite(z) || z == 0.0f) {
    if (tid == 0) atomicOr(err, ERRF_NONFINITE);
    return;
  }
  for (int j = tid; j < len; j += SD_THREADS) {
    const float p = fdiv(sm_row[j], z);
    if (!finite(p)) atomicOr(err, ERRF_NONFINITE);
    s[j] = p;
  }
  const int zend = min(s_ld, (len + 31 + 31) & ~31);
  for (int j = len + tid; j < zend; j += SD_THREADS) s[j] = 0.0f;
}

template <int HD>
__global__ void attn_pv_decode_kernel(const float* __restrict__ P, const float* __restrict__ vc, const int* pos0p,
                                      int n_head, int gsz, int n_ctx, int s_ld, float* __restrict__ out,
                                      uint32_t* err) {
  pdl_enter();
  extern __shared__ __align__(16) float pd_smem[];
  float* ps = pd_smem;                     // [PD_STAGES][gsz][PD_KEYS]
  float* vs = pd_smem + pd_ps_floats(gsz);  // [PD_STAGES][PD_KEYS][PD_DIMS]
  const int kvh = blockIdx.x, d0 = blockIdx.y * PD_DIMS, t = blockIdx.z;
  const int tid = threadIdx.x, nt = blockDim.x;
  const int h = tid / PD_DIMS, dd = tid - h * PD_DIMS;
  const int len = *pos0p + t + 1;
  const float* vb = vc + (size_t)kvh * n_ctx * HD;
  float* ob = out + ((size_t)t * n_head + kvh * gsz + h) * HD + d0 + dd;
  if (len == 1) {  // score_len == 1 copies v_0 (lib.rs:2319-2322)
    *ob = vb[d0 + dd];
    return;
  }
  const float* prow0 = P + ((size_t)t * n_head + kvh * gsz) * s_ld;
  const int ntile = (len + PD_KEYS - 1) / PD_KEYS;
  // tile k into stage k % PD_STAGES; an empty commit group past the last
  // tile keeps the wait count uniform
  auto load_tile = [&](int k) {
    if (k < ntile) {
      const int jc = k * PD_KEYS, bf = k % PD_STAGES;
      float* pb = ps + bf * gsz * PD_KEYS;
      float* vbuf = vs + bf * PD_KEYS * PD_DIMS;
      for (int i = tid; i < gsz * (PD_KEYS / 4); i += nt) {
        const int r = i / (PD_KEYS / 4), c4 = (i - r * (PD_KEYS / 4)) * 4;
        // a chunk that starts at or past the score length is zero (never
        // read: it may lie past the row's zeroed tail)
        if (jc + c4 < len)
          cp_async16(pb + r * PD_KEYS + c4, prow0 + (size_t)r * s_ld + jc + c4);
        else
          *reinterpret_cast<float4*>(pb + r * PD_KEYS + c4) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      for (int i = tid; i < PD_KEYS * (PD_DIMS / 4); i += nt) {
        const int jj = i / (PD_DIMS / 4), c4 = (i - jj * (PD_DIMS / 4)) * 4;
        if (jc + jj < len)
          cp_async16(vbuf + jj * PD_DIMS + c4, vb + (size_t)(jc + jj) * HD + d0 + c4);
        else
          *reinterpret_cast<float4*>(vbuf + jj * PD_DIMS + c4) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    cp_async_commit();
  };
  float acc = 0.0f;
  for (int k = 0; k < PD_STAGES - 1; k++) load_tile(k);
  for (int k = 0; k < ntile; k++) {
    load_tile(k + PD_STAGES - 1);
    cp_async_wait<PD_STAGES - 1>();  // tile k has landed
    __syncthreads();
    const int bf = k % PD_STAGES;
    const float* pr = ps + (bf * gsz + h) * PD_KEYS;
    const float* vr = vs + bf * PD_KEYS * PD_DIMS + dd;
#pragma unroll 8
    for (int jj = 0; jj < PD_KEYS; jj++) acc = fadd(acc, fmul(pr[jj], vr[jj * PD_DIMS]));
    __syncthreads();  // stage bf is refilled by the next iteration's load
  }
  if (!finite(acc)) atomicOr(err, ERRF_NONFINITE);
  *ob = acc;
}

// ---- one position, fused ------------------------------------------------------
// For a chunk of one position (decode) the three steps run in one kernel: a
// cluster of AD_CS CTAs per query head, each CTA owning a contiguous quarter
// of the keys (whole 64-key tiles, in order), so each SM streams a quarter
// of the head's K and V rows:
//   scores  the CTA's K tiles stream through an AD_STAGES-slot cp.async ring;
//           four threads share a key, thread quarter r owning the lane
//           chains 2r and 2r + 1 of the dot (elements 8i + 2r, 8i + 2r + 1,
//           i ascending), so ((l0 + l1) + (l2 + l3)) + ((l4 + l5) + (l6 +
//           l7)) is two in-thread adds and two shuffles;
//   softmax the max over the cluster (each CTA's max read through
//           distributed shared memory), e_j, then the eight ordered z lane
//           chains relayed CTA to CTA in key order (CTA c starts its lanes
//           from CTA c - 1's partial sums), z = finish8 of the last, p = e/z;
//   PV      the CTA's V tiles stream in during the softmax; the chain o[d]
//           is relayed the same way: CTA c continues CTA c - 1's sums over
//           its own keys, and the last CTA stores them.
// Each relay step is one cluster barrier, taken by every thread of every
// CTA, so the chains keep the reference's order exactly.  Tile rows are
// HD + 8 floats apart, so the 8-byte reads of a half-warp (four keys x four
// quarters) and the 4-byte reads of consecutive d fall in distinct banks.
constexpr int AD_THREADS = 256;
constexpr int AD_KEYS = 64;
constexpr int AD_STAGES = 3;
constexpr int AD_CS = 4;           // CTAs per head (cluster size)
constexpr int AD_MAX_CTX = 16384;  // each CTA's score slice in shared memory
template <int HD>
__host__ __device__ constexpr int ad_tile_floats() {
  return AD_KEYS * (HD + 8);
}
// the most keys one CTA owns: whole tiles, ceil(tiles / AD_CS) of them
inline int ad_slice_keys(int n_ctx) { return ((n_ctx + AD_KEYS - 1) / AD_KEYS + AD_CS - 1) / AD_CS * AD_KEYS; }
template <int HD>
size_t ad_smem_bytes(int n_ctx) {
  // ring, q row, score slice, relay buffer (HD PV sums)
  return ((size_t)AD_STAGES * ad_tile_floats<HD>() + 2 * HD + (size_t)ad_slice_keys(n_ctx)) * sizeof(float);
}

DI void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
DI uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// a float of CTA `rank`'s shared memory at the address of `local` in this CTA
DI float ld_dsmem(const float* local, uint32_t rank) {
  uint32_t a = (uint32_t)__cvta_generic_to_shared(local), ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
}

template <int HD>
__global__ void __launch_bounds__(AD_THREADS) attn_decode_kernel(const float* __restrict__ q,
                                                                 const float* __restrict__ kc,
                                                                 const float* __restrict__ vc, const int* pos0p,
                                                                 int gsz, int n_ctx, float scale,
                                                                 float* __restrict__ out, uint32_t* err) {
  constexpr int LD = HD + 8;
  pdl_enter();
  extern __shared__ __align__(16) float ad_smem[];
  float* ring = ad_smem;                                 // [AD_STAGES][AD_KEYS][LD]
  float* qs = ring + AD_STAGES * ad_tile_floats<HD>();  // [HD]
  float* relay = qs + HD;                                // [HD]: PV sums handed to the next CTA
  float* sc = relay + HD;                                // [slice]: scores, then e, then p
  __shared__ float red[AD_THREADS / 32];
  __shared__ float cmax;
  __shared__ float l8[8];  // z lane sums handed to the next CTA
  const uint32_t rank = cluster_rank();
  const int h = (int)blockIdx.x / AD_CS, kvh = h / gsz;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int len = *pos0p + 1;
  const float* kb = kc + (size_t)kvh * n_ctx * HD;
  const float* vb = vc + (size_t)kvh * n_ctx * HD;
  float* ob = out + (size_t)h * HD;
  if (len == 1) {  // score_len == 1 copies v_0 (lib.rs:2319-2322); the same in every CTA of the cluster
    if (rank == 0)
      for (int d = tid; d < HD; d += AD_THREADS) ob[d] = vb[d];
    return;
  }
  // this CTA's tiles [t0, t1) of the score row
  const int ntile_all = (len + AD_KEYS - 1) / AD_KEYS;
  const int t0 = (int)(((long long)ntile_all * rank) / AD_CS), t1 = (int)(((long long)ntile_all * (rank + 1)) / AD_CS);
  const int ntile = t1 - t0, j0 = t0 * AD_KEYS, jn = min(len, t1 * AD_KEYS) - j0;  // local keys [0, jn)
  // local tile k of `base` into slot k % AD_STAGES, rows past the score
  // length zero; an empty group past the last tile keeps the wait counts
  // uniform
  auto load_tile = [&](const float* base, int k) {
    if (k < ntile) {
      float* dst = ring + (k % AD_STAGES) * ad_tile_floats<HD>();
      for (int i = tid; i < AD_KEYS * (HD / 4); i += AD_THREADS) {
        const int jj = i / (HD / 4), c4 = (i - jj * (HD / 4)) * 4;
        const int j = j0 + k * AD_KEYS + jj;
        if (j < len)
          cp_async16(dst + jj * LD + c4, base + (size_t)j * HD + c4);
        else
          *reinterpret_cast<float4*>(dst + jj * LD + c4) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    cp_async_commit();
  };
  for (int k = 0; k < AD_STAGES - 1; k++) load_tile(kb, k);
  for (int d = tid; d < HD; d += AD_THREADS) {
    const float v = q[(size_t)h * HD + d];
    if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
    qs[d] = v;
  }

  // scores: s_j = dot_f32_ref(q, k_j) * scale
  const int jj = tid >> 2, qr = tid & 3;
  for (int k = 0; k < ntile; k++) {
    load_tile(kb, k + AD_STAGES - 1);
    cp_async_wait<AD_STAGES - 1>();  // tile k has landed
    __syncthreads();
    const float* kr = ring + (k % AD_STAGES) * ad_tile_floats<HD>() + jj * LD + 2 * qr;
    float a0 = 0.0f, a1 = 0.0f;  // lane chains 2 qr and 2 qr + 1
#pragma unroll
    for (int i = 0; i < HD / 8; i++) {
      const float2 kv = *reinterpret_cast<const float2*>(kr + 8 * i);
      const float2 qv = *reinterpret_cast<const float2*>(qs + 8 * i + 2 * qr);
      const float2 pr = mul2(qv.x, qv.y, kv.x, kv.y);
      a0 = fadd(a0, pr.x);
      a1 = fadd(a1, pr.y);
    }
    const float pair = fadd(a0, a1);                                        // l(2qr) + l(2qr + 1)
    const float quad = fadd(pair, __shfl_xor_sync(0xffffffffu, pair, 1));  // (l0 + l1) + (l2 + l3), ...
    const float dot = fadd(quad, __shfl_xor_sync(0xffffffffu, quad, 2));
    const int jl = k * AD_KEYS + jj;
    if (qr == 0 && jl < jn) {
      const float sv = fmul(dot, scale);
      if (!finite(sv)) atomicOr(err, ERRF_NONFINITE);
      sc[jl] = sv;
    }
    __syncthreads();  // slot k % AD_STAGES is refilled by the next iteration
  }
  for (int k = 0; k < AD_STAGES - 1; k++) load_tile(vb, k);  // V, during the softmax

  // softmax (attention_one_head: e_j = exp(max(s_j - max, -88)), z = sum_f32_ref(e))
  float mx = -INFINITY;
  for (int j = tid; j < jn; j += AD_THREADS) mx = fmaxf(mx, sc[j]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  if (tid == 0) {
    float m = red[0];
#pragma unroll
    for (int w = 1; w < AD_THREADS / 32; w++) m = fmaxf(m, red[w]);
    cmax = m;
  }
  cluster_sync();  // every CTA's max is published
  mx = ld_dsmem(&cmax, 0);
#pragma unroll
  for (int r = 1; r < AD_CS; r++) mx = fmaxf(mx, ld_dsmem(&cmax, (uint32_t)r));
  for (int j = tid; j < jn; j += AD_THREADS) {
    const float d = fsub(sc[j], mx);
    sc[j] = expf_det(d > -88.0f ? d : -88.0f);
  }
  __syncthreads();
  // sum_f32_ref: lane l sums e_j over j = l (mod 8) in key order, CTA after CTA
  for (int c = 0; c < AD_CS; c++) {
    if ((int)rank == c && tid < 8) {
      float acc = c == 0 ? 0.0f : ld_dsmem(&l8[tid], (uint32_t)(c - 1));
      // local key jl has global index j0 + jl; j0 is a multiple of 8, so the
      // lane of local key jl is jl mod 8
      int j = tid;
      for (; j + 56 < jn; j += 64) {
        float e[8];
#pragma unroll
        for (int k = 0; k < 8; k++) e[k] = sc[j + 8 * k];
#pragma unroll
        for (int k = 0; k < 8; k++) acc = fadd(acc, e[k]);
      }
      for (; j < jn; j += 8) acc = fadd(acc, sc[j]);
      l8[tid] = acc;
    }
    cluster_sync();
  }
  float lz[8];
#pragma unroll
  for (int k = 0; k < 8; k++) lz[k] = ld_dsmem(&l8[k], AD_CS - 1);
  const float z = finish8(lz);
  if (!finite(z) || z == 0.0f) {  // the same z in every CTA: the whole cluster stops here
    if (tid == 0 && rank == 0) atomicOr(err, ERRF_NONFINITE);
    cp_async_wait<0>();  // no copy into this CTA's shared memory outlives it
    cluster_sync();      // no CTA leaves while another may still read its shared memory
    return;
  }
  for (int j = tid; j < jn; j += AD_THREADS) {
    const float pj = fdiv(sc[j], z);
    if (!finite(pj)) atomicOr(err, ERRF_NONFINITE);
    sc[j] = pj;
  }
  __syncthreads();

  // o[d] = sum over j of p_j * v_j[d], in key order, CTA after CTA
  for (int c = 0; c < AD_CS; c++) {
    if ((int)rank == c) {
      float acc = 0.0f;
      if (c > 0 && tid < HD) acc = ld_dsmem(&relay[tid], (uint32_t)(c - 1));
      for (int k = 0; k < ntile; k++) {
        load_tile(vb, k + AD_STAGES - 1);
        cp_async_wait<AD_STAGES - 1>();
        __syncthreads();  // tile k visible
        if (tid < HD) {
          const float* vr = ring + (k % AD_STAGES) * ad_tile_floats<HD>() + tid;
          const float* pr = sc + k * AD_KEYS;
          const int n = min(AD_KEYS, jn - k * AD_KEYS);
          int i = 0;
          for (; i + 8 <= n; i += 8) {
            float pv[8], vv[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
              pv[u] = pr[i + u];
              vv[u] = vr[(i + u) * LD];
            }
#pragma unroll
            for (int u = 0; u < 8; u++) acc = fadd(acc, fmul(pv[u], vv[u]));
          }
          for (; i < n; i++) acc = fadd(acc, fmul(pr[i], vr[i * LD]));
        }
        __syncthreads();
      }
      if (tid < HD) {
        if (c == AD_CS - 1) {
          if (!finite(acc)) atomicOr(err, ERRF_NONFINITE);
          ob[tid] = acc;
        } else {
          relay[tid] = acc;
        }
      }
    }
    cluster_sync();
  }
  cp_async_wait<0>();
}

template <int HD>
constexpr int qk_smem_bytes() {
  return (QK_ROWS + QK_KEYS) * (HD + 4) * (int)sizeof(float);
}

template <int HD>
cudaError_t launch_tiled(const Launch& L, const float* q, const float* kc, const float* vc, int T, const int* pos0,
                         int n_head, int n_head_kv, int n_ctx, float scale, float* out, float* S) {
  const int gsz = n_head / n_head_kv;
  const int qb = QK_ROWS / gsz;
  constexpr int smem = qk_smem_bytes<HD>();
  static std::atomic<unsigned long long> attr_set{0};  // one bit per device (sessions may run on several host threads)
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && (dev >= 64 || !(attr_set.load() >> dev & 1ull))) {
    cudaError_t e = cudaFuncSetAttribute(attn_scores_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set.fetch_or(1ull << dev);
  }
  const int s_ld = score_ld(n_ctx);
  if (T == 1 && n_ctx <= AD_MAX_CTX) {  // one position: the fused kernel, a cluster of AD_CS CTAs per head
    if (cudaError_t e = raise_smem_cap((const void*)attn_decode_kernel<HD>, ad_smem_bytes<HD>(AD_MAX_CTX))) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_head * AD_CS);
    cfg.blockDim = dim3(AD_THREADS);
    cfg.dynamicSmemBytes = ad_smem_bytes<HD>(n_ctx);
    cfg.stream = L.stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = AD_CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = L.pdl && pdl_enabled() ? 2 : 1;
    const cudaError_t e_ = cudaLaunchKernelEx(&cfg, attn_decode_kernel<HD>, q, kc, vc, pos0, gsz, n_ctx, scale, out,
                                              L.err);
    if (e_ != cudaSuccess) return e_;
    if (L.launches) *L.launches += 1;
    return cudaGetLastError();
  }
  dim3 g1((n_ctx + QK_KEYS - 1) / QK_KEYS, (T + qb - 1) / qb, n_head_kv);
  {
    const cudaError_t e_ = launch_k(L, attn_scores_kernel<HD>, g1, QK_THREADS, smem, q, kc, pos0, T, n_head, gsz, qb,
        n_ctx, s_ld, scale, S, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int rows = T * n_head;
  const int rpc = std::max(1, std::min(4, SM_SMEM_FLOATS / s_ld));
  if (T <= 8 && s_ld <= SM_SMEM_FLOATS) {  // decode: a CTA per row, a thread per PV chain
    {
      const cudaError_t e_ = launch_k(L, attn_softmax_row_kernel, rows, SD_THREADS, (size_t)s_ld * sizeof(float), S,
                                      pos0, n_head, s_ld, L.err);
      if (e_ != cudaSuccess) return e_;
    }
    {
      const cudaError_t e_ = launch_k(L, attn_pv_decode_kernel<HD>, dim3(n_head_kv, HD / PD_DIMS, T), gsz * PD_DIMS,
                                      pd_smem_bytes(gsz), S, vc, pos0, n_head, gsz, n_ctx, s_ld, out, L.err);
      if (e_ != cudaSuccess) return e_;
    }
    if (L.launches) *L.launches += 3;
    return cudaGetLastError();
  }
  if (rpc >= 4) {  // rows short enough to stage four per CTA in shared memory
    {
      const cudaError_t e_ = launch_k(L, attn_softmax_kernel<true>, (rows + rpc - 1) / rpc, rpc * 32,
          (size_t)rpc * s_ld * sizeof(float),  S, pos0, T, n_head, s_ld, rpc, L.err);
      if (e_ != cudaSuccess) return e_;
    }
  } else {
    {
      const cudaError_t e_ = launch_k(L, attn_softmax_long_kernel, (rows + SL_WARPS - 1) / SL_WARPS, SL_WARPS * 32, 0,
                                      S, pos0, T, n_head, s_ld, L.err);
      if (e_ != cudaSuccess) return e_;
    }
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int qb2 = PV_ROWS / gsz;
  dim3 g3((T + qb2 - 1) / qb2, n_head_kv);
  {
    const cudaError_t e_ = launch_k(L, attn_pv_kernel<HD>, g3, (PV_ROWS / 4) * (HD / 4), 0, S, vc, pos0, T, n_head,
        gsz, qb2, n_ctx, s_ld, 1.0f, out, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  if (L.launches) *L.launches += 3;
  return cudaGetLastError();
}

}  // namespace

size_t attention_tiled_scratch_floats(int T, int n_head, int n_ctx) { return (size_t)T * n_head * score_ld(n_ctx); }

bool attention_tiled_supported(int n_head, int n_head_kv, int head_dim) {
  if (n_head_kv <= 0 || n_head % n_head_kv) return false;
  const int gsz = n_head / n_head_kv;
  return (head_dim == 64 || head_dim == 128) && gsz <= PV_ROWS;
}

cudaError_t launch_attention_tiled(const Launch& L, const float* q, const float* kc, const float* vc, int T,
                                   const int* pos0, int n_head, int n_head_kv, int head_dim, int n_ctx, float scale,
                                   float* out, float* S) {
  if (head_dim == 64) return launch_tiled<64>(L, q, kc, vc, T, pos0, n_head, n_head_kv, n_ctx, scale, out, S);
  return launch_tiled<128>(L, q, kc, vc, T, pos0, n_head, n_head_kv, n_ctx, scale, out, S);
}

}  // namespace det
