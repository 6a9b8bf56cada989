// kernels.cu -- sm_100a kernels of libdetgpu.so (layer ops, attention, CDF).
//
// Each kernel reproduces the reference's arithmetic in the reference's order;
// the comment on each names the Rust function it follows.  All f32 math goes
// through det::fadd/fmul/fdiv (explicitly rounded, never contracted).  Any
// non-finite intermediate the reference would reject sets a bit in the
// session's device error flag, which the host turns into DET_ERR_NONFINITE.
#include <cuda_runtime.h>

#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "dev_math.cuh"
#include "../../include/detgpu.h"
#include "internal.h"

namespace det {

namespace {

DI void flag(uint32_t* err, uint32_t bit) { atomicOr(err, bit); }

template <int NT>
DI float block_max(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < NT / 32 ? red[l] : -INFINITY;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

template <int NT>
DI unsigned long long block_sum_u64(unsigned long long v, unsigned long long* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < NT / 32 ? red[l] : 0ull;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// ---- dequantisation helpers (det-quant lib.rs:506-568) --------------------

// q4_k_value on a raw 144-byte super-block
DI float q4k_value(const uint8_t* blk, int index) {
  const float d = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
  const float dmin = f16_bits_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
  const int sub = index >> 5, within = index & 31;
  int sc, mn;
  q4k_scale_min(blk + 4, sub, sc, mn);
  const uint8_t byte = blk[16 + (sub >> 1) * 32 + within];
  const int q = (sub & 1) ? (byte >> 4) : (byte & 0x0f);
  return fsub(fmul(fmul(d, (float)sc), (float)q), fmul(dmin, (float)mn));
}

// q6_k_quant on a 208-byte body (ql[128] | qh[64] | scales[16])
DI int q6k_scale_index(int index) {
  const int half = index >> 7, within = index & 127, l = within & 31, part = within >> 5;
  return half * 8 + (l >> 4) + 2 * part;
}

DI float q6k_value(const uint8_t* body, float d, int index) {
  const int8_t sc = (int8_t)body[192 + q6k_scale_index(index)];
  return fmul(fmul(d, (float)sc), (float)q6k_quant(body, index));
}

// ---- RoPE table: RopeTables::llama (det-model lib.rs:813-846) ------------
__global__ void rope_table_kernel(float* cos_t, float* sin_t, int positions, int half, int rope_dim,
                                  float rope_base) {
  pdl_enter();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)positions * half) return;
  const int pos = (int)(i / half), j = (int)(i % half);
  const double ln_base = log_det((double)rope_base);
  const double exponent = ddiv(-(double)(2 * j), (double)rope_dim);
  const double omega = exp_det(dmul(exponent, ln_base));
  const double phi = dmul((double)pos, omega);
  cos_t[i] = __double2float_rn(cos_det(phi));
  sin_t[i] = __double2float_rn(sin_det(phi));
}

// ---- embedding row: write_row_validated (det-model lib.rs:667-746) --------
__global__ void embed_kernel(DevMatrix m, const uint32_t* tokens, int T, float* x, uint32_t* err) {
  pdl_enter();
  const int t = blockIdx.x;
  if (t >= T) return;
  const uint32_t tok = tokens[t];
  if (tok >= (uint32_t)m.rows) {
    if (threadIdx.x == 0) flag(err, ERRF_SHAPE);
    return;
  }
  const int K = m.cols;
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    float v;
    switch (m.type) {
      case GT_F32: v = m.f[(size_t)tok * K + i]; break;
      case GT_Q8_0:
      case GT_Q4_0: {  // tile records (gemm.cu): element (tok, i) of the block
        const bool q8 = m.type == GT_Q8_0;
        const int rb = q8 ? 544 : 288, qb = q8 ? 512 : 256;
        const int rr = (int)(tok & 15), g = rr & 7, hi = rr >> 3, b = i >> 5, c = i & 31;
        const uint8_t* rec = (const uint8_t*)m.q + ((size_t)(tok >> 4) * m.nb + b) * rb;
        const int lane = g * 4 + ((c & 15) >> 2);
        int qv;
        if (q8) {
          qv = (int8_t)rec[lane * 16 + hi * 4 + (c >= 16 ? 8 : 0) + (c & 3)];
        } else {  // Q4_0: element j < 16 low nibble of byte j, else high nibble
          const uint8_t byte = rec[lane * 8 + hi * 4 + (c & 3)];
          qv = (c < 16 ? (byte & 0x0f) : (byte >> 4)) - 8;
        }
        const uint32_t sw = *reinterpret_cast<const uint32_t*>(rec + qb + 4 * g);
        const float d = f16_bits_to_f32((uint16_t)(hi ? (sw >> 16) : (sw & 0xffffu)));
        v = fmul(d, (float)qv);
        break;
      }
      case GT_Q4_K:
        v = q4k_value((const uint8_t*)m.q + ((size_t)tok * m.nb + (i >> 8)) * 144, i & 255);
        break;
      default: {  // GT_Q6_K
        const size_t b = (size_t)tok * m.nb + (i >> 8);
        v = q6k_value((const uint8_t*)m.q + b * 208, f16_bits_to_f32(m.d[b]), i & 255);
        break;
      }
    }
    if (!finite(v)) flag(err, ERRF_NONFINITE);
    x[(size_t)t * K + i] = v;
  }
}

// ---- Q8A quantiser: try_quantize_q8a_block (det-quant lib.rs:111-137) ------
// One warp quantises one 32-element block, lane l holding element l; amax by
// shuffle (max is order-free); the output goes to the Q8A layout
// (dev_math.cuh).  Callers have checked v for finiteness.
DI void q8a_block_warp(float v, int l, int nbk, int t, int kb, float* __restrict__ qd, int8_t* __restrict__ qq) {
  float amax = fabsf(v);
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  int q = 0;
  float d = 0.0f;
  if (amax != 0.0f) {
    d = fdiv(amax, 127.0f);
    const float s = fdiv(v, d);
    int r = v < 0.0f ? __float2int_rz(fsub(s, 0.5f)) : __float2int_rz(fadd(s, 0.5f));
    q = max(-127, min(127, r));
  }
  qq[q8a_elem(nbk, t, kb, l)] = (int8_t)q;
  if (l == 0) qd[q8a_dslot(nbk, t, kb)] = d;
}

// one warp per block of x (T x K, row-major)
__global__ void quant_q8a_kernel(const float* __restrict__ x, int nblocks, int nbk, float* __restrict__ qd,
                                 int8_t* __restrict__ qq, uint32_t* err) {
  pdl_enter();
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (b >= nblocks) return;
  const int l = threadIdx.x & 31;
  const int t = b / nbk, kb = b - t * nbk;
  const float v = x[(size_t)b * 32 + l];
  if (!finite(v)) flag(err, ERRF_NONFINITE);
  q8a_block_warp(v, l, nbk, t, kb, qd, qq);
}

// swiglu (det-model lib.rs:2420-2434) with the Q8A quantisation of its
// output fused in: one warp per 32-element block of the T x n output
__global__ void swiglu_q8a_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ out,
                                  int nblocks, int nbk, float* __restrict__ qd, int8_t* __restrict__ qq,
                                  uint32_t* err) {
  pdl_enter();
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (b >= nblocks) return;
  const int l = threadIdx.x & 31;
  const int t = b / nbk, kb = b - t * nbk;
  const size_t i = (size_t)b * 32 + l;
  const float gv = g[i], uv = u[i];
  const float y = fmul(silu_det(gv), uv);
  if (!finite(y) || !finite(gv) || !finite(uv)) flag(err, ERRF_NONFINITE);
  out[i] = y;
  q8a_block_warp(y, l, nbk, t, kb, qd, qq);
}

// ---- rmsnorm (det-model lib.rs:2053-2073) ----------------------------------
// sum_squares_f32_ref: lane l accumulates x[i]^2 for i = l (mod 8) in order.
// The row and the norm weights are staged in shared memory by all threads
// (coalesced, one load latency), then eight threads run the eight ordered
// lane chains out of shared memory.
constexpr int RMS_MAX_SMEM = 16384;  // floats staged per row (larger rows read global)

// When qd / qq are given (n a multiple of 32), the normalised row is also
// quantised to Q8A: warp w takes blocks w, w + 8, ... of the row.
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, int n, float eps,
                               float* __restrict__ h, float* __restrict__ qd, int8_t* __restrict__ qq,
                               uint32_t* err) {
  pdl_enter();
  extern __shared__ float xs[];  // [n] x, then [n] w
  const int t = blockIdx.x;
  const float* xr = x + (size_t)t * n;
  __shared__ float lanes[8];
  __shared__ float r_s;
  const bool staged = n <= RMS_MAX_SMEM;
  if (staged) {
    if ((n & 3) == 0 && (((uintptr_t)xr | (uintptr_t)w) & 15) == 0) {  // float4 copies, two per thread in flight
      const float4* x4 = reinterpret_cast<const float4*>(xr);
      const float4* w4 = reinterpret_cast<const float4*>(w);
      for (int i = threadIdx.x; i < n / 4; i += blockDim.x) {
        const float4 a = x4[i], b = w4[i];
        reinterpret_cast<float4*>(xs)[i] = a;
        reinterpret_cast<float4*>(xs + n)[i] = b;
      }
    } else {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        xs[i] = xr[i];
        xs[n + i] = w[i];
      }
    }
  }
  __syncthreads();
  const float* src = staged ? xs : xr;
  const float* wv = staged ? xs + n : w;
  if (threadIdx.x < 8) {  // sum_squares_f32_ref: the ordered chain of lane threadIdx.x
    float acc = 0.0f;
    int i = threadIdx.x;
    // two groups of eight loads in flight ahead of the adds
    for (; i + 120 < n; i += 128) {
      float a[16];
#pragma unroll
      for (int k = 0; k < 16; k++) a[k] = src[i + 8 * k];
#pragma unroll
      for (int k = 0; k < 16; k++) acc = fadd(acc, fmul(a[k], a[k]));
    }
    for (; i < n; i += 8) acc = fadd(acc, fmul(src[i], src[i]));
    lanes[threadIdx.x] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const float ss = finish8(lanes);
    const float m = fdiv(ss, __int2float_rn(n));
    const float r = fdiv(1.0f, __fsqrt_rn(fadd(m, eps)));
    if (!finite(r)) flag(err, ERRF_NONFINITE);
    r_s = r;
  }
  __syncthreads();
  const float r = r_s;
  if (qq) {
    const int nbk = n / 32, l = threadIdx.x & 31;
    for (int kb = threadIdx.x >> 5; kb < nbk; kb += blockDim.x >> 5) {
      const int i = kb * 32 + l;
      const float xi = src[i];
      const float v = fmul(fmul(xi, r), wv[i]);
      if (!finite(v) || !finite(xi)) flag(err, ERRF_NONFINITE);
      h[(size_t)t * n + i] = v;
      q8a_block_warp(v, l, nbk, t, kb, qd, qq);
    }
    return;
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float xi = src[i];
    const float v = fmul(fmul(xi, r), wv[i]);
    if (!finite(v) || !finite(xi)) flag(err, ERRF_NONFINITE);
    h[(size_t)t * n + i] = v;
  }
}

// ---- Q8_K quantiser: try_quantize_q8k_block (det-quant lib.rs:139-172) ----
// one warp per 256-element block; the signed max is x at the FIRST index with
// the largest |x| (carried as (|x|, index) through the reduction).
// qp non-null: also the class-permuted record of gemm_q6k_tc.cu per
// (64-position group, block): byte (c, p, j) = q[8 j + c] of position p,
// 16-byte halves swapped for positions with bit 2 set, then a.d per position
__global__ void quant_q8k_kernel(const float* __restrict__ x, int nblocks, int nbk, float* __restrict__ qd,
                                 int8_t* __restrict__ qq, uint8_t* __restrict__ qp, uint32_t* err) {
  pdl_enter();
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (b >= nblocks) return;
  const int l = threadIdx.x & 31;
  const float* xb = x + (size_t)b * 256;
  // this lane's elements 8 l .. 8 l + 7 are column l of classes 0..7
  uint8_t* prec = nullptr;
  int pcol = 0;
  if (qp) {
    const int t = b / nbk, kb = b - t * nbk, p = t & 63;
    prec = qp + ((size_t)(t >> 6) * nbk + kb) * (8 * 64 * 32 + 64 * 4);
    pcol = p * 32 + (l ^ (((p >> 2) & 1) << 4));
  }
  float v[8];
  float amax = 0.0f;
  int idx = 0x7fffffff;
  for (int k = 0; k < 8; k++) {
    const int i = l * 8 + k;
    v[k] = xb[i];
    if (!finite(v[k])) flag(err, ERRF_NONFINITE);
    const float ax = fabsf(v[k]);
    if (ax > amax) {
      amax = ax;
      idx = i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (oa > amax || (oa == amax && oi < idx)) {
      amax = oa;
      idx = oi;
    }
  }
  if (amax == 0.0f) {
    for (int k = 0; k < 8; k++) qq[(size_t)b * 256 + l * 8 + k] = 0;
    if (l == 0) qd[b] = 0.0f;
    if (prec) {
      for (int k = 0; k < 8; k++) prec[k * 2048 + pcol] = 0;
      if (l == 0) reinterpret_cast<float*>(prec + 16384)[(b / nbk) & 63] = 0.0f;
    }
    return;
  }
  const float mx = xb[idx];
  const float iscale = fdiv(-127.0f, mx);
  for (int k = 0; k < 8; k++) {
    const float val = fadd(fmul(iscale, v[k]), 12582912.0f);
    int r = (int)(__float_as_uint(val) & 0x007fffffu) - 0x00400000;
    const int8_t q = (int8_t)min(127, r);
    qq[(size_t)b * 256 + l * 8 + k] = q;
    if (prec) prec[k * 2048 + pcol] = (uint8_t)q;
  }
  if (l == 0) {
    const float dv = fdiv(1.0f, iscale);
    qd[b] = dv;
    if (prec) reinterpret_cast<float*>(prec + 16384)[(b / nbk) & 63] = dv;
  }
}

// ---- generic GEMV: one thread per (row, position) running the reference's
// own loop.  Exact for every type; used for F32, Q4_K and Q6_K and as the
// fallback shape for the others. ------------------------------------------
DI float dot_row(const DevMatrix& m, const DevActs& a, int r, int t) {
  const int K = m.cols;
  switch (m.type) {
    case GT_F32: {  // dot_f32_ref (det-num reduce.rs:2-11)
      const float* w = m.f + (size_t)r * K;
      const float* x = a.x + (size_t)t * K;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int i = 0; i < K; i++) acc[i & 7] = fadd(acc[i & 7], fmul(w[i], x[i]));
      return finish8(acc);
    }
    case GT_Q4_K: {  // dot_q4_k_q8a (det-quant lib.rs:281-315): one f32 chain
      const uint8_t* w = (const uint8_t*)m.q + (size_t)r * m.nb * 144;
      const int nbk = K / 32;
      float sum = 0.0f;
      for (int b = 0; b < m.nb; b++) {
        const uint8_t* blk = w + (size_t)b * 144;
        const float d = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        const float dmin = f16_bits_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
        for (int sub = 0; sub < 8; sub++) {
          int sc, mn;
          q4k_scale_min(blk + 4, sub, sc, mn);
          const float dsc = fmul(d, (float)sc), dmn = fmul(dmin, (float)mn);
          const int kb = b * 8 + sub;
          const float a_d = a.qa_d[q8a_dslot(nbk, t, kb)];
          const uint8_t* qs = blk + 16 + (sub >> 1) * 32;
          const int8_t* aq = a.qa_q + q8a_slot(nbk, t, kb) * 32;
          const int swz = q8a_swz(t);
          for (int i = 0; i < 32; i++) {
            const int qv = (sub & 1) ? (qs[i] >> 4) : (qs[i] & 0x0f);
            const float weight = fsub(fmul(dsc, (float)qv), dmn);
            const float act = fmul(a_d, (float)aq[i ^ swz]);
            sum = fadd(sum, fmul(weight, act));
          }
        }
      }
      return sum;
    }
    default: {  // GT_Q6_K: dot_q6_k_q8k (det-quant lib.rs:353-397)
      const uint8_t* w = (const uint8_t*)m.q + (size_t)r * m.nb * 208;
      const uint16_t* wd = m.d + (size_t)r * m.nb;
      const int8_t* q = a.qk_q + (size_t)t * K;
      const float* ad = a.qk_d + (size_t)t * m.nb;
      float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int b = 0; b < m.nb; b++) {
        const uint8_t* body = w + (size_t)b * 208;
        int aux[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int s = 0; s < 16; s++) {
          const int scale = (int8_t)body[192 + s];
          for (int rep = 0; rep < 2; rep++) {
            const int off = s * 16 + rep * 8;
#pragma unroll
            for (int ln = 0; ln < 8; ln++)
              aux[ln] += scale * (int)q[b * 256 + off + ln] * q6k_quant(body, off + ln);
          }
        }
        const float dd = fmul(f16_bits_to_f32(wd[b]), ad[b]);
#pragma unroll
        for (int ln = 0; ln < 8; ln++) sums[ln] = fadd(sums[ln], fmul(dd, __int2float_rn(aux[ln])));
      }
      float sum = 0.0f;
#pragma unroll
      for (int ln = 0; ln < 8; ln++) sum = fadd(sum, sums[ln]);
      return sum;
    }
  }
}

DI void epilogue_store(float v, int r, int t, float* out, int out_ld, int epi, const float* bias, uint32_t* err) {
  if (!finite(v)) flag(err, ERRF_NONFINITE);
  float* dst = out + (size_t)t * out_ld + r;
  if (epi == EPI_BIAS) {
    v = fadd(v, bias[r]);
    if (!finite(v)) flag(err, ERRF_NONFINITE);
    *dst = v;
  } else if (epi == EPI_RESIDUAL) {
    const float y = fadd(*dst, v);
    if (!finite(y)) flag(err, ERRF_NONFINITE);
    *dst = y;
  } else {
    *dst = v;
  }
}

// grid: x = position-major tiles so consecutive CTAs share rows (L2 reuse)
__global__ void gemv_generic_kernel(DevMatrix m, DevActs a, int T, float* out, int out_ld, int epi,
                                    const float* bias, uint32_t* err) {
  pdl_enter();
  const int r = blockIdx.y * blockDim.x + threadIdx.x;
  const int t = blockIdx.x;
  if (r >= m.rows || t >= T) return;
  epilogue_store(dot_row(m, a, r, t), r, t, out, out_ld, epi, bias, err);
}

// ---- RoPE + KV store: apply_rope (det-model lib.rs:2011-2051) and
// KvCache::store (:883-913) ------------------------------------------------
// One thread per item, all items of a position in flight at once: a (q or k)
// rotation pair, or a K/V element past the rotated dims.  A k pair also
// stores its two rotated values and the V values at the same two dims in
// the cache, so no second pass (and no barrier) is needed.
__global__ void rope_store_kernel(float* q, float* k, const float* v, const int* pos0p, int n_head, int n_head_kv,
                                  int hd, int half, int pairing, const float* cos_t, const float* sin_t, float* kc,
                                  float* vc, int n_ctx, uint32_t* err) {
  pdl_enter();
  const int t = blockIdx.x;
  const int pos = *pos0p + t;
  float* qt = q + (size_t)t * n_head * hd;
  float* kt = k + (size_t)t * n_head_kv * hd;
  const float* vt = v + (size_t)t * n_head_kv * hd;
  const int nq = n_head * half, nk = n_head_kv * half, rest = hd - 2 * half;
  const int i = blockIdx.y * blockDim.x + threadIdx.x;
  if (i < nq + nk) {
    const bool isk = i >= nq;
    float* base = isk ? kt : qt;
    const int ii = isk ? i - nq : i;
    const int head = ii / half, j = ii - head * half;
    int a, b;
    if (pairing == 0) {
      a = head * hd + 2 * j;
      b = a + 1;
    } else {
      a = head * hd + j;
      b = a + half;
    }
    const float x0 = base[a], x1 = base[b];
    const float c = cos_t[(size_t)pos * half + j], sv = sin_t[(size_t)pos * half + j];
    const float y0 = fsub(fmul(x0, c), fmul(x1, sv));
    const float y1 = fadd(fmul(x0, sv), fmul(x1, c));
    if (!finite(y0) || !finite(y1) || !finite(x0) || !finite(x1)) flag(err, ERRF_NONFINITE);
    base[a] = y0;
    base[b] = y1;
    if (isk) {  // the KV store of these two dims (K after RoPE)
      const float va = vt[a], vb = vt[b];
      if (!finite(va) || !finite(vb)) flag(err, ERRF_NONFINITE);
      const size_t row = ((size_t)head * n_ctx + pos) * hd;
      kc[row + (a - head * hd)] = y0;
      kc[row + (b - head * hd)] = y1;
      vc[row + (a - head * hd)] = va;
      vc[row + (b - head * hd)] = vb;
    }
  } else if (i < nq + nk + n_head_kv * rest) {  // K / V dims past the rotated ones: stored as they are
    const int ii = i - nq - nk;
    const int kh = ii / rest, dd = 2 * half + (ii - kh * rest);
    const float kv = kt[kh * hd + dd], vv = vt[kh * hd + dd];
    if (!finite(kv) || !finite(vv)) flag(err, ERRF_NONFINITE);
    const size_t off = ((size_t)kh * n_ctx + pos) * hd + dd;
    kc[off] = kv;
    vc[off] = vv;
  }
}

// ---- attention for one (position, head): attention_one_head
// (det-model lib.rs:2300-2418) ---------------------------------------------
constexpr int ATT_THREADS = 256;

__global__ void attention_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                 const float* __restrict__ vc, const int* pos0p, int n_head, int n_head_kv, int hd,
                                 int n_ctx, float scale, float* __restrict__ out, float* __restrict__ scratch,
                                 int smem_scores, uint32_t* err) {
  pdl_enter();
  extern __shared__ float sm[];
  __shared__ float red[32];
  __shared__ float lanes[8];
  __shared__ float z_s;
  const int t = blockIdx.x, head = blockIdx.y;
  const int len = *pos0p + t + 1;
  const int kvh = head / (n_head / n_head_kv);
  const float* kb = kc + (size_t)kvh * n_ctx * hd;
  const float* vb = vc + (size_t)kvh * n_ctx * hd;
  float* o = out + ((size_t)t * n_head + head) * hd;
  if (len == 1) {  // score_len == 1 copies V (:2319-2322)
    for (int d = threadIdx.x; d < hd; d += blockDim.x) o[d] = vb[d];
    return;
  }
  float* qs = sm;  // hd floats
  float* sc = smem_scores ? sm + hd : scratch + ((size_t)t * n_head + head) * n_ctx;
  const float* qh = q + ((size_t)t * n_head + head) * hd;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    qs[d] = qh[d];
    if (!finite(qh[d])) flag(err, ERRF_NONFINITE);
  }
  __syncthreads();
  // scores: dot_f32_ref(q, k_j) * scale (:2335-2359)
  float lmax = -INFINITY;
  for (int j = threadIdx.x; j < len; j += blockDim.x) {
    const float* kj = kb + (size_t)j * hd;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (hd & 7) {  // head dims that are not a multiple of 8 (tiny fixtures)
      for (int i = 0; i < hd; i++) acc[i & 7] = fadd(acc[i & 7], fmul(qs[i], kj[i]));
    } else for (int i = 0; i < hd; i += 8) {
      const float4 k0 = *reinterpret_cast<const float4*>(kj + i);
      const float4 k1 = *reinterpret_cast<const float4*>(kj + i + 4);
      acc[0] = fadd(acc[0], fmul(qs[i + 0], k0.x));
      acc[1] = fadd(acc[1], fmul(qs[i + 1], k0.y));
      acc[2] = fadd(acc[2], fmul(qs[i + 2], k0.z));
      acc[3] = fadd(acc[3], fmul(qs[i + 3], k0.w));
      acc[4] = fadd(acc[4], fmul(qs[i + 4], k1.x));
      acc[5] = fadd(acc[5], fmul(qs[i + 5], k1.y));
      acc[6] = fadd(acc[6], fmul(qs[i + 6], k1.z));
      acc[7] = fadd(acc[7], fmul(qs[i + 7], k1.w));
    }
    const float s = fmul(finish8(acc), scale);
    if (!finite(s)) flag(err, ERRF_NONFINITE);
    sc[j] = s;
    lmax = fmaxf(lmax, s);
  }
  const float mx = block_max<ATT_THREADS>(lmax, red);
  // softmax_in_place (:2361-2388): e = expf(max(s - m, -88))
  for (int j = threadIdx.x; j < len; j += blockDim.x) {
    const float dlt = fsub(sc[j], mx);
    sc[j] = expf_det(dlt > -88.0f ? dlt : -88.0f);
  }
  __syncthreads();
  if (threadIdx.x < 8) {  // sum_f32_ref: 8 ordered lane chains
    float acc = 0.0f;
    for (int j = threadIdx.x; j < len; j += 8) acc = fadd(acc, sc[j]);
    lanes[threadIdx.x] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const float z = finish8(lanes);
    if (!finite(z) || z == 0.0f) flag(err, ERRF_NONFINITE);
    z_s = z;
  }
  __syncthreads();
  const float z = z_s;
  for (int j = threadIdx.x; j < len; j += blockDim.x) sc[j] = fdiv(sc[j], z);
  __syncthreads();
  // attention_weighted_value (:2390-2418): o[d] += p_j * v_j[d], j ascending
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.0f;
    for (int j = 0; j < len; j++) acc = fadd(acc, fmul(sc[j], vb[(size_t)j * hd + d]));
    if (!finite(acc)) flag(err, ERRF_NONFINITE);
    o[d] = acc;
  }
}

// ---- attention, GQA-grouped: one CTA per (position, KV head) computes every
// query head that shares the KV head, so each K/V row is staged in shared
// memory once for the whole group.  Same arithmetic as attention_kernel:
// scores by dot_f32_ref * scale, softmax with expf(max(s - m, -88)) and the
// 8-lane Z, then o[d] += p_j * v_j[d] for j ascending (one thread per chain).
constexpr int ATG_THREADS = 512;
constexpr int ATG_J = 64;  // K/V rows per staged chunk

__global__ void __launch_bounds__(ATG_THREADS)
    attention_gqa_kernel(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                         const int* pos0p, int n_head, int n_head_kv, int hd, int n_ctx, float scale,
                         float* __restrict__ out, float* __restrict__ scratch, int smem_scores, uint32_t* err) {
  pdl_enter();
  extern __shared__ __align__(16) float sm[];
  const int t = blockIdx.x, kvh = blockIdx.y, tid = threadIdx.x;
  const int gsz = n_head / n_head_kv, h0 = kvh * gsz;
  const int len = *pos0p + t + 1;
  const float* kb = kc + (size_t)kvh * n_ctx * hd;
  const float* vb = vc + (size_t)kvh * n_ctx * hd;
  float* ob = out + ((size_t)t * n_head + h0) * hd;
  if (len == 1) {  // score_len == 1 copies V (:2319-2322)
    for (int i = tid; i < gsz * hd; i += ATG_THREADS) ob[i] = vb[i % hd];
    return;
  }
  const bool vec = (hd & 7) == 0;
  const int ks = vec ? hd + 4 : hd + 1;  // padded K row stride (floats)
  float* qs = sm;                         // [gsz][hd]
  float* kvs = qs + gsz * hd;             // [ATG_J][ks]  (K chunk, then V chunk)
  float* sc = smem_scores ? kvs + ATG_J * ks : scratch + ((size_t)t * n_head + h0) * n_ctx;  // [gsz][n_ctx]
  const float* qg = q + ((size_t)t * n_head + h0) * hd;
  for (int i = tid; i < gsz * hd; i += ATG_THREADS) {
    const float v = qg[i];
    if (!finite(v)) flag(err, ERRF_NONFINITE);
    qs[i] = v;
  }
  // ---- scores (:2335-2359)
  for (int jc = 0; jc < len; jc += ATG_J) {
    const int cnt = min(ATG_J, len - jc);
    __syncthreads();  // previous chunk consumed
    for (int i = tid; i < cnt * hd; i += ATG_THREADS) {
      const int jj = i / hd, d = i - jj * hd;
      kvs[jj * ks + d] = kb[(size_t)(jc + jj) * hd + d];
    }
    __syncthreads();
    for (int pr = tid; pr < gsz * cnt; pr += ATG_THREADS) {
      const int h = pr / cnt, jj = pr - h * cnt;
      const float* qh = qs + h * hd;
      const float* kr = kvs + jj * ks;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (vec) {
        for (int i = 0; i < hd; i += 8) {
          const float4 k0 = *reinterpret_cast<const float4*>(kr + i);
          const float4 k1 = *reinterpret_cast<const float4*>(kr + i + 4);
          acc[0] = fadd(acc[0], fmul(qh[i + 0], k0.x));
          acc[1] = fadd(acc[1], fmul(qh[i + 1], k0.y));
          acc[2] = fadd(acc[2], fmul(qh[i + 2], k0.z));
          acc[3] = fadd(acc[3], fmul(qh[i + 3], k0.w));
          acc[4] = fadd(acc[4], fmul(qh[i + 4], k1.x));
          acc[5] = fadd(acc[5], fmul(qh[i + 5], k1.y));
          acc[6] = fadd(acc[6], fmul(qh[i + 6], k1.z));
          acc[7] = fadd(acc[7], fmul(qh[i + 7], k1.w));
        }
      } else {
        for (int i = 0; i < hd; i++) acc[i & 7] = fadd(acc[i & 7], fmul(qh[i], kr[i]));
      }
      const float s = fmul(finish8(acc), scale);
      if (!finite(s)) flag(err, ERRF_NONFINITE);
      sc[(size_t)h * n_ctx + jc + jj] = s;
    }
  }
  __syncthreads();
  // ---- softmax per head (:2361-2388): one warp per head
  const int warp = tid >> 5, lane = tid & 31;
  for (int h = warp; h < gsz; h += ATG_THREADS / 32) {
    float* s = sc + (size_t)h * n_ctx;
    float m = -INFINITY;
    for (int j = lane; j < len; j += 32) m = fmaxf(m, s[j]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    for (int j = lane; j < len; j += 32) {
      const float dlt = fsub(s[j], m);
      s[j] = expf_det(dlt > -88.0f ? dlt : -88.0f);
    }
    __syncwarp();
    float acc = 0.0f;  // sum_f32_ref: lanes 0..7 run the ordered lane chains
    if (lane < 8) {
      int j = lane;
      for (; j + 56 < len; j += 64) {
        float e[8];
#pragma unroll
        for (int k = 0; k < 8; k++) e[k] = s[j + 8 * k];
#pragma unroll
        for (int k = 0; k < 8; k++) acc = fadd(acc, e[k]);
      }
      for (; j < len; j += 8) acc = fadd(acc, s[j]);
    }
    float a[8];
#pragma unroll
    for (int k = 0; k < 8; k++) a[k] = __shfl_sync(0xffffffffu, acc, k);
    const float z = finish8(a);
    if (lane == 0 && (!finite(z) || z == 0.0f)) flag(err, ERRF_NONFINITE);
    for (int j = lane; j < len; j += 32) s[j] = fdiv(s[j], z);
  }
  // ---- o[d] += p_j * v_j[d], j ascending (:2390-2418): one thread per chain
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  const int nch = gsz * hd;
  for (int jc = 0; jc < len; jc += ATG_J) {
    const int cnt = min(ATG_J, len - jc);
    __syncthreads();  // scores final / previous V chunk consumed
    for (int i = tid; i < cnt * hd; i += ATG_THREADS) kvs[i] = vb[(size_t)jc * hd + i];
    __syncthreads();
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int idx = tid + c * ATG_THREADS;
      if (idx < nch) {
        const int h = idx / hd, d = idx - h * hd;
        const float* p = sc + (size_t)h * n_ctx + jc;
        float acc = o[c];
        for (int jj = 0; jj < cnt; jj++) acc = fadd(acc, fmul(p[jj], kvs[jj * hd + d]));
        o[c] = acc;
      }
    }
  }
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const int idx = tid + c * ATG_THREADS;
    if (idx < nch) {
      if (!finite(o[c])) flag(err, ERRF_NONFINITE);
      ob[idx] = o[c];
    }
  }
}

// ---- swiglu (det-model lib.rs:2420-2434) ---------------------------------
__global__ void swiglu_kernel(const float* g, const float* u, float* out, long long n, uint32_t* err) {
  pdl_enter();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float gv = g[i], uv = u[i];
  const float y = fmul(silu_det(gv), uv);
  if (!finite(y) || !finite(gv) || !finite(uv)) flag(err, ERRF_NONFINITE);
  out[i] = y;
}

// ---- logits -> CDF (det-coder cdf.rs:138-245) ----------------------------
constexpr int CDF_THREADS = 512;
constexpr int CDF_CHUNK = 4096;  // floats per shared-memory chunk (multiple of 8)

// per row: max, e_i = expf(max(l_i - m, -88)), Z = sum_f32_ref(e)
__global__ void cdf_prepare_kernel(const float* __restrict__ logits, int V, const uint32_t* rows,
                                   float* __restrict__ e, float* __restrict__ z, uint32_t* err) {
  pdl_enter();
  __shared__ float red[32];
  __shared__ float lanes[8];
  const uint32_t row = rows[blockIdx.x];
  const float* l = logits + (size_t)row * V;
  float* er = e + (size_t)row * V;
  float lmax = -INFINITY;
  bool bad = false;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = l[i];
    if (!finite(v)) bad = true;
    lmax = fmaxf(lmax, v);
  }
  if (bad) flag(err, ERRF_CDF_NONFINITE);
  const float mx = block_max<CDF_THREADS>(lmax, red);
  // Double-buffered through shared memory: while lanes 0..7 of warp 0 run
  // the eight ordered Z chains (sum_f32_ref) over chunk c-1, warps 1..15
  // compute e_i = expf(max(l_i - m, -88)) for chunk c (and store it for the
  // frequency pass).  CDF_CHUNK is a multiple of 8, so chunk boundaries keep
  // every lane's elements in order.
  __shared__ float ebuf[2][CDF_CHUNK];
  const int nchunk = (V + CDF_CHUNK - 1) / CDF_CHUNK;
  float acc = 0.0f;
  for (int c = 0; c <= nchunk; c++) {
    if (threadIdx.x >= 32 && c < nchunk) {
      const int base = c * CDF_CHUNK, cnt = min(CDF_CHUNK, V - base);
      for (int i = threadIdx.x - 32; i < cnt; i += blockDim.x - 32) {
        const float d = fsub(l[base + i], mx);
        const float e = expf_det(d > -88.0f ? d : -88.0f);
        ebuf[c & 1][i] = e;
        er[base + i] = e;
      }
    } else if (threadIdx.x < 8 && c > 0) {
      const int base = (c - 1) * CDF_CHUNK, cnt = min(CDF_CHUNK, V - base);
      const float* eb = ebuf[(c - 1) & 1];
      int i = threadIdx.x;
      for (; i + 56 < cnt; i += 64) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = eb[i + 8 * k];
#pragma unroll
        for (int k = 0; k < 8; k++) acc = fadd(acc, v[k]);
      }
      for (; i < cnt; i += 8) acc = fadd(acc, eb[i]);
    }
    __syncthreads();
  }
  if (threadIdx.x < 8) lanes[threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.x == 0) z[row] = finish8(lanes);
}

DI uint32_t freq_of(float e, float z) {  // ((e / Z) * 2^24) as u32 + 1
  return __float2uint_rz(fmul(fdiv(e, z), 16777216.0f)) + 1u;
}

// one CTA per query: (cum, freq, total) of symbols[i] under row rows[i]
__global__ void cdf_ranges_kernel(const float* __restrict__ e, const float* __restrict__ z, int V, int tail,
                                  const uint32_t* rows, const uint32_t* symbols, uint64_t* out3, uint32_t* err) {
  pdl_enter();
  __shared__ unsigned long long red[32];
  const uint32_t row = rows[blockIdx.x];
  const uint32_t sym = symbols[blockIdx.x];
  const float* er = e + (size_t)row * V;
  const float zz = z[row];
  unsigned long long tot = 0, cum = 0;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const uint32_t f = freq_of(er[i], zz);
    tot += f;
    if ((uint32_t)i < sym) cum += f;
  }
  tot = block_sum_u64<CDF_THREADS>(tot, red);
  cum = block_sum_u64<CDF_THREADS>(cum, red);
  if (threadIdx.x == 0) {
    uint64_t freq;
    if (sym < (uint32_t)V) {
      freq = freq_of(er[sym], zz);
    } else {
      cum = tot + (sym - (uint32_t)V);
      freq = 1;
    }
    const uint64_t total = tot + (uint64_t)tail;
    if (total >= (1ull << 31)) flag(err, ERRF_CDF_TOTAL);
    out3[3 * blockIdx.x + 0] = cum;
    out3[3 * blockIdx.x + 1] = freq;
    out3[3 * blockIdx.x + 2] = total;
  }
}

// decoder: symbol with cum <= value < cum + freq (DecoderDistribution::
// symbol_range, cdf.rs:392-425), by block-wide exclusive scans of the
// (exact integer) frequencies.  out4 = {symbol, cum, freq, total}
__global__ void decoder_lookup_kernel(const float* __restrict__ e, const float* __restrict__ z, int V, int tail,
                                      uint32_t row, const uint64_t* value_p, uint64_t* out4, uint32_t* err) {
  pdl_enter();
  __shared__ unsigned long long wsum[32];
  __shared__ unsigned long long base_s;
  __shared__ int found;
  const float* er = e + (size_t)row * V;
  const float zz = z[row];
  const unsigned long long value = *value_p;
  if (threadIdx.x == 0) {
    base_s = 0;
    found = 0;
  }
  __syncthreads();
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  for (int start = 0; start < V; start += blockDim.x) {
    const int i = start + threadIdx.x;
    const unsigned long long f = i < V ? freq_of(er[i], zz) : 0ull;
    unsigned long long inc = f;
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long n = __shfl_up_sync(0xffffffffu, inc, o);
      if (l >= o) inc += n;
    }
    if (l == 31) wsum[w] = inc;
    __syncthreads();
    if (w == 0) {
      unsigned long long s = l < (int)(blockDim.x >> 5) ? wsum[l] : 0ull;
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long n = __shfl_up_sync(0xffffffffu, s, o);
        if (l >= o) s += n;
      }
      wsum[l] = s;  // inclusive warp prefix
    }
    __syncthreads();
    const unsigned long long base = base_s;
    const unsigned long long excl = base + (w ? wsum[w - 1] : 0ull) + inc - f;
    if (i < V && excl <= value && value < excl + f) {
      out4[0] = (uint64_t)i;
      out4[1] = excl;
      out4[2] = f;
      found = 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) base_s = base + wsum[(blockDim.x >> 5) - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const unsigned long long tot = base_s;
    const unsigned long long total = tot + (unsigned long long)tail;
    out4[3] = total;
    if (!found) {
      const unsigned long long off = value - tot;
      if (value >= tot && off < (unsigned long long)tail) {
        out4[0] = (uint64_t)V + off;
        out4[1] = value;
        out4[2] = 1;
      } else {
        flag(err, ERRF_DECODE);
      }
    }
  }
}

// ---- the decompress loop on the device -------------------------------------
// One decoded symbol per launch (one CTA of RC_THREADS): the symbol range of
// the next symbol under logits row 0 (or the uniform CDF while the window is
// empty), the range decoder's decode_freq / advance with its renormalisation
// (det-coder range.rs:110-178), the symbol's byte count, and the next
// one-position forward's token and position in device memory.  A launch
// after the loop has stopped (done, window full, error, batch full) changes
// nothing, and neither does the forward that follows it: that forward then
// recomputes the previous one (same token, same position) bit for bit.
constexpr int RC_THREADS = 1024;
constexpr unsigned long long RC_TOP = 1ull << 56, RC_BOTTOM = 1ull << 48;

// normalize_step (range.rs:169-178)
DI bool rc_normalize_step(unsigned long long low, unsigned long long& range) {
  if ((low ^ (low + range)) < RC_TOP) return true;
  if (range < RC_BOTTOM) {
    range = (0ull - low) & (RC_BOTTOM - 1);
    return true;
  }
  return false;
}

__global__ void __launch_bounds__(RC_THREADS) rc_step_kernel(RcState* __restrict__ S, const float* __restrict__ e,
                                                             const float* __restrict__ z, int V,
                                                             const uint8_t* __restrict__ payload,
                                                             const uint16_t* __restrict__ piece_len,
                                                             uint32_t* __restrict__ tok, int* __restrict__ posp,
                                                             uint32_t* err) {
  pdl_enter();
  __shared__ unsigned long long wsum[32];
  __shared__ unsigned long long sh_total, sh_value, sh_r, sh_base, sh_sym, sh_cum, sh_freq;
  __shared__ int sh_run, sh_uniform, sh_found, sh_fail;
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  const int tail = (int)S->tail;
  if (tid == 0) {
    sh_run = S->status == RC_RUNNING && S->count < S->max_count;
    sh_uniform = S->clen == 0;
    sh_found = 0;
    sh_fail = 0;
    sh_base = 0;
  }
  __syncthreads();
  if (!sh_run) return;
  const float zz = sh_uniform ? 1.0f : z[0];
  // total of the distribution (symbols_total for the uniform CDF)
  unsigned long long tot = 0;
  if (!sh_uniform)
    for (int i = tid; i < V; i += RC_THREADS) tot += freq_of(e[i], zz);
  tot = block_sum_u64<RC_THREADS>(tot, wsum);
  if (tid == 0) {
    const unsigned long long total = (unsigned long long)V + (unsigned long long)tail;
    sh_total = sh_uniform ? total : tot + (unsigned long long)tail;
    // decode_freq (range.rs:110-128)
    const unsigned long long t = sh_total;
    unsigned long long r = 0, value = 0;
    int bad = 0;
    if (!sh_uniform && t >= (1ull << 31)) {
      bad = DET_ERR_CDF_TOTAL_TOO_LARGE;
    } else if (t == 0 || t >= (1ull << 31)) {
      bad = DET_ERR_RANGE_INVALID_FREQUENCY;
    } else {
      r = S->range / t;
      if (r == 0) bad = DET_ERR_RANGE_INVALID_FREQUENCY;
      else {
        value = (S->code - S->low) / r;
        if (value >= t) bad = DET_ERR_RANGE_INVALID_FREQUENCY;
      }
    }
    if (bad) {
      S->status = RC_FAILED;
      S->error = (uint32_t)bad;
      sh_fail = 1;
    }
    sh_value = value;
    sh_r = r;
    if (sh_uniform) {  // uniform_symbol_range (cdf.rs:247-253)
      sh_sym = value;
      sh_cum = value;
      sh_freq = 1;
      sh_found = 1;
    }
  }
  __syncthreads();
  if (sh_fail) return;
  const unsigned long long value = sh_value;
  if (!sh_uniform) {
    // DecoderDistribution::symbol_range (cdf.rs:392-425): exclusive scans of
    // the exact integer frequencies
    for (int start = 0; start < V; start += RC_THREADS) {
      const int i = start + tid;
      const unsigned long long f = i < V ? freq_of(e[i], zz) : 0ull;
      unsigned long long inc = f;
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long n = __shfl_up_sync(0xffffffffu, inc, o);
        if (l >= o) inc += n;
      }
      __syncthreads();
      if (l == 31) wsum[w] = inc;
      __syncthreads();
      if (w == 0) {
        unsigned long long s = wsum[l];
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned long long n = __shfl_up_sync(0xffffffffu, s, o);
          if (l >= o) s += n;
        }
        wsum[l] = s;
      }
      __syncthreads();
      const unsigned long long base = sh_base;
      const unsigned long long excl = base + (w ? wsum[w - 1] : 0ull) + inc - f;
      if (i < V && excl <= value && value < excl + f) {
        sh_sym = (unsigned long long)i;
        sh_cum = excl;
        sh_freq = f;
        sh_found = 1;
      }
      __syncthreads();
      if (tid == 0) sh_base = base + wsum[31];
      __syncthreads();
    }
  }
  if (tid != 0) return;
  unsigned long long sym = sh_sym, cum = sh_cum, freq = sh_freq;
  const unsigned long long total = sh_total;
  if (!sh_found) {  // the byte-escape tail
    const unsigned long long tot_f = sh_base;
    if (value >= tot_f && value - tot_f < (unsigned long long)tail) {
      sym = (unsigned long long)V + (value - tot_f);
      cum = value;
      freq = 1;
    } else {
      flag(err, ERRF_DECODE);
      S->status = RC_FAILED;
      S->error = DET_ERR_DECODE;
      return;
    }
  }
  // advance (range.rs:130-148) with validate (:180-186) and renorm
  const unsigned long long end = cum + freq;
  if (end < cum || freq == 0 || total == 0 || total >= (1ull << 31) || end > total) {
    S->status = RC_FAILED;
    S->error = DET_ERR_RANGE_INVALID_FREQUENCY;
    return;
  }
  unsigned long long low = S->low, code = S->code, range = sh_r, pos = S->pos;
  low += range * cum;
  range *= freq;
  while (rc_normalize_step(low, range)) {
    if (pos >= S->len) {
      S->status = RC_FAILED;
      S->error = DET_ERR_RANGE_UNEXPECTED_EOF;
      return;
    }
    code = (code << 8) | (unsigned long long)payload[pos++];
    low <<= 8;
    range <<= 8;
  }
  S->low = low;
  S->code = code;
  S->range = range;
  S->pos = pos;
  // the symbol's bytes; a symbol without bytes is an error (det-cli
  // main.rs:614-616)
  const unsigned plen = piece_len[sym];
  S->syms[S->count++] = (uint32_t)sym;
  if (plen == 0) {
    S->status = RC_FAILED;
    S->error = DET_ERR_TOKENIZER;
    return;
  }
  S->bytes += plen;
  const bool token = !(tail && sym >= (unsigned long long)V);
  if (token) {
    if (S->clen >= S->n_ctx) {
      S->status = RC_FAILED;
      S->error = DET_ERR_WINDOW;
      return;
    }
    tok[0] = (uint32_t)sym;
    *posp = (int)S->clen;
    S->clen++;
  }
  if (S->bytes >= S->orig_len) S->status = RC_DONE;
  else if (token && S->clen >= S->n_ctx) S->status = RC_WINDOW_FULL;
}

__global__ void expf_kernel(const float* x, float* y, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = expf_det(x[i]);
}

}  // namespace

// One warp runs n pairs of dependent rounded adds between two clock reads:
// the cycles per add are the latency floor of every ordered f32 chain.
__global__ void add_chain_kernel(const float* __restrict__ x, float* __restrict__ out, long long* cycles, int n) {
  float s = 0.0f;
  const float a = x[threadIdx.x], b = x[threadIdx.x + 32];
  const long long t0 = clock64();
#pragma unroll 16
  for (int i = 0; i < n; i++) {
    s = fadd(s, a);
    s = fadd(s, b);
  }
  const long long t1 = clock64();
  out[threadIdx.x] = s;
  if (threadIdx.x == 0) *cycles = t1 - t0;
}

cudaError_t launch_add_chain(const float* x, float* out, long long* cycles, int n) {
  add_chain_kernel<<<1, 32>>>(x, out, cycles, n);
  return cudaGetLastError();
}

cudaError_t launch_expf(cudaStream_t st, const float* x, float* y, long long n) {
  expf_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, y, n);
  return cudaGetLastError();
}

// ---- launchers ---------------------------------------------------------------
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("DETGPU_NO_PDL");
    return !(e && *e && *e != '0');
  }();
  return on;
}

static inline cudaError_t post(const Launch& L) {
  if (L.launches) ++*L.launches;
  return cudaGetLastError();
}

cudaError_t launch_rope_table(const Launch& L, float* cos_t, float* sin_t, int positions, int half, int rope_dim,
                              float rope_base) {
  const long long n = (long long)positions * half;
  {
    const cudaError_t e_ = launch_k(L, rope_table_kernel, (unsigned)((n + 255) / 256), 256, 0, cos_t, sin_t,
        positions, half, rope_dim, rope_base);
    if (e_ != cudaSuccess) return e_;
  }
  return post(L);
}

cudaError_t launch_embed(const Launch& L, const DevMatrix& m, const uint32_t* tokens, int T, float* x) {
  {
    const cudaError_t e_ = launch_k(L, embed_kernel, T, 256, 0, m, tokens, T, x, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  return post(L);
}

int device_sms() {
  static const int sms = [] {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        n <= 0)
      return 148;
    return n;
  }();
  return sms;
}

cudaError_t raise_smem_cap(const void* kern, size_t bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> caps;
  std::lock_guard<std::mutex> lock(mu);
  size_t& cap = caps[{kern, dev}];
  if (cap >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) cap = bytes;
  return e;
}

cudaError_t launch_rmsnorm(const Launch& L, const float* x, const float* w, int n, float eps, int T, float* h,
                           float* qd, int8_t* qq) {
  const size_t smem = n <= RMS_MAX_SMEM ? 2 * (size_t)n * sizeof(float) : 0;
  if (cudaError_t e = raise_smem_cap((const void*)rmsnorm_kernel, smem)) return e;
  if (n % 32) qd = nullptr, qq = nullptr;
  // a short chunk is one or a few CTAs: more warps share the quantisation
  const int threads = T <= 16 ? 1024 : 256;
  {
    const cudaError_t e_ = launch_k(L, rmsnorm_kernel, T, threads, smem, x, w, n, eps, h, qd, qq, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  return post(L);
}

cudaError_t launch_quant_q8a(const Launch& L, const float* x, int K, int T, float* qd, int8_t* qq) {
  const int nb = T * (K / 32);
  {
    const cudaError_t e_ = launch_k(L, quant_q8a_kernel, (nb + 7) / 8, 256, 0, x, nb, K / 32, qd, qq, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  return post(L);
}

cudaError_t launch_quant_q8k(const Launch& L, const float* x, int K, int T, float* qd, int8_t* qq, uint8_t* qp) {
  const int nb = T * (K / 256);
  {
    const cudaError_t e_ = launch_k(L, quant_q8k_kernel, (nb + 7) / 8, 256, 0, x, nb, K / 256, qd, qq, qp, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  return post(L);
}

cudaError_t launch_gemv_fast(const Launch& L, const DevMatrix& m, const DevActs& a, int T, float* out, int out_ld,
                             int epi, const float* bias, bool* handled);

cudaError_t launch_gemv(const Launch& L, const DevMatrix& m, const DevActs& a, int T, float* out, int out_ld,
                        int epi, const float* bias) {
  bool handled = false;
  cudaError_t e = launch_gemv_fast(L, m, a, T, out, out_ld, epi, bias, &handled);
  if (handled || e != cudaSuccess) return e;
  if (m.type == GT_Q4_K && T > 16) return launch_gemm_q4k(L, m, a, T, out, out_ld, epi, bias);
  if (m.type == GT_Q6_K && T > 16) return launch_gemm_q6k_tc(L, m, a, T, out, out_ld, epi, bias);
  if ((m.type == GT_Q4_K || m.type == GT_Q6_K) && T == 1 && kq_decode_supported(m))
    return launch_gemv_kq_decode(L, m, a, out, epi, bias);
  dim3 grid(T, (m.rows + 127) / 128);
  {
    const cudaError_t e_ = launch_k(L, gemv_generic_kernel, grid, 128, 0, m, a, T, out, out_ld, epi, bias, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  return post(L);
}

cudaError_t launch_rope_store(const Launch& L, float* q, float* k, const float* v, int T, const int* pos0, int n_head,
                              int n_head_kv, int head_dim, int rope_dim, int pairing, const float* cos_t,
                              const float* sin_t, float* kc, float* vc, int n_ctx) {
  {
    const int items = (n_head + n_head_kv) * (rope_dim / 2) + n_head_kv * (head_dim - rope_dim);
    const cudaError_t e_ = launch_k(L, rope_store_kernel, dim3(T, (items + 255) / 256), 256, 0, q, k, v, pos0,
                                    n_head, n_head_kv, head_dim, rope_dim / 2, pairing, cos_t, sin_t, kc, vc, n_ctx,
                                    L.err);
    if (e_ != cudaSuccess) return e_;
  }
  return post(L);
}

namespace {
// shared-memory plan of attention_gqa_kernel: returns false when the group
// is too wide for it (more than 4 chains per thread)
bool gqa_plan(int n_head, int n_head_kv, int hd, int n_ctx, size_t* smem, int* smem_scores) {
  const int gsz = n_head / n_head_kv;
  if ((size_t)gsz * hd > 4 * (size_t)ATG_THREADS) return false;
  const int ks = (hd & 7) == 0 ? hd + 4 : hd + 1;
  const size_t base = ((size_t)gsz * hd + (size_t)ATG_J * ks) * sizeof(float);
  const size_t with_scores = base + (size_t)gsz * n_ctx * sizeof(float);
  *smem_scores = with_scores <= 200 * 1024 ? 1 : 0;
  *smem = *smem_scores ? with_scores : base;
  return true;
}
}  // namespace

size_t attention_scratch_floats(int T, int n_head, int n_head_kv, int hd, int n_ctx) {
  if (attention_tiled_supported(n_head, n_head_kv, hd)) return attention_tiled_scratch_floats(T, n_head, n_ctx);
  size_t smem;
  int in_smem;
  if (gqa_plan(n_head, n_head_kv, hd, n_ctx, &smem, &in_smem)) return in_smem ? 0 : (size_t)T * n_head * n_ctx;
  return (size_t)(hd + n_ctx) * sizeof(float) <= 160 * 1024 ? 0 : (size_t)T * n_head * n_ctx;
}

cudaError_t launch_attention(const Launch& L, const float* q, const float* kc, const float* vc, int T, const int* pos0,
                             int n_head, int n_head_kv, int head_dim, int n_ctx, float scale, float* out,
                             float* score_scratch) {
  if (attention_tiled_supported(n_head, n_head_kv, head_dim))
    return launch_attention_tiled(L, q, kc, vc, T, pos0, n_head, n_head_kv, head_dim, n_ctx, scale, out,
                                  score_scratch);
  size_t gsmem;
  int gscores;
  if (gqa_plan(n_head, n_head_kv, head_dim, n_ctx, &gsmem, &gscores)) {
    if (cudaError_t e = raise_smem_cap((const void*)attention_gqa_kernel, gsmem)) return e;
    dim3 grid(T, n_head_kv);
    {
      const cudaError_t e_ = launch_k(L, attention_gqa_kernel, grid, ATG_THREADS, gsmem, q, kc, vc, pos0, n_head,
          n_head_kv, head_dim, n_ctx, scale, out, score_scratch, gscores, L.err);
      if (e_ != cudaSuccess) return e_;
    }
    return post(L);
  }
  const size_t need = (size_t)(head_dim + n_ctx) * sizeof(float);
  const int smem_scores = need <= 160 * 1024 ? 1 : 0;
  const size_t smem = smem_scores ? need : head_dim * sizeof(float);
  if (cudaError_t e = raise_smem_cap((const void*)attention_kernel, smem)) return e;
  dim3 grid(T, n_head);
  {
    const cudaError_t e_ = launch_k(L, attention_kernel, grid, ATT_THREADS, smem, q, kc, vc, pos0, n_head, n_head_kv,
        head_dim, n_ctx, scale, out, score_scratch, smem_scores, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  return post(L);
}

cudaError_t launch_swiglu(const Launch& L, const float* g, const float* u, float* out, int n, int T, float* qd,
                          int8_t* qq) {
  if (qq && n % 32 == 0) {
    const int nb = T * (n / 32);
    {
      const cudaError_t e_ = launch_k(L, swiglu_q8a_kernel, (nb + 7) / 8, 256, 0, g, u, out, nb, n / 32, qd, qq, L.err);
      if (e_ != cudaSuccess) return e_;
    }
    return post(L);
  }
  const long long tot = (long long)n * T;
  {
    const cudaError_t e_ = launch_k(L, swiglu_kernel, (unsigned)((tot + 255) / 256), 256, 0, g, u, out, tot, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  return post(L);
}

cudaError_t launch_cdf_prepare(const Launch& L, const float* logits, int V, const uint32_t* rows, int nrows,
                               float* e, float* z) {
  {
    const cudaError_t e_ = launch_k(L, cdf_prepare_kernel, nrows, CDF_THREADS, 0, logits, V, rows, e, z, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  return post(L);
}

cudaError_t launch_cdf_ranges(const Launch& L, const float* e, const float* z, int V, int tail,
                              const uint32_t* rows, const uint32_t* symbols, int n, uint64_t* out3) {
  {
    const cudaError_t e_ = launch_k(L, cdf_ranges_kernel, n, CDF_THREADS, 0, e, z, V, tail, rows, symbols, out3, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  return post(L);
}

cudaError_t launch_rc_step(const Launch& L, RcState* S, const float* e, const float* z, int V, const uint8_t* payload,
                           const uint16_t* piece_len, uint32_t* tok, int* pos) {
  {
    const cudaError_t e_ =
        launch_k(L, rc_step_kernel, 1, RC_THREADS, 0, S, e, z, V, payload, piece_len, tok, pos, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  return post(L);
}

cudaError_t launch_decoder_lookup(const Launch& L, const float* e, const float* z, int V, int tail, uint32_t row,
                                  const uint64_t* value, uint64_t* out4) {
  {
    const cudaError_t e_ = launch_k(L, decoder_lookup_kernel, 1, 1024, 0, e, z, V, tail, row, value, out4, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  return post(L);
}

}  // namespace det
