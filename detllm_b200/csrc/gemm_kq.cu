// gemm_kq.cu -- Q4_K x Q8A chunk GEMM (teacher-forced chunks of T > 16).
//
// Reference: dot_q4_k_q8a (crates/det-quant/src/lib.rs:281-315).  There is
// no integer shortcut: every row is ONE f32 chain over all K elements,
//   sum += ((d * sc) * q - (dmin * m)) * (a.d * a.q)
// with each product and difference separately rounded.  The weight factor
// depends only on (row, element) and the activation factor only on
// (position, element), so a CTA dequantises a 64-row x 32-element weight
// tile and a 64-position x 32-element activation tile into shared memory
// with exactly the reference's operations, once per stage, and the rest is
// an ordered f32 GEMM: each thread owns 4 rows x 4 positions = 16 chains
// and advances them element by element in the reference's order.  The
// products run packed (mul.rn.f32x2); the adds are fma(p, one, acc) with
// `one` == 1.0 a kernel argument -- exact, and not contractible with the
// multiply (a packed add fed by a packed multiply is contracted by the code
// generator).
#include <cuda_runtime.h>

#include "dev_math.cuh"
#include "internal.h"

namespace det {
namespace {

DI unsigned long long pk2(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
DI float2 up2(unsigned long long r) {
  float2 o;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(o.x), "=f"(o.y) : "l"(r));
  return o;
}
// acc + w * (a0, a1): two separately rounded products, two exact adds
DI float2 madd2(float w, float a0, float a1, float one, float2 acc) {
  unsigned long long p, r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(p) : "l"(pk2(w, w)), "l"(pk2(a0, a1)));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(p), "l"(pk2(one, one)), "l"(pk2(acc.x, acc.y)));
  return up2(r);
}

constexpr int KQ_ROWS = 64;
constexpr int KQ_POS = 64;  // one Q8A group
constexpr int KQ_E = 32;    // elements per stage: one Q4_K sub-block = one Q8A block
constexpr int KQ_THREADS = 256;
constexpr int KQ_WS = KQ_ROWS + 4;  // padded tile rows (floats)

__global__ void __launch_bounds__(KQ_THREADS) gemm_q4k_kernel(const uint8_t* __restrict__ W, int rows, int nbs,
                                                              const int8_t* __restrict__ aq,
                                                              const float* __restrict__ ad, int T,
                                                              float* __restrict__ out, int out_ld, int epi,
                                                              const float* __restrict__ bias, float one,
                                                              uint32_t* err) {
  pdl_enter();
  __shared__ __align__(16) float ws[KQ_E][KQ_WS];  // dequantised weights [element][row]
  __shared__ __align__(16) float as[KQ_E][KQ_WS];  // dequantised activations [element][position]
  const int tid = threadIdx.x;
  const int r0 = blockIdx.x * KQ_ROWS, p0 = blockIdx.y * KQ_POS;
  const int nbk = nbs * 8;  // Q8A blocks per position
  // staging: row / position tid >> 2, elements 8 * (tid & 3) .. + 8
  const int sr = tid >> 2, se = 8 * (tid & 3);
  const bool row_ok = r0 + sr < rows;
  const int t_st = p0 + sr;
  const bool pos_ok = t_st < T;
  const uint8_t* wrow = W + (size_t)(row_ok ? r0 + sr : 0) * nbs * 144;
  // compute: rows rt * 4 .. + 3, positions pt * 4 .. + 3
  const int rt = tid >> 4, pt = tid & 15;
  float2 acc[4][2];
#pragma unroll
  for (int r = 0; r < 4; r++) acc[r][0] = acc[r][1] = make_float2(0.f, 0.f);

  for (int b = 0; b < nbs; b++) {
    const uint8_t* blk = wrow + (size_t)b * 144;
    const float d = row_ok ? f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8))) : 0.0f;
    const float dmin = row_ok ? f16_bits_to_f32((uint16_t)(blk[2] | (blk[3] << 8))) : 0.0f;
    for (int sub = 0; sub < 8; sub++) {
      __syncthreads();  // previous stage consumed
      // weights: w = (d * sc) * q - dmin * m
      if (row_ok) {
        int sc, mn;
        q4k_scale_min(blk + 4, sub, sc, mn);
        const float dsc = fmul(d, (float)sc), dmn = fmul(dmin, (float)mn);
        const uint2 qv = *reinterpret_cast<const uint2*>(blk + 16 + (sub >> 1) * 32 + se);
        const int sh = (sub & 1) * 4;
#pragma unroll
        for (int k = 0; k < 8; k++) {
          const uint32_t word = k < 4 ? qv.x : qv.y;
          const int q = (int)((word >> (8 * (k & 3) + sh)) & 0x0fu);
          ws[se + k][sr] = fsub(fmul(dsc, (float)q), dmn);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 8; k++) ws[se + k][sr] = 0.0f;
      }
      // activations: a.d * a.q (Q8A block b * 8 + sub of position t_st)
      if (pos_ok) {
        const int kb = b * 8 + sub;
        const float a_d = ad[q8a_dslot(nbk, t_st, kb)];
        const uint2 qa = *reinterpret_cast<const uint2*>(aq + q8a_slot(nbk, t_st, kb) * 32 + (se ^ q8a_swz(t_st)));
#pragma unroll
        for (int k = 0; k < 8; k++) {
          const uint32_t word = k < 4 ? qa.x : qa.y;
          as[se + k][sr] = fmul(a_d, (float)(int8_t)(word >> (8 * (k & 3))));
        }
      } else {
#pragma unroll
        for (int k = 0; k < 8; k++) as[se + k][sr] = 0.0f;
      }
      __syncthreads();
#pragma unroll 8
      for (int e = 0; e < KQ_E; e++) {
        const float4 w4 = *reinterpret_cast<const float4*>(&ws[e][rt * 4]);
        const float4 a4 = *reinterpret_cast<const float4*>(&as[e][pt * 4]);
        const float wr[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int r = 0; r < 4; r++) {
          acc[r][0] = madd2(wr[r], a4.x, a4.y, one, acc[r][0]);
          acc[r][1] = madd2(wr[r], a4.z, a4.w, one, acc[r][1]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const int row = r0 + rt * 4 + r;
    if (row >= rows) continue;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int t = p0 + pt * 4 + c;
      if (t >= T) continue;
      float v = (c & 1) ? acc[r][c >> 1].y : acc[r][c >> 1].x;
      if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
      float* dst = out + (size_t)t * out_ld + row;
      if (epi == EPI_BIAS) {
        v = fadd(v, bias[row]);
        if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
      } else if (epi == EPI_RESIDUAL) {
        v = fadd(*dst, v);
        if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
      }
      *dst = v;
    }
  }
}

// ---- Q6_K x Q8_K chunk GEMM -------------------------------------------------------
// Reference: dot_q6_k_q8k (crates/det-quant/src/lib.rs:353-397).  Per
// 256-element block, lane ln (elements i = 16 s + 8 rep + ln) accumulates the
// exact integer aux[ln] = sum over s, rep of scale_s * a.q[i] * q6[i]; then
// sums[ln] += (w.d * a.d) * (f32)aux[ln] block by block, and the result is
// ((((0 + sums[0]) + sums[1]) + ...) + sums[7]).  A CTA stages one block of
// 32 rows and 64 positions: per (row, ln, s) the int16 pair
// (scale_s * q6[16s + ln], scale_s * q6[16s + 8 + ln]) and per (position,
// ln, s, s + 1) the four matching int8 activations, so one dp2a adds both
// products of a (lane, sub-block) pair.  A thread owns 2 rows x 4 positions
// and runs lane by lane: integer aux (exact in any order), then the f32
// lane sums in block order.
constexpr int K6_ROWS = 32;
constexpr int K6_POS = 64;
constexpr int K6_THREADS = 256;

__global__ void __launch_bounds__(K6_THREADS) gemm_q6k_kernel(const uint8_t* __restrict__ W,
                                                              const uint16_t* __restrict__ Wd, int rows, int nb,
                                                              const int8_t* __restrict__ aq,
                                                              const float* __restrict__ ad, int T,
                                                              float* __restrict__ out, int out_ld, int epi,
                                                              const float* __restrict__ bias, uint32_t* err) {
  pdl_enter();
  __shared__ __align__(16) int wp[8][16][K6_ROWS];      // [ln][s][row]: int16 pair
  __shared__ __align__(16) int ap[8][8][K6_POS];        // [ln][s / 2][pos]: 4 x int8
  __shared__ float sdw[K6_ROWS], sad[K6_POS];
  const int tid = threadIdx.x;
  const int r0 = blockIdx.x * K6_ROWS, p0 = blockIdx.y * K6_POS;
  const int K = nb * 256;
  const int rt = tid >> 4, pt = tid & 15;  // rows 2 rt .. + 1, positions 4 pt .. + 3
  float sums[2][4][8];
#pragma unroll
  for (int r = 0; r < 2; r++)
#pragma unroll
    for (int c = 0; c < 4; c++)
#pragma unroll
      for (int l = 0; l < 8; l++) sums[r][c][l] = 0.0f;

  for (int b = 0; b < nb; b++) {
    __syncthreads();  // previous block consumed
    // weights: 32 rows x 128 (ln, s) pairs; thread: row tid >> 3, pairs (tid & 7) * 16 .. + 16
    {
      const int r = tid >> 3, pr0 = (tid & 7) * 16;
      const bool ok = r0 + r < rows;
      const uint8_t* body = W + ((size_t)(ok ? r0 + r : 0) * nb + b) * 208;
#pragma unroll 4
      for (int k = 0; k < 16; k++) {
        const int pr = pr0 + k, ln = pr >> 4, sb = pr & 15;
        int v = 0;
        if (ok) {
          const int scale = (int8_t)body[192 + sb];
          const int lo = scale * q6k_quant(body, sb * 16 + ln), hi = scale * q6k_quant(body, sb * 16 + 8 + ln);
          v = (int)(((uint32_t)lo & 0xffffu) | ((uint32_t)hi << 16));
        }
        wp[ln][sb][r] = v;
      }
      if (tid < K6_ROWS) sdw[tid] = r0 + tid < rows ? f16_bits_to_f32(Wd[(size_t)(r0 + tid) * nb + b]) : 0.0f;
    }
    // activations: 64 positions x 64 (ln, s-pair) words; thread: position tid >> 2, 16 words
    {
      const int p = tid >> 2, w0 = (tid & 3) * 16;
      const int t = p0 + p;
      const bool ok = t < T;
      const int8_t* qa = aq + (size_t)(ok ? t : 0) * K + (size_t)b * 256;
#pragma unroll 4
      for (int k = 0; k < 16; k++) {
        const int wi = w0 + k, ln = wi >> 3, s2 = wi & 7, s = 2 * s2;
        uint32_t v = 0;
        if (ok)
          v = (uint32_t)(uint8_t)qa[s * 16 + ln] | ((uint32_t)(uint8_t)qa[s * 16 + 8 + ln] << 8) |
              ((uint32_t)(uint8_t)qa[(s + 1) * 16 + ln] << 16) | ((uint32_t)(uint8_t)qa[(s + 1) * 16 + 8 + ln] << 24);
        ap[ln][s2][p] = (int)v;
      }
      if (tid < K6_POS) sad[tid] = p0 + tid < T ? ad[(size_t)(p0 + tid) * nb + b] : 0.0f;
    }
    __syncthreads();
    float dd[2][4];
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
      for (int c = 0; c < 4; c++) dd[r][c] = fmul(sdw[2 * rt + r], sad[4 * pt + c]);
#pragma unroll
    for (int ln = 0; ln < 8; ln++) {
      int aux[2][4];
#pragma unroll
      for (int r = 0; r < 2; r++)
#pragma unroll
        for (int c = 0; c < 4; c++) aux[r][c] = 0;
#pragma unroll
      for (int s2 = 0; s2 < 8; s2++) {
        const int2 w0 = *reinterpret_cast<const int2*>(&wp[ln][2 * s2][2 * rt]);
        const int2 w1 = *reinterpret_cast<const int2*>(&wp[ln][2 * s2 + 1][2 * rt]);
        const int4 a4 = *reinterpret_cast<const int4*>(&ap[ln][s2][4 * pt]);
        const int av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
        for (int c = 0; c < 4; c++) {
          aux[0][c] = __dp2a_hi(w1.x, av[c], __dp2a_lo(w0.x, av[c], aux[0][c]));
          aux[1][c] = __dp2a_hi(w1.y, av[c], __dp2a_lo(w0.y, av[c], aux[1][c]));
        }
      }
#pragma unroll
      for (int r = 0; r < 2; r++)
#pragma unroll
        for (int c = 0; c < 4; c++) sums[r][c][ln] = fadd(sums[r][c][ln], fmul(dd[r][c], __int2float_rn(aux[r][c])));
    }
  }
#pragma unroll
  for (int r = 0; r < 2; r++) {
    const int row = r0 + 2 * rt + r;
    if (row >= rows) continue;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int t = p0 + 4 * pt + c;
      if (t >= T) continue;
      float v = 0.0f;
#pragma unroll
      for (int l = 0; l < 8; l++) v = fadd(v, sums[r][c][l]);
      if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
      float* dst = out + (size_t)t * out_ld + row;
      if (epi == EPI_BIAS) {
        v = fadd(v, bias[row]);
        if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
      } else if (epi == EPI_RESIDUAL) {
        v = fadd(*dst, v);
        if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
      }
      *dst = v;
    }
  }
}

// ---- one position (decode) ---------------------------------------------------------
// Q4_K: the reference's chain is sequential over all K elements, so each
// thread runs one row's chain; the position's dequantised activations
// (a.d * a.q, the reference's exact value) sit in shared memory, so the chain
// only waits on its own f32 adds.
constexpr int D4_THREADS = 128;

__global__ void __launch_bounds__(D4_THREADS) gemv_q4k_decode_kernel(const uint8_t* __restrict__ W, int rows, int nbs,
                                                                     const int8_t* __restrict__ aq,
                                                                     const float* __restrict__ ad,
                                                                     float* __restrict__ out, int epi,
                                                                     const float* __restrict__ bias, uint32_t* err) {
  pdl_enter();
  extern __shared__ float act[];  // [K]
  const int K = nbs * 256, nbk = nbs * 8;
  for (int i = threadIdx.x; i < K; i += D4_THREADS) {
    const int kb = i >> 5, e = i & 31;
    act[i] = fmul(ad[q8a_dslot(nbk, 0, kb)], (float)aq[q8a_elem(nbk, 0, kb, e)]);
  }
  __syncthreads();
  const int row = blockIdx.x * D4_THREADS + threadIdx.x;
  if (row >= rows) return;
  const uint8_t* w = W + (size_t)row * nbs * 144;
  float sum = 0.0f;
  for (int b = 0; b < nbs; b++) {
    const uint8_t* blk = w + (size_t)b * 144;
    const uint4 h = *reinterpret_cast<const uint4*>(blk);  // d, dmin, scales[12]
    uint8_t hb[16];
    *reinterpret_cast<uint4*>(hb) = h;
    const float d = f16_bits_to_f32((uint16_t)(hb[0] | (hb[1] << 8)));
    const float dmin = f16_bits_to_f32((uint16_t)(hb[2] | (hb[3] << 8)));
#pragma unroll 1
    for (int pair = 0; pair < 4; pair++) {  // sub-blocks 2 pair, 2 pair + 1 share 32 quant bytes
      uint32_t qw[8];
#pragma unroll
      for (int k = 0; k < 2; k++) {
        const uint4 v = *reinterpret_cast<const uint4*>(blk + 16 + pair * 32 + 16 * k);
        qw[4 * k] = v.x; qw[4 * k + 1] = v.y; qw[4 * k + 2] = v.z; qw[4 * k + 3] = v.w;
      }
#pragma unroll
      for (int half = 0; half < 2; half++) {
        const int sub = 2 * pair + half;
        int sc, mn;
        q4k_scale_min(hb + 4, sub, sc, mn);
        const float dsc = fmul(d, (float)sc), dmn = fmul(dmin, (float)mn);
        const float* a = act + b * 256 + sub * 32;
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const int q = (int)((qw[i >> 2] >> (8 * (i & 3) + 4 * half)) & 0x0fu);
          sum = fadd(sum, fmul(fsub(fmul(dsc, (float)q), dmn), a[i]));
        }
      }
    }
  }
  if (!finite(sum)) atomicOr(err, ERRF_NONFINITE);
  float v = sum;
  if (epi == EPI_BIAS) {
    v = fadd(v, bias[row]);
    if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
  } else if (epi == EPI_RESIDUAL) {
    v = fadd(out[row], v);
    if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
  }
  out[row] = v;
}

// Q6_K: the integer lane sums are order-free, so a warp takes a row and its
// lanes split each block (lane l: elements 8 l .. 8 l + 7, one per lane
// class ln), reduce the 8 class sums exactly with shuffles, and lane 0 keeps
// the 8 f32 lane sums in block order.
constexpr int D6_WARPS = 4;

__global__ void __launch_bounds__(D6_WARPS * 32) gemv_q6k_decode_kernel(const uint8_t* __restrict__ W,
                                                                        const uint16_t* __restrict__ Wd, int rows,
                                                                        int nb, const int8_t* __restrict__ aq,
                                                                        const float* __restrict__ ad,
                                                                        float* __restrict__ out, int epi,
                                                                        const float* __restrict__ bias,
                                                                        uint32_t* err) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * D6_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint8_t* w = W + (size_t)row * nb * 208;
  float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int b = 0; b < nb; b++) {
    const uint8_t* body = w + (size_t)b * 208;
    const int8_t* a = aq + (size_t)b * 256;
    int aux[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int i = 8 * lane + k;  // ln = k
      aux[k] = (int)(int8_t)body[192 + (i >> 4)] * (int)a[i] * q6k_quant(body, i);
    }
#pragma unroll
    for (int k = 0; k < 8; k++)
      for (int o = 16; o > 0; o >>= 1) aux[k] += __shfl_xor_sync(0xffffffffu, aux[k], o);
    const float dd = fmul(f16_bits_to_f32(Wd[(size_t)row * nb + b]), ad[b]);
#pragma unroll
    for (int k = 0; k < 8; k++) sums[k] = fadd(sums[k], fmul(dd, __int2float_rn(aux[k])));
  }
  if (lane != 0) return;
  float v = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; k++) v = fadd(v, sums[k]);
  if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
  if (epi == EPI_BIAS) {
    v = fadd(v, bias[row]);
    if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
  } else if (epi == EPI_RESIDUAL) {
    v = fadd(out[row], v);
    if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
  }
  out[row] = v;
}

}  // namespace

cudaError_t launch_gemv_kq_decode(const Launch& L, const DevMatrix& m, const DevActs& a, float* out, int epi,
                                  const float* bias) {
  cudaError_t e;
  if (m.type == GT_Q4_K) {
    const size_t smem = (size_t)m.nb * 256 * sizeof(float);
    if (smem > 48 * 1024) {
      e = cudaFuncSetAttribute(gemv_q4k_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    e = launch_k(L, gemv_q4k_decode_kernel, (m.rows + D4_THREADS - 1) / D4_THREADS, D4_THREADS, smem,
                 (const uint8_t*)m.q, m.rows, m.nb, a.qa_q, a.qa_d, out, epi, bias, L.err);
  } else {
    e = launch_k(L, gemv_q6k_decode_kernel, (m.rows + D6_WARPS - 1) / D6_WARPS, D6_WARPS * 32, 0,
                 (const uint8_t*)m.q, m.d, m.rows, m.nb, a.qk_q, a.qk_d, out, epi, bias, L.err);
  }
  if (e != cudaSuccess) return e;
  if (L.launches) ++*L.launches;
  return cudaGetLastError();
}

cudaError_t launch_gemm_q6k(const Launch& L, const DevMatrix& m, const DevActs& a, int T, float* out, int out_ld,
                            int epi, const float* bias) {
  const dim3 grid((m.rows + K6_ROWS - 1) / K6_ROWS, (T + K6_POS - 1) / K6_POS);
  const cudaError_t e = launch_k(L, gemm_q6k_kernel, grid, K6_THREADS, 0, (const uint8_t*)m.q, m.d, m.rows, m.nb,
                                 a.qk_q, a.qk_d, T, out, out_ld, epi, bias, L.err);
  if (e != cudaSuccess) return e;
  if (L.launches) ++*L.launches;
  return cudaGetLastError();
}

cudaError_t launch_gemm_q4k(const Launch& L, const DevMatrix& m, const DevActs& a, int T, float* out, int out_ld,
                            int epi, const float* bias) {
  const dim3 grid((m.rows + KQ_ROWS - 1) / KQ_ROWS, (T + KQ_POS - 1) / KQ_POS);
  const cudaError_t e = launch_k(L, gemm_q4k_kernel, grid, KQ_THREADS, 0, (const uint8_t*)m.q, m.rows, m.nb, a.qa_q,
                                 a.qa_d, T, out, out_ld, epi, bias, 1.0f, L.err);
  if (e != cudaSuccess) return e;
  if (L.launches) ++*L.launches;
  return cudaGetLastError();
}

}  // namespace det
