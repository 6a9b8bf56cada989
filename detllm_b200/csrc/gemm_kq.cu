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
#include <algorithm>
#include <atomic>
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

// Up to three matrices that read the same activation (q / k / v, gate / up)
// in one launch: segment i owns the row tiles from cta0[i] on (blockIdx.x).
struct Q4Segs {
  const uint8_t* W[3];
  int rows[3], cta0[3], out_ld[3], epi[3];
  float* out[3];
  const float* bias[3];
};

__global__ void __launch_bounds__(KQ_THREADS, 5) gemm_q4k_kernel(const Q4Segs G, int nbs,
                                                              const int8_t* __restrict__ aq,
                                                              const float* __restrict__ ad, int T, float one,
                                                              uint32_t* err) {
  pdl_enter();
  const int seg = (int)(blockIdx.x >= (unsigned)G.cta0[1]) + (int)(blockIdx.x >= (unsigned)G.cta0[2]);
  // constant indices only (a runtime index would copy G to local memory)
#define KQ_PICK(f) (seg == 0 ? G.f[0] : (seg == 1 ? G.f[1] : G.f[2]))
  const uint8_t* __restrict__ W = KQ_PICK(W);
  const int rows = KQ_PICK(rows), out_ld = KQ_PICK(out_ld), epi = KQ_PICK(epi);
  float* __restrict__ out = KQ_PICK(out);
  const float* __restrict__ bias = KQ_PICK(bias);
  const int tile = (int)blockIdx.x - KQ_PICK(cta0);
#undef KQ_PICK
  // two stage buffers: stage s + 1 is dequantised into one while the chains
  // run over the other, from raw bytes loaded into registers before stage s
  __shared__ __align__(16) float ws[2][KQ_E][KQ_WS];  // dequantised weights [element][row]
  __shared__ __align__(16) float as[2][KQ_E][KQ_WS];  // dequantised activations [element][position]
  const int tid = threadIdx.x;
  const int r0 = tile * KQ_ROWS, p0 = blockIdx.y * KQ_POS;
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

  // raw bytes of stage st (super-block st >> 3, sub-block st & 7)
  uint4 hdr = make_uint4(0, 0, 0, 0);  // the current super-block's d, dmin and scales
  uint2 qv = make_uint2(0, 0), qa = make_uint2(0, 0);
  float a_d = 0.0f;
  auto load = [&](int st) {
    const int b = st >> 3, sub = st & 7;
    if (row_ok) {
      const uint8_t* blk = wrow + (size_t)b * 144;
      if (sub == 0) hdr = *reinterpret_cast<const uint4*>(blk);
      qv = *reinterpret_cast<const uint2*>(blk + 16 + (sub >> 1) * 32 + se);
    }
    if (pos_ok) {
      const int kb = b * 8 + sub;
      a_d = ad[q8a_dslot(nbk, t_st, kb)];
      qa = *reinterpret_cast<const uint2*>(aq + q8a_slot(nbk, t_st, kb) * 32 + (se ^ q8a_swz(t_st)));
    }
  };
  // w = (d * sc) * q - dmin * m and a.d * a.q, with the reference's rounding
  auto dequant = [&](int st, int buf) {
    const int sub = st & 7;
    if (row_ok) {
      const float d = f16_bits_to_f32((uint16_t)(hdr.x & 0xffffu));
      const float dmin = f16_bits_to_f32((uint16_t)(hdr.x >> 16));
      // get_scale_min_k4 (det-quant lib.rs:506-518) on the scale bytes
      // held in hdr.y .. hdr.w (bytes 4..15 of the block)
      auto sbyte = [&](int k) -> int {
        const uint32_t w = k < 4 ? hdr.y : (k < 8 ? hdr.z : hdr.w);
        return (int)((w >> (8 * (k & 3))) & 0xffu);
      };
      int sc, mn;
      if (sub < 4) {
        sc = sbyte(sub) & 0x3f;
        mn = sbyte(sub + 4) & 0x3f;
      } else {
        sc = (sbyte(sub + 4) & 0x0f) | ((sbyte(sub - 4) >> 6) << 4);
        mn = (sbyte(sub + 4) >> 4) | ((sbyte(sub) >> 6) << 4);
      }
      const float dsc = fmul(d, (float)sc), dmn = fmul(dmin, (float)mn);
      const int sh = (sub & 1) * 4;
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const uint32_t word = k < 4 ? qv.x : qv.y;
        const int q = (int)((word >> (8 * (k & 3) + sh)) & 0x0fu);
        // (d*sc)*q is exact (17 + 4 significant bits), so the fused form
        // rounds once, exactly where the reference's subtraction does
        ws[buf][se + k][sr ^ se] = __fmaf_rn(dsc, (float)q, -dmn);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; k++) ws[buf][se + k][sr ^ se] = 0.0f;
    }
    if (pos_ok) {
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const uint32_t word = k < 4 ? qa.x : qa.y;
        as[buf][se + k][sr ^ se] = fmul(a_d, (float)(int8_t)(word >> (8 * (k & 3))));
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; k++) as[buf][se + k][sr ^ se] = 0.0f;
    }
  };

  const int nst = nbs * 8;
  load(0);
  dequant(0, 0);
  __syncthreads();
  for (int st = 0; st < nst; st++) {
    const int buf = st & 1;
    if (st + 1 < nst) load(st + 1);  // in flight while the chains run
#pragma unroll 8
    for (int e = 0; e < KQ_E; e++) {
      // rows / positions of element e are stored XOR 8 * (e / 8) (bank
      // spread for the staging stores; 4-row groups stay contiguous)
      const int sw = (e >> 3) << 3;
      const float4 w4 = *reinterpret_cast<const float4*>(&ws[buf][e][(rt * 4) ^ sw]);
      const float4 a4 = *reinterpret_cast<const float4*>(&as[buf][e][(pt * 4) ^ sw]);
      const float wr[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int r = 0; r < 4; r++) {
        acc[r][0] = madd2(wr[r], a4.x, a4.y, one, acc[r][0]);
        acc[r][1] = madd2(wr[r], a4.z, a4.w, one, acc[r][1]);
      }
    }
    if (st + 1 < nst) dequant(st + 1, buf ^ 1);
    __syncthreads();
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

// ---- one position (decode) ---------------------------------------------------------
// Up to three matrices that read the same activation (q, k, v or gate, up)
// in one launch: segment i owns CTAs [cta0, next cta0).
DI KqSeg kq_seg(const KqSegs& S) {
  const int i = (int)(blockIdx.x >= (unsigned)S.s[1].cta0) + (int)(blockIdx.x >= (unsigned)S.s[2].cta0);
  return i == 0 ? S.s[0] : (i == 1 ? S.s[1] : S.s[2]);
}

// byte k (0..11) of a Q4_K block's packed scales (bytes 4..15 of the block)
DI uint32_t q4k_sbyte(const uint4& h, int k) {
  const uint32_t w = k < 4 ? h.y : (k < 8 ? h.z : h.w);
  return (w >> (8 * (k & 3))) & 0xffu;
}

DI void kq_store(const KqSeg& g, int row, float sum, uint32_t* err) {
  if (!finite(sum)) atomicOr(err, ERRF_NONFINITE);
  float v = sum;
  if (g.epi == EPI_BIAS) {
    v = fadd(v, g.bias[row]);
    if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
  } else if (g.epi == EPI_RESIDUAL) {
    v = fadd(g.out[row], v);
    if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
  }
  g.out[row] = v;
}

// Q4_K, one position.  Each row is one f32 chain over all K elements
// (sum += w * act, in order; det-quant lib.rs:281-315), so a row costs K
// dependent adds however it is split.  Every lane therefore owns one row and
// runs its whole chain in registers: it dequantises its row's weights out of
// shared memory, multiplies them by the activation and adds the products in
// element order.  A CTA is one warp (32 rows), so the scheduler spreads the
// warps of a wide matrix over every SM and sub-partition at once; each warp
// streams its rows' super-blocks (32 rows x 144 B) through a G4R_STAGES-slot
// ring with cp.async, G4R_STAGES - 1 super-blocks ahead, and holds the
// activation, dequantised once (act[i] = a.d * a.q, the reference's value),
// in shared memory, where every lane reads the same float4 (a broadcast).
// It serves wide matrices (more CTAs than two per SM; gemv_q4k_split_kernel
// below takes the narrow ones): 3 ring slots keep the CTA at 30 KB, so that
// seven fit per SM and the matrix runs in one wave.
// Lane l reads its row's bytes at 144 l: a quarter-warp's eight 16-byte
// reads fall in distinct bank groups.  The dequantisation and the products
// run as f32x2 pairs; the chain adds one element at a time.
constexpr int G4R_ROWS = 32;
constexpr int G4R_STAGE = G4R_ROWS * 144;  // bytes of one super-block of 32 rows
constexpr int G4_MAX_NB = 64;              // K <= 16384 (activation staged in shared memory)
inline size_t g4r_smem_bytes(int stages, int nbs) { return (size_t)stages * G4R_STAGE + (size_t)nbs * 256 * 4; }

DI void g4_cp_async16(void* sdst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"((uint32_t)__cvta_generic_to_shared(sdst)), "l"(gsrc) : "memory");
}
DI void g4_cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
DI void g4_cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

DI unsigned long long add2(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
DI unsigned long long mul2(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
DI unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// The activation of position 0, dequantised: act[i] = a.d * a.q (the
// reference's value), by threads tid = 0 .. nthreads - 1 with each thread's
// loads in flight together (a block's 32 quants of position 0 are
// contiguous and unswizzled).
DI void q4k_stage_act(float* act, const int8_t* __restrict__ aq, const float* __restrict__ ad, int nbk, int tid,
                      int nthreads) {
  for (int kb0 = 0; kb0 < nbk; kb0 += 4 * nthreads) {
    uint4 qv[4][2];
    float dv[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int kb = kb0 + nthreads * u + tid;
      if (kb < nbk) {
        const uint4* src = reinterpret_cast<const uint4*>(aq + q8a_elem(nbk, 0, kb, 0));
        qv[u][0] = src[0];
        qv[u][1] = src[1];
        dv[u] = ad[q8a_dslot(nbk, 0, kb)];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int kb = kb0 + nthreads * u + tid;
      if (kb < nbk) {
        const uint32_t w[8] = {qv[u][0].x, qv[u][0].y, qv[u][0].z, qv[u][0].w,
                               qv[u][1].x, qv[u][1].y, qv[u][1].z, qv[u][1].w};
        float4* dst = reinterpret_cast<float4*>(act + kb * 32);
#pragma unroll
        for (int k = 0; k < 8; k++) {
          const int x = (int)w[k];
          dst[k] = make_float4(fmul(dv[u], (float)((x << 24) >> 24)), fmul(dv[u], (float)((x << 16) >> 24)),
                               fmul(dv[u], (float)((x << 8) >> 24)), fmul(dv[u], (float)(x >> 24)));
        }
      }
    }
  }
}

// (d * sc, -(dmin * m)) of sub-block j (q4_k_scale_min, det-quant
// lib.rs:516-529, on the packed scale bytes of header h), as f32x2 pairs
DI void q4k_sub_scales(const uint4& h, float d, float dmin, int j, unsigned long long& dsc2,
                       unsigned long long& ndmn2) {
  int sc, mn;
  if (j < 4) {
    sc = (int)(q4k_sbyte(h, j) & 63u);
    mn = (int)(q4k_sbyte(h, j + 4) & 63u);
  } else {
    sc = (int)((q4k_sbyte(h, j + 4) & 0x0fu) | ((q4k_sbyte(h, j - 4) >> 6) << 4));
    mn = (int)((q4k_sbyte(h, j + 4) >> 4) | ((q4k_sbyte(h, j) >> 6) << 4));
  }
  const float dsc = fmul(d, (float)sc), dmn = fmul(dmin, (float)mn);
  dsc2 = pk2(dsc, dsc);
  ndmn2 = pk2(-dmn, -dmn);
}

// products w * act of the four elements whose nibbles are the low nibbles
// of the bytes of `nib` (already shifted and masked).  w = (d*sc)*q -
// (dmin*m): d*sc and q have at most 17 and 4 significant bits, so the
// product is exact and one fused multiply-add rounds exactly where the
// reference's subtraction does; then w * act, rounded.
DI float4 q4k_prod4(uint32_t nib, unsigned long long dsc2, unsigned long long ndmn2, float4 a) {
  const unsigned long long nmag2 = pk2(-8388608.0f, -8388608.0f);
  // 2^23 + q as f32 bits, minus 2^23: q exactly
  const float m0 = __uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7540));
  const float m1 = __uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7541));
  const float m2 = __uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7542));
  const float m3 = __uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7543));
  const unsigned long long w01 = fma2(dsc2, add2(pk2(m0, m1), nmag2), ndmn2);  // exact product, one rounding
  const unsigned long long w23 = fma2(dsc2, add2(pk2(m2, m3), nmag2), ndmn2);  // exact product, one rounding
  const float2 r01 = up2(mul2(w01, pk2(a.x, a.y)));
  const float2 r23 = up2(mul2(w23, pk2(a.z, a.w)));
  return make_float4(r01.x, r01.y, r23.x, r23.y);
}

template <int G4R_STAGES>
__global__ void __launch_bounds__(32) gemv_q4k_rows_kernel(KqSegs S, const int8_t* __restrict__ aq,
                                                           const float* __restrict__ ad, uint32_t* err) {
  extern __shared__ __align__(16) uint8_t g4r_smem[];
  uint8_t* ring = g4r_smem;                                                      // [stage][32 rows][144]
  float* act = reinterpret_cast<float*>(g4r_smem + (size_t)G4R_STAGES * G4R_STAGE);  // [K]
  const KqSeg g = kq_seg(S);
  const int r0 = ((int)blockIdx.x - g.cta0) * G4R_ROWS;
  const int nbs = S.nb, nbk = nbs * 8;
  const int lane = threadIdx.x;

  // raw bytes of super-block s of the 32 rows into slot s % G4R_STAGES;
  // rows past the matrix are zeros (zero weights, zero products).  Every
  // lane commits one group per call, so the wait counts stay uniform.
  auto issue = [&](int s) {
    if (s < nbs) {
      uint8_t* dst0 = ring + (size_t)(s % G4R_STAGES) * G4R_STAGE;
#pragma unroll
      for (int i = 0; i < 9; i++) {
        const int c = lane + 32 * i, r = c / 9, part = c - 9 * r;
        uint8_t* dst = dst0 + r * 144 + part * 16;
        if (r0 + r < g.rows)
          g4_cp_async16(dst, g.q + ((size_t)(r0 + r) * nbs + s) * 144 + part * 16);
        else
          *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    g4_cp_commit();
  };
  for (int s = 0; s < G4R_STAGES - 1; s++) issue(s);  // weights are constant: before the predecessor ends
  pdl_enter();
  q4k_stage_act(act, aq, ad, nbk, lane, 32);
  __syncwarp();

  float sum = 0.0f;
  for (int s = 0; s < nbs; s++) {
    issue(s + G4R_STAGES - 1);             // into the slot read in iteration s - 1
    g4_cp_wait<G4R_STAGES - 1>();          // this lane's copies of super-block s have landed
    __syncwarp();                          // ... and every lane's
    const uint8_t* blk = ring + (size_t)(s % G4R_STAGES) * G4R_STAGE + lane * 144;
    const uint4 h = *reinterpret_cast<const uint4*>(blk);  // d, dmin, scales[12]
    const float d = f16_bits_to_f32((uint16_t)(h.x & 0xffffu));
    const float dmin = f16_bits_to_f32((uint16_t)(h.x >> 16));
    const float4* av = reinterpret_cast<const float4*>(act + s * 256);
    // the super-block's 128 quant bytes at once, and the activation one
    // sub-block ahead of the arithmetic, so no shared-memory load latency
    // sits on the chain
    uint4 qv[8];
#pragma unroll
    for (int i = 0; i < 8; i++) qv[i] = reinterpret_cast<const uint4*>(blk + 16)[i];
    float4 acur[8];
#pragma unroll
    for (int k = 0; k < 8; k++) acur[k] = av[k];
#pragma unroll
    for (int j = 0; j < 8; j++) {  // sub-block j: bytes 32 (j / 2) .., low nibbles for even j
      float4 anext[8];
      if (j < 7) {
#pragma unroll
        for (int k = 0; k < 8; k++) anext[k] = av[(j + 1) * 8 + k];
      }
      unsigned long long dsc2, ndmn2;
      q4k_sub_scales(h, d, dmin, j, dsc2, ndmn2);
      const uint4 v0 = qv[(j >> 1) * 2], v1 = qv[(j >> 1) * 2 + 1];
      const uint32_t qw[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
      for (int k = 0; k < 8; k++) {  // elements 4k .. 4k + 3 of sub-block j, then the chain
        const float4 r = q4k_prod4((qw[k] >> (4 * (j & 1))) & 0x0f0f0f0fu, dsc2, ndmn2, acur[k]);
        sum = fadd(sum, r.x);
        sum = fadd(sum, r.y);
        sum = fadd(sum, r.z);
        sum = fadd(sum, r.w);
      }
      if (j < 7) {
#pragma unroll
        for (int k = 0; k < 8; k++) acur[k] = anext[k];
      }
    }
    __syncwarp();  // every lane is done with the slot before it is refilled
  }
  const int row = r0 + lane;
  if (row < g.rows) kq_store(g, row, sum, err);
}

// Q4_K, one position, for narrow matrices (at most two CTAs per SM): the
// same per-row chain, with the products made by other warps.  A lane of the
// kernel above both forms its row's products and adds them, so with one
// warp per SM sub-partition the row runs at the warp's issue rate, about
// twice the chain's own latency of one dependent add per element.  Here a
// CTA of 32 rows has four producer warps and one chain warp: producer thread
// (row r, sub-block s of a half block) dequantises its 32 weights and forms
// the exact products w * act (q4k_prod4), written to a three-slot ring of
// half-block product tiles [32 rows][128 elements]; the chain warp's lane r
// then only loads row r's products and adds them in element order.  The
// raw blocks come in by cp.async, issued by the producers seven blocks ahead;
// the product slots hand over on mbarriers (full: 128 producer arrivals,
// empty: the chain warp), every wait bounded by %globaltimer and abandoned
// at once after any timeout.
constexpr int G4S_PROD_WARPS = 4;
constexpr int G4S_THREADS = (G4S_PROD_WARPS + 1) * 32;
constexpr int G4S_RAW = 8;                      // raw block slots: 7 blocks in flight
constexpr int G4S_PS = 3;                       // product slots (half blocks)
constexpr int G4S_PLD = 128 + 4;                // product row stride (floats): rows 4 banks apart
constexpr int G4S_PSLOT = G4R_ROWS * G4S_PLD;   // floats per product slot
// raw ring | product ring | activation [K] | full[PS], empty[PS] | abort flag
inline size_t g4s_smem_bytes(int nbs) {
  return (size_t)G4S_RAW * G4R_STAGE + (size_t)G4S_PS * G4S_PSLOT * 4 + (size_t)nbs * 256 * 4 + 2 * G4S_PS * 8 + 16;
}

// bounded wait for phase `parity`; returns at once once the CTA has given up
DI void g4s_wait(uint32_t bar, uint32_t parity, volatile int* gave_up, uint32_t* err) {
  unsigned long long t0 = 0;
  for (unsigned it = 0;; it++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok || *gave_up) return;
    if ((it & 63) == 0) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
      if (it == 0) {
        t0 = t;
      } else if (t - t0 > 2000000000ull) {
        atomicOr(err, ERRF_TIMEOUT);
        *gave_up = 1;
        return;
      }
    }
  }
}
DI void g4s_arrive(uint32_t bar) { asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory"); }

__global__ void __launch_bounds__(G4S_THREADS) gemv_q4k_split_kernel(KqSegs S, const int8_t* __restrict__ aq,
                                                                     const float* __restrict__ ad, uint32_t* err) {
  extern __shared__ __align__(16) uint8_t g4s_smem[];
  const int nbs = S.nb, nbk = nbs * 8;
  uint8_t* raw = g4s_smem;                                                          // [RAW][32 rows][144]
  float* prod = reinterpret_cast<float*>(raw + (size_t)G4S_RAW * G4R_STAGE);        // [PS][32][PLD]
  float* act = prod + (size_t)G4S_PS * G4S_PSLOT;                                   // [K]
  uint64_t* bars = reinterpret_cast<uint64_t*>(act + (size_t)nbs * 256);
  volatile int* gave_up = reinterpret_cast<volatile int*>(bars + 2 * G4S_PS);
  const uint32_t full0 = (uint32_t)__cvta_generic_to_shared(bars), empty0 = full0 + 8 * G4S_PS;
  const KqSeg g = kq_seg(S);
  const int r0 = ((int)blockIdx.x - g.cta0) * G4R_ROWS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool producer = warp < G4S_PROD_WARPS;
  if (tid == 0) {
    for (int i = 0; i < G4S_PS; i++) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(full0 + 8 * i), "r"(G4S_PROD_WARPS * 32) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(empty0 + 8 * i) : "memory");
    }
    *gave_up = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  // raw bytes of block b of the 32 rows into slot b % G4S_RAW (producers;
  // rows past the matrix are zeros); one commit group per call
  auto issue = [&](int b) {
    if (b < nbs) {
      uint8_t* dst0 = raw + (size_t)(b % G4S_RAW) * G4R_STAGE;
      for (int c = tid; c < G4R_ROWS * 9; c += G4S_PROD_WARPS * 32) {
        const int r = c / 9, part = c - 9 * r;
        uint8_t* dst = dst0 + r * 144 + part * 16;
        if (r0 + r < g.rows)
          g4_cp_async16(dst, g.q + ((size_t)(r0 + r) * nbs + b) * 144 + part * 16);
        else
          *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    g4_cp_commit();
  };
  if (producer)
    for (int b = 0; b < G4S_RAW - 1; b++) issue(b);  // weights are constant: before the predecessor ends
  pdl_enter();
  q4k_stage_act(act, aq, ad, nbk, tid, G4S_THREADS);
  __syncthreads();  // activation and barrier initialisation visible

  if (producer) {
    const int pr = tid & 31, ps = tid >> 5;  // row, sub-block of the half block
    for (int b = 0; b < nbs; b++) {
      asm volatile("bar.sync 1, %0;\n" ::"n"(G4S_PROD_WARPS * 32) : "memory");  // slot (b - 1) % RAW is read
      issue(b + G4S_RAW - 1);
      g4_cp_wait<G4S_RAW - 1>();  // this thread's copies of block b have landed
      asm volatile("bar.sync 1, %0;\n" ::"n"(G4S_PROD_WARPS * 32) : "memory");  // ... and every producer's
      const uint8_t* blk = raw + (size_t)(b % G4S_RAW) * G4R_STAGE + pr * 144;
      const uint4 h = *reinterpret_cast<const uint4*>(blk);  // d, dmin, scales[12]
      const float d = f16_bits_to_f32((uint16_t)(h.x & 0xffffu));
      const float dmin = f16_bits_to_f32((uint16_t)(h.x >> 16));
#pragma unroll
      for (int hf = 0; hf < 2; hf++) {
        const int hh = 2 * b + hf, slot = hh % G4S_PS;
        g4s_wait(empty0 + 8 * slot, (uint32_t)(((hh / G4S_PS) & 1) ^ 1), gave_up, err);
        const int j = 4 * hf + ps;  // sub-block: bytes 32 (j / 2) .., low nibbles for even j
        unsigned long long dsc2, ndmn2;
        q4k_sub_scales(h, d, dmin, j, dsc2, ndmn2);
        const uint4 v0 = *reinterpret_cast<const uint4*>(blk + 16 + 32 * (j >> 1));
        const uint4 v1 = *reinterpret_cast<const uint4*>(blk + 32 + 32 * (j >> 1));
        const uint32_t qw[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        const float4* av = reinterpret_cast<const float4*>(act + (size_t)b * 256 + 32 * j);
        float4* dst = reinterpret_cast<float4*>(prod + (size_t)slot * G4S_PSLOT + pr * G4S_PLD + 32 * ps);
#pragma unroll
        for (int k = 0; k < 8; k++) dst[k] = q4k_prod4((qw[k] >> (4 * (j & 1))) & 0x0f0f0f0fu, dsc2, ndmn2, av[k]);
        g4s_arrive(full0 + 8 * slot);
      }
    }
    g4_cp_wait<0>();
  } else {
    // lane = row: the chain over the half blocks' products in element order
    float sum = 0.0f;
    for (int hh = 0; hh < 2 * nbs; hh++) {
      const int slot = hh % G4S_PS;
      g4s_wait(full0 + 8 * slot, (uint32_t)((hh / G4S_PS) & 1), gave_up, err);
      const float4* src = reinterpret_cast<const float4*>(prod + (size_t)slot * G4S_PSLOT + lane * G4S_PLD);
#pragma unroll
      for (int k0 = 0; k0 < 32; k0 += 8) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) v[u] = src[k0 + u];
#pragma unroll
        for (int u = 0; u < 8; u++) {
          sum = fadd(sum, v[u].x);
          sum = fadd(sum, v[u].y);
          sum = fadd(sum, v[u].z);
          sum = fadd(sum, v[u].w);
        }
      }
      __syncwarp();
      if (lane == 0) g4s_arrive(empty0 + 8 * slot);  // the slot's products are read
    }
    const int row = r0 + lane;
    if (row < g.rows) kq_store(g, row, sum, err);
  }
}

// Q6_K: per block the reference forms eight exact integer lane sums
// aux[c] = sum over elements i = c (mod 8) of sc[i / 16] * a[i] * (q[i] - 32)
// and then advances eight f32 chains sums[c] += (d * a.d) * aux[c] in block
// order.  The integer sums are order-free, so a CTA computes them for all
// (row, block) items of its R rows in parallel, two items per thread with
// both items' loads issued first (the lanes of a warp take consecutive rows
// of one block, so their activation reads are broadcasts): within a
// 16-element scale group, class c
// owns elements c and c + 8, whose 6-bit values a byte permute pairs up for
// dp2a against the activation pairs (a[c], a[c + 8]); the -32 offset is
// folded in as sc * (a[c] + a[c + 8]) sums, also by dp2a.  Then thread
// (row, class) runs its f32 chain over the blocks out of shared memory, and
// the row's eight chains are summed in lane order.
constexpr int G6_THREADS = 256;
constexpr int G6_NBC = 32;                 // blocks per pass
constexpr int G6_AUX_LD = G6_NBC * 8 + 1;  // aux row stride (ints): rows in distinct banks
constexpr int G6_DD_LD = G6_NBC + 1;
template <int R>
constexpr size_t g6_smem() {
  return (size_t)G6_NBC * (128 + 64) * 4 + (size_t)R * G6_AUX_LD * 4 + (size_t)R * G6_DD_LD * 4;
}

DI int dp2a_lo_su(uint32_t a, uint32_t b, int c) {  // a: two s16, b: bytes 0, 1 unsigned
  int d;
  asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
DI int dp2a_hi_su(uint32_t a, uint32_t b, int c) {  // bytes 2, 3
  int d;
  asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
DI int dp2a_lo_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
DI int dp2a_hi_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
DI uint32_t s16pair(int lo, int hi) { return ((uint32_t)lo & 0xffffu) | ((uint32_t)hi << 16); }
// prmt.b32 with sign replication (a selector nibble with bit 3 set copies
// the selected byte's sign bit into the whole target byte)
DI uint32_t prmt_sx(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

struct Q6Item {
  uint32_t w[52];  // ql words 0..31, qh words 32..47, scale words 48..51
  uint32_t d;      // f16 bits of the block scale
};

DI void q6_load(const KqSeg& g, int nb, int row, int b, Q6Item& it) {
  const uint4* src = reinterpret_cast<const uint4*>(g.q + ((size_t)row * nb + b) * 208);
#pragma unroll
  for (int k = 0; k < 13; k++) {
    const uint4 v = src[k];
    it.w[4 * k] = v.x;
    it.w[4 * k + 1] = v.y;
    it.w[4 * k + 2] = v.z;
    it.w[4 * k + 3] = v.w;
  }
  it.d = g.d[(size_t)row * nb + b];
}

// the eight integer lane sums of one block (A, Sp: its activation pairs)
DI void q6_aux(const Q6Item& it, const uint32_t* A, const uint32_t* Sp, int* dst) {
  const uint32_t* w = it.w;
  int acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
  for (int half = 0; half < 2; half++)
#pragma unroll
    for (int lh = 0; lh < 2; lh++)
#pragma unroll
      for (int part = 0; part < 4; part++) {
        const int gg = half * 8 + part * 2 + lh;  // scale group of these 16 elements
        uint32_t x[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
          uint32_t lw = w[half * 16 + (part & 1) * 8 + lh * 4 + k];
          if (part >= 2) lw >>= 4;
          const uint32_t hw = w[32 + half * 8 + lh * 4 + k];
          const uint32_t hs = part == 0 ? hw << 4 : part == 1 ? hw << 2 : part == 2 ? hw : hw >> 2;
          x[k] = (lw & 0x0f0f0f0fu) | (hs & 0x30303030u);  // 6-bit values of elements 4k .. 4k + 3
        }
        const uint32_t p0 = __byte_perm(x[0], x[2], 0x5140), p1 = __byte_perm(x[0], x[2], 0x7362);
        const uint32_t p2 = __byte_perm(x[1], x[3], 0x5140), p3 = __byte_perm(x[1], x[3], 0x7362);
        const uint4 aa = *reinterpret_cast<const uint4*>(A + gg * 8);
        const uint4 ab = *reinterpret_cast<const uint4*>(A + gg * 8 + 4);
        const int sc = (int)(int8_t)(w[48 + (gg >> 2)] >> (8 * (gg & 3)));
        acc[0] += sc * dp2a_lo_su(aa.x, p0, 0);
        acc[1] += sc * dp2a_hi_su(aa.y, p0, 0);
        acc[2] += sc * dp2a_lo_su(aa.z, p1, 0);
        acc[3] += sc * dp2a_hi_su(aa.w, p1, 0);
        acc[4] += sc * dp2a_lo_su(ab.x, p2, 0);
        acc[5] += sc * dp2a_hi_su(ab.y, p2, 0);
        acc[6] += sc * dp2a_lo_su(ab.z, p3, 0);
        acc[7] += sc * dp2a_hi_su(ab.w, p3, 0);
      }
#pragma unroll
  for (int c = 0; c < 8; c++) {
    int corr = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      corr = dp2a_lo_ss(Sp[(2 * k) * 8 + c], w[48 + k], corr);
      corr = dp2a_hi_ss(Sp[(2 * k + 1) * 8 + c], w[48 + k], corr);
    }
    dst[c] = acc[c] - 32 * corr;
  }
}

// Q6_K, one position, on int8 tensor cores (mma.sync m16n8k16).  Per block
// the reference's lane sums (dot_q6_k_q8k, det-quant lib.rs:353-397) are
//   aux[r][l] = sum over the 16 scale groups j of scale[r][j] * C_j[r][l],
//   C_j[r][l] = sum over e in {16 j + l, 16 j + 8 + l} of (q6[r][e] - 32) * a[e],
// so one group of 16 rows is one m16n8k16 MMA: A = the rows' 6-bit codes of
// the group as unsigned bytes (MMA column k = element 16 j + k), B = the
// activation placed so that output column l sees only the group's two
// elements of lane l (B[k][l] = a[16 j + k] when k % 8 == l, else 0).  Every
// C_j' = sum of q6 * a fits 16 bits (|C| <= 16,128), so the scale step takes
// a group pair at once: dp2a of the packed (C'_2Q, C'_2Q+1) with scale bytes
// 2Q and 2Q + 1.  The -32 offset is one more product per tile,
//   sum over j of scale[r][j] * (a[16 j + l] + a[16 j + 8 + l]),
// two m16n8k16 MMAs of the rows' 16 scales (as A, k = group) by the
// activation's two elements of each (group, lane) (as B), taken 32 times
// off the integer sums.  The float work is the reference's: d = w.d *
// a.d, p = d * (f32)aux, each (row, lane) chain adds p in block order, and
// the row's result sums its eight chains in lane order.
//
// A CTA owns ceil(rows / SMs) contiguous rows, so the weight stream is
// spread evenly over every SM.  It walks them in groups of 32 rows, each
// group's blocks in chunks of 8; one stage is one (group, chunk), whose
// rows are contiguous 1,664-byte runs (one cp.async.bulk per row) moved into
// a Q6M_STAGES-slot ring on per-slot mbarriers.  Each of the 16 warps takes
// one (16-row tile, block) unit per stage and leaves its 16 x 8 products in
// shared memory; after the stage's barrier, threads (row, lane) add them to
// their chains while the warps go on to the next stage.  The activation is
// staged once per CTA: the B bytes of every (block, thread slot) and the
// offset operands of every (block, thread).  Waits are bounded by
// %globaltimer.
constexpr int Q6M_THREADS = 512;
constexpr int Q6M_GROUP = 32;                          // rows per group (two MMA tiles)
constexpr int Q6M_CHUNK = 8;                           // blocks per stage
constexpr int Q6M_STAGES = 3;
constexpr int Q6M_ROW = Q6M_CHUNK * 208;               // one row of a stage: 1,664 B
constexpr int Q6M_ROW_LD = Q6M_ROW + 16;               // its slot: 420 words, so rows g = 0..7 start 4 banks apart
constexpr int Q6M_STAGE = Q6M_GROUP * Q6M_ROW_LD;      // 53,760 B
constexpr int Q6M_MAX_NB = 64;                         // K <= 16384 (activation tables in shared memory)
constexpr int Q6M_PLD = Q6M_CHUNK * 8 + 8;             // product row stride (floats): conflict-free chain reads
constexpr int Q6M_PBUF = 2 * Q6M_GROUP * Q6M_PLD * 4;  // two stages of products
// ring | mbarriers (32 B) | B bytes [nb][16][16] | offset B words [nb][32][2] | products | a.d [nb]
inline size_t q6m_smem_bytes(int nb) {
  return (size_t)Q6M_STAGES * Q6M_STAGE + 32 + (size_t)nb * 256 + (size_t)nb * 256 + Q6M_PBUF + (size_t)nb * 4;
}
static_assert(Q6M_PBUF >= Q6M_MAX_NB * 256, "the activation is staged in the product buffers");

DI bool q6m_wait(uint32_t bar, uint32_t parity) {
  unsigned long long t0 = 0;
  for (unsigned it = 0;; it++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((it & 63) == 0) {  // the clock every 64 polls
      unsigned long long t;
      asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
      if (it == 0) t0 = t;
      else if (t - t0 > 2000000000ull) return false;
    }
  }
}

// the segment of concatenated row r and r's index in it
DI KqSeg q6m_seg(const KqSegs& S, int r, int& rr) {
  const int p1 = S.s[0].rows, p2 = p1 + S.s[1].rows;
  if (r < p1) {
    rr = r;
    return S.s[0];
  }
  if (r < p2) {
    rr = r - p1;
    return S.s[1];
  }
  rr = r - p2;
  return S.s[2];
}

// the unsigned 6-bit codes of quarter qd (nibble nib of the ql word, bits
// 2 qd, 2 qd + 1 of the qh word) for four consecutive elements
template <int NIB, int QD>
DI uint32_t q6m_code(uint32_t ql, uint32_t qh) {
  const uint32_t lo = NIB ? ql >> 4 : ql;
  const uint32_t hi = QD == 0 ? qh << 4 : (QD == 1 ? qh << 2 : (QD == 2 ? qh : qh >> 2));
  return (lo & 0x0f0f0f0fu) | (hi & 0x30303030u);
}

// four 8 x 16-byte matrices: lane 8 m + r gives row r of matrix m; lane
// (g, t) receives word t of row g of each
DI void q6m_ldsm(const uint8_t* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"((uint32_t)__cvta_generic_to_shared(p))
               : "memory");
}

// c = A B with unsigned A (the codes), signed B
DI void q6m_mma(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};\n"
      : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(a0), "r"(a1), "r"(b), "r"(0));
}
// c += A B, both signed (the offset product)
DI void q6m_mma_ss(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(b));
}

__global__ void __launch_bounds__(Q6M_THREADS, 1) gemv_q6k_mma_kernel(KqSegs S, int total, int per_cta,
                                                                      const int8_t* __restrict__ aq,
                                                                      const float* __restrict__ ad, uint32_t* err) {
  extern __shared__ __align__(16) uint8_t q6m_smem[];
  const int nb = S.nb;
  uint8_t* ring = q6m_smem;                                                      // [stages][32 rows][1680]
  const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(ring + (size_t)Q6M_STAGES * Q6M_STAGE);
  uint8_t* bact = ring + (size_t)Q6M_STAGES * Q6M_STAGE + 32;                   // [nb][16 slots][16 groups]
  // offset B words: lane (g, t) holds bytes a[16 (4t + i) + g] and
  // a[16 (4t + i) + 8 + g], i = 0..3, of each block
  uint2* offb = reinterpret_cast<uint2*>(bact + (size_t)nb * 256);
  float* pbuf = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(offb) + (size_t)nb * 256);  // [2][32][PLD]
  float* adv = pbuf + 2 * Q6M_GROUP * Q6M_PLD;                                  // [nb]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;     // MMA fragment coordinates
  const int mt = warp >> 3, bb = warp & 7;   // this warp's unit: 16-row tile, block of the chunk
  const int row0 = (int)blockIdx.x * per_cta, rows = min(per_cta, total - row0);
  const int nch = (nb + Q6M_CHUNK - 1) / Q6M_CHUNK;
  const int nst = (rows + Q6M_GROUP - 1) / Q6M_GROUP * nch;
  if (tid == 0) {
    for (int s = 0; s < Q6M_STAGES; s++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(bar0 + 8 * s) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();

  // stage coordinates (row group, chunk), advanced one stage at a time
  struct At {
    int grp, ch;
  };
  auto next = [&](At& a) {
    if (++a.ch == nch) {
      a.ch = 0;
      a.grp++;
    }
  };
  // stage s (at a) into slot s % Q6M_STAGES: one bulk copy per row; thread
  // 0 arrives with the stage's byte count (complete_tx may come first)
  auto issue = [&](int s, const At& a) {
    const int r0 = a.grp * Q6M_GROUP, nr = min(Q6M_GROUP, rows - r0);
    const int b0 = a.ch * Q6M_CHUNK, nbk = min(Q6M_CHUNK, nb - b0);
    const uint32_t bar = bar0 + 8 * (s % Q6M_STAGES);
    if (tid == 0)
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"((uint32_t)(nr * nbk * 208))
                   : "memory");
    if (tid < nr) {
      int rr;
      const KqSeg sg = q6m_seg(S, row0 + r0 + tid, rr);
      const uint8_t* src = sg.q + ((size_t)rr * nb + b0) * 208;
      const uint32_t dst =
          (uint32_t)__cvta_generic_to_shared(ring + (size_t)(s % Q6M_STAGES) * Q6M_STAGE + (size_t)tid * Q6M_ROW_LD);
      // the slot was last read with ordinary loads (stage s - Q6M_STAGES)
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
                   "l"(src), "r"((uint32_t)(nbk * 208)), "r"(bar)
                   : "memory");
    }
  };
  // the f16 block scales of this thread's rows g and g + 8 in the unit of
  // the stage at a (row pointers cached per group; 0 past the rows)
  int dgrp = -1;
  const uint16_t *dpa = nullptr, *dpb = nullptr;
  auto load_d = [&](const At& a, uint32_t& da, uint32_t& db) {
    da = db = 0u;
    if (a.grp != dgrp) {
      dgrp = a.grp;
      const int la = a.grp * Q6M_GROUP + mt * 16 + g;
      int rr;
      dpa = dpb = nullptr;
      if (la < rows) {
        const KqSeg sg = q6m_seg(S, row0 + la, rr);
        dpa = sg.d + (size_t)rr * nb;
      }
      if (la + 8 < rows) {
        const KqSeg sg = q6m_seg(S, row0 + la + 8, rr);
        dpb = sg.d + (size_t)rr * nb;
      }
    }
    const int b = a.ch * Q6M_CHUNK + bb;
    if (b < nb) {
      if (dpa) da = dpa[b];
      if (dpb) db = dpb[b];
    }
  };
  int issued = 0;
  At ia{0, 0};  // the next stage to issue
  for (; issued < nst && issued < Q6M_STAGES; issued++, next(ia)) issue(issued, ia);  // weights are constant: before the predecessor ends
  uint32_t da, db;
  load_d(At{0, 0}, da, db);
  pdl_enter();

  // activation tables: the raw bytes staged in the product buffers first
  {
    int8_t* raw = reinterpret_cast<int8_t*>(pbuf);
    for (int i = tid; i < nb * 16; i += Q6M_THREADS)
      reinterpret_cast<uint4*>(raw)[i] = reinterpret_cast<const uint4*>(aq)[i];
    for (int b = tid; b < nb; b += Q6M_THREADS) adv[b] = ad[b];
    __syncthreads();
    // B bytes: slot sl = 4 t + (g & 3) holds a[16 j + sl] for j = 0..15
    for (int i = tid; i < nb * 16; i += Q6M_THREADS) {
      const int b = i >> 4, sl = i & 15;
      const int8_t* a = raw + b * 256 + sl;
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; k++)
        w[k] = (uint32_t)(uint8_t)a[64 * k] | ((uint32_t)(uint8_t)a[64 * k + 16] << 8) |
               ((uint32_t)(uint8_t)a[64 * k + 32] << 16) | ((uint32_t)(uint8_t)a[64 * k + 48] << 24);
      reinterpret_cast<uint4*>(bact)[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    for (int i = tid; i < nb * 32; i += Q6M_THREADS) {
      const int b = i >> 5, lg = (i & 31) >> 2, lt = i & 3;
      const int8_t* a = raw + b * 256 + 64 * lt + lg;
      uint32_t w0 = 0u, w1 = 0u;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        w0 |= (uint32_t)(uint8_t)a[16 * k] << (8 * k);
        w1 |= (uint32_t)(uint8_t)a[16 * k + 8] << (8 * k);
      }
      offb[i] = make_uint2(w0, w1);
    }
    __syncthreads();  // the product buffers are free again
  }

  // B placement: byte x of an activation word to byte g & 3 when this
  // thread's k rows (4 t .. 4 t + 3) hold lane g's elements, else zero
  const bool bl = (g >> 2) == (t & 1);
  uint32_t bsel[4];
#pragma unroll
  for (int x = 0; x < 4; x++)
    bsel[x] = bl ? ((0x4444u & ~(0xfu << (4 * (g & 3)))) | ((uint32_t)x << (4 * (g & 3)))) : 0x4444u;

  // threads (row tid >> 3, lane tid & 7) < 256 add the products of the
  // stage at a (buffer sp & 1) to their chains in block order; after a
  // group's last chunk each row sums its eight chains in lane order and is
  // stored.  A stage's products stay in place until the barrier of the next.
  float csum = 0.0f;
  auto chain = [&](int sp, const At& a) {
    if (tid >= 256) return;
    const int crow = tid >> 3;
    const int nbk = min(Q6M_CHUNK, nb - a.ch * Q6M_CHUNK);
    const float* pr = pbuf + (size_t)(sp & 1) * Q6M_GROUP * Q6M_PLD + (size_t)crow * Q6M_PLD + (tid & 7);
    float pv[Q6M_CHUNK];
#pragma unroll
    for (int k = 0; k < Q6M_CHUNK; k++) pv[k] = pr[k * 8];  // in the buffer for every k; used below nbk
#pragma unroll
    for (int k = 0; k < Q6M_CHUNK; k++)
      if (k < nbk) csum = fadd(csum, pv[k]);
    if (a.ch == nch - 1) {
      // ((((0 + s0) + s1) + ...) + s7) within each group of eight lanes
      float v = 0.0f;
#pragma unroll
      for (int k = 0; k < 8; k++) v = fadd(v, __shfl_sync(0xffffffffu, csum, (lane & ~7) + k));
      const int r = a.grp * Q6M_GROUP + crow;
      if ((tid & 7) == 0 && r < rows) {
        int rr;
        const KqSeg sg = q6m_seg(S, row0 + r, rr);
        kq_store(sg, rr, v, err);
      }
      csum = 0.0f;
    }
  };
  bool ok = true;
  int s = 0;
  At at{0, 0}, prev{0, 0};  // stage s, stage s - 1
  for (; s < nst; s++) {
    const int slot = s % Q6M_STAGES, buf = s & 1;
    At nx = at;
    next(nx);
    uint32_t dna = 0u, dnb = 0u;
    if (s + 1 < nst) load_d(nx, dna, dnb);
    if (!q6m_wait(bar0 + 8 * slot, (uint32_t)((s / Q6M_STAGES) & 1))) {
      atomicOr(err, ERRF_TIMEOUT);
      ok = false;
    }
    const int b = at.ch * Q6M_CHUNK + bb;
    if (ok && b < nb && at.grp * Q6M_GROUP + mt * 16 < rows) {
      const uint8_t* wa = ring + (size_t)slot * Q6M_STAGE + (size_t)(mt * 16 + g) * Q6M_ROW_LD + bb * 208;
      const uint8_t* wb = wa + 8 * Q6M_ROW_LD;
      const uint4 sca = *reinterpret_cast<const uint4*>(wa + 192);
      const uint4 scb = *reinterpret_cast<const uint4*>(wb + 192);
      const uint4 av = *reinterpret_cast<const uint4*>(bact + ((size_t)b * 16 + 4 * t + (g & 3)) * 16);
      const uint32_t avw[4] = {av.x, av.y, av.z, av.w};
      const uint32_t scwa[4] = {sca.x, sca.y, sca.z, sca.w}, scwb[4] = {scb.x, scb.y, scb.z, scb.w};
      // ldmatrix rows: lanes 8m .. 8m + 7 give matrix m = (rows 0-7 | 8-15 of the tile, bytes 0-15 | 16-31 of a run)
      const uint8_t* lrow = ring + (size_t)slot * Q6M_STAGE +
                            (size_t)(mt * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * Q6M_ROW_LD + bb * 208 +
                            16 * (lane >> 4);
      int xa0 = 0, xa1 = 0, xb0 = 0, xb1 = 0;  // aux of (g, 2t), (g, 2t+1), (g+8, 2t), (g+8, 2t+1)
#pragma unroll
      for (int h = 0; h < 2; h++) {
        uint32_t hE_a, hE_b, hO_a, hO_b;  // qh words t (group E) and 4 + t (group O) of rows g, g + 8
        q6m_ldsm(lrow + 128 + 32 * h, hE_a, hE_b, hO_a, hO_b);
#pragma unroll
        for (int p = 0; p < 2; p++) {
          uint32_t lE_a, lE_b, lO_a, lO_b;  // ql words of run (h, p), likewise
          q6m_ldsm(lrow + 64 * h + 32 * p, lE_a, lE_b, lO_a, lO_b);
#pragma unroll
          for (int nib = 0; nib < 2; nib++) {
            const int qd = p + 2 * nib, Q = 4 * h + qd;  // groups 2Q, 2Q + 1
            uint32_t aE0, aE1, aO0, aO1;
            if (nib == 0 && p == 0) {
              aE0 = q6m_code<0, 0>(lE_a, hE_a), aE1 = q6m_code<0, 0>(lE_b, hE_b);
              aO0 = q6m_code<0, 0>(lO_a, hO_a), aO1 = q6m_code<0, 0>(lO_b, hO_b);
            } else if (nib == 0) {
              aE0 = q6m_code<0, 1>(lE_a, hE_a), aE1 = q6m_code<0, 1>(lE_b, hE_b);
              aO0 = q6m_code<0, 1>(lO_a, hO_a), aO1 = q6m_code<0, 1>(lO_b, hO_b);
            } else if (p == 0) {
              aE0 = q6m_code<1, 2>(lE_a, hE_a), aE1 = q6m_code<1, 2>(lE_b, hE_b);
              aO0 = q6m_code<1, 2>(lO_a, hO_a), aO1 = q6m_code<1, 2>(lO_b, hO_b);
            } else {
              aE0 = q6m_code<1, 3>(lE_a, hE_a), aE1 = q6m_code<1, 3>(lE_b, hE_b);
              aO0 = q6m_code<1, 3>(lO_a, hO_a), aO1 = q6m_code<1, 3>(lO_b, hO_b);
            }
            int cE[4], cO[4];
            q6m_mma(cE, aE0, aE1, __byte_perm(avw[Q >> 1], 0u, bsel[(2 * Q) & 3]));
            q6m_mma(cO, aO0, aO1, __byte_perm(avw[Q >> 1], 0u, bsel[(2 * Q + 1) & 3]));
            const uint32_t pa0 = __byte_perm((uint32_t)cE[0], (uint32_t)cO[0], 0x5410u);
            const uint32_t pa1 = __byte_perm((uint32_t)cE[1], (uint32_t)cO[1], 0x5410u);
            const uint32_t pb0 = __byte_perm((uint32_t)cE[2], (uint32_t)cO[2], 0x5410u);
            const uint32_t pb1 = __byte_perm((uint32_t)cE[3], (uint32_t)cO[3], 0x5410u);
            if (Q & 1) {  // scale bytes 2, 3 of word Q >> 1
              xa0 = dp2a_hi_ss(pa0, scwa[Q >> 1], xa0);
              xa1 = dp2a_hi_ss(pa1, scwa[Q >> 1], xa1);
              xb0 = dp2a_hi_ss(pb0, scwb[Q >> 1], xb0);
              xb1 = dp2a_hi_ss(pb1, scwb[Q >> 1], xb1);
            } else {  // bytes 0, 1
              xa0 = dp2a_lo_ss(pa0, scwa[Q >> 1], xa0);
              xa1 = dp2a_lo_ss(pa1, scwa[Q >> 1], xa1);
              xb0 = dp2a_lo_ss(pb0, scwb[Q >> 1], xb0);
              xb1 = dp2a_lo_ss(pb1, scwb[Q >> 1], xb1);
            }
          }
        }
      }
      {  // the -32 offset: 32 * sum over j of scale[r][j] * (a[16 j + l] + a[16 j + 8 + l])
        const uint2 ow = offb[(size_t)b * 32 + lane];
        const uint32_t swa = *reinterpret_cast<const uint32_t*>(wa + 192 + 4 * t);
        const uint32_t swb = *reinterpret_cast<const uint32_t*>(wb + 192 + 4 * t);
        int co[4] = {0, 0, 0, 0};
        q6m_mma_ss(co, swa, swb, ow.x);
        q6m_mma_ss(co, swa, swb, ow.y);
        xa0 -= 32 * co[0];
        xa1 -= 32 * co[1];
        xb0 -= 32 * co[2];
        xb1 -= 32 * co[3];
      }
      const float adb = adv[b];
      const float dda = fmul(f16_bits_to_f32((uint16_t)da), adb), ddb = fmul(f16_bits_to_f32((uint16_t)db), adb);
      float* pr = pbuf + (size_t)buf * Q6M_GROUP * Q6M_PLD + (size_t)(mt * 16 + g) * Q6M_PLD + bb * 8 + 2 * t;
      *reinterpret_cast<float2*>(pr) = make_float2(fmul(dda, __int2float_rn(xa0)), fmul(dda, __int2float_rn(xa1)));
      *reinterpret_cast<float2*>(pr + 8 * Q6M_PLD) =
          make_float2(fmul(ddb, __int2float_rn(xb0)), fmul(ddb, __int2float_rn(xb1)));
    }
    if (s > 0) chain(s - 1, prev);  // overlaps the other warps' units of stage s
    da = dna;
    db = dnb;
    prev = at;
    at = nx;
    if (!__syncthreads_and(ok)) break;  // the stage's products are complete and its slot is free
    if (issued < nst) {
      issue(issued, ia);
      issued++;
      next(ia);
    }
  }
  if (ok && nst > 0) chain(nst - 1, prev);
  if (!ok)  // every copy issued has landed before the CTA's shared memory goes away (bounded)
    for (int q = s; q < issued; q++) q6m_wait(bar0 + 8 * (q % Q6M_STAGES), (uint32_t)((q / Q6M_STAGES) & 1));
}

template <int R>
__global__ void __launch_bounds__(G6_THREADS, 1) gemv_q6k_aux_kernel(KqSegs S, const int8_t* __restrict__ aq,
                                                                     const float* __restrict__ ad, uint32_t* err) {
  pdl_enter();
  extern __shared__ uint32_t g6_smem[];
  uint32_t* apair = g6_smem;                               // [G6_NBC][16 groups][8 classes]: (a[c], a[c + 8])
  uint32_t* spair = apair + G6_NBC * 128;                  // [G6_NBC][8 group pairs][8 classes]
  int* aux = reinterpret_cast<int*>(spair + G6_NBC * 64);  // [R][G6_AUX_LD]
  float* ddv = reinterpret_cast<float*>(aux + R * G6_AUX_LD);  // [R][G6_DD_LD]: d * a.d
  const KqSeg g = kq_seg(S);
  const int r0 = ((int)blockIdx.x - g.cta0) * R;
  const int nb = S.nb;
  const int t = threadIdx.x;
  const int cr = t >> 3, cc = t & 7;  // chain: row, class
  float sum = 0.0f;
  for (int b0 = 0; b0 < nb; b0 += G6_NBC) {
    const int nbc = min(G6_NBC, nb - b0);
    const int nit = R * nbc;
    // this thread's two (row, block) items: loads first
    Q6Item i0, i1;
    const int it0 = t, it1 = t + G6_THREADS;  // item it: row it % R, block it / R
    const int rw0 = r0 + it0 % R, rw1 = r0 + it1 % R;
    const bool h0 = it0 < nit && rw0 < g.rows, h1 = it1 < nit && rw1 < g.rows;
    if (h0) q6_load(g, nb, rw0, b0 + it0 / R, i0);
    if (h1) q6_load(g, nb, rw1, b0 + it1 / R, i1);
    // activation pairs of the pass: one (block, group pair) per thread
    for (int i = t; i < nbc * 8; i += G6_THREADS) {
      const int bb = i >> 3, j = i & 7;
      const uint4 v0 = *reinterpret_cast<const uint4*>(aq + (size_t)(b0 + bb) * 256 + j * 32);
      const uint4 v1 = *reinterpret_cast<const uint4*>(aq + (size_t)(b0 + bb) * 256 + j * 32 + 16);
      uint32_t* A = apair + bb * 128 + (2 * j) * 8;
#pragma unroll
      for (int c = 0; c < 8; c++) {
        const uint32_t k = (uint32_t)(c & 3);
        // bytes c and c + 8 of the group, each sign-extended to 16 bits
        const uint32_t sel = k | ((k | 8u) << 4) | ((4u + k) << 8) | (((4u + k) | 8u) << 12);
        const uint32_t a0 = prmt_sx(c < 4 ? v0.x : v0.y, c < 4 ? v0.z : v0.w, sel);
        const uint32_t a1 = prmt_sx(c < 4 ? v1.x : v1.y, c < 4 ? v1.z : v1.w, sel);
        A[c] = a0;
        A[8 + c] = a1;
        const int s0 = (int)(int16_t)(a0 & 0xffffu) + ((int)a0 >> 16);
        const int s1 = (int)(int16_t)(a1 & 0xffffu) + ((int)a1 >> 16);
        spair[bb * 64 + j * 8 + c] = s16pair(s0, s1);
      }
    }
    __syncthreads();
    if (h0) {
      const int r = it0 % R, bb = it0 / R;
      q6_aux(i0, apair + bb * 128, spair + bb * 64, aux + r * G6_AUX_LD + bb * 8);
      ddv[r * G6_DD_LD + bb] = fmul(f16_bits_to_f32((uint16_t)i0.d), ad[b0 + bb]);
    }
    if (h1) {
      const int r = it1 % R, bb = it1 / R;
      q6_aux(i1, apair + bb * 128, spair + bb * 64, aux + r * G6_AUX_LD + bb * 8);
      ddv[r * G6_DD_LD + bb] = fmul(f16_bits_to_f32((uint16_t)i1.d), ad[b0 + bb]);
    }
    __syncthreads();
    if (cr < R && r0 + cr < g.rows) {
      const int* src = aux + cr * G6_AUX_LD + cc;
      const float* dd = ddv + cr * G6_DD_LD;
      for (int bb = 0; bb < nbc; bb++) sum = fadd(sum, fmul(dd[bb], __int2float_rn(src[bb * 8])));
    }
    __syncthreads();
  }
  // ((((0 + s0) + s1) + ...) + s7) within each group of eight lanes
  float v = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; k++) v = fadd(v, __shfl_sync(0xffffffffu, sum, (t & 31 & ~7) + k));
  const int row = r0 + cr;
  if (cr < R && cc == 0 && row < g.rows) kq_store(g, row, v, err);
}

}  // namespace

bool kq_decode_supported(const DevMatrix& m) {
  return m.type == GT_Q6_K || (m.type == GT_Q4_K && m.nb <= G4_MAX_NB);
}

cudaError_t launch_gemv_kq_decode_segs(const Launch& L, const DevMatrix* const* m, int n, const DevActs& a,
                                       float* const* out, const int* epi, const float* const* bias) {
  if (n < 1 || n > 3) return cudaErrorInvalidValue;
  for (int i = 0; i < n; i++)
    if (!kq_decode_supported(*m[i])) return cudaErrorInvalidValue;
  const bool q4 = m[0]->type == GT_Q4_K;
  // Q6_K: the tensor-core kernel when the activation tables fit in shared
  // memory, else two (row, block) items per thread per pass of up to 32
  // blocks, 16 rows per CTA
  const bool q6m = !q4 && m[0]->nb <= Q6M_MAX_NB;
  const int per = q4 ? G4R_ROWS : 16;
  KqSegs S;
  S.nb = m[0]->nb;
  int ctas = 0, total = 0;  // CTAs of the per-tile kernels; rows
  for (int i = 0; i < 3; i++) {
    KqSeg& g = S.s[i];
    if (i < n) {
      if (m[i]->type != m[0]->type || m[i]->nb != S.nb) return cudaErrorInvalidValue;
      g = KqSeg{(const uint8_t*)m[i]->q, m[i]->d, m[i]->rows, ctas, out[i], epi[i], bias[i]};
      ctas += (m[i]->rows + per - 1) / per;
      total += m[i]->rows;
    } else {
      g = KqSeg{nullptr, nullptr, 0, 0x7fffffff, nullptr, EPI_STORE, nullptr};
    }
  }
  if (ctas == 0) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  const int sms = device_sms();
  if (q4) {
    if (ctas > 2 * sms) {
      if ((e = raise_smem_cap((const void*)gemv_q4k_rows_kernel<3>, g4r_smem_bytes(3, G4_MAX_NB))) == cudaSuccess)
        e = launch_k(L, gemv_q4k_rows_kernel<3>, ctas, G4R_ROWS, g4r_smem_bytes(3, S.nb), S, a.qa_q, a.qa_d,
                     L.err);
    } else if ((e = raise_smem_cap((const void*)gemv_q4k_split_kernel, g4s_smem_bytes(G4_MAX_NB))) == cudaSuccess) {
      e = launch_k(L, gemv_q4k_split_kernel, ctas, G4S_THREADS, g4s_smem_bytes(S.nb), S, a.qa_q, a.qa_d, L.err);
    }
  } else if (q6m) {
    // ceil(rows / SMs) contiguous rows per CTA
    const int per_cta = (total + sms - 1) / sms, grid = (total + per_cta - 1) / per_cta;
    if ((e = raise_smem_cap((const void*)gemv_q6k_mma_kernel, q6m_smem_bytes(Q6M_MAX_NB))) == cudaSuccess)
      e = launch_k(L, gemv_q6k_mma_kernel, grid, Q6M_THREADS, q6m_smem_bytes(S.nb), S, total, per_cta, a.qk_q,
                   a.qk_d, L.err);
  } else {
    if ((e = raise_smem_cap((const void*)gemv_q6k_aux_kernel<16>, g6_smem<16>())) == cudaSuccess)
      e = launch_k(L, gemv_q6k_aux_kernel<16>, ctas, G6_THREADS, g6_smem<16>(), S, a.qk_q, a.qk_d, L.err);
  }
  if (e != cudaSuccess) return e;
  if (L.launches) ++*L.launches;
  return cudaGetLastError();
}

cudaError_t launch_gemv_kq_decode(const Launch& L, const DevMatrix& m, const DevActs& a, float* out, int epi,
                                  const float* bias) {
  const DevMatrix* mm[1] = {&m};
  float* oo[1] = {out};
  const int ee[1] = {epi};
  const float* bb[1] = {bias};
  return launch_gemv_kq_decode_segs(L, mm, 1, a, oo, ee, bb);
}


cudaError_t launch_gemm_q4k_segs(const Launch& L, const DevMatrix* const* m, int n, const DevActs& a, int T,
                                 float* const* out, const int* out_ld, const int* epi, const float* const* bias) {
  if (n < 1 || n > 3) return cudaErrorInvalidValue;
  Q4Segs G{};
  int ctas = 0;
  for (int i = 0; i < 3; i++) {
    const int k = i < n ? i : n - 1;  // unused segments repeat the last one and own no tiles
    if (m[k]->type != GT_Q4_K || m[k]->nb != m[0]->nb) return cudaErrorInvalidValue;
    G.W[i] = static_cast<const uint8_t*>(m[k]->q);
    G.rows[i] = m[k]->rows;
    G.out[i] = out[k];
    G.out_ld[i] = out_ld[k];
    G.epi[i] = epi[k];
    G.bias[i] = bias[k];
    G.cta0[i] = i < n ? ctas : 1 << 30;
    if (i < n) ctas += (m[k]->rows + KQ_ROWS - 1) / KQ_ROWS;
  }
  const dim3 grid(ctas, (T + KQ_POS - 1) / KQ_POS);
  const cudaError_t e =
      launch_k(L, gemm_q4k_kernel, grid, KQ_THREADS, 0, G, m[0]->nb, a.qa_q, a.qa_d, T, 1.0f, L.err);
  if (e != cudaSuccess) return e;
  if (L.launches) ++*L.launches;
  return cudaGetLastError();
}

cudaError_t launch_gemm_q4k(const Launch& L, const DevMatrix& m, const DevActs& a, int T, float* out, int out_ld,
                            int epi, const float* bias) {
  const DevMatrix* mm[1] = {&m};
  float* const oo[1] = {out};
  const int ll[1] = {out_ld}, ee[1] = {epi};
  const float* const bb[1] = {bias};
  return launch_gemm_q4k_segs(L, mm, 1, a, T, oo, ll, ee, bb);
}

}  // namespace det
