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
// A wide matrix (more CTAs than two per SM) gets 3 ring slots, which keep
// the CTA at 30 KB so that seven fit per SM and the matrix runs in one wave;
// a narrow one gets 8, so that its few warps keep 7 super-blocks in flight.
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
  const unsigned long long w01 = fma2(dsc2, add2(pk2(m0, m1), nmag2), ndmn2);
  const unsigned long long w23 = fma2(dsc2, add2(pk2(m2, m3), nmag2), ndmn2);
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

// Activation pairs of Q8_K block b, group pair j (elements 32 j .. 32 j + 31):
// A[c] and A[8 + c] hold (a[c], a[c + 8]) of the pair's two 16-element
// groups as sign-extended 16-bit halves, Sp[c] their two sums.
DI void q6_pairs(const int8_t* __restrict__ aq, int b, int j, uint32_t* A, uint32_t* Sp) {
  const uint4 v0 = *reinterpret_cast<const uint4*>(aq + (size_t)b * 256 + j * 32);
  const uint4 v1 = *reinterpret_cast<const uint4*>(aq + (size_t)b * 256 + j * 32 + 16);
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
    Sp[c] = s16pair(s0, s1);
  }
}

// Q6_K, one position, streamed: the same integer lane sums and chains as
// gemv_q6k_aux_kernel, with the weight stream overlapping the integer work.
// A persistent CTA (one per SM) walks 32-row tiles; each tile is read in
// passes of 8 blocks, one (row, block) item of 208 bytes per thread, and
// every thread moves the item it will use in the NEXT pass into its own
// slot of a two-pass shared-memory buffer with one cp.async.bulk while it
// works on the current one (the passes run on across tile boundaries); a
// buffer's mbarrier counts the pass's bytes (thread 0 arrives with the
// expected total).  The activation's pairs for all blocks are staged once
// per CTA.  After a pass, thread (row, class) advances its f32 chain over
// the pass's blocks in order; after a tile's last pass the row's eight
// chains are summed in lane order.  Waits are bounded by %globaltimer.
constexpr int Q6S_ROWS = 32;
constexpr int Q6S_NBP = 8;  // blocks per pass
constexpr int Q6S_THREADS = Q6S_ROWS * Q6S_NBP;
constexpr int Q6S_AUX_LD = Q6S_NBP * 8 + 1;  // aux row stride (ints)
constexpr int Q6S_MAX_NB = 64;               // K <= 16384 (activation pairs staged in shared memory)
inline size_t q6s_smem_bytes(int nb) {
  return (size_t)2 * Q6S_THREADS * 208 + (size_t)nb * (128 + 64) * 4 + (size_t)Q6S_ROWS * Q6S_AUX_LD * 4 +
         (size_t)Q6S_ROWS * (Q6S_NBP + 1) * 4 + 16;
}

// the segment that holds tile `tile` (its first tile is its cta0)
DI KqSeg kq_seg_at(const KqSegs& S, int tile) {
  const int i = (int)(tile >= S.s[1].cta0) + (int)(tile >= S.s[2].cta0);
  return i == 0 ? S.s[0] : (i == 1 ? S.s[1] : S.s[2]);
}

DI bool q6s_wait(uint32_t bar, uint32_t parity) {
  unsigned long long t0 = 0;
  for (unsigned it = 0;; it++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    if (it == 0) t0 = t;
    else if (t - t0 > 2000000000ull) return false;
  }
}

__global__ void __launch_bounds__(Q6S_THREADS, 1) gemv_q6k_stream_kernel(KqSegs S, int tiles,
                                                                        const int8_t* __restrict__ aq,
                                                                        const float* __restrict__ ad,
                                                                        uint32_t* err) {
  extern __shared__ __align__(16) uint8_t q6s_smem[];
  uint8_t* items = q6s_smem;                                                      // [2][256][208]
  uint32_t* apair = reinterpret_cast<uint32_t*>(items + (size_t)2 * Q6S_THREADS * 208);  // [nb][16][8]
  const int nb = S.nb;
  uint32_t* spair = apair + (size_t)nb * 128;                                     // [nb][8][8]
  int* aux = reinterpret_cast<int*>(spair + (size_t)nb * 64);                     // [32][Q6S_AUX_LD]
  float* ddv = reinterpret_cast<float*>(aux + Q6S_ROWS * Q6S_AUX_LD);             // [32][Q6S_NBP + 1]
  const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(ddv + Q6S_ROWS * (Q6S_NBP + 1));  // [2] mbarriers
  const int t = threadIdx.x;
  const int ir = t & 31, ib = t >> 5;  // this thread's item: row ir, block ib of each pass
  const int cr = t >> 3, cc = t & 7;   // chain: row, class
  const int npass = (nb + Q6S_NBP - 1) / Q6S_NBP;
  // the passes of this CTA, in order: tile blockIdx.x + k gridDim.x, pass p
  const int my_tiles = tiles > (int)blockIdx.x ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int nq = my_tiles * npass;
  if (t == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(bar0) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(bar0 + 8) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();

  // pass q's item of this thread into buffer q & 1 (one bulk copy), and its
  // block scale; thread 0 arrives on the buffer's barrier with the pass's
  // byte count (complete_tx may come first: the count then runs negative)
  auto issue = [&](int q, uint32_t& dbits) {
    if (q >= nq) return;
    const int tile = (int)blockIdx.x + (q / npass) * (int)gridDim.x, p = q % npass, b = p * Q6S_NBP + ib;
    const KqSeg g = kq_seg_at(S, tile);
    const int r0 = (tile - g.cta0) * Q6S_ROWS, row = r0 + ir;
    const uint32_t bar = bar0 + 8 * (q & 1);
    if (t == 0) {
      const uint32_t nrow = (uint32_t)min(Q6S_ROWS, g.rows - r0), nblk = (uint32_t)min(Q6S_NBP, nb - p * Q6S_NBP);
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(nrow * nblk * 208u)
                   : "memory");
    }
    if (b < nb && row < g.rows) {
      const uint8_t* src = g.q + ((size_t)row * nb + b) * 208;
      const uint32_t dst = (uint32_t)__cvta_generic_to_shared(items + ((size_t)(q & 1) * Q6S_THREADS + t) * 208);
      // the slot was last read with ordinary loads (pass q - 2)
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], 208, [%2];\n" ::"r"(dst),
                   "l"(src), "r"(bar)
                   : "memory");
      dbits = g.d[(size_t)row * nb + b];
    }
  };
  uint32_t dnext = 0;
  issue(0, dnext);  // weights are constant: before the predecessor ends
  pdl_enter();
  for (int i = t; i < nb * 8; i += Q6S_THREADS)
    q6_pairs(aq, i >> 3, i & 7, apair + (i >> 3) * 128 + (2 * (i & 7)) * 8, spair + (i >> 3) * 64 + (i & 7) * 8);
  __syncthreads();

  float sum = 0.0f;
  bool ok = true;
  int issued = nq > 0 ? 0 : -1;  // the last pass whose copies were issued
  for (int q = 0; q < nq; q++) {
    const int tile = (int)blockIdx.x + (q / npass) * (int)gridDim.x, p = q % npass;
    const KqSeg g = kq_seg_at(S, tile);
    const int r0 = (tile - g.cta0) * Q6S_ROWS, b0 = p * Q6S_NBP;
    const uint32_t dcur = dnext;
    issue(q + 1, dnext);
    if (q + 1 < nq) issued = q + 1;
    const int b = b0 + ib;
    const bool has = b < nb && r0 + ir < g.rows;
    const float adb = has ? ad[b] : 0.0f;
    if (!q6s_wait(bar0 + 8 * (q & 1), (uint32_t)((q >> 1) & 1))) {  // pass q's items have landed
      atomicOr(err, ERRF_TIMEOUT);
      ok = false;
    }
    if (!__syncthreads_and(ok)) break;
    if (has) {
      Q6Item it;
      const uint4* src = reinterpret_cast<const uint4*>(items + ((size_t)(q & 1) * Q6S_THREADS + t) * 208);
#pragma unroll
      for (int k = 0; k < 13; k++) {
        const uint4 v = src[k];
        it.w[4 * k] = v.x;
        it.w[4 * k + 1] = v.y;
        it.w[4 * k + 2] = v.z;
        it.w[4 * k + 3] = v.w;
      }
      q6_aux(it, apair + b * 128, spair + b * 64, aux + ir * Q6S_AUX_LD + ib * 8);
      ddv[ir * (Q6S_NBP + 1) + ib] = fmul(f16_bits_to_f32((uint16_t)dcur), adb);
    }
    __syncthreads();  // aux / ddv of the pass complete
    if (r0 + cr < g.rows) {
      const int nbp = min(Q6S_NBP, nb - b0);
      const int* src = aux + cr * Q6S_AUX_LD + cc;
      const float* dd = ddv + cr * (Q6S_NBP + 1);
      for (int bb = 0; bb < nbp; bb++) sum = fadd(sum, fmul(dd[bb], __int2float_rn(src[bb * 8])));
    }
    if (p == npass - 1) {
      // ((((0 + s0) + s1) + ...) + s7) within each group of eight lanes
      float v = 0.0f;
#pragma unroll
      for (int k = 0; k < 8; k++) v = fadd(v, __shfl_sync(0xffffffffu, sum, (t & 31 & ~7) + k));
      const int row = r0 + cr;
      if (cc == 0 && row < g.rows) kq_store(g, row, v, err);
      sum = 0.0f;
    }
    __syncthreads();  // aux / ddv free for the next pass
  }
  if (!ok)  // every copy issued has landed before the CTA's shared memory goes away (bounded)
    for (int q = max(0, issued - 1); q <= issued; q++) q6s_wait(bar0 + 8 * (q & 1), (uint32_t)((q >> 1) & 1));
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
  // Q6_K: the streamed kernel when the activation pairs fit in shared memory,
  // else two (row, block) items per thread per pass of up to 32 blocks, 16
  // rows per CTA
  const bool q6s = !q4 && m[0]->nb <= Q6S_MAX_NB;
  const int per = q4 ? G4R_ROWS : (q6s ? Q6S_ROWS : 16);
  KqSegs S;
  S.nb = m[0]->nb;
  int ctas = 0;  // CTAs of the per-tile kernels, tiles of the streamed one
  for (int i = 0; i < 3; i++) {
    KqSeg& g = S.s[i];
    if (i < n) {
      if (m[i]->type != m[0]->type || m[i]->nb != S.nb) return cudaErrorInvalidValue;
      g = KqSeg{(const uint8_t*)m[i]->q, m[i]->d, m[i]->rows, ctas, out[i], epi[i], bias[i]};
      ctas += (m[i]->rows + per - 1) / per;
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
    } else if ((e = raise_smem_cap((const void*)gemv_q4k_rows_kernel<8>, g4r_smem_bytes(8, G4_MAX_NB))) ==
               cudaSuccess) {
      e = launch_k(L, gemv_q4k_rows_kernel<8>, ctas, G4R_ROWS, g4r_smem_bytes(8, S.nb), S, a.qa_q, a.qa_d, L.err);
    }
  } else if (q6s) {
    if ((e = raise_smem_cap((const void*)gemv_q6k_stream_kernel, q6s_smem_bytes(Q6S_MAX_NB))) == cudaSuccess)
      e = launch_k(L, gemv_q6k_stream_kernel, std::min(ctas, sms), Q6S_THREADS, q6s_smem_bytes(S.nb), S, ctas,
                   a.qk_q, a.qk_d, L.err);
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
