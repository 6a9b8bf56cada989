// gemm.cu -- Q8_0 / Q4_0 x Q8A GEMV and teacher-forced GEMM on tensor cores.
//
// Reference: dot_q8_0_q8a / dot_q4_0_q8a (crates/det-quant/src/lib.rs:
// 237-279, 423-466).  Per 32-element block the reference computes an exact
// i32 dot `isum`, then `c = (w.d * a.d) * (isum as f32)` and folds
// `sum += c` block by block from 0.0.  Integer dots are exact in any order,
// so each block's isum comes from one int8 MMA (m16n8k32: 16 weight rows x 8
// positions x one 32-element block); the f32 fold then runs in registers in
// block order, exactly as the reference does, for every (row, position).
//
// Weight layout (repacked once at model load): 16-row tiles; per tile, per
// block, one record of
//   Q8_0: 512 B of A fragments (lane-major, 16 B per lane) + 32 B scales
//   Q4_0: 256 B of nibbles (8 B per lane)                 + 32 B scales
// where lane (g = lane/4, t = lane%4) holds rows g and g+8, columns 4t..4t+3
// and 4t+16..4t+19 of the block (the PTX m16n8k32 .s8 A-fragment map), and
// scale word g = f16 d[g] | f16 d[g+8] << 16.  A record is exactly
// 16 rows x (34 or 18) bytes, the GGUF size, so HBM bytes per weight are
// unchanged.
//
// The int32 accumulator is seeded with 0x4B400000: for |isum| < 2^22 (a
// block's |isum| <= 32*127*127) the MMA result read as f32 is
// 12582912 + isum exactly, so one FADD recovers (f32)isum.
//
// Chunk kernel (T > 8 positions): a CTA owns 32 rows (2 warps x 16-row tile)
// and 64 positions; weights, activation blocks and activation scales stream
// through a 4-stage cp.async pipeline in shared memory, so each weight byte
// leaves HBM once per chunk and the activations are shared by both warps.
// The fold epilogue (4 IEEE ops per row x position x block) runs on packed
// f32x2 instructions, each lane of which is an ordinary round-to-nearest
// f32 add or multiply.
#include <cuda_runtime.h>

#include "dev_math.cuh"
#include "internal.h"

namespace det {
namespace {

DI void mma_s8(int (&c)[4], const int (&a)[4], int b0, int b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// packed IEEE f32 pairs (sm_100): each half is one round-to-nearest op
DI unsigned long long pack2(float2 a) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a.x), "f"(a.y));
  return r;
}
DI float2 unpack2(unsigned long long r) {
  float2 a;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a.x), "=f"(a.y) : "l"(r));
  return a;
}
DI float2 add2(float2 a, float2 b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pack2(a)), "l"(pack2(b)));
  return unpack2(r);
}
DI float2 mul2(float2 a, float2 b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pack2(a)), "l"(pack2(b)));
  return unpack2(r);
}

// One fold step for two (row, position) pairs sharing a weight scale:
//   acc += (d * ad) * isum      (two roundings in the product, one in the add)
// The multiplies run packed; the accumulate uses scalar __fadd_rn, which the
// compiler never contracts with the preceding multiply into an FMA.
#ifndef DET_FOLD_VARIANT
#define DET_FOLD_VARIANT 4
#endif
DI void fold2(float2& acc, float2 d, float2 adv, float2 iv) {
#if DET_FOLD_VARIANT == 1
  acc = add2(acc, mul2(mul2(d, adv), iv));
#elif DET_FOLD_VARIANT == 4
  const float2 c = mul2(mul2(d, adv), iv);
  acc.x = __fadd_rn(acc.x, c.x);
  acc.y = __fadd_rn(acc.y, c.y);
#else
  acc.x = fadd(acc.x, fmul(fmul(d.x, adv.x), iv.x));
  acc.y = fadd(acc.y, fmul(fmul(d.y, adv.y), iv.y));
#endif
}

template <int QT>
struct Rec;
template <>
struct Rec<GT_Q8_0> {
  static constexpr int bytes = 544, qbytes = 512;
  DI static void frag(const uint8_t* r, int lane, int (&a)[4]) {
    const int4 v = *reinterpret_cast<const int4*>(r + lane * 16);
    a[0] = v.x; a[1] = v.y; a[2] = v.z; a[3] = v.w;
  }
};
template <>
struct Rec<GT_Q4_0> {
  static constexpr int bytes = 288, qbytes = 256;
  // element j < 16 is the low nibble of byte j, j >= 16 the high nibble of
  // byte j-16; values are nibble - 8 (det-quant lib.rs:455-466)
  DI static void frag(const uint8_t* r, int lane, int (&a)[4]) {
    const int2 v = *reinterpret_cast<const int2*>(r + lane * 8);
    a[0] = (int)__vsub4((unsigned)v.x & 0x0f0f0f0fu, 0x08080808u);
    a[1] = (int)__vsub4((unsigned)v.y & 0x0f0f0f0fu, 0x08080808u);
    a[2] = (int)__vsub4(((unsigned)v.x >> 4) & 0x0f0f0f0fu, 0x08080808u);
    a[3] = (int)__vsub4(((unsigned)v.y >> 4) & 0x0f0f0f0fu, 0x08080808u);
  }
};

DI float lo_half(uint32_t w) { return f16_bits_to_f32((uint16_t)(w & 0xffffu)); }
DI float hi_half(uint32_t w) { return f16_bits_to_f32((uint16_t)(w >> 16)); }

DI void store_out(float v, int r, int p, float* out, int out_ld, int epi, const float* bias, uint32_t* err) {
  if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
  float* dst = out + (size_t)p * out_ld + r;
  if (epi == EPI_BIAS) {
    v = fadd(v, bias[r]);
    if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
  } else if (epi == EPI_RESIDUAL) {
    v = fadd(*dst, v);
    if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
  }
  *dst = v;
}

// ---- small-T kernel (decode and short chunks): 4 warps per 16-row tile,
// 16 positions per warp, operands straight from global/L1 ---------------------
constexpr int SM_WARPS = 4;
constexpr int SM_POS = SM_WARPS * 16;

template <int QT>
__global__ void __launch_bounds__(SM_WARPS * 32) gemm_small_kernel(const uint8_t* __restrict__ W, int rows, int nb,
                                                                   const int8_t* __restrict__ aq,
                                                                   const float* __restrict__ ad, int T,
                                                                   float* __restrict__ out, int out_ld, int epi,
                                                                   const float* __restrict__ bias, uint32_t* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tg = lane & 3;
  const int pbase = blockIdx.y * SM_POS + warp * 16;
  if (pbase >= T) return;
  const int K = nb * 32;
  const uint8_t* rec = W + (size_t)blockIdx.x * nb * Rec<QT>::bytes;
  const int pb0 = pbase + g, pb1 = pbase + 8 + g;
  const int pc[2][2] = {{pbase + 2 * tg, pbase + 2 * tg + 1}, {pbase + 8 + 2 * tg, pbase + 8 + 2 * tg + 1}};
  const bool okb0 = pb0 < T, okb1 = pb1 < T;
  const int8_t* a0p = aq + (size_t)(okb0 ? pb0 : 0) * K + tg * 4;
  const int8_t* a1p = aq + (size_t)(okb1 ? pb1 : 0) * K + tg * 4;
  const float* adp[2][2];
#pragma unroll
  for (int n = 0; n < 2; n++)
#pragma unroll
    for (int j = 0; j < 2; j++) adp[n][j] = ad + (size_t)(pc[n][j] < T ? pc[n][j] : 0) * nb;
  float sum[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 4
  for (int b = 0; b < nb; b++) {
    const uint8_t* r = rec + (size_t)b * Rec<QT>::bytes;
    int a[4];
    Rec<QT>::frag(r, lane, a);
    const uint32_t sw = __ldg(reinterpret_cast<const uint32_t*>(r + Rec<QT>::qbytes) + g);
    const float dlo = lo_half(sw), dhi = hi_half(sw);
    const int bo = b * 32;
    const int b00 = okb0 ? __ldg(reinterpret_cast<const int*>(a0p + bo)) : 0;
    const int b01 = okb0 ? __ldg(reinterpret_cast<const int*>(a0p + bo + 16)) : 0;
    const int b10 = okb1 ? __ldg(reinterpret_cast<const int*>(a1p + bo)) : 0;
    const int b11 = okb1 ? __ldg(reinterpret_cast<const int*>(a1p + bo + 16)) : 0;
    int c0[4] = {0x4B400000, 0x4B400000, 0x4B400000, 0x4B400000};
    int c1[4] = {0x4B400000, 0x4B400000, 0x4B400000, 0x4B400000};
    mma_s8(c0, a, b00, b01);
    mma_s8(c1, a, b10, b11);
#pragma unroll
    for (int n = 0; n < 2; n++) {
      const int* c = n ? c1 : c0;
      const float ad0 = __ldg(adp[n][0] + b), ad1 = __ldg(adp[n][1] + b);
      sum[n][0] = fadd(sum[n][0], fmul(fmul(dlo, ad0), fsub(__int_as_float(c[0]), 12582912.0f)));
      sum[n][1] = fadd(sum[n][1], fmul(fmul(dlo, ad1), fsub(__int_as_float(c[1]), 12582912.0f)));
      sum[n][2] = fadd(sum[n][2], fmul(fmul(dhi, ad0), fsub(__int_as_float(c[2]), 12582912.0f)));
      sum[n][3] = fadd(sum[n][3], fmul(fmul(dhi, ad1), fsub(__int_as_float(c[3]), 12582912.0f)));
    }
  }
  const int r0 = blockIdx.x * 16 + g, r1 = r0 + 8;
#pragma unroll
  for (int n = 0; n < 2; n++)
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int r = (e < 2) ? r0 : r1;
      const int p = pc[n][e & 1];
      if (r < rows && p < T) store_out(sum[n][e], r, p, out, out_ld, epi, bias, err);
    }
}

// ---- chunk kernel: one 16-row tile x 64 positions per CTA, 4 warps of 16
// positions each, 4-stage cp.async pipeline of SB blocks per stage -------------
constexpr int CK_WARPS = 4;
constexpr int CK_NT = 2;       // n8 tiles (8 positions each) per warp
constexpr int CK_POS = CK_WARPS * CK_NT * 8;  // 64
constexpr int CK_THREADS = CK_WARPS * 32;
constexpr int CK_SB = 4;       // blocks per stage
constexpr int CK_STAGES = 4;
constexpr int ACT_STRIDE = 48; // bytes per (block, position) in smem: 32 used, padded against bank conflicts

template <int QT>
struct ChunkSmem {
  static constexpr int w_bytes = CK_SB * Rec<QT>::bytes;
  static constexpr int a_bytes = CK_SB * CK_POS * ACT_STRIDE;
  static constexpr int s_bytes = CK_SB * CK_POS * 4;
  static constexpr int stage = w_bytes + a_bytes + s_bytes;
  static constexpr int total = stage * CK_STAGES;
};

DI void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
DI void cp_async4(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem));
}
DI void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
DI void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Issue the loads of stage `st` (blocks [st*SB, st*SB+SB) clamped to nb).
// Rows beyond the matrix are padded tiles of the record array; positions
// beyond T re-read position T-1 (their outputs are never stored).
template <int QT>
DI void load_stage(uint8_t* sbuf, int st, int nb, const uint8_t* __restrict__ wtile, const int8_t* __restrict__ aq,
                   const float* __restrict__ ad, int K, int p0, int T) {
  using S = ChunkSmem<QT>;
  const int tid = threadIdx.x;
  const int b0 = st * CK_SB;
  // weights: the SB consecutive records of this tile are contiguous in HBM
  constexpr int w16 = S::w_bytes / 16;
  const int nrec = min(CK_SB, nb - b0);  // records that exist in this stage
  for (int i = tid; i < w16; i += CK_THREADS)
    if (i / (Rec<QT>::bytes / 16) < nrec)  // slots of missing records are never read
      cp_async16(sbuf + i * 16, wtile + (size_t)b0 * Rec<QT>::bytes + (size_t)i * 16);
  // activation blocks: SB x 64 positions x 32 bytes (two 16-byte pieces);
  // CK_SB * CK_POS * 2 == 4 * CK_THREADS
  uint8_t* abuf = sbuf + S::w_bytes;
#pragma unroll
  for (int k = 0; k < (CK_SB * CK_POS * 2) / CK_THREADS; k++) {
    const int i = tid + k * CK_THREADS;
    const int bb = i >> 7, p = (i & 127) >> 1, half = i & 1;
    const int b = min(b0 + bb, nb - 1);
    const int pp = min(p0 + p, T - 1);
    cp_async16(abuf + (bb * CK_POS + p) * ACT_STRIDE + half * 16, aq + (size_t)pp * K + b * 32 + half * 16);
  }
  // activation scales: SB x 64 floats (2 per thread)
  float* sbf = reinterpret_cast<float*>(sbuf + S::w_bytes + S::a_bytes);
#pragma unroll
  for (int k = 0; k < (CK_SB * CK_POS) / CK_THREADS; k++) {
    const int i = tid + k * CK_THREADS;
    const int bb = i >> 6, p = i & 63;
    const int b = min(b0 + bb, nb - 1);
    const int pp = min(p0 + p, T - 1);
    cp_async4(sbf + bb * CK_POS + p, ad + (size_t)pp * nb + b);
  }
}

template <int QT>
__global__ void __launch_bounds__(CK_THREADS) gemm_chunk_kernel(const uint8_t* __restrict__ W, int rows, int nb,
                                                                const int8_t* __restrict__ aq,
                                                                const float* __restrict__ ad, int T,
                                                                float* __restrict__ out, int out_ld, int epi,
                                                                const float* __restrict__ bias, uint32_t* err) {
  using S = ChunkSmem<QT>;
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tg = lane & 3;
  const int p0 = blockIdx.y * CK_POS;
  const int K = nb * 32;
  const uint8_t* wtile = W + (size_t)blockIdx.x * nb * Rec<QT>::bytes;
  const int nst = (nb + CK_SB - 1) / CK_SB;
  const int pw = warp * CK_NT * 8;  // this warp's first position within the CTA's 64

  float2 acc[CK_NT][2];  // [n-tile][row g | row g+8] = (pos 2tg, 2tg+1)
#pragma unroll
  for (int j = 0; j < CK_NT; j++) acc[j][0] = acc[j][1] = make_float2(0.f, 0.f);
  const float2 bias2 = make_float2(-12582912.0f, -12582912.0f);

#pragma unroll
  for (int s = 0; s < CK_STAGES - 1; s++) {
    if (s < nst) load_stage<QT>(smem + s * S::stage, s, nb, wtile, aq, ad, K, p0, T);
    cp_commit();
  }
  for (int st = 0; st < nst; st++) {
    cp_wait<CK_STAGES - 2>();
    __syncthreads();
    {
      const int ns = st + CK_STAGES - 1;
      if (ns < nst) load_stage<QT>(smem + (ns % CK_STAGES) * S::stage, ns, nb, wtile, aq, ad, K, p0, T);
      cp_commit();
    }
    const uint8_t* sbuf = smem + (st % CK_STAGES) * S::stage;
    const uint8_t* abuf = sbuf + S::w_bytes;
    const float* sbf = reinterpret_cast<const float*>(sbuf + S::w_bytes + S::a_bytes);
    const int nblk = min(CK_SB, nb - st * CK_SB);
    for (int bb = 0; bb < nblk; bb++) {
      const uint8_t* r = sbuf + bb * Rec<QT>::bytes;
      int a[4];
      Rec<QT>::frag(r, lane, a);
      const uint32_t sw = *reinterpret_cast<const uint32_t*>(r + Rec<QT>::qbytes + 4 * g);
      const float2 dlo = make_float2(lo_half(sw), lo_half(sw));
      const float2 dhi = make_float2(hi_half(sw), hi_half(sw));
      const uint8_t* ab = abuf + (bb * CK_POS + pw) * ACT_STRIDE;
      const float* sb = sbf + bb * CK_POS + pw;
#pragma unroll
      for (int j = 0; j < CK_NT; j++) {
        const uint8_t* ap = ab + (j * 8 + g) * ACT_STRIDE + tg * 4;
        const int b0v = *reinterpret_cast<const int*>(ap);
        const int b1v = *reinterpret_cast<const int*>(ap + 16);
        int c[4] = {0x4B400000, 0x4B400000, 0x4B400000, 0x4B400000};
        mma_s8(c, a, b0v, b1v);
        const float2 adv = *reinterpret_cast<const float2*>(sb + j * 8 + 2 * tg);
        const float2 i01 = add2(make_float2(__int_as_float(c[0]), __int_as_float(c[1])), bias2);
        const float2 i23 = add2(make_float2(__int_as_float(c[2]), __int_as_float(c[3])), bias2);
        fold2(acc[j][0], dlo, adv, i01);
        fold2(acc[j][1], dhi, adv, i23);
      }
    }
  }
  cp_wait<0>();
  const int r0 = blockIdx.x * 16 + g, r1 = r0 + 8;
#pragma unroll
  for (int j = 0; j < CK_NT; j++) {
    const int pa = p0 + pw + j * 8 + 2 * tg, pb = pa + 1;
    if (r0 < rows) {
      if (pa < T) store_out(acc[j][0].x, r0, pa, out, out_ld, epi, bias, err);
      if (pb < T) store_out(acc[j][0].y, r0, pb, out, out_ld, epi, bias, err);
    }
    if (r1 < rows) {
      if (pa < T) store_out(acc[j][1].x, r1, pa, out, out_ld, epi, bias, err);
      if (pb < T) store_out(acc[j][1].y, r1, pb, out, out_ld, epi, bias, err);
    }
  }
}

template <int QT>
cudaError_t launch_chunk(const Launch& L, const DevMatrix& m, const DevActs& a, int T, float* out, int out_ld,
                         int epi, const float* bias) {
  constexpr int smem = ChunkSmem<QT>::total;
  static unsigned long long attr_set = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(attr_set >> dev & 1ull)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_chunk_kernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set |= 1ull << dev;
  }
  dim3 grid((m.rows + 15) / 16, (T + CK_POS - 1) / CK_POS);
  gemm_chunk_kernel<QT><<<grid, CK_THREADS, smem, L.stream>>>((const uint8_t*)m.q, m.rows, m.nb, a.qa_q, a.qa_d, T,
                                                              out, out_ld, epi, bias, L.err);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemv_fast(const Launch& L, const DevMatrix& m, const DevActs& a, int T, float* out, int out_ld,
                             int epi, const float* bias, bool* handled) {
  *handled = false;
  if (m.layout != LAYOUT_MMA16) return cudaSuccess;
  *handled = true;
  cudaError_t e;
  if (T > 16) {
    e = m.type == GT_Q8_0 ? launch_chunk<GT_Q8_0>(L, m, a, T, out, out_ld, epi, bias)
                          : launch_chunk<GT_Q4_0>(L, m, a, T, out, out_ld, epi, bias);
  } else {
    dim3 grid((m.rows + 15) / 16, (T + SM_POS - 1) / SM_POS);
    if (m.type == GT_Q8_0)
      gemm_small_kernel<GT_Q8_0><<<grid, SM_WARPS * 32, 0, L.stream>>>(
          (const uint8_t*)m.q, m.rows, m.nb, a.qa_q, a.qa_d, T, out, out_ld, epi, bias, L.err);
    else
      gemm_small_kernel<GT_Q4_0><<<grid, SM_WARPS * 32, 0, L.stream>>>(
          (const uint8_t*)m.q, m.rows, m.nb, a.qa_q, a.qa_d, T, out, out_ld, epi, bias, L.err);
    e = cudaGetLastError();
  }
  if (L.launches) ++*L.launches;
  return e;
}

}  // namespace det
