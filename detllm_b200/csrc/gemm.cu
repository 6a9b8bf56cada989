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
// unchanged, and a tile's records are contiguous.  Matrices that read the
// same activations (q/k/v, gate/up) are stored back to back as one matrix
// and run as one launch whose rows map to several outputs (OutSegs).
//
// Activations use the Q8A layout of dev_math.cuh (64-position groups,
// block-major, 16-byte-half swizzle).
//
// The int32 accumulator is seeded with 0x4B400000: for |isum| < 2^22 (a
// block's |isum| <= 32*127*127) the MMA result read as f32 is
// 12582912 + isum exactly, so one FADD recovers (f32)isum.
//
// Chunk kernel (T > 16 positions): a CTA owns two 16-row tiles and one group
// of 64 positions; each of its 4 compute warps owns 16 rows x 32 positions,
// so one A fragment feeds four MMAs, and B fragments come from shared memory
// by ldmatrix.  Each pipeline stage is SB (8) blocks: the two tiles' SB weight
// records, the SB (group, block) activation slabs and their scales --
// contiguous ranges moved by TMA bulk copies (cp.async.bulk) that a producer
// warp issues, completing on a "full" mbarrier; compute warps release a slot
// through an "empty" mbarrier.  Every mbarrier wait is bounded
// (globaltimer); on timeout the kernel flags ERRF_TIMEOUT and stops.
#include <atomic>
#include <cuda_runtime.h>

#include <algorithm>

#include "dev_math.cuh"
#include "../../include/detgpu.h"
#include "internal.h"

namespace det {
namespace {

DI void mma_s8(int (&c)[4], const int (&a)[4], int b0, int b1) {
  asm(
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

DI float2 fma2(float2 a, float2 b, float2 c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(pack2(a)), "l"(pack2(b)), "l"(pack2(c)));
  return unpack2(r);
}

// One fold step for two (row, position) pairs sharing a weight scale:
//   acc += (d * ad) * isum      (two roundings in the product, one in the add)
// The multiplies run packed.  A packed add fed by a packed multiply is
// contracted into a fused multiply-add by the code generator (one rounding
// fewer), so the add is written as fma(c, one, acc) with `one` == 1.0 a
// kernel argument: c * 1 is exact, the fma rounds once, like the add, and
// the compiler cannot see that the multiplier is 1.
DI void fold2(float2& acc, float2 d, float2 adv, float2 iv, float2 one) {
  const float2 c = mul2(mul2(d, adv), iv);
  acc = fma2(c, one, acc);
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

// The output segment that holds matrix row `row` (segments are whole tiles,
// except that the last one may end inside its last tile).
struct SegView {
  float* out;
  const float* bias;
  int ld, epi, row0, rows;
};
DI SegView seg_for(const OutSegs& o, int row) {
  SegView v{o.s[0].out, o.s[0].bias, o.s[0].ld, o.s[0].epi, 0, o.s[0].rows};
  int base = o.s[0].rows;
#pragma unroll
  for (int k = 1; k < kMaxOutSegs; k++) {
    if (k < o.n && row >= base) v = SegView{o.s[k].out, o.s[k].bias, o.s[k].ld, o.s[k].epi, base, o.s[k].rows};
    base += o.s[k].rows;
  }
  return v;
}

DI void store_out(float v, int lr, int p, const SegView& sg, uint32_t* err) {
  if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
  float* dst = sg.out + (size_t)p * sg.ld + lr;
  if (sg.epi == EPI_BIAS) {
    v = fadd(v, sg.bias[lr]);
    if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
  } else if (sg.epi == EPI_RESIDUAL) {
    v = fadd(*dst, v);
    if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
  }
  *dst = v;
}

// acc[j] holds rows (g, g+8) x positions (pbase + 8j + 2tg, +1)
template <int NJ>
DI void store_tile(const float2 (&acc)[NJ][2], int tile, int pbase, int T, const OutSegs& o, int g, int tg,
                   uint32_t* err) {
  const SegView sg = seg_for(o, tile * 16);
  const int r0 = tile * 16 - sg.row0 + g, r1 = r0 + 8;
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const int pa = pbase + 8 * j + 2 * tg, pb = pa + 1;
    if (r0 < sg.rows) {
      if (pa < T) store_out(acc[j][0].x, r0, pa, sg, err);
      if (pb < T) store_out(acc[j][0].y, r0, pb, sg, err);
    }
    if (r1 < sg.rows) {
      if (pa < T) store_out(acc[j][1].x, r1, pa, sg, err);
      if (pb < T) store_out(acc[j][1].y, r1, pb, sg, err);
    }
  }
}

// The activation scales of positions (pos + 2tg, +1) and (pos + 8 + 2tg, +1)
// of a slab (pos a multiple of 16): adjacent in the permuted scale order.
DI float4 adv_pair16(const float* sb, int pos, int tg) {
  return *reinterpret_cast<const float4*>(sb + (pos & 32) + 8 * tg + ((pos & 16) >> 2));
}

// int32 MMA results (biased) -> exact f32 isums, then the two folds
DI void fold_n8(const int (&c)[4], float2 dlo, float2 dhi, float2 adv, float2 one, float2 (&acc)[2]) {
  const float2 bias2 = make_float2(-12582912.0f, -12582912.0f);
  const float2 i01 = add2(make_float2(__int_as_float(c[0]), __int_as_float(c[1])), bias2);
  const float2 i23 = add2(make_float2(__int_as_float(c[2]), __int_as_float(c[3])), bias2);
  fold2(acc[0], dlo, adv, i01, one);
  fold2(acc[1], dhi, adv, i23, one);
}

// One n8 tile: B fragments of positions (pos .. pos+7) of block slab `ab`
// (64 x 32 B, swizzled) from global memory, and the fold into acc.
DI void n8_step(const int (&a)[4], float2 dlo, float2 dhi, const uint8_t* ab, float2 adv, int pos, int g, int tg,
                float2 one, float2 (&acc)[2]) {
  const int pl = pos + g;
  const int swz = ((pl >> 2) & 1) << 4;
  const uint8_t* ap = ab + pl * 32 + tg * 4;
  const int b0v = *reinterpret_cast<const int*>(ap + swz);
  const int b1v = *reinterpret_cast<const int*>(ap + (16 ^ swz));
  int c[4] = {0x4B400000, 0x4B400000, 0x4B400000, 0x4B400000};
  mma_s8(c, a, b0v, b1v);
  fold_n8(c, dlo, dhi, adv, one, acc);
}

// B fragments of two n8 tiles (positions pos .. pos+15 of slab `ab`) with one
// ldmatrix.x4: matrices (pos..pos+7, bytes 0-15), (pos..pos+7, 16-31),
// (pos+8..pos+15, 0-15), (pos+8..pos+15, 16-31); lane i gives the row address
// of row i%8 of matrix i/8, so the half swizzle is applied per row.
DI void ldsm_b_pair(const uint8_t* ab, int pos, int lane, int (&b)[4]) {
  const int mi = lane >> 3, p = pos + ((mi >> 1) << 3) + (lane & 7);
  const uint32_t addr = (uint32_t)__cvta_generic_to_shared(ab + p * 32 + (((mi & 1) << 4) ^ (((p >> 2) & 1) << 4)));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
               : "r"(addr));
}

// One chunk-kernel warp's work on NB blocks of a stage: 16 rows (one record
// per block) x 32 positions starting at `pos` (0 or 32), B fragments by
// ldmatrix.  All MMAs of the stage are issued first, then the folds run in
// block order, so the MMA latency overlaps the previous folds.
template <int QT, int NB>
DI void stage_blocks(const uint8_t* wbuf, const uint8_t* abuf, const float* sbf, int pos, int lane, int g, int tg,
                     float2 one, float2 (&acc)[4][2]) {
  int c[NB][4][4];
#pragma unroll
  for (int bb = 0; bb < NB; bb++) {
    int a[4];
    Rec<QT>::frag(wbuf + bb * Rec<QT>::bytes, lane, a);
    int b[2][4];
    ldsm_b_pair(abuf + bb * Q8A_GROUP * 32, pos, lane, b[0]);
    ldsm_b_pair(abuf + bb * Q8A_GROUP * 32, pos + 16, lane, b[1]);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      c[bb][j][0] = c[bb][j][1] = c[bb][j][2] = c[bb][j][3] = 0x4B400000;
      mma_s8(c[bb][j], a, b[j >> 1][2 * (j & 1)], b[j >> 1][2 * (j & 1) + 1]);
    }
  }
#pragma unroll
  for (int bb = 0; bb < NB; bb++) {
    const uint32_t sw = *reinterpret_cast<const uint32_t*>(wbuf + bb * Rec<QT>::bytes + Rec<QT>::qbytes + 4 * g);
    const float2 dlo = make_float2(lo_half(sw), lo_half(sw)), dhi = make_float2(hi_half(sw), hi_half(sw));
    const float4 s0 = adv_pair16(sbf + bb * Q8A_GROUP, pos, tg);
    const float4 s1 = adv_pair16(sbf + bb * Q8A_GROUP, pos + 16, tg);
    fold_n8(c[bb][0], dlo, dhi, make_float2(s0.x, s0.y), one, acc[0]);
    fold_n8(c[bb][1], dlo, dhi, make_float2(s0.z, s0.w), one, acc[1]);
    fold_n8(c[bb][2], dlo, dhi, make_float2(s1.x, s1.y), one, acc[2]);
    fold_n8(c[bb][3], dlo, dhi, make_float2(s1.z, s1.w), one, acc[3]);
  }
}

// A fragment + scales of one record, then NJ n8 tiles starting at `pos`
template <int QT>
DI void block_step(const uint8_t* r, const uint8_t* ab, const float* sb, int pos, int lane, int g, int tg, float2 one,
                   float2 (&acc)[2][2]) {
  int a[4];
  Rec<QT>::frag(r, lane, a);
  const uint32_t sw = __ldg(reinterpret_cast<const uint32_t*>(r + Rec<QT>::qbytes) + g);
  const float2 dlo = make_float2(lo_half(sw), lo_half(sw)), dhi = make_float2(hi_half(sw), hi_half(sw));
  const float4 s = adv_pair16(sb, pos, tg);
  n8_step(a, dlo, dhi, ab, make_float2(s.x, s.y), pos, g, tg, one, acc[0]);
  n8_step(a, dlo, dhi, ab, make_float2(s.z, s.w), pos + 8, g, tg, one, acc[1]);
}

// ---- small-T kernel (decode and short chunks): 4 warps per 16-row tile,
// 16 positions per warp, operands straight from global/L1 ---------------------
constexpr int SM_WARPS = 4;

template <int QT>
__global__ void __launch_bounds__(SM_WARPS * 32) gemm_small_kernel(const uint8_t* __restrict__ W, int nb,
                                                                   const int8_t* __restrict__ aq,
                                                                   const float* __restrict__ ad, int T,
                                                                   const OutSegs o, uint32_t* err) {
  pdl_enter();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tg = lane & 3;
  const int pw = warp * 16;  // positions pw .. pw+15 of the first 64-group
  if (pw >= T) return;
  const uint8_t* rec = W + (size_t)blockIdx.x * nb * Rec<QT>::bytes;
  float2 acc[2][2];
#pragma unroll
  for (int j = 0; j < 2; j++) acc[j][0] = acc[j][1] = make_float2(0.f, 0.f);
#pragma unroll 2
  for (int b = 0; b < nb; b++) {
    const uint8_t* ab = reinterpret_cast<const uint8_t*>(aq) + (size_t)b * Q8A_GROUP * 32;  // group 0
    const float* sb = ad + (size_t)b * Q8A_GROUP;
    block_step<QT>(rec + (size_t)b * Rec<QT>::bytes, ab, sb, pw, lane, g, tg, make_float2(o.one, o.one), acc);
  }
  store_tile<2>(acc, blockIdx.x, pw, T, o, g, tg, err);
}

// ---- chunk kernel: warp-specialised TMA bulk-copy pipeline ------------------
// Warps 0-3 compute (warp w: tile w >> 1, positions 32 * (w & 1) ..); warp 4
// is the producer, one lane of which issues the stage copies.  full[s]
// completes when stage s's bytes have landed; empty[s] when all four compute
// warps have finished with it.  No CTA-wide barrier inside the loop.
constexpr int CK_TILES = 2;   // 16-row tiles per CTA
constexpr int CK_CWARPS = 4;  // compute warps
constexpr int CK_THREADS = (CK_CWARPS + 1) * 32;
constexpr int CK_NJ = 4;      // n8 tiles per compute warp (32 positions)
// pipeline shape: SB blocks per stage, STAGES stages in flight
template <int SB_, int STAGES_>
struct CkCfg {
  static constexpr int SB = SB_, STAGES = STAGES_;
};
constexpr unsigned long long kWaitNs = 2000000000ull;  // mbarrier wait bound (2 s)

template <int QT, class C>
struct ChunkSmem {
  static constexpr int w_tile = C::SB * Rec<QT>::bytes;
  static constexpr int w_bytes = CK_TILES * w_tile;
  static constexpr int a_bytes = C::SB * Q8A_GROUP * 32;
  static constexpr int s_bytes = C::SB * Q8A_GROUP * 4;
  static constexpr int stage = w_bytes + a_bytes + s_bytes;
  static constexpr int bars = 2 * C::STAGES * 8;
  static constexpr int total = stage * C::STAGES + bars;
};

DI uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

DI void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
DI void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
DI void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
DI void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
DI unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// bounded wait for phase `parity` of the mbarrier; false on timeout
DI bool mbar_wait(uint32_t bar, uint32_t parity) {
  unsigned long long t0 = 0;
  for (unsigned it = 0;; it++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if (it == 0) t0 = globaltimer();
    else if ((it & 63) == 0 && globaltimer() - t0 > kWaitNs) return false;
  }
}

template <int QT, class C>
DI void issue_stage(uint8_t* sbuf, uint32_t bar, int st, int nb, int ntile, const uint8_t* wtile,
                    const int8_t* aslab, const float* sslab) {
  using S = ChunkSmem<QT, C>;
  const int b0 = st * C::SB, nrec = min(C::SB, nb - b0);
  const uint32_t wb = (uint32_t)(nrec * Rec<QT>::bytes), abytes = (uint32_t)(nrec * Q8A_GROUP * 32),
                 sbytes = (uint32_t)(nrec * Q8A_GROUP * 4);
  mbar_expect_tx(bar, wb * ntile + abytes + sbytes);
  for (int i = 0; i < ntile; i++)
    bulk_g2s(smem_u32(sbuf + i * S::w_tile), wtile + ((size_t)i * nb + b0) * Rec<QT>::bytes, wb, bar);
  bulk_g2s(smem_u32(sbuf + S::w_bytes), aslab + (size_t)b0 * Q8A_GROUP * 32, abytes, bar);
  bulk_g2s(smem_u32(sbuf + S::w_bytes + S::a_bytes), sslab + (size_t)b0 * Q8A_GROUP, sbytes, bar);
}

template <int QT, class C>
__global__ void __launch_bounds__(CK_THREADS) gemm_chunk_kernel(const uint8_t* __restrict__ W, int tiles, int nb,
                                                                const int8_t* __restrict__ aq,
                                                                const float* __restrict__ ad, int T,
                                                                const OutSegs o, uint32_t* err) {
  pdl_enter();
  using S = ChunkSmem<QT, C>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile0 = blockIdx.x * CK_TILES;
  const int ntile = min(CK_TILES, tiles - tile0);
  const int grp = blockIdx.y;  // 64-position group
  const int nst = (nb + C::SB - 1) / C::SB;
  const uint32_t full0 = smem_u32(smem + S::stage * C::STAGES);
  const uint32_t empty0 = full0 + 8 * C::STAGES;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, CK_CWARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();

  if (warp == CK_CWARPS) {  // ---- producer
    if (lane != 0) return;
    const uint8_t* wtile = W + (size_t)tile0 * nb * Rec<QT>::bytes;
    const int8_t* aslab = aq + (size_t)grp * nb * Q8A_GROUP * 32;
    const float* sslab = ad + (size_t)grp * nb * Q8A_GROUP;
    int st = 0;
    for (; st < nst; st++) {
      const int slot = st % C::STAGES;
      if (st >= C::STAGES && !mbar_wait(empty0 + 8 * slot, (uint32_t)((st / C::STAGES - 1) & 1))) {
        atomicOr(err, ERRF_TIMEOUT);
        break;
      }
      issue_stage<QT, C>(smem + slot * S::stage, full0 + 8 * slot, st, nb, ntile, wtile, aslab, sslab);
    }
    // the CTA's shared memory must outlive every copy issued into it
    for (int s2 = max(0, st - C::STAGES); s2 < st; s2++)
      mbar_wait(full0 + 8 * (s2 % C::STAGES), (uint32_t)((s2 / C::STAGES) & 1));
    return;
  }

  // ---- compute warps
  const int g = lane >> 2, tg = lane & 3;
  const int wt = warp >> 1;        // this warp's tile within the CTA
  const int pw = 32 * (warp & 1);  // this warp's positions within the group
  const bool active = wt < ntile && grp * Q8A_GROUP + pw < T;
  const float2 one = make_float2(o.one, o.one);
  float2 acc[CK_NJ][2];
#pragma unroll
  for (int j = 0; j < CK_NJ; j++) acc[j][0] = acc[j][1] = make_float2(0.f, 0.f);

  for (int st = 0; st < nst; st++) {
    const int slot = st % C::STAGES;
    if (!mbar_wait(full0 + 8 * slot, (uint32_t)((st / C::STAGES) & 1))) {
      if (lane == 0) atomicOr(err, ERRF_TIMEOUT);
      return;
    }
    if (active) {
      const uint8_t* sbuf = smem + slot * S::stage;
      const uint8_t* wbuf = sbuf + wt * S::w_tile;
      const uint8_t* abuf = sbuf + S::w_bytes;
      const float* sbf = reinterpret_cast<const float*>(sbuf + S::w_bytes + S::a_bytes);
      const int nblk = min(C::SB, nb - st * C::SB);
      if (nblk == C::SB) {
        stage_blocks<QT, C::SB>(wbuf, abuf, sbf, pw, lane, g, tg, one, acc);
      } else {
        for (int bb = 0; bb < nblk; bb++)
          stage_blocks<QT, 1>(wbuf + bb * Rec<QT>::bytes, abuf + bb * Q8A_GROUP * 32, sbf + bb * Q8A_GROUP, pw, lane,
                              g, tg, one, acc);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * slot);
  }
  if (active) store_tile<CK_NJ>(acc, tile0 + wt, grp * Q8A_GROUP + pw, T, o, g, tg, err);
}

template <int QT, class C>
cudaError_t launch_chunk_cfg(const Launch& L, const DevMatrix& m, const DevActs& a, int T, const OutSegs& o) {
  constexpr int smem = ChunkSmem<QT, C>::total;
  static std::atomic<unsigned long long> attr_set{0};  // one bit per device (sessions may run on several host threads)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(attr_set.load() >> dev & 1ull)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_chunk_kernel<QT, C>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set.fetch_or(1ull << dev);
  }
  const int tiles = (m.rows + 15) / 16;
  dim3 grid((tiles + CK_TILES - 1) / CK_TILES, (T + Q8A_GROUP - 1) / Q8A_GROUP);
  {
    const cudaError_t e_ = launch_k(L, gemm_chunk_kernel<QT, C>, grid, CK_THREADS, smem, (const uint8_t*)m.q, tiles,
        m.nb, a.qa_q, a.qa_d, T, o, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  return cudaGetLastError();
}

// 8 blocks per stage, 2 stages: 54 KB of shared memory, 4 CTAs per SM; the
// 32 MMAs a warp issues per stage hide their latency behind the folds
// (measured against 2..16 blocks per stage and 2..6 stages)
template <int QT>
cudaError_t launch_chunk(const Launch& L, const DevMatrix& m, const DevActs& a, int T, const OutSegs& o) {
  return launch_chunk_cfg<QT, CkCfg<8, 2>>(L, m, a, T, o);
}

// ---- decode kernel (T <= 8, e.g. one token): weight stream at HBM rate ----------
// One CTA per 16-row tile.  Thread 0 moves the tile's records (contiguous)
// into shared memory with bulk copies on one mbarrier -- in passes of at most
// DG_PASS_BYTES -- so each CTA has its whole tile in flight and several CTAs
// per SM overlap.  The per-block products c_b = (d * ad) * isum are
// independent: the 8 warps split the blocks (isums by MMA; the 8 columns are
// the positions, zero past T) and leave c_b in shared memory.  Then one
// thread per (row, position) runs the reference's ordered fold
// sum = ((0 + c_0) + c_1) + ... with its loads batched ahead of the adds.
constexpr int DG_WARPS = 8;
constexpr int DG_THREADS = DG_WARPS * 32;
constexpr int DG_PASS_BYTES = 112 * 1024;
constexpr int DG_COPY_BYTES = 32 * 1024;  // one bulk copy

template <int QT>
struct DecodeSmem {
  __host__ __device__ static int pass_recs(int nb) {
    return nb < DG_PASS_BYTES / Rec<QT>::bytes ? nb : DG_PASS_BYTES / Rec<QT>::bytes;
  }
  __host__ __device__ static int recs_bytes(int nb) { return pass_recs(nb) * Rec<QT>::bytes; }
  // products [T * 16][nb + 1] f32, then the staged activations: quants
  // [nb][T][32 B] (as stored, halves swizzled) and scales [nb][T]
  __host__ __device__ static int prod_off(int nb) { return recs_bytes(nb) + 16; }
  __host__ __device__ static int act_off(int T, int nb) { return prod_off(nb) + T * 16 * (nb + 1) * 4; }
  __host__ __device__ static int ads_off(int T, int nb) { return act_off(T, nb) + nb * T * 32; }
  __host__ __device__ static int total(int T, int nb) { return ads_off(T, nb) + nb * T * 4; }
};

template <int QT>
__global__ void __launch_bounds__(DG_THREADS) gemv_decode_kernel(const uint8_t* __restrict__ W, int nb,
                                                                 const int8_t* __restrict__ aq,
                                                                 const float* __restrict__ ad, int T,
                                                                 const OutSegs o, uint32_t* err) {
  using S = DecodeSmem<QT>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int g = lane >> 2, tg = lane & 3;
  const int precs = S::pass_recs(nb);
  const uint32_t bar = smem_u32(smem + S::recs_bytes(nb));
  float* prod = reinterpret_cast<float*>(smem + S::prod_off(nb));  // [T * 16][nb + 1]
  uint8_t* act = smem + S::act_off(T, nb);
  float* ads = reinterpret_cast<float*>(smem + S::ads_off(T, nb));
  const int ps = nb + 1;
  const uint8_t* tile = W + (size_t)blockIdx.x * nb * Rec<QT>::bytes;
  const bool col = g < T;  // B column g = position g
  const int swz = ((g >> 2) & 1) << 4;
  const float bias = -12582912.0f;

  // thread 0: bulk copies of the weight records [p0, p0 + nrec) of the tile
  auto issue = [&](int p0, int nrec) {
    const uint32_t bytes = (uint32_t)(nrec * Rec<QT>::bytes);
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    mbar_expect_tx(bar, bytes);
    for (uint32_t off = 0; off < bytes; off += DG_COPY_BYTES)
      bulk_g2s(smem_u32(smem + off), tile + (size_t)p0 * Rec<QT>::bytes + off,
               min(bytes - off, (uint32_t)DG_COPY_BYTES), bar);
  };
  if (tid == 0) {
    mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    issue(0, precs);  // weights are constant: stream them before the predecessor ends
  }
  pdl_enter();
  // the T positions' activations (group 0 of the Q8A layout), while the
  // first weight pass is in flight
  for (int i = tid; i < nb * T * 8; i += DG_THREADS) {
    const int w = i & 7, bp = i >> 3, b = bp / T, p = bp - b * T;
    reinterpret_cast<uint32_t*>(act)[i] = __ldg(reinterpret_cast<const uint32_t*>(aq + ((size_t)b * Q8A_GROUP + p) * 32) + w);
  }
  for (int i = tid; i < nb * T; i += DG_THREADS) {
    const int b = i / T, p = i - b * T;
    ads[i] = __ldg(ad + (size_t)b * Q8A_GROUP + q8a_sperm(p));
  }
  __syncthreads();
  int pass = 0;
  for (int p0 = 0; p0 < nb; p0 += precs, pass++) {
    const int nrec = min(precs, nb - p0);
    if (pass > 0 && tid == 0) issue(p0, nrec);
    const bool ok = mbar_wait(bar, (uint32_t)(pass & 1));
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        atomicOr(err, ERRF_TIMEOUT);
        mbar_wait(bar, (uint32_t)(pass & 1));  // let the copy land before the CTA exits
      }
      return;
    }
    for (int b = p0 + warp; b < p0 + nrec; b += DG_WARPS) {
      const uint8_t* r = smem + (size_t)(b - p0) * Rec<QT>::bytes;
      int a[4];
      Rec<QT>::frag(r, lane, a);
      const uint32_t sw = *reinterpret_cast<const uint32_t*>(r + Rec<QT>::qbytes + 4 * g);
      const uint8_t* abk = act + ((size_t)b * T + g) * 32;
      const int bv0 = col ? *reinterpret_cast<const int*>(abk + ((4 * tg) ^ swz)) : 0;
      const int bv1 = col ? *reinterpret_cast<const int*>(abk + ((16 + 4 * tg) ^ swz)) : 0;
      int c[4] = {0x4B400000, 0x4B400000, 0x4B400000, 0x4B400000};
      mma_s8(c, a, bv0, bv1);
      const float dl = lo_half(sw), dh = hi_half(sw);
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int p = 2 * tg + e;
        if (p < T) {
          const float adp = ads[b * T + p];
          prod[(p * 16 + g) * ps + b] = fmul(fmul(dl, adp), fadd(__int_as_float(c[e]), bias));
          prod[(p * 16 + g + 8) * ps + b] = fmul(fmul(dh, adp), fadd(__int_as_float(c[2 + e]), bias));
        }
      }
    }
    __syncthreads();  // records consumed / products complete
  }
  if (tid < 16 * T) {
    const int p = tid >> 4, rr = tid & 15;
    const float* pr = prod + (p * 16 + rr) * ps;
    float sum = 0.0f;
    int bb = 0;
    for (; bb + 8 <= nb; bb += 8) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; k++) v[k] = pr[bb + k];
#pragma unroll
      for (int k = 0; k < 8; k++) sum = fadd(sum, v[k]);
    }
    for (; bb < nb; bb++) sum = fadd(sum, pr[bb]);
    const SegView sg = seg_for(o, blockIdx.x * 16);
    const int lr = blockIdx.x * 16 - sg.row0 + rr;
    if (lr < sg.rows) store_out(sum, lr, p, sg, err);
  }
}

template <int QT>
cudaError_t launch_decode(const Launch& L, const DevMatrix& m, const DevActs& a, int T, const OutSegs& o) {
  const int smem = DecodeSmem<QT>::total(T, m.nb);
  if (cudaError_t e = raise_smem_cap((const void*)gemv_decode_kernel<QT>, smem)) return e;
  {
    const cudaError_t e_ = launch_k(L, gemv_decode_kernel<QT>, (m.rows + 15) / 16, DG_THREADS, smem,
        (const uint8_t*)m.q, m.nb, a.qa_q, a.qa_d, T, o, L.err);
    if (e_ != cudaSuccess) return e_;
  }
  return cudaGetLastError();
}

// Which chunk GEMM runs for Q8_0 / Q4_0 matrices that have tensor-core
// records: 1 the tcgen05 kernel (gemm_q8_tc.cu), 0 the mma.sync kernel
// above.  Both give the same bits.  Both are bound by the per-block f32 folds
// (four rounded operations per row, position and block), not by the integer
// dots, and the mma.sync kernel, with four CTAs of 8 warps per SM, hides
// their latency better: at TinyLlama shape and 1,024 positions its gate|up
// launch takes 157 us against 233 us, so it is the default.
std::atomic<int> g_q8_tc{0};

}  // namespace

bool q8_tensor_cores() { return g_q8_tc.load(std::memory_order_relaxed) != 0; }

cudaError_t launch_gemm_mma16(const Launch& L, const DevMatrix& m, const DevActs& a, int T, const OutSegs& o) {
  cudaError_t e;
  if (T > 16 && m.tc && q8_tensor_cores()) {
    e = launch_gemm_q8_tc(L, m, a, T, o);
  } else if (T > 16) {
    e = m.type == GT_Q8_0 ? launch_chunk<GT_Q8_0>(L, m, a, T, o) : launch_chunk<GT_Q4_0>(L, m, a, T, o);
  } else if (T <= 8 && (m.type == GT_Q8_0 ? DecodeSmem<GT_Q8_0>::total(T, m.nb)
                                           : DecodeSmem<GT_Q4_0>::total(T, m.nb)) <= 200 * 1024) {
    e = m.type == GT_Q8_0 ? launch_decode<GT_Q8_0>(L, m, a, T, o) : launch_decode<GT_Q4_0>(L, m, a, T, o);
  } else {
    const dim3 grid((m.rows + 15) / 16);
    if (m.type == GT_Q8_0)
      {
        const cudaError_t e_ = launch_k(L, gemm_small_kernel<GT_Q8_0>, grid, SM_WARPS * 32, 0, (const uint8_t*)m.q,
            m.nb, a.qa_q, a.qa_d, T, o, L.err);
        if (e_ != cudaSuccess) return e_;
      }
    else
      {
        const cudaError_t e_ = launch_k(L, gemm_small_kernel<GT_Q4_0>, grid, SM_WARPS * 32, 0, (const uint8_t*)m.q,
            m.nb, a.qa_q, a.qa_d, T, o, L.err);
        if (e_ != cudaSuccess) return e_;
      }
    e = cudaGetLastError();
  }
  if (L.launches) ++*L.launches;
  return e;
}

cudaError_t launch_gemv_fast(const Launch& L, const DevMatrix& m, const DevActs& a, int T, float* out, int out_ld,
                             int epi, const float* bias, bool* handled) {
  *handled = false;
  if (m.layout != LAYOUT_MMA16) return cudaSuccess;
  *handled = true;
  OutSegs o;
  o.n = 1;
  o.s[0] = OutSeg{m.rows, out, out_ld, epi, bias};
  return launch_gemm_mma16(L, m, a, T, o);
}

}  // namespace det

extern "C" det_status det_set_q8_tensor_cores(int enable, int* previous) {
  const int prev = det::g_q8_tc.exchange(enable ? 1 : 0, std::memory_order_relaxed);
  if (previous) *previous = prev;
  return DET_OK;
}
