// gemm_q8_tc.cu -- Q8_0 / Q4_0 x Q8A chunk GEMM on the 5th-generation tensor
// cores (tcgen05.mma kind::i8, accumulators in tensor memory).
//
// Reference: dot_q8_0_q8a / dot_q4_0_q8a (crates/det-quant/src/lib.rs:
// 237-279, 407-466).  Per 32-element block the reference forms the exact
// integer dot isum, then c = (w.d * a.d) * (f32)isum, and folds sum += c in
// block order from 0.0.  The integer dots are exact in any order, so each
// block's isums for 128 rows x 128 positions come from tcgen05 MMAs
// (M = 128, N = 64 per 64-position group, K = 32 = one block) into a fresh
// tensor-memory accumulator; the f32 folds then run in registers in block
// order, exactly as the reference does.
//
// Roles (one CTA per 128 rows x 128 positions, 18 warps):
//   warp 16       producer: one thread moves each stage (4 blocks) of weight
//                 records, weight scales, activation slabs and activation
//                 scales into a 4-slot shared-memory ring with cp.async.bulk
//                 (full mbarrier, transaction bytes);
//   warp 17       allocates 512 tensor-memory columns; one thread issues the
//                 MMAs of a block into one of 4 accumulator buffers (128
//                 columns each) and commits them to that buffer's mbarrier;
//   warps 0..15   drain: warp w reads TMEM lanes 32 (w % 4) .. + 31 (its 32
//                 rows) and columns 32 (w / 4) .. + 31 (its 32 positions)
//                 with tcgen05.ld, releases the buffer, recovers each isum
//                 exactly (|isum| <= 32 * 127 * 127 < 2^22: add 0x4B400000 to
//                 the bits, subtract 12582912.0f) and folds it.
// A ring slot is free once its MMAs have completed (tcgen05.commit) and the
// 16 drain warps have read its scales; an accumulator buffer is free once
// the 16 drain warps have read it.  Every mbarrier wait is bounded by
// %globaltimer (2 s); a timeout sets ERRF_TIMEOUT, the CTA stops, waits
// (bounded) for its copies and MMAs in flight, frees its tensor memory and
// returns without writing outputs.
//
// Operand layout: K-major with the 32-byte swizzle (row r of a tile at
// 32 r, its two 16-byte halves swapped when bit 2 of r is set).  That is the
// Q8A activation layout of dev_math.cuh as stored, so the activation slabs
// are the B operands unchanged; the weights get a copy in the same layout
// (q8_tc_repack_kernel, from the LAYOUT_MMA16 records at load): per
// (128-row tile, block) 4 KiB of int8 values, then per (tile, block) 128
// f32 scales w.d.
#include <atomic>
#include <cuda_runtime.h>

#include "dev_math.cuh"
#include "internal.h"

namespace det {
namespace {

constexpr int QT_ROWS = 128;
constexpr int QT_POS = 128;         // two Q8A groups
constexpr int QT_SB = 4;            // blocks per stage
constexpr int QT_STAGES = 4;
constexpr int QT_BUFS = 4;          // accumulator buffers of 128 columns
constexpr int QT_DRAIN = 16;        // drain warps
constexpr int QT_PRODUCER = 16;     // warp ids
constexpr int QT_MMA = 17;
constexpr int QT_THREADS = 18 * 32;
constexpr int QT_TMEM_COLS = 512;
constexpr int QT_AQ = 4096;         // bytes of a weight block tile (128 rows x 32)
constexpr int QT_BQ = 2048;         // bytes of an activation slab (64 positions x 32)
// stage layout: weight tiles [SB][4096], activation slabs [group 2][SB][2048],
// weight scales [SB][128] f32, activation scales [group 2][SB][64] f32
constexpr int QT_OFF_B = QT_SB * QT_AQ;
constexpr int QT_OFF_WS = QT_OFF_B + 2 * QT_SB * QT_BQ;
constexpr int QT_OFF_AS = QT_OFF_WS + QT_SB * QT_ROWS * 4;
constexpr int QT_STAGE = QT_OFF_AS + 2 * QT_SB * 64 * 4;
constexpr int QT_BARS = 2 * QT_STAGES + 2 * QT_BUFS + 1;  // full, empty, tfull, tempty, done
constexpr int QT_SMEM = QT_STAGE * QT_STAGES + QT_BARS * 8 + 16 + 1024;  // + tmem address, alignment slack
constexpr unsigned long long kQtWaitNs = 2000000000ull;

// instruction descriptor of tcgen05.mma kind::i8: D s32 (bits 4-5 = 2), A and
// B signed 8-bit (bits 7-9, 10-12 = 1), both K-major (bits 15, 16 = 0),
// N >> 3 at bits 17-22, M >> 4 at bits 24-28
__host__ __device__ constexpr uint32_t qt_idesc(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// shared-memory matrix descriptor: K-major, 32-byte swizzle (layout type 6,
// bits 61-63), 8-row groups 256 bytes apart (SBO, bits 32-45, in 16-byte
// units), leading offset 1 (bits 16-29; unused within one swizzle row),
// descriptor version 1 (bits 46-47), start address >> 4 (bits 0-13)
DI unsigned long long qt_sdesc(uint32_t saddr) {
  return (unsigned long long)((saddr >> 4) & 0x3fffu) | (1ull << 16) | (16ull << 32) | (1ull << 46) | (6ull << 61);
}

DI uint32_t qsu32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
DI void q_mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
DI void q_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
DI void q_arrive(uint32_t bar) { asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory"); }
DI void q_bulk(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
DI unsigned long long q_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
DI bool q_wait(uint32_t bar, uint32_t parity) {
  unsigned long long t0 = 0;
  for (unsigned it = 0;; it++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if (it == 0) t0 = q_now();
    else if ((it & 63) == 0 && q_now() - t0 > kQtWaitNs) return false;
  }
}
DI void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
DI void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
DI void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}
DI void tc_mma_i8(uint32_t dtmem, unsigned long long adesc, unsigned long long bdesc, uint32_t idesc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(dtmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}
// 32 lanes x 16 columns, without the wait: the registers are not valid until
// tc_wait16 on the same array
DI void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
// waits for every tcgen05.ld of the thread; v is an in/out operand so the
// compiler cannot read it before the wait
DI void tc_wait16(uint32_t (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                 "+r"(v[15])
               :
               : "memory");
}

// The output segment that holds matrix row `row` (segments hold multiples
// of 16 rows, except the last)
struct QtSeg {
  float* out;
  const float* bias;
  int ld, epi, row0, rows;
};
DI QtSeg qt_seg(const OutSegs& o, int row) {
  QtSeg v{o.s[0].out, o.s[0].bias, o.s[0].ld, o.s[0].epi, 0, o.s[0].rows};
  int base = o.s[0].rows;
#pragma unroll
  for (int k = 1; k < kMaxOutSegs; k++) {
    if (k < o.n && row >= base) v = QtSeg{o.s[k].out, o.s[k].bias, o.s[k].ld, o.s[k].epi, base, o.s[k].rows};
    base += o.s[k].rows;
  }
  return v;
}

__global__ void __launch_bounds__(QT_THREADS, 1)
    gemm_q8_tc_kernel(const uint8_t* __restrict__ Wq, const float* __restrict__ Ws, int rows, int nb,
                      const int8_t* __restrict__ aq, const float* __restrict__ ad, int T, const OutSegs o,
                      uint32_t* err) {
  pdl_enter();
  extern __shared__ uint8_t qt_raw[];
  // 1024-byte aligned ring (the swizzled tiles want aligned bases)
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)qt_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t bar0 = qsu32(smem + QT_STAGE * QT_STAGES);
  const uint32_t full0 = bar0, empty0 = bar0 + 8 * QT_STAGES, tfull0 = bar0 + 16 * QT_STAGES,
                 tempty0 = tfull0 + 8 * QT_BUFS, done_bar = tempty0 + 8 * QT_BUFS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + QT_STAGE * QT_STAGES + QT_BARS * 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.y, grp0 = 2 * blockIdx.x;  // 128 rows, two 64-position groups
  const int ngroups_total = (T + 63) / 64;
  const int ngroups = min(2, ngroups_total - grp0);
  const int nst = (nb + QT_SB - 1) / QT_SB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < QT_STAGES; s++) {
      q_mbar_init(full0 + 8 * s, 1);
      q_mbar_init(empty0 + 8 * s, 1 + QT_DRAIN);  // the MMAs' commit + every drain warp
    }
    for (int b = 0; b < QT_BUFS; b++) {
      q_mbar_init(tfull0 + 8 * b, 1);
      q_mbar_init(tempty0 + 8 * b, QT_DRAIN);
    }
    q_mbar_init(done_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == QT_MMA) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(qsu32(tmem_slot)),
                 "r"(QT_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == QT_PRODUCER) {
    if (lane == 0) {
      int st = 0;
      for (; st < nst; st++) {
        const int slot = st % QT_STAGES, b0 = st * QT_SB, nblk = min(QT_SB, nb - b0);
        if (st >= QT_STAGES && !q_wait(empty0 + 8 * slot, (uint32_t)((st / QT_STAGES - 1) & 1))) {
          atomicOr(err, ERRF_TIMEOUT);
          ok = false;
          break;
        }
        uint8_t* sb = smem + slot * QT_STAGE;
        const uint32_t fb = full0 + 8 * slot;
        q_expect_tx(fb, (uint32_t)(nblk * (QT_AQ + QT_ROWS * 4) + ngroups * nblk * (QT_BQ + 64 * 4)));
        q_bulk(qsu32(sb), Wq + ((size_t)tile * nb + b0) * QT_AQ, nblk * QT_AQ, fb);
        q_bulk(qsu32(sb + QT_OFF_WS), Ws + ((size_t)tile * nb + b0) * QT_ROWS, nblk * QT_ROWS * 4, fb);
        for (int g = 0; g < ngroups; g++) {
          q_bulk(qsu32(sb + QT_OFF_B + g * QT_SB * QT_BQ), aq + ((size_t)(grp0 + g) * nb + b0) * QT_BQ,
                 nblk * QT_BQ, fb);
          q_bulk(qsu32(sb + QT_OFF_AS + g * QT_SB * 64 * 4), ad + ((size_t)(grp0 + g) * nb + b0) * 64,
                 nblk * 64 * 4, fb);
        }
      }
      // the CTA's shared memory must outlive every copy issued into it
      for (int s2 = max(0, st - QT_STAGES); s2 < st; s2++)
        q_wait(full0 + 8 * (s2 % QT_STAGES), (uint32_t)((s2 / QT_STAGES) & 1));
    }
  } else if (warp == QT_MMA) {
    if (lane == 0) {
      const uint32_t idesc = qt_idesc(QT_ROWS, 64);
      int b = 0;
      for (int st = 0; st < nst && ok; st++) {
        const int slot = st % QT_STAGES, b0 = st * QT_SB, nblk = min(QT_SB, nb - b0);
        if (!q_wait(full0 + 8 * slot, (uint32_t)((st / QT_STAGES) & 1))) {
          atomicOr(err, ERRF_TIMEOUT);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint8_t* sb = smem + slot * QT_STAGE;
        for (int k = 0; k < nblk; k++, b++) {
          const int buf = b % QT_BUFS;
          if (b >= QT_BUFS && !q_wait(tempty0 + 8 * buf, (uint32_t)((b / QT_BUFS - 1) & 1))) {
            atomicOr(err, ERRF_TIMEOUT);
            ok = false;
            break;
          }
          tc_fence_after();
          const unsigned long long adesc = qt_sdesc(qsu32(sb + k * QT_AQ));
          for (int g = 0; g < ngroups; g++)
            tc_mma_i8(tmem + (uint32_t)(buf * 128 + 64 * g), adesc,
                      qt_sdesc(qsu32(sb + QT_OFF_B + g * QT_SB * QT_BQ + k * QT_BQ)), idesc);
          tc_commit(tfull0 + 8 * buf);
        }
        if (!ok) break;
        tc_commit(empty0 + 8 * slot);  // the stage's MMAs have read its tiles
      }
      // every MMA issued has completed before the tensor memory is freed
      tc_commit(done_bar);
      q_wait(done_bar, 0);
    }
  } else {
    // ---- drain warps
    const int q = warp & 3, cg = warp >> 2;  // TMEM lane quarter (rows), column group (positions)
    const int row_l = 32 * q + lane;
    const bool cols_live = cg < 2 * ngroups;  // columns of an absent group are never written
    float acc[32];
#pragma unroll
    for (int j = 0; j < 32; j++) acc[j] = 0.0f;
    // `one` comes from the host (OutSegs::one == 1.0): with a literal 1.0 the
    // compiler may turn fma(c, 1, acc) into c + acc and contract it with the
    // product before it, which would skip the product's rounding
    const float one = o.one;
    // One block b at a time, in order.  The block's 32 columns are read in
    // two 16-column halves, and each read is issued before the arithmetic
    // on the previous half, so its latency hides behind that arithmetic:
    //   ld A(b) ... wait, ld B(b), fold A(b), wait, release buffer,
    //   ld A(b + 1), fold B(b).
    // A stage's scales are released after the fold of its last block.
    // Column j of the warp's 32 is position 32 (cg & 1) + j of the group;
    // its activation scale sits at slot 8 ((j >> 1) & 3) + 2 (j >> 3) +
    // (j & 1) of the group's permuted half (q8a_sperm): half A (j < 16)
    // reads float4s 0, 2, 4, 6 of the half, half B float4s 1, 3, 5, 7.
    const uint32_t tlane = (uint32_t)(32 * q) << 16;
    auto full_wait = [&](int st) {
      if (q_wait(full0 + 8 * (st % QT_STAGES), (uint32_t)((st / QT_STAGES) & 1))) return true;
      if (lane == 0) atomicOr(err, ERRF_TIMEOUT);
      return false;
    };
    auto tfull_wait = [&](int b) {
      if (q_wait(tfull0 + 8 * (b % QT_BUFS), (uint32_t)((b / QT_BUFS) & 1))) return true;
      if (lane == 0) atomicOr(err, ERRF_TIMEOUT);
      return false;
    };
    auto fold = [&](const uint32_t (&v)[16], int b, int half) {
      const int st = b / QT_SB, k = b - st * QT_SB;
      const uint8_t* sb = smem + (st % QT_STAGES) * QT_STAGE;
      const float wd = reinterpret_cast<const float*>(sb + QT_OFF_WS)[k * QT_ROWS + row_l];
      const float4* as4 = reinterpret_cast<const float4*>(
          reinterpret_cast<const float*>(sb + QT_OFF_AS) + (cg >> 1) * QT_SB * 64 + k * 64 + 32 * (cg & 1));
      float adv[16];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float4 f = as4[2 * i + half];
        adv[4 * i] = f.x;
        adv[4 * i + 1] = f.y;
        adv[4 * i + 2] = f.z;
        adv[4 * i + 3] = f.w;
      }
#pragma unroll
      for (int jj = 0; jj < 16; jj++) {
        const int j = 16 * half + jj;
        // slot within this half's four float4s: 8u + 2a + e -> 4 (u) + (2a + e) % 4
        const int u = (j >> 1) & 3, ae = ((j >> 3) & 1) * 2 + (j & 1);
        const float isum = __fsub_rn(__uint_as_float(v[jj] + 0x4B400000u), 12582912.0f);  // exact
        const float c = __fmul_rn(__fmul_rn(wd, adv[4 * u + ae]), isum);
        acc[j] = __fmaf_rn(c, one, acc[j]);  // acc + c, rounded once
      }
    };
    if (cols_live) {
      uint32_t va[16], vb[16];
      if (nb > 0 && (ok = full_wait(0) && tfull_wait(0))) {
        tc_fence_after();
        tc_ld16(tmem + tlane + (uint32_t)(32 * cg), va);
      }
      for (int b = 0; b < nb && ok; b++) {
        const int buf = b % QT_BUFS;
        tc_wait16(va);
        tc_ld16(tmem + tlane + (uint32_t)(buf * 128 + 32 * cg + 16), vb);
        fold(va, b, 0);
        tc_wait16(vb);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) q_arrive(tempty0 + 8 * buf);
        if (b + 1 < nb) {
          if ((b + 1) % QT_SB == 0 && !full_wait((b + 1) / QT_SB)) ok = false;
          if (ok && !tfull_wait(b + 1)) ok = false;
          if (ok) {
            tc_fence_after();
            tc_ld16(tmem + tlane + (uint32_t)(((b + 1) % QT_BUFS) * 128 + 32 * cg), va);
          }
        }
        fold(vb, b, 1);
        if (b + 1 == nb || (b + 1) % QT_SB == 0) {
          __syncwarp();
          if (lane == 0) q_arrive(empty0 + 8 * ((b / QT_SB) % QT_STAGES));  // done with the stage's scales
        }
      }
      // no read of the tensor memory may be in flight past this point
      asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
    } else {
      // columns of an absent group: keep the barrier counts
      int b = 0;
      for (int st = 0; st < nst && ok; st++) {
        const int nblk = min(QT_SB, nb - st * QT_SB);
        if (!full_wait(st)) {
          ok = false;
          break;
        }
        for (int k = 0; k < nblk; k++, b++) {
          if (!tfull_wait(b)) {
            ok = false;
            break;
          }
          __syncwarp();
          if (lane == 0) q_arrive(tempty0 + 8 * (b % QT_BUFS));
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) q_arrive(empty0 + 8 * (st % QT_STAGES));
      }
    }
    // outputs of row (tile * 128 + row_l), positions grp0 * 64 + 32 cg + j
    if (__all_sync(0xffffffffu, ok) && cols_live) {
      const int row = tile * QT_ROWS + row_l;
      if (row < rows) {
        const QtSeg sg = qt_seg(o, row);
        const int lr = row - sg.row0;
#pragma unroll
        for (int j = 0; j < 32; j++) {
          {
            const int p = grp0 * 64 + 32 * cg + j;
            if (p >= T) continue;
            float v = acc[j];
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
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == QT_MMA)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(QT_TMEM_COLS)
                 : "memory");
}

// Tensor-core copy of a LAYOUT_MMA16 Q8_0 / Q4_0 matrix: per (128-row tile,
// block) the 128 rows' 32 int8 values in the 32-byte swizzled layout (row r
// at 32 r, halves swapped when bit 2 of r is set; Q4_0 nibbles as
// nibble - 8, det-quant lib.rs:455-466), then per (tile, block) the rows'
// w.d as f32.  Rows past the matrix are zeros.  One thread per (tile, block,
// row).
__global__ void q8_tc_repack_kernel(const uint8_t* __restrict__ rec, int type, int rows, int nb, int tiles,
                                    uint8_t* __restrict__ outq, float* __restrict__ outs) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)tiles * nb * QT_ROWS) return;
  const int r = (int)(i % QT_ROWS);
  const long long tb = i / QT_ROWS;
  const int b = (int)(tb % nb), tl = (int)(tb / nb);
  const int row = tl * QT_ROWS + r;
  uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float d = 0.0f;
  if (row < rows) {
    const int t16 = row >> 4, rr = row & 15, g = rr & 7, hi = rr >> 3;
    const size_t rb = type == GT_Q8_0 ? 544 : 288, qb = type == GT_Q8_0 ? 512 : 256;
    const uint8_t* R = rec + ((size_t)t16 * nb + b) * rb;
    for (int tg = 0; tg < 4; tg++) {
      const int lane = g * 4 + tg;
      if (type == GT_Q8_0) {
        // lane (g, tg): 16 B = row g cols 4tg.., row g+8 cols 4tg.., row g cols 16+4tg.., row g+8 cols 16+4tg..
        w[tg] = *reinterpret_cast<const uint32_t*>(R + lane * 16 + hi * 4);
        w[4 + tg] = *reinterpret_cast<const uint32_t*>(R + lane * 16 + 8 + hi * 4);
      } else {
        // lane (g, tg): 8 B = nibble bytes 4tg.. of rows g and g+8; element
        // j < 16 is the low nibble of byte j, j >= 16 the high nibble of j - 16
        const uint32_t nib = *reinterpret_cast<const uint32_t*>(R + lane * 8 + hi * 4);
        w[tg] = __vsub4(nib & 0x0f0f0f0fu, 0x08080808u);
        w[4 + tg] = __vsub4((nib >> 4) & 0x0f0f0f0fu, 0x08080808u);
      }
    }
    const uint32_t sw = *reinterpret_cast<const uint32_t*>(R + qb + 4 * g);
    d = f16_bits_to_f32((uint16_t)(hi ? sw >> 16 : sw & 0xffffu));
  }
  uint8_t* dst = outq + ((size_t)tl * nb + b) * QT_AQ + r * 32;
  const int swz = ((r >> 2) & 1);
  *reinterpret_cast<uint4*>(dst + 16 * swz) = make_uint4(w[0], w[1], w[2], w[3]);
  *reinterpret_cast<uint4*>(dst + 16 * (swz ^ 1)) = make_uint4(w[4], w[5], w[6], w[7]);
  outs[((size_t)tl * nb + b) * QT_ROWS + r] = d;
}

}  // namespace

size_t q8_tc_bytes(int rows, int nb) {
  const size_t tiles = (size_t)(rows + QT_ROWS - 1) / QT_ROWS;
  return tiles * nb * (QT_AQ + QT_ROWS * 4);
}

cudaError_t launch_q8_tc_repack(cudaStream_t st, const DevMatrix& m, uint8_t* out) {
  if (m.layout != LAYOUT_MMA16 || (m.type != GT_Q8_0 && m.type != GT_Q4_0)) return cudaErrorInvalidValue;
  const int tiles = (m.rows + QT_ROWS - 1) / QT_ROWS;
  const long long n = (long long)tiles * m.nb * QT_ROWS;
  float* outs = reinterpret_cast<float*>(out + (size_t)tiles * m.nb * QT_AQ);
  q8_tc_repack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(static_cast<const uint8_t*>(m.q), m.type,
                                                                     m.rows, m.nb, tiles, out, outs);
  return cudaGetLastError();
}

cudaError_t launch_gemm_q8_tc(const Launch& L, const DevMatrix& m, const DevActs& a, int T, const OutSegs& o) {
  if (!m.tc) return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> attr_set{0};  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(attr_set.load() >> dev & 1ull)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_q8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, QT_SMEM);
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set.fetch_or(1ull << dev);
  }
  const int tiles = (m.rows + QT_ROWS - 1) / QT_ROWS;
  const float* ws = reinterpret_cast<const float*>(m.tc + (size_t)tiles * m.nb * QT_AQ);
  const dim3 grid((T + QT_POS - 1) / QT_POS, tiles);
  const cudaError_t e = launch_k(L, gemm_q8_tc_kernel, grid, QT_THREADS, QT_SMEM, m.tc, ws, m.rows, m.nb, a.qa_q,
                                 a.qa_d, T, o, L.err);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace det
