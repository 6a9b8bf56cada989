// decode_fused.cu -- the one-position forward (decode) as one persistent kernel.
//
// Reference: forward_one_with_workspace (crates/det-model/src/lib.rs:1249-1400)
// for one token, with the operations of rmsnorm (:2053-2073),
// try_quantize_q8a_block (crates/det-quant/src/lib.rs:111-137),
// dot_q8_0_q8a / dot_q4_0_q8a (det-quant :237-279), add_optional_bias and
// apply_rope (det-model :1982-2051), KvCache::store (:883-913),
// attention_one_head (:2300-2418), residual_add (:1967-1980) and swiglu
// (:2420-2434).  Every value is computed by the same sequence of separately
// rounded f32 operations as the per-op kernels (kernels.cu, gemm.cu,
// attention.cu), so the logits are bit-identical to theirs; only the
// scheduling differs.
//
// One CTA per SM (cooperative launch, so all CTAs are resident) runs every
// phase of the forward:
//
//   A  RMSNorm + Q8A of x (every CTA, into shared memory), q|k|v tiles
//   B1 RoPE of q (and of k at the current position), KV store, scores
//   B2 softmax rows          B3 P.V chains
//   C  Q8A of the attention output, o tiles (+ residual)
//   D  RMSNorm + Q8A, gate|up tiles (gate rows store silu(g))
//   E  silu(g) * u + Q8A, down tiles (+ residual)
//   after the last layer: RMSNorm + Q8A, lm_head tiles
//
// with a grid barrier after each phase.  Weight tiles (16 rows in the MMA16
// record layout of gemm.cu) are dealt round robin over the CTAs in one
// global order.  A producer warp walks its CTA's tile list for the WHOLE
// forward and moves the records into a shared-memory ring with bulk copies
// (cp.async.bulk, full/empty mbarriers), so weights keep streaming while
// the CTA computes norms and attention or waits at a barrier.  Sixteen
// compute warps in four groups run the CTA's tiles side by side: per ring
// slot a group forms the block products c_b = (d * ad) * isum (exact dp4a
// integer dots) and one thread per row folds them in the reference's order.
//
// Every wait is bounded by %globaltimer (2 s): a ring slot, a grid barrier,
// the final drain of in-flight copies.  A wait that runs out sets
// ERRF_TIMEOUT and an abort word that every other wait polls, so all CTAs
// leave at their next wait; the producer lets its copies land before its
// CTA exits.
#include <cuda_runtime.h>

#include <algorithm>

#include "dev_math.cuh"
#include "internal.h"

namespace det {

namespace {

constexpr int FD_WARPS = 16;                 // compute warps
constexpr int FD_GROUPS = 4;                 // warp groups that run weight tiles independently
constexpr int FD_GW = FD_WARPS / FD_GROUPS;  // warps per group
constexpr int FD_CT = FD_WARPS * 32;         // compute threads
constexpr int FD_THREADS = FD_CT + 32;       // + one producer warp
constexpr int FD_CB = 16;                    // weight blocks per ring slot
constexpr int FD_SLOT = FD_CB * 544;         // bytes per slot (16 Q8_0 records)
constexpr int FD_PS = FD_CB + 4;             // product row stride (16-byte rows, conflict-free)
constexpr int FD_KEYS = 64;                  // keys per score item and per PV tile
constexpr int FD_PV_DIMS = 8;                // head dims per PV item
constexpr int FD_PV_STAGES = 8;              // PV tiles in flight
constexpr int FD_MAX_SLOTS = 32;
constexpr unsigned long long FD_WAIT_NS = 2000000000ull;

struct FdSmem {
  int ns, nbmax, scratch;
  __host__ __device__ int bars() const { return ns * FD_SLOT; }      // full[ns], empty[ns]
  __host__ __device__ int prod() const { return bars() + 16 * ns; }  // [FD_GROUPS][2][16 rows][FD_PS] f32
  __host__ __device__ int actq() const { return prod() + FD_GROUPS * 2 * 16 * FD_PS * 4; }  // [nbmax][32] int8
  __host__ __device__ int actd() const { return actq() + nbmax * 32; }                     // [nbmax] f32
  __host__ __device__ int scr() const { return (actd() + nbmax * 4 + 15) & ~15; }         // [scratch] f32
  __host__ __device__ int misc() const { return scr() + scratch * 4; }                     // 32 words
  __host__ __device__ int total() const { return misc() + 32 * 4; }
};

// ---- PTX helpers ----------------------------------------------------------------
DI uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
DI void mb_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
DI void mb_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
DI void mb_arrive(uint32_t bar) { asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory"); }
// non-blocking test of phase `parity`
DI bool mb_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
DI bool mb_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
DI void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// fetch [src, src + bytes) into L2 (16-byte aligned, bytes % 16 == 0)
DI void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(src), "r"(bytes) : "memory");
}
DI unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// barrier of the compute warps only (the producer warp never joins it)
DI void csync() { asm volatile("bar.sync 1, %0;\n" ::"n"(FD_CT) : "memory"); }
// the same barrier, returning whether `v` holds for any compute thread
DI bool csync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(FD_CT)
      : "memory");
  return r != 0;
}
// barrier of warp group `grp` (named barriers 2..5)
DI void gsync(int grp) { asm volatile("bar.sync %0, %1;\n" ::"r"(2 + grp), "n"(FD_GW * 32) : "memory"); }
DI bool gsync_or(int grp, bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(2 + grp), "n"(FD_GW * 32)
      : "memory");
  return r != 0;
}
DI unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
DI unsigned ld_relaxed(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// 16-byte copy global -> shared through L2 only (.cg): the source may have
// been written by another SM earlier in this kernel
DI void cpa16(void* sdst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(su32(sdst)), "l"(gsrc) : "memory");
}
DI void cpa_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
DI void cpa_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
DI void flag(uint32_t* err, uint32_t bit) { atomicOr(err, bit); }

// dst[0, n) = src[0, n) by all compute threads, every thread's loads issued
// before its stores.  CG: the source was written earlier in this kernel
// (read through L2 only); else it is constant.  n % 4 == 0, 16-byte aligned.
template <bool CG>
DI void fd_stage(float* dst, const float* src, int n) {
  const int tid = threadIdx.x, n4 = n >> 2;
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  for (int base = 0; base < n4; base += 4 * FD_CT) {
    float4 v[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int i = base + k * FD_CT + tid;
      v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < n4) v[k] = CG ? __ldcg(s4 + i) : __ldg(s4 + i);
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int i = base + k * FD_CT + tid;
      if (i < n4) d4[i] = v[k];
    }
  }
}

// ---- error / abort ------------------------------------------------------------
DI void fd_abort(unsigned* sync, uint32_t* err) {
  atomicOr(err, ERRF_TIMEOUT);
  atomicExch(sync + 1, 1u);
}
// bounded wait for phase `parity` of an mbarrier; false on timeout or when
// another CTA has aborted the forward
DI bool fd_wait(uint32_t bar, uint32_t parity, unsigned* sync, uint32_t* err) {
  if (mb_test(bar, parity)) return true;  // the common case: the slot is ready
  const unsigned long long t0 = gtime();
  for (unsigned it = 1;; it++) {
    if (mb_try(bar, parity)) return true;
    if ((it & 63) == 0) {
      if (ld_relaxed(sync + 1)) return false;
      if (gtime() - t0 > FD_WAIT_NS) {
        fd_abort(sync, err);
        return false;
      }
    }
  }
}

// the first tile of a matrix this CTA owns: tiles are dealt round robin in
// one global order (`base` = tiles of all earlier matrices of the forward)
DI int fd_first(int base) {
  const int G = gridDim.x;
  return ((int)blockIdx.x - base % G + G) % G;
}

// ---- producer: the CTA's weight tiles of the whole forward, in order -------
DI void fd_producer(const FdParams& p, uint8_t* smem, const FdSmem& sm) {
  const uint32_t full0 = su32(smem + sm.bars()), empty0 = full0 + 8 * p.ns;
  int n = 0;             // chunks issued
  int s = 0, round = 0;  // ring slot of chunk n, and passes over the ring before it
  int base = 0;
  bool ok = true;
  auto mat = [&](const FdMat& m) {
    const int tiles = (m.rows + 15) >> 4, rb = m.type == GT_Q8_0 ? 544 : 288;
    const int nch = (m.nb + FD_CB - 1) / FD_CB;
    for (int t = fd_first(base); ok && t < tiles; t += gridDim.x)
      for (int ch = 0; ch < nch; ch++) {
        // the slot's previous chunk (one pass earlier) must have been released
        if (round > 0 && !fd_wait(empty0 + 8 * s, (uint32_t)((round - 1) & 1), p.sync, p.err)) {
          ok = false;
          break;
        }
        const int b0 = ch * FD_CB, nblk = min(FD_CB, m.nb - b0);
        const uint32_t bytes = (uint32_t)(nblk * rb);
        // the compute warps read this slot through the generic proxy before
        // they released it; order those reads before the async-proxy write
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        mb_expect_tx(full0 + 8 * s, bytes);
        bulk_copy(su32(smem + (size_t)s * FD_SLOT), m.q + ((size_t)t * m.nb + b0) * rb, bytes, full0 + 8 * s);
        n++;
        if (++s == p.ns) {
          s = 0;
          round++;
        }
      }
    base += tiles;
  };
  for (int l = 0; l < p.L && ok; l++) {
    const FdLayer& Ly = p.layers[l];
    mat(Ly.qkv);
    mat(Ly.o);
    mat(Ly.gu);
    mat(Ly.down);
  }
  mat(p.out);
  // no copy may be in flight when the CTA exits: wait (bounded, ignoring
  // the abort word) for the last slots issued; on a normal run the compute
  // warps have already consumed them and these return at once
  for (int k = n > p.ns ? n - p.ns : 0; k < n; k++) {
    const uint32_t bar = full0 + 8 * (uint32_t)(k % p.ns), par = (uint32_t)((k / p.ns) & 1);
    const unsigned long long t0 = gtime();
    while (!mb_try(bar, par))
      if (gtime() - t0 > FD_WAIT_NS) {
        fd_abort(p.sync, p.err);
        break;
      }
  }
}

// ---- compute side ---------------------------------------------------------------
struct FdCtx {
  int chunk = 0;    // ring chunks of earlier tiles (position of the next)
  int base = 0;     // tiles of earlier matrices (round-robin order)
  unsigned nbar = 0;
};

// Grid barrier of the compute warps of all CTAs: arrival counter sync[0]
// (zeroed before the launch), abort word sync[1].  False when the forward
// was aborted (timeout here or elsewhere).
DI bool fd_sync(const FdParams& p, FdCtx& cx, float* misc) {
  csync();
  cx.nbar++;
  volatile int* okp = reinterpret_cast<volatile int*>(misc + 9);
  if (threadIdx.x == 0) {
    int ok = 1;
    // arrival: a release add (orders this CTA's writes, which bar.sync made
    // this thread's, before it) that does not wait for a reply
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;\n" ::"l"(p.sync) : "memory");
    const unsigned target = cx.nbar * gridDim.x;
    const unsigned long long t0 = gtime();
    for (unsigned it = 0;; it++) {
      if (ld_acquire(p.sync) >= target) break;
      if (ld_relaxed(p.sync + 1)) {
        ok = 0;
        break;
      }
      if ((it & 15) == 15 && gtime() - t0 > FD_WAIT_NS) {
        fd_abort(p.sync, p.err);
        ok = 0;
        break;
      }
    }
    __threadfence();
    *okp = ok;
  }
  csync();
  return *okp != 0;
}

// try_quantize_q8a_block (det-quant lib.rs:111-137) for up to four blocks
// held by one warp: lane l holds element l of block kb[k] (ok[k] false: no
// block).  amax = max |x| by one redux over the bit patterns (for finite
// non-negative floats the unsigned order is the float order, and max is
// order-free), d = amax / 127, q = clamp(round-half-away(x / d), +-127), as
// q8a_block_warp; the four blocks' division chains overlap.
DI void fd_q8a4(const float (&v)[4], const int (&kb)[4], const bool (&ok)[4], int l, int8_t* aq, float* ad) {
  float amax[4], d[4], sq[4];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    amax[k] = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v[k]))));
    d[k] = amax[k] != 0.0f ? fdiv(amax[k], 127.0f) : 0.0f;
  }
#pragma unroll
  for (int k = 0; k < 4; k++) sq[k] = amax[k] != 0.0f ? fdiv(v[k], d[k]) : 0.0f;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    if (!ok[k]) continue;
    int q = 0;
    if (amax[k] != 0.0f) {
      const int r = v[k] < 0.0f ? __float2int_rz(fsub(sq[k], 0.5f)) : __float2int_rz(fadd(sq[k], 0.5f));
      q = max(-127, min(127, r));
    }
    aq[kb[k] * 32 + l] = (int8_t)q;
    if (l == 0) ad[kb[k]] = d[k];
  }
}

struct FdShared {
  int8_t* aq;
  float* ad;
  float* prod;
  float* scr;
  float* misc;
  uint32_t full0, empty0;
  uint8_t* ring;
};

// Q8A of nblk blocks, four per warp at a time; value(i) gives element i
// (and flags non-finite inputs itself)
template <class F>
DI void fd_quant_blocks(int nblk, const FdShared& sh, F&& value) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int base = warp; base < nblk; base += 4 * FD_WARPS) {
    float v[4];
    int kb[4];
    bool ok[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      kb[k] = base + k * FD_WARPS;
      ok[k] = kb[k] < nblk;
      v[k] = ok[k] ? value(kb[k] * 32 + lane) : 0.0f;
    }
    fd_q8a4(v, kb, ok, lane, sh.aq, sh.ad);
  }
}

// lane-major staging: element i at row i % 8, column i / 8 of rows of
// `rs` floats (rs = columns rounded up to 32, + 4: the scattered writes of
// 32 consecutive elements hit 32 banks, and rows stay 16-byte aligned), so
// each of the eight ordered reduction lanes reads its elements as float4s
DI int fd_lane_rs(int n) { return ((((n + 7) >> 3) + 31) & ~31) + 4; }
DI float& fd_lm(float* base, int rs, int i) { return base[(i & 7) * rs + (i >> 3)]; }

// one ordered lane chain over `cnt` elements of a lane-major row:
// acc = ((0 + f(e0)) + f(e1)) + ...; SQ: f(e) = e * e, else f(e) = e
template <bool SQ>
DI float fd_lane_chain(const float* row, int cnt) {
  const float4* r4 = reinterpret_cast<const float4*>(row);
  float acc = 0.0f;
  int c = 0;
  for (; c + 16 <= cnt; c += 16) {
    float4 a[4];
#pragma unroll
    for (int k = 0; k < 4; k++) a[k] = r4[(c >> 2) + k];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float e[4] = {a[k].x, a[k].y, a[k].z, a[k].w};
#pragma unroll
      for (int u = 0; u < 4; u++) acc = fadd(acc, SQ ? fmul(e[u], e[u]) : e[u]);
    }
  }
  for (; c < cnt; c++) acc = fadd(acc, SQ ? fmul(row[c], row[c]) : row[c]);
  return acc;
}

// rmsnorm of x (p.d floats) with weights w, quantised to Q8A in shared
// memory (rmsnorm_kernel with its fused Q8A).  x is staged lane-major so the
// eight ordered sum_squares chains read float4s.
DI void fd_norm_quant(const FdParams& p, const float* w, const FdShared& sh) {
  const int tid = threadIdx.x, n = p.d, n4 = n >> 2, rs = fd_lane_rs(n);
  float* xl = sh.scr;           // [8][rs] lane-major x
  float* ws = sh.scr + 8 * rs;  // [n] weights
  const float4* x4 = reinterpret_cast<const float4*>(p.x);
  for (int base = 0; base < n4; base += 4 * FD_CT) {
    float4 v[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int i4 = base + k * FD_CT + tid;
      v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i4 < n4) v[k] = __ldcg(x4 + i4);
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int i = 4 * (base + k * FD_CT + tid);
      if (i < n) {
        fd_lm(xl, rs, i) = v[k].x;
        fd_lm(xl, rs, i + 1) = v[k].y;
        fd_lm(xl, rs, i + 2) = v[k].z;
        fd_lm(xl, rs, i + 3) = v[k].w;
      }
    }
  }
  fd_stage<false>(ws, w, n);
  csync();
  if (tid < 8) sh.misc[tid] = fd_lane_chain<true>(xl + tid * rs, (n - tid + 7) >> 3);  // sum_squares_f32_ref lanes
  csync();
  if (tid == 0) {
    const float ss = finish8(sh.misc);
    const float m = fdiv(ss, __int2float_rn(n));
    const float r = fdiv(1.0f, __fsqrt_rn(fadd(m, p.eps)));
    if (!finite(r)) flag(p.err, ERRF_NONFINITE);
    sh.misc[8] = r;
  }
  csync();
  const float r = sh.misc[8];
  fd_quant_blocks(n / 32, sh, [&](int i) {
    const float xi = fd_lm(xl, rs, i);
    const float v = fmul(fmul(xi, r), ws[i]);
    if (!finite(v) || !finite(xi)) flag(p.err, ERRF_NONFINITE);
    return v;
  });
  csync();
}

// Q8A of n floats written earlier in this forward (the attention output)
DI void fd_quant(const FdParams& p, const float* x, int n, const FdShared& sh) {
  fd_stage<true>(sh.scr, x, n);
  csync();
  fd_quant_blocks(n / 32, sh, [&](int i) {
    const float v = sh.scr[i];
    if (!finite(v)) flag(p.err, ERRF_NONFINITE);
    return v;
  });
  csync();
}

// swiglu: silu(g) * u with the Q8A of its output.  The gate rows' epilogue
// (FD_EPI_SILU) already stored silu(g), so y = silu(g) * u here, by all
// threads (loads batched ahead of the math) into shared memory; then the
// blocks are quantised.  The operations are swiglu_q8a_kernel's.
DI void fd_swiglu_quant(const FdParams& p, const FdShared& sh) {
  const int tid = threadIdx.x, n4 = p.dff >> 2;
  float* y = sh.scr;
  const float4* g4 = reinterpret_cast<const float4*>(p.gate);
  const float4* u4 = reinterpret_cast<const float4*>(p.up);
  for (int base = 0; base < n4; base += 4 * FD_CT) {
    float4 gv[4], uv[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int i = base + k * FD_CT + tid;
      gv[k] = uv[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < n4) {
        gv[k] = __ldcg(g4 + i);
        uv[k] = __ldcg(u4 + i);
      }
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int i = base + k * FD_CT + tid;
      if (i < n4) {
        const float ga[4] = {gv[k].x, gv[k].y, gv[k].z, gv[k].w}, ua[4] = {uv[k].x, uv[k].y, uv[k].z, uv[k].w};
        float ya[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
          ya[e] = fmul(ga[e], ua[e]);
          if (!finite(ya[e]) || !finite(ga[e]) || !finite(ua[e])) flag(p.err, ERRF_NONFINITE);
        }
        reinterpret_cast<float4*>(y)[i] = make_float4(ya[0], ya[1], ya[2], ya[3]);
      }
    }
  }
  csync();
  fd_quant_blocks(p.dff / 32, sh, [&](int i) { return y[i]; });
  csync();
}

// output rows of a matrix: consecutive segments, each stored as the GEMV
// epilogues of gemm.cu do (store_out); FD_EPI_SILU stores silu(sum) (the
// gate rows: SwiGLU then only multiplies by up)
constexpr int FD_EPI_SILU = 3;
struct FdOut {
  float* out;
  const float* bias;
  int rows, epi;
};
struct FdEpi {
  FdOut s[3];
  int n;
};

DI void fd_store(const FdEpi& e, int row, float v, uint32_t* err) {
  int k = 0, r = row;
  while (k + 1 < e.n && r >= e.s[k].rows) {
    r -= e.s[k].rows;
    k++;
  }
  const FdOut o = e.s[k];
  if (!finite(v)) flag(err, ERRF_NONFINITE);
  float* dst = o.out + r;
  if (o.epi == EPI_BIAS) {
    v = fadd(v, o.bias[r]);
    if (!finite(v)) flag(err, ERRF_NONFINITE);
  } else if (o.epi == EPI_RESIDUAL) {
    v = fadd(__ldcg(dst), v);
    if (!finite(v)) flag(err, ERRF_NONFINITE);
  } else if (o.epi == FD_EPI_SILU) {
    v = silu_det(v);
  }
  *dst = v;
}

// Tile t of matrix m, run by warp group `grp`; its chunks are ring
// positions c0 .. c0 + nch - 1.  Per 16-block chunk the group's four warps
// form the block products c_b = (d * ad) * isum of the tile's 16 rows into
// one of the group's two product buffers, then release the slot; lanes
// 0..15 of the group's first warp fold the previous chunk's products into
// their row sums meanwhile, in block order: sum = ((0 + c_0) + c_1) + ...
// (gemv_decode_kernel at T = 1).  A warp's block: lane (g, t) holds the
// A-fragment bytes of rows g and g + 8, columns 4t..4t+3 and 16+4t..16+4t+3
// (the record layout of gemm.cu); four dp4a and two lane shuffles give the
// exact integer isum of both rows (integer sums are exact in any order),
// and (float)isum is exact (|isum| <= 32 * 127 * 127 < 2^24).
DI bool fd_tile(const FdParams& p, const FdMat& m, int t, int c0, const FdEpi& ep, const FdShared& sh, int grp) {
  const int lane = threadIdx.x & 31, gw = (threadIdx.x >> 5) % FD_GW, g = lane >> 2, tg = lane & 3;
  const bool q8 = m.type == GT_Q8_0;
  const int rb = q8 ? 544 : 288, qb = q8 ? 512 : 256;
  const int nb = m.nb, nch = (nb + FD_CB - 1) / FD_CB;
  float* buf = sh.prod + grp * 2 * 16 * FD_PS;  // [2][16 rows][FD_PS]
  const bool folder = gw == 0 && lane < 16;    // row `lane` of the tile
  float sum = 0.0f;
  auto fold = [&](int ch) {  // the products of chunk ch, in block order
    const float* r = buf + (ch & 1) * 16 * FD_PS + lane * FD_PS;
    const int n = min(FD_CB, nb - ch * FD_CB);
    if (n == FD_CB) {
      const float4* r4 = reinterpret_cast<const float4*>(r);
      float4 v[FD_CB / 4];
#pragma unroll
      for (int k = 0; k < FD_CB / 4; k++) v[k] = r4[k];
#pragma unroll
      for (int k = 0; k < FD_CB / 4; k++) {
        sum = fadd(sum, v[k].x);
        sum = fadd(sum, v[k].y);
        sum = fadd(sum, v[k].z);
        sum = fadd(sum, v[k].w);
      }
    } else {
      for (int k = 0; k < n; k++) sum = fadd(sum, r[k]);
    }
  };
  for (int ch = 0; ch < nch; ch++) {
    const int c = c0 + ch, s = c % p.ns;
    const bool ok = fd_wait(sh.full0 + 8 * s, (uint32_t)((c / p.ns) & 1), p.sync, p.err);
    // the group agrees on a failed wait (timeout or abort) and stops; this
    // barrier also orders the previous chunk's products before their fold
    if (gsync_or(grp, !ok)) return false;
    if (folder && ch > 0) fold(ch - 1);
    const uint8_t* slot = sh.ring + (size_t)s * FD_SLOT;
    float* pb = buf + (ch & 1) * 16 * FD_PS;
    const int b0 = ch * FD_CB, nblk = min(FD_CB, nb - b0);
#pragma unroll 2
    for (int bi = gw; bi < nblk; bi += FD_GW) {
      const uint8_t* r = slot + bi * rb;
      const int b = b0 + bi;
      int a[4];
      if (q8) {
        const int4 v = *reinterpret_cast<const int4*>(r + lane * 16);
        a[0] = v.x;
        a[1] = v.y;
        a[2] = v.z;
        a[3] = v.w;
      } else {  // Q4_0: element j < 16 low nibble of byte j, else high nibble; nibble - 8
        const int2 v = *reinterpret_cast<const int2*>(r + lane * 8);
        a[0] = (int)__vsub4((unsigned)v.x & 0x0f0f0f0fu, 0x08080808u);
        a[1] = (int)__vsub4((unsigned)v.y & 0x0f0f0f0fu, 0x08080808u);
        a[2] = (int)__vsub4(((unsigned)v.x >> 4) & 0x0f0f0f0fu, 0x08080808u);
        a[3] = (int)__vsub4(((unsigned)v.y >> 4) & 0x0f0f0f0fu, 0x08080808u);
      }
      const uint32_t sw = *reinterpret_cast<const uint32_t*>(r + qb + 4 * g);
      const int blo = *reinterpret_cast<const int*>(sh.aq + b * 32 + 4 * tg);
      const int bhi = *reinterpret_cast<const int*>(sh.aq + b * 32 + 16 + 4 * tg);
      int s0 = __dp4a(a[0], blo, __dp4a(a[2], bhi, 0));  // row g
      int s1 = __dp4a(a[1], blo, __dp4a(a[3], bhi, 0));  // row g + 8
      s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
      s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
      s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
      s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
      if (tg == 0) {
        const float adp = sh.ad[b];
        const float dl = f16_bits_to_f32((uint16_t)(sw & 0xffffu)), dh = f16_bits_to_f32((uint16_t)(sw >> 16));
        pb[g * FD_PS + bi] = fmul(fmul(dl, adp), __int2float_rn(s0));
        pb[(g + 8) * FD_PS + bi] = fmul(fmul(dh, adp), __int2float_rn(s1));
      }
    }
    __syncwarp();
    if (lane == 0) mb_arrive(sh.empty0 + 8 * s);
  }
  gsync(grp);  // the last chunk's products
  if (folder) {
    fold(nch - 1);
    const int row = t * 16 + lane;
    if (row < m.rows) fd_store(ep, row, sum, p.err);
  }
  return true;
}

// The CTA's tiles of matrix m (prologue first: the activation they read);
// its k-th tile goes to warp group k % FD_GROUPS, so groups run tiles side
// by side.  Tile k's chunks are ring positions cx.chunk + k * nch onwards
// (the producer issues the CTA's tiles in this order).
template <class Pro>
DI bool fd_matrix(const FdParams& p, const FdMat& m, const FdEpi& ep, Pro&& prologue, const FdShared& sh,
                  FdCtx& cx) {
  const int tiles = (m.rows + 15) >> 4, G = gridDim.x;
  const int t0 = fd_first(cx.base), nch = (m.nb + FD_CB - 1) / FD_CB;
  const int mine = t0 < tiles ? (tiles - t0 + G - 1) / G : 0;
  bool ok = true;
  if (mine > 0) {
    prologue();
    const int grp = (threadIdx.x >> 5) / FD_GW;
    bool bad = false;
    for (int k = grp; !bad && k < mine; k += FD_GROUPS)
      bad = !fd_tile(p, m, t0 + k * G, cx.chunk + k * nch, ep, sh, grp);
    ok = !csync_or(bad);  // every group done; all agree on a failure
    cx.chunk += mine * nch;
  }
  cx.base += tiles;
  return ok;
}

// B1: items (KV head, 64-key tile).  Each item rotates the group's query
// rows (apply_rope, as rope_store_kernel), takes keys j < pos from the
// cache and key pos from this forward's k (rotated here), stores k and v of
// position pos when the tile holds it, and writes the scores
// s_j = dot_f32_ref(q, k_j) * scale (8 ordered lane chains, finish_8lane).
DI void fd_scores(const FdParams& p, float* kc, float* vc, int pos, const FdShared& sh) {
  const int tid = threadIdx.x;
  const int len = pos + 1, ntile = (len + FD_KEYS - 1) / FD_KEYS, gsz = p.nh / p.nkv, hd = p.hd, kst = hd + 1;
  float* qs = sh.scr;             // [gsz][hd]
  float* ks = sh.scr + gsz * hd;  // [FD_KEYS][hd + 1]
  const float* cs = p.cos_t + (size_t)pos * p.half;
  const float* sn = p.sin_t + (size_t)pos * p.half;
  for (int it = blockIdx.x; it < p.nkv * ntile; it += gridDim.x) {
    const int kvh = it / ntile, kt = it - kvh * ntile, j0 = kt * FD_KEYS, nk = min(FD_KEYS, len - j0);
    const bool has_pos = j0 + nk == len;
    for (int e = tid; e < gsz * hd / 4; e += FD_CT)
      reinterpret_cast<float4*>(qs)[e] = __ldcg(reinterpret_cast<const float4*>(p.q + (size_t)kvh * gsz * hd) + e);
    for (int e = tid; e < nk * (hd / 4); e += FD_CT) {
      const int jj = e / (hd / 4), d4 = (e - jj * (hd / 4)) * 4, j = j0 + jj;
      const float* src = j < pos ? kc + ((size_t)kvh * p.n_ctx + j) * hd + d4 : p.k + (size_t)kvh * hd + d4;
      const float4 v = __ldcg(reinterpret_cast<const float4*>(src));
      float* dst = ks + jj * kst + d4;
      dst[0] = v.x;
      dst[1] = v.y;
      dst[2] = v.z;
      dst[3] = v.w;
    }
    csync();
    const int nq = gsz * p.half, nr = nq + (has_pos ? p.half : 0);
    for (int e = tid; e < nr; e += FD_CT) {
      float* base;
      int j;
      if (e < nq) {
        const int r = e / p.half;
        j = e - r * p.half;
        base = qs + r * hd;
      } else {
        j = e - nq;
        base = ks + (pos - j0) * kst;
      }
      int a, b;
      if (p.pairing == 0) {
        a = 2 * j;
        b = a + 1;
      } else {
        a = j;
        b = j + p.half;
      }
      const float x0 = base[a], x1 = base[b];
      const float c = cs[j], s = sn[j];
      const float y0 = fsub(fmul(x0, c), fmul(x1, s));
      const float y1 = fadd(fmul(x0, s), fmul(x1, c));
      if (!finite(y0) || !finite(y1) || !finite(x0) || !finite(x1)) flag(p.err, ERRF_NONFINITE);
      base[a] = y0;
      base[b] = y1;
    }
    csync();
    if (has_pos)
      for (int dd = tid; dd < hd; dd += FD_CT) {
        const size_t off = ((size_t)kvh * p.n_ctx + pos) * hd + dd;
        const float kv = ks[(pos - j0) * kst + dd], vv = __ldcg(p.v + (size_t)kvh * hd + dd);
        if (!finite(kv) || !finite(vv)) flag(p.err, ERRF_NONFINITE);
        kc[off] = kv;
        vc[off] = vv;
      }
    if (len > 1)
      for (int e = tid; e < gsz * FD_KEYS; e += FD_CT) {
        const int r = e / FD_KEYS, jj = e - r * FD_KEYS;
        if (jj >= nk) continue;
        const float* qr = qs + r * hd;
        const float* kr = ks + jj * kst;
        float acc[8];
#pragma unroll
        for (int l = 0; l < 8; l++) acc[l] = 0.0f;
        for (int i = 0; i < hd; i += 8) {
#pragma unroll
          for (int l = 0; l < 8; l++) acc[l] = fadd(acc[l], fmul(qr[i + l], kr[i + l]));
        }
        const float sc = fmul(finish8(acc), p.scale);
        if (!finite(sc)) flag(p.err, ERRF_NONFINITE);
        p.S[(size_t)(kvh * gsz + r) * p.s_ld + j0 + jj] = sc;
      }
    csync();  // qs / ks are reused by the next item
  }
}

// B2: one CTA per head row: max, e_j = expf(max(s_j - m, -88)), the eight
// ordered Z chains, p_j = e_j / Z written back (attn_softmax_row_kernel).
// The row is staged lane-major so each Z lane chain reads float4s.
DI void fd_softmax(const FdParams& p, int pos, const FdShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int len = pos + 1, rs = fd_lane_rs(len);
  if (len == 1) return;  // score_len == 1 copies v_0 (no scores)
  float* el = sh.scr;  // [8][rs]
  float* red = sh.misc + 16;
  for (int h = blockIdx.x; h < p.nh; h += gridDim.x) {
    float* s = p.S + (size_t)h * p.s_ld;
    float mx = -INFINITY;
    for (int j = tid; j < len; j += FD_CT) {
      const float v = __ldcg(s + j);
      fd_lm(el, rs, j) = v;
      mx = fmaxf(mx, v);
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    csync();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < FD_WARPS; w++) mx = fmaxf(mx, red[w]);
    for (int j = tid; j < len; j += FD_CT) {
      float& e = fd_lm(el, rs, j);
      const float d = fsub(e, mx);
      e = expf_det(d > -88.0f ? d : -88.0f);
    }
    csync();
    if (tid < 8) sh.misc[tid] = fd_lane_chain<false>(el + tid * rs, (len - tid + 7) >> 3);  // sum_f32_ref lanes
    csync();
    const float z = finish8(sh.misc);
    if (!finite(z) || z == 0.0f) {
      if (tid == 0) flag(p.err, ERRF_NONFINITE);
    } else {
      for (int j = tid; j < len; j += FD_CT) {
        const float pv = fdiv(fd_lm(el, rs, j), z);
        if (!finite(pv)) flag(p.err, ERRF_NONFINITE);
        s[j] = pv;
      }
    }
    csync();  // el / misc are reused by the next head
  }
}

// B3: items (KV head, 8 dims): one ordered chain o[d] += p_j * v_j[d] per
// (query head, dim), j ascending, over 64-key tiles of P and V staged with
// cp.async, FD_PV_STAGES tiles in flight (attn_pv_decode_kernel)
DI void fd_pv(const FdParams& p, const float* vc, int pos, const FdShared& sh) {
  const int tid = threadIdx.x;
  const int len = pos + 1, gsz = p.nh / p.nkv, hd = p.hd, nds = hd / FD_PV_DIMS;
  const int stage_f = gsz * FD_KEYS + FD_KEYS * FD_PV_DIMS;
  const int h = tid / FD_PV_DIMS, dd = tid - h * FD_PV_DIMS;
  const bool chain = tid < gsz * FD_PV_DIMS;
  for (int it = blockIdx.x; it < p.nkv * nds; it += gridDim.x) {
    const int kvh = it / nds, d0 = (it - kvh * nds) * FD_PV_DIMS;
    const float* vb = vc + (size_t)kvh * p.n_ctx * hd;
    float* ob = p.attn + (size_t)(kvh * gsz + h) * hd + d0 + dd;
    if (len == 1) {  // score_len == 1 copies v_0 (lib.rs:2319-2322)
      if (chain) *ob = __ldcg(vb + d0 + dd);
      continue;
    }
    const float* prow0 = p.S + (size_t)kvh * gsz * p.s_ld;
    const int ntile = (len + FD_KEYS - 1) / FD_KEYS;
    auto load = [&](int k) {
      if (k < ntile) {
        const int jc = k * FD_KEYS;
        float* pb = sh.scr + (k % FD_PV_STAGES) * stage_f;
        float* vbuf = pb + gsz * FD_KEYS;
        for (int i = tid; i < gsz * (FD_KEYS / 4); i += FD_CT) {
          const int r = i / (FD_KEYS / 4), c4 = (i - r * (FD_KEYS / 4)) * 4;
          if (jc + c4 < len) cpa16(pb + r * FD_KEYS + c4, prow0 + (size_t)r * p.s_ld + jc + c4);
        }
        for (int i = tid; i < FD_KEYS * (FD_PV_DIMS / 4); i += FD_CT) {
          const int jj = i / (FD_PV_DIMS / 4), c4 = (i - jj * (FD_PV_DIMS / 4)) * 4;
          if (jc + jj < len) cpa16(vbuf + jj * FD_PV_DIMS + c4, vb + (size_t)(jc + jj) * hd + d0 + c4);
        }
      }
      cpa_commit();  // an empty group past the last tile keeps the wait count uniform
    };
    float acc = 0.0f;
    for (int k = 0; k < FD_PV_STAGES - 1; k++) load(k);
    for (int k = 0; k < ntile; k++) {
      load(k + FD_PV_STAGES - 1);
      cpa_wait<FD_PV_STAGES - 1>();  // tile k has landed
      csync();
      if (chain) {
        const float* pb = sh.scr + (k % FD_PV_STAGES) * stage_f;
        const float* pr = pb + h * FD_KEYS;
        const float* vr = pb + gsz * FD_KEYS + dd;
        const int nj = min(FD_KEYS, len - k * FD_KEYS);
        if (nj == FD_KEYS) {
          // 16 keys at a time: operands and products first, then the 16
          // ordered adds (the chain only waits on its own adds)
#pragma unroll
          for (int j0 = 0; j0 < FD_KEYS; j0 += 16) {
            float pv[16];
#pragma unroll
            for (int jj = 0; jj < 16; jj++) pv[jj] = fmul(pr[j0 + jj], vr[(j0 + jj) * FD_PV_DIMS]);
#pragma unroll
            for (int jj = 0; jj < 16; jj++) acc = fadd(acc, pv[jj]);
          }
        } else {
          for (int jj = 0; jj < nj; jj++) acc = fadd(acc, fmul(pr[jj], vr[jj * FD_PV_DIMS]));
        }
      }
      csync();  // stage k % FD_PV_STAGES is refilled by a later load
    }
    if (chain) {
      if (!finite(acc)) flag(p.err, ERRF_NONFINITE);
      *ob = acc;
    }
  }
}

__global__ void __launch_bounds__(FD_THREADS, 1) decode_fused_kernel(const FdParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const FdSmem sm{p.ns, p.nbmax, p.scratch};
  FdShared sh;
  sh.ring = smem;
  sh.full0 = su32(smem + sm.bars());
  sh.empty0 = sh.full0 + 8 * p.ns;
  sh.prod = reinterpret_cast<float*>(smem + sm.prod());
  sh.aq = reinterpret_cast<int8_t*>(smem + sm.actq());
  sh.ad = reinterpret_cast<float*>(smem + sm.actd());
  sh.scr = reinterpret_cast<float*>(smem + sm.scr());
  sh.misc = reinterpret_cast<float*>(smem + sm.misc());
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.ns; s++) {
      mb_init(sh.full0 + 8 * s, 1);
      mb_init(sh.empty0 + 8 * s, FD_GW);  // one chunk is consumed by one warp group
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x >= FD_CT) {
    if (threadIdx.x == FD_CT) fd_producer(p, smem, sm);
    return;
  }
  const int pos = *p.pos;
  FdCtx cx;
  const int qd = p.nh * p.hd, kvd = p.nkv * p.hd;
  for (int l = 0; l < p.L; l++) {
    const FdLayer& Ly = p.layers[l];
    const size_t kv_layer = (size_t)p.nkv * p.n_ctx * p.hd;
    float* kc = p.kc + (size_t)l * kv_layer;
    float* vc = p.vc + (size_t)l * kv_layer;
    if (threadIdx.x == 0 && pos > 0) {
      // the K and V rows 0..pos-1 this layer's attention reads, 64 rows per
      // item, into L2 while phase A runs
      const int ntile = (pos + FD_KEYS - 1) / FD_KEYS;
      for (int it = blockIdx.x; it < 2 * p.nkv * ntile; it += gridDim.x) {
        const int kv = it / (p.nkv * ntile), r = it - kv * p.nkv * ntile, h = r / ntile, j0 = (r - h * ntile) * FD_KEYS;
        const float* base = (kv ? vc : kc) + ((size_t)h * p.n_ctx + j0) * p.hd;
        bulk_prefetch_l2(base, (uint32_t)(min(FD_KEYS, pos - j0) * p.hd * 4));
      }
    }
    // A: q | k | v with their bias epilogues
    FdEpi eq;
    eq.n = 3;
    eq.s[0] = FdOut{p.q, Ly.bq, qd, Ly.bq ? EPI_BIAS : EPI_STORE};
    eq.s[1] = FdOut{p.k, Ly.bk, kvd, Ly.bk ? EPI_BIAS : EPI_STORE};
    eq.s[2] = FdOut{p.v, Ly.bv, kvd, Ly.bv ? EPI_BIAS : EPI_STORE};
    if (!fd_matrix(p, Ly.qkv, eq, [&] { fd_norm_quant(p, Ly.attn_norm, sh); }, sh, cx)) return;
    if (!fd_sync(p, cx, sh.misc)) return;
    // B: attention over the layer's KV cache
    fd_scores(p, kc, vc, pos, sh);
    if (!fd_sync(p, cx, sh.misc)) return;
    fd_softmax(p, pos, sh);
    if (!fd_sync(p, cx, sh.misc)) return;
    fd_pv(p, vc, pos, sh);
    if (!fd_sync(p, cx, sh.misc)) return;
    // C: o tiles, residual into x
    FdEpi ex;
    ex.n = 1;
    ex.s[0] = FdOut{p.x, nullptr, p.d, EPI_RESIDUAL};
    if (!fd_matrix(p, Ly.o, ex, [&] { fd_quant(p, p.attn, qd, sh); }, sh, cx)) return;
    if (!fd_sync(p, cx, sh.misc)) return;
    // D: gate | up (gate rows store silu(g))
    FdEpi eg;
    eg.n = 2;
    eg.s[0] = FdOut{p.gate, nullptr, p.dff, FD_EPI_SILU};
    eg.s[1] = FdOut{p.up, nullptr, p.dff, EPI_STORE};
    if (!fd_matrix(p, Ly.gu, eg, [&] { fd_norm_quant(p, Ly.ffn_norm, sh); }, sh, cx)) return;
    if (!fd_sync(p, cx, sh.misc)) return;
    // E: down, residual into x
    if (!fd_matrix(p, Ly.down, ex, [&] { fd_swiglu_quant(p, sh); }, sh, cx)) return;
    if (!fd_sync(p, cx, sh.misc)) return;
  }
  FdEpi eo;
  eo.n = 1;
  eo.s[0] = FdOut{p.logits, nullptr, p.vocab, EPI_STORE};
  fd_matrix(p, p.out, eo, [&] { fd_norm_quant(p, p.out_norm, sh); }, sh, cx);
}

}  // namespace

// ---- host side -----------------------------------------------------------------
int fused_decode_smem(const FdParams& p) { return FdSmem{p.ns, p.nbmax, p.scratch}.total(); }

bool fused_decode_plan(int d, int dff, int nh, int nkv, int hd, int s_ld, FdParams* p) {
  if (nkv <= 0 || nh % nkv || hd % 8 || hd > 256 || d % 32 || dff % 32 || (nh * hd) % 32) return false;
  const int gsz = nh / nkv;
  if (gsz * FD_PV_DIMS > FD_CT) return false;
  int dev = 0, optin = 0, coop = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess || !coop) return false;
  p->nbmax = std::max(std::max(d, dff), nh * hd) / 32;
  int scratch = std::max(std::max(2 * d, dff), nh * hd);  // norm x + w, SwiGLU y, attention output
  scratch = std::max(scratch, gsz * hd + FD_KEYS * (hd + 1));
  const int lane_rows = 8 * (((((std::max(d, s_ld) + 7) >> 3) + 31) & ~31) + 4);  // lane-major staging
  scratch = std::max(scratch, lane_rows + d);                                      // norm: x + weights
  scratch = std::max(scratch, FD_PV_STAGES * (gsz * FD_KEYS + FD_KEYS * FD_PV_DIMS));
  p->scratch = (scratch + 3) & ~3;
  p->ns = 0;
  const int fixed = FdSmem{0, p->nbmax, p->scratch}.total();
  const int ns = (optin - fixed) / (FD_SLOT + 16);
  if (ns < 4) return false;
  p->ns = std::min(ns, FD_MAX_SLOTS);
  return fused_decode_smem(*p) <= optin;
}

cudaError_t fused_decode_prepare(const FdParams& p, int* grid) {
  const int smem = fused_decode_smem(p);
  cudaError_t e = raise_smem_cap((const void*)decode_fused_kernel, smem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0, occ = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_fused_kernel, FD_THREADS, smem)) != cudaSuccess)
    return e;
  if (occ < 1) return cudaErrorCooperativeLaunchTooLarge;
  *grid = sms;  // one CTA per SM: every CTA is resident (cooperative launch)
  return cudaSuccess;
}

cudaError_t launch_decode_fused(const Launch& L, const FdParams& p, int grid) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(FD_THREADS);
  cfg.dynamicSmemBytes = fused_decode_smem(p);
  cfg.stream = L.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_fused_kernel, p);
  if (L.launches) ++*L.launches;
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace det
