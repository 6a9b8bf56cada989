// gemm_q6k_tc.cu -- Q6_K x Q8_K chunk GEMM on int8 tensor cores.
//
// Reference: dot_q6_k_q8k (crates/det-quant/src/lib.rs:353-397).  Per
// 256-element block, lane class c (the elements i with i % 8 == c)
// accumulates the exact integer
//   aux[c] = sum over those i of scale[i / 16] * q6[i] * a.q[i],
// then sums[c] += (w.d * a.d) * (f32)aux[c] block by block, and the row's
// result is ((((0 + sums[0]) + sums[1]) + ...) + sums[7]).
//
// aux[c] is an integer dot product over the 32 elements of class c, so it is
// one int8 MMA (m16n8k32) whose K dimension is that class: element
// i = 8 j + c sits at MMA column j.  The weight factor w' = scale * q6 needs
// 13 bits, so it is split as w' = 64 * hi + lo with hi = w' >> 6 (in
// [-62, 64]) and lo = w' & 63: two MMAs per (block, class), and
// aux = 64 * hi_sum + lo_sum.  Each partial sum is below 2^22 in magnitude
// (32 * 64 * 127 and 32 * 63 * 127), so its int32 accumulator is seeded with
// 0x4B400000 and read back as the f32 12582912 + sum: one exact subtraction
// gives the f32 value, and 64 * hi + lo is exact in f32 because
// |aux| <= 32 * 4096 * 127 < 2^24.  The float work is then exactly the
// reference's: one product (w.d * a.d), one product with aux, one add per
// (row, position, block, class), in block order.
//
// Layouts (both built once per use, both bulk-copied whole per stage):
// * weights (q6k_tc_repack_kernel, at model load): per 64-row group and
//   block, a 33,024-byte record: for 4 row tiles x 8 classes x {hi, lo} the
//   m16n8k32 A fragments (32 lanes x 16 B, lane (g, t) holds rows g and g+8,
//   columns 4t..4t+3 and 4t+16..4t+19), then the 64 rows' w.d as f32;
// * activations (quant_q8k_kernel with a permuted output): per 64-position
//   group and block, a 16,640-byte record: for 8 classes x 64 positions the
//   class's 32 bytes (16-byte halves swapped for positions with bit 2 set,
//   so ldmatrix reads are bank-conflict free), then the 64 positions' a.d.
//
// A CTA owns 64 rows x 64 positions: thread 0 moves one block's two records
// per stage with cp.async.bulk (full / empty mbarriers, every wait bounded by
// %globaltimer); the 16 warps each own one 16-row tile, two classes and all
// 64 positions.  The per-class sums meet in shared memory at
// the end, where each output adds its eight lane sums in lane order.
#include <atomic>
#include <cuda_runtime.h>

#include "../../include/detgpu.h"
#include "dev_math.cuh"
#include "internal.h"

namespace det {
namespace {

constexpr int TC_ROWS = 64, TC_POS = 64;
constexpr int TC_CWARPS = 16;
constexpr int TC_THREADS = TC_CWARPS * 32;
constexpr int TC_STAGES = 4;
constexpr int TC_A_FRAG = 32768;                  // 4 tiles x 8 classes x 2 halves x 512 B
constexpr int TC_A_REC = TC_A_FRAG + TC_ROWS * 4;  // + w.d of the 64 rows
constexpr int TC_B_Q = 8 * TC_POS * 32;            // 8 classes x 64 positions x 32 B
constexpr int TC_B_REC = TC_B_Q + TC_POS * 4;      // + a.d of the 64 positions
constexpr int TC_STAGE = TC_A_REC + TC_B_REC;
constexpr int TC_RED_LD = TC_ROWS + 4;  // reduction rows (floats): conflict-free writes and reads
constexpr int TC_SMEM = TC_STAGE * TC_STAGES + 2 * TC_STAGES * 8;
static_assert(8 * TC_POS * TC_RED_LD * 4 <= TC_STAGE * TC_STAGES, "reduction fits the ring");
constexpr unsigned long long kTcWaitNs = 2000000000ull;  // mbarrier wait bound (2 s)
constexpr unsigned long long kTcSelftestWaitNs = 20000000ull;  // the self-test's bound (20 ms)

DI uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
DI void tc_mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
DI void tc_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
DI void tc_arrive(uint32_t bar) { asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory"); }
DI void tc_bulk(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
DI unsigned long long tc_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// bounded wait for phase `parity`; false after `bound_ns`
DI bool tc_wait(uint32_t bar, uint32_t parity, unsigned long long bound_ns) {
  unsigned long long t0 = 0;
  for (unsigned it = 0;; it++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if (it == 0) t0 = tc_now();
    else if ((it & 63) == 0 && tc_now() - t0 > bound_ns) return false;
  }
}

DI void tc_mma(int (&c)[4], const int4& a, int b0, int b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// packed f32 pairs: each half is one IEEE round-to-nearest operation
DI unsigned long long p2(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
DI unsigned long long i2(int a, int b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(a), "r"(b));
  return r;
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
DI float2 un2(unsigned long long r) {
  float2 o;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(o.x), "=f"(o.y) : "l"(r));
  return o;
}

// ldmatrix.x4 of class rows (positions p0..p0+15, 32 B each, halves swapped
// for positions with bit 2 set): the B fragments of two N8 tiles
DI void ldsm_b(const uint8_t* cls, int p0, int lane, int (&b)[4]) {
  const int p = p0 + ((lane >> 4) << 3) + (lane & 7), h = (lane >> 3) & 1;
  const uint32_t addr = su32(cls + p * 32 + ((h ^ ((p >> 2) & 1)) << 4));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
               : "r"(addr));
}

__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_q6k_tc_kernel(const uint8_t* __restrict__ W, int rows, int nb, const uint8_t* __restrict__ A, int T,
                       float* __restrict__ out, int out_ld, int epi, const float* __restrict__ bias, float one,
                       uint32_t* err, int withhold, unsigned long long wait_ns) {
  // withhold >= 0 (det_q6k_pipeline_timeout_selftest only): that stage is
  // never copied, so every wait on it runs out after wait_ns
  pdl_enter();
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = blockIdx.x, rg = blockIdx.y;  // position group, row group
  const uint32_t full0 = su32(smem + TC_STAGE * TC_STAGES), empty0 = full0 + 8 * TC_STAGES;
  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; s++) {
      tc_mbar_init(full0 + 8 * s, 1);
      tc_mbar_init(empty0 + 8 * s, TC_CWARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();

  // thread 0 also produces: stage b goes into slot b % TC_STAGES once all
  // 16 warps have released stage b - TC_STAGES from it
  const uint8_t* wrec = W + (size_t)rg * nb * TC_A_REC;
  const uint8_t* arec = A + (size_t)grp * nb * TC_B_REC;
  auto issue = [&](int b) {
    if (b == withhold) return;
    const int slot = b % TC_STAGES;
    uint8_t* sb = smem + slot * TC_STAGE;
    tc_expect_tx(full0 + 8 * slot, TC_STAGE);
    tc_bulk(su32(sb), wrec + (size_t)b * TC_A_REC, TC_A_REC, full0 + 8 * slot);
    tc_bulk(su32(sb + TC_A_REC), arec + (size_t)b * TC_B_REC, TC_B_REC, full0 + 8 * slot);
  };
  const bool producer = threadIdx.x == 0;
  int issued = 0;
  if (producer)
    for (; issued < nb && issued < TC_STAGES; issued++) issue(issued);

  // ---- compute warps: row tile rt, classes c0 and c0 + 1, all 64 positions
  const int rt = warp >> 2, c0 = 2 * (warp & 3);
  const int g = lane >> 2, t = lane & 3;
  const unsigned long long ONE = p2(one, one), NEG_M = p2(-12582912.0f, -12582912.0f), K64 = p2(64.0f, 64.0f);
  const int SEED = 0x4B400000;
  // sums[class][tile n][row half][position pair], packed
  unsigned long long sums[2][8][2];
#pragma unroll
  for (int k = 0; k < 2; k++)
#pragma unroll
    for (int n = 0; n < 8; n++) sums[k][n][0] = sums[k][n][1] = 0ull;
  bool ok = true;
  for (int b = 0; b < nb; b++) {
    const int slot = b % TC_STAGES;
    if (ok && !tc_wait(full0 + 8 * slot, (uint32_t)((b / TC_STAGES) & 1), wait_ns)) {
      if (lane == 0) atomicOr(err, ERRF_TIMEOUT);
      ok = false;
    }
    if (!ok) break;
    const uint8_t* sb = smem + slot * TC_STAGE;
    const float* wd = reinterpret_cast<const float*>(sb + TC_A_FRAG);
    const uint8_t* bq = sb + TC_A_REC;
    const float* ad = reinterpret_cast<const float*>(bq + TC_B_Q);
    const float wd0 = wd[16 * rt + g], wd1 = wd[16 * rt + g + 8];
#pragma unroll
    for (int tp = 0; tp < 4; tp++) {  // tile pairs: positions 16 tp .. 16 tp + 15
      unsigned long long dd[2][2];     // [tile][row half]: (w.d * a.d) for the pair of positions
#pragma unroll
      for (int n = 0; n < 2; n++) {
        const float2 a2 = *reinterpret_cast<const float2*>(ad + 16 * tp + 8 * n + 2 * t);
        const unsigned long long av = p2(a2.x, a2.y);
        dd[n][0] = mul2(p2(wd0, wd0), av);
        dd[n][1] = mul2(p2(wd1, wd1), av);
      }
#pragma unroll
      for (int k = 0; k < 2; k++) {
        const int c = c0 + k;
        const int4 ahi = *reinterpret_cast<const int4*>(sb + ((rt * 8 + c) * 2 + 0) * 512 + lane * 16);
        const int4 alo = *reinterpret_cast<const int4*>(sb + ((rt * 8 + c) * 2 + 1) * 512 + lane * 16);
        int bf[4];
        ldsm_b(bq + c * (TC_POS * 32), 16 * tp, lane, bf);
#pragma unroll
        for (int n = 0; n < 2; n++) {
          int ch[4] = {SEED, SEED, SEED, SEED}, cl[4] = {SEED, SEED, SEED, SEED};
          tc_mma(ch, ahi, bf[2 * n], bf[2 * n + 1]);
          tc_mma(cl, alo, bf[2 * n], bf[2 * n + 1]);
#pragma unroll
          for (int h = 0; h < 2; h++) {  // row g (c[0], c[1]) and row g + 8 (c[2], c[3])
            const unsigned long long fh = add2(i2(ch[2 * h], ch[2 * h + 1]), NEG_M);
            const unsigned long long fl = add2(i2(cl[2 * h], cl[2 * h + 1]), NEG_M);
            const unsigned long long aux = fma2(fh, K64, fl);   // exact: 64 * hi + lo
            const unsigned long long pr = mul2(dd[n][h], aux);  // (w.d * a.d) * aux
            sums[k][2 * tp + n][h] = fma2(pr, ONE, sums[k][2 * tp + n][h]);  // exact add of pr
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) tc_arrive(empty0 + 8 * slot);
    if (producer && issued < nb) {
      if (!tc_wait(empty0 + 8 * slot, (uint32_t)((b / TC_STAGES) & 1), wait_ns)) {
        atomicOr(err, ERRF_TIMEOUT);
        ok = false;
      } else {
        issue(issued++);
      }
    }
  }
  // the CTA's shared memory must outlive every copy issued into it: wait for
  // the stages a failed warp left unread (bounded), then agree on the outcome
  if (producer)
    for (int s2 = max(0, issued - TC_STAGES); s2 < issued; s2++)
      if (s2 != withhold) tc_wait(full0 + 8 * (s2 % TC_STAGES), (uint32_t)((s2 / TC_STAGES) & 1), wait_ns);
  if (!__syncthreads_and(ok)) return;
  float* red = reinterpret_cast<float*>(smem);  // [class][position][row]
#pragma unroll
  for (int k = 0; k < 2; k++)
#pragma unroll
    for (int n = 0; n < 8; n++)
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const float2 v = un2(sums[k][n][h]);
        const int r = 16 * rt + g + 8 * h, p = 8 * n + 2 * t;
        red[((c0 + k) * TC_POS + p) * TC_RED_LD + r] = v.x;
        red[((c0 + k) * TC_POS + p + 1) * TC_RED_LD + r] = v.y;
      }
  __syncthreads();
  for (int i = threadIdx.x; i < TC_ROWS * TC_POS; i += TC_THREADS) {
    const int r = i & (TC_ROWS - 1), p = i / TC_ROWS;
    const int row = rg * TC_ROWS + r, pos = grp * TC_POS + p;
    if (row >= rows || pos >= T) continue;
    float v = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; c++) v = fadd(v, red[(c * TC_POS + p) * TC_RED_LD + r]);
    if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
    float* dst = out + (size_t)pos * out_ld + row;
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

// Weight records of one (64-row group, block): slot s = ((tile * 8 + class)
// * 2 + half) * 32 + lane holds 16 bytes: A-fragment words (row g, columns
// 4t..4t+3), (row g+8, same), (row g, 4t+16..4t+19), (row g+8, same), with
// column j of class c standing for element 8 j + c and half 0 / 1 holding
// w' >> 6 / w' & 63 of w' = scale * q6 (det-quant lib.rs:536-568).
__global__ void q6k_tc_repack_kernel(const uint8_t* __restrict__ q, const uint16_t* __restrict__ d, int rows,
                                     int nb, uint8_t* __restrict__ out) {
  const int rg = blockIdx.x, b = blockIdx.y;
  uint8_t* rec = out + ((size_t)rg * nb + b) * TC_A_REC;
  for (int s = threadIdx.x; s < 2048; s += blockDim.x) {
    const int lane = s & 31, half = (s >> 5) & 1, c = (s >> 6) & 7, tile = s >> 9;
    const int g = lane >> 2, t = lane & 3;
    uint32_t words[4];
#pragma unroll
    for (int w = 0; w < 4; w++) {
      const int row = rg * TC_ROWS + tile * 16 + g + 8 * (w & 1);
      const int j0 = 4 * t + 16 * (w >> 1);
      uint32_t word = 0;
      if (row < rows) {
        const uint8_t* body = q + ((size_t)row * nb + b) * 208;
        for (int k = 0; k < 4; k++) {
          const int i = 8 * (j0 + k) + c;
          const int wq = (int)(int8_t)body[192 + (i >> 4)] * q6k_quant(body, i);
          const int v = half == 0 ? (wq >> 6) : (wq & 63);
          word |= (uint32_t)(uint8_t)(int8_t)v << (8 * k);
        }
      }
      words[w] = word;
    }
    *reinterpret_cast<uint4*>(rec + (size_t)s * 16) = make_uint4(words[0], words[1], words[2], words[3]);
  }
  float* wd = reinterpret_cast<float*>(rec + TC_A_FRAG);
  for (int r = threadIdx.x; r < TC_ROWS; r += blockDim.x) {
    const int row = rg * TC_ROWS + r;
    wd[r] = row < rows ? f16_bits_to_f32(d[(size_t)row * nb + b]) : 0.0f;
  }
}

}  // namespace

size_t q6k_tc_bytes(int rows, int nb) { return (size_t)((rows + TC_ROWS - 1) / TC_ROWS) * nb * TC_A_REC; }
size_t q6k_tc_act_bytes(int T, int K) { return (size_t)((T + TC_POS - 1) / TC_POS) * (K / 256) * TC_B_REC; }
size_t q6k_tc_row_offset(int r0, int nb) { return (size_t)(r0 / TC_ROWS) * nb * TC_A_REC; }

cudaError_t launch_q6k_tc_repack(cudaStream_t st, const DevMatrix& m, uint8_t* out) {
  if (m.type != GT_Q6_K || !m.q || !m.d) return cudaErrorInvalidValue;
  dim3 grid((m.rows + TC_ROWS - 1) / TC_ROWS, m.nb);
  q6k_tc_repack_kernel<<<grid, 256, 0, st>>>(static_cast<const uint8_t*>(m.q), m.d, m.rows, m.nb, out);
  return cudaGetLastError();
}

cudaError_t launch_gemm_q6k_tc(const Launch& L, const DevMatrix& m, const DevActs& a, int T, float* out, int out_ld,
                               int epi, const float* bias) {
  if (!m.tc || !a.qk_p) return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> attr_set{0};  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(attr_set.load() >> dev & 1ull)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_q6k_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set.fetch_or(1ull << dev);
  }
  dim3 grid((T + TC_POS - 1) / TC_POS, (m.rows + TC_ROWS - 1) / TC_ROWS);
  const cudaError_t e = launch_k(L, gemm_q6k_tc_kernel, grid, TC_THREADS, TC_SMEM, m.tc, m.rows, m.nb, a.qk_p, T,
                                 out, out_ld, epi, bias, 1.0f, L.err, -1, kTcWaitNs);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace det

// The pipeline's bounded waits, exercised: one CTA over zero-filled records
// of 64 rows x 4 blocks and 64 positions, first with stage 1 never copied
// (every wait on it gives up after 20 ms and the kernel reports
// ERRF_TIMEOUT without writing its outputs), then complete (outputs 0, no
// error), on the same device and stream.
extern "C" det_status det_q6k_pipeline_timeout_selftest(int device) {
  using namespace det;
  int cnt = 0;
  if (cudaGetDeviceCount(&cnt) != cudaSuccess || cnt == 0) return DET_ERR_NO_DEVICE;
  if (device < 0 || device >= cnt) return DET_ERR_INVALID_ARGUMENT;
  if (cudaSetDevice(device) != cudaSuccess) return DET_ERR_CUDA;
  constexpr int nb = 4;
  const size_t wbytes = (size_t)nb * TC_A_REC, abytes = (size_t)nb * TC_B_REC, obytes = (size_t)TC_ROWS * TC_POS * 4;
  uint8_t* mem = nullptr;
  if (cudaMalloc(&mem, wbytes + abytes + obytes + 256) != cudaSuccess) return DET_ERR_DEVICE_OOM;
  uint8_t* w = mem;
  uint8_t* a = mem + wbytes;
  float* out = reinterpret_cast<float*>(mem + wbytes + abytes);
  uint32_t* err = reinterpret_cast<uint32_t*>(mem + wbytes + abytes + obytes);
  cudaError_t e = cudaMemset(mem, 0, wbytes + abytes + obytes + 256);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemm_q6k_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
  uint32_t flag[2] = {0, 0};
  for (int run = 0; run < 2 && e == cudaSuccess; run++) {
    gemm_q6k_tc_kernel<<<dim3(1, 1), TC_THREADS, TC_SMEM>>>(w, TC_ROWS, nb, a, TC_POS, out, TC_ROWS, EPI_STORE,
                                                           nullptr, 1.0f, err, run == 0 ? 1 : -1,
                                                           kTcSelftestWaitNs);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(&flag[run], err, 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(err, 0, 4);
  }
  cudaFree(mem);
  if (e != cudaSuccess) return DET_ERR_CUDA;
  if (flag[1] != 0) return DET_ERR_CUDA;  // the complete run must not flag anything
  return (flag[0] & ERRF_TIMEOUT) ? DET_ERR_TIMEOUT : DET_OK;
}
