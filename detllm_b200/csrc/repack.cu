// repack.cu -- GGUF weight tensors into the device layouts, on the device.
//
// The loader copies a tensor's bytes as they sit in the GGUF file into a
// device staging buffer (one host-to-device copy, no host-side pass over the
// blocks) and these kernels write the layouts the GEMV / GEMM kernels read
// (internal.h), checking every block scale on the way as read_q8/q4/q4k/
// q6k_matrix do (crates/det-model/src/lib.rs:1812-1953: a non-finite f16
// scale fails the load with NonFinite):
//   * Q8_0 / Q4_0 -> LAYOUT_MMA16 records: per (16-row tile, block) the
//     m16n8k32 A fragments of the 16 rows (lane (g, t): rows g and g + 8,
//     quant bytes 4t..4t+3 and, for Q8_0, 16+4t..16+4t+3), then the rows'
//     f16 scales in pairs (row g, row g + 8); rows past the matrix are zeros;
//   * Q4_K -> the blocks as stored (144 B: d, dmin, scales, quants), checked;
//   * Q6_K -> ql | qh | scales (208 B) per block and the f16 d split out;
//   * F16 -> f32, by the exact widening of f16_to_f32 (det-num f16.rs:6-34).
// Each kernel sets ERRF_NONFINITE in the error word for a non-finite scale
// (or value, for F16 / F32 tensors).
#include <cuda_runtime.h>

#include "dev_math.cuh"
#include "internal.h"

namespace det {
namespace {

constexpr int RP_THREADS = 256;

DI bool f16_bits_finite(uint32_t b) { return (b & 0x7c00u) != 0x7c00u; }
DI uint32_t rd16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }
DI uint32_t rd32u(const uint8_t* p) {  // any alignment
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// one thread per (tile, block, lane) of the records: the lane's 16 (Q8_0) or
// 8 (Q4_0) fragment bytes; lanes 0..7 also write the scale pair of rows
// (g, g + 8) with g = lane
__global__ void __launch_bounds__(RP_THREADS) mma16_records_kernel(const uint8_t* __restrict__ raw, int q8, int rows,
                                                                   int nb, long long total,
                                                                   uint8_t* __restrict__ recs, uint32_t* err) {
  const long long i = (long long)blockIdx.x * RP_THREADS + threadIdx.x;
  if (i >= total) return;
  const int lane = (int)(i & 31);
  const long long tb = i >> 5;  // tile * nb + block
  const int b = (int)(tb % nb);
  const long long tile = tb / nb;
  const int tbytes = q8 ? 34 : 18, qb = q8 ? 512 : 256, rb = qb + 32;
  uint8_t* r = recs + tb * rb;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int hi = 0; hi < 2; hi++) {
    const long long row = tile * 16 + g + 8 * hi;
    uint32_t w0 = 0, w1 = 0;
    if (row < rows) {
      const uint8_t* blk = raw + ((size_t)row * nb + b) * tbytes + 2;  // quants after the f16 scale
      w0 = rd32u(blk + 4 * t);
      if (q8) w1 = rd32u(blk + 16 + 4 * t);
    }
    if (q8) {
      *reinterpret_cast<uint32_t*>(r + lane * 16 + hi * 4) = w0;
      *reinterpret_cast<uint32_t*>(r + lane * 16 + 8 + hi * 4) = w1;
    } else {
      *reinterpret_cast<uint32_t*>(r + lane * 8 + hi * 4) = w0;
    }
  }
  if (lane < 8) {
    const long long r0 = tile * 16 + lane, r1 = r0 + 8;
    const uint32_t d0 = r0 < rows ? rd16(raw + ((size_t)r0 * nb + b) * tbytes) : 0u;
    const uint32_t d1 = r1 < rows ? rd16(raw + ((size_t)r1 * nb + b) * tbytes) : 0u;
    if (!f16_bits_finite(d0) || !f16_bits_finite(d1)) atomicOr(err, ERRF_NONFINITE);
    *reinterpret_cast<uint32_t*>(r + qb + 4 * lane) = d0 | (d1 << 16);
  }
}

// one thread per Q4_K block: d and dmin finite
__global__ void __launch_bounds__(RP_THREADS) q4k_check_kernel(const uint8_t* __restrict__ blocks, long long n,
                                                               uint32_t* err) {
  const long long i = (long long)blockIdx.x * RP_THREADS + threadIdx.x;
  if (i >= n) return;
  const uint32_t w = *reinterpret_cast<const uint32_t*>(blocks + i * 144);  // 144 = 16 * 9: aligned
  if (!f16_bits_finite(w & 0xffffu) || !f16_bits_finite(w >> 16)) atomicOr(err, ERRF_NONFINITE);
}

// one thread per (Q6_K block, 16-byte piece of its first 208 bytes); piece 0
// also moves the block's d
__global__ void __launch_bounds__(RP_THREADS) q6k_split_kernel(const uint8_t* __restrict__ raw, long long n,
                                                               uint8_t* __restrict__ q, uint16_t* __restrict__ d,
                                                               uint32_t* err) {
  const long long i = (long long)blockIdx.x * RP_THREADS + threadIdx.x;
  if (i >= n * 13) return;
  const long long blk = i / 13;
  const int piece = (int)(i - blk * 13);
  const uint8_t* src = raw + blk * 210 + piece * 16;  // 210-byte blocks: 2-byte aligned
  uint4 v;
  v.x = rd32u(src);
  v.y = rd32u(src + 4);
  v.z = rd32u(src + 8);
  v.w = rd32u(src + 12);
  *reinterpret_cast<uint4*>(q + blk * 208 + piece * 16) = v;
  if (piece == 0) {
    const uint32_t db = rd16(raw + blk * 210 + 208);
    if (!f16_bits_finite(db)) atomicOr(err, ERRF_NONFINITE);
    d[blk] = (uint16_t)db;
  }
}

// f16_to_f32 (det-num f16.rs:6-34): exact widening, subnormals normalised
DI float f16_widen(uint32_t bits) {
  const uint32_t sign = (bits & 0x8000u) << 16;
  const uint32_t ex = (bits >> 10) & 0x1f, frac = bits & 0x3ffu;
  uint32_t out;
  if (ex == 0) {
    if (frac == 0) {
      out = sign;
    } else {
      uint32_t f = frac;
      int e = -14;
      while ((f & 0x400u) == 0) {
        f <<= 1;
        e--;
      }
      out = sign | ((uint32_t)(e + 127) << 23) | ((f & 0x3ffu) << 13);
    }
  } else if (ex == 0x1f) {
    out = sign | 0x7f800000u | (frac << 13);
  } else {
    out = sign | ((ex - 15 + 127) << 23) | (frac << 13);
  }
  return __uint_as_float(out);
}

// F16 or F32 values -> f32, every value finite
__global__ void __launch_bounds__(RP_THREADS) dense_f32_kernel(const uint8_t* __restrict__ raw, int f16, long long n,
                                                               float* __restrict__ out, uint32_t* err) {
  const long long i = (long long)blockIdx.x * RP_THREADS + threadIdx.x;
  if (i >= n) return;
  float v;
  if (f16) {
    const uint32_t b = rd16(raw + 2 * i);
    if (!f16_bits_finite(b)) atomicOr(err, ERRF_NONFINITE);
    v = f16_widen(b);
  } else {
    v = __uint_as_float(rd32u(raw + 4 * i));
    if (!finite(v)) atomicOr(err, ERRF_NONFINITE);
  }
  out[i] = v;
}

unsigned grid_for(long long n) { return (unsigned)((n + RP_THREADS - 1) / RP_THREADS); }

}  // namespace

cudaError_t launch_repack_mma16(const uint8_t* raw, int q8, int rows, int nb, uint8_t* recs, uint32_t* err) {
  const long long total = (long long)((rows + 15) / 16) * nb * 32;
  if (total == 0) return cudaSuccess;
  mma16_records_kernel<<<grid_for(total), RP_THREADS>>>(raw, q8, rows, nb, total, recs, err);
  return cudaGetLastError();
}

cudaError_t launch_check_q4k(const uint8_t* blocks, long long nblk, uint32_t* err) {
  if (nblk == 0) return cudaSuccess;
  q4k_check_kernel<<<grid_for(nblk), RP_THREADS>>>(blocks, nblk, err);
  return cudaGetLastError();
}

cudaError_t launch_split_q6k(const uint8_t* raw, long long nblk, uint8_t* q, uint16_t* d, uint32_t* err) {
  if (nblk == 0) return cudaSuccess;
  q6k_split_kernel<<<grid_for(nblk * 13), RP_THREADS>>>(raw, nblk, q, d, err);
  return cudaGetLastError();
}

cudaError_t launch_dense_f32(const uint8_t* raw, int f16, long long n, float* out, uint32_t* err) {
  if (n == 0) return cudaSuccess;
  dense_f32_kernel<<<grid_for(n), RP_THREADS>>>(raw, f16, n, out, err);
  return cudaGetLastError();
}

}  // namespace det
