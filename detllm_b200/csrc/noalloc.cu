// noalloc.cu -- det_symbol_ranges_noalloc: symbol ranges for logits that are
// already in device memory, computed without allocating anything.
//
// Some callers cannot allocate device memory inside a call: a host engine
// that owns a fixed memory budget and forbids allocation after start-up, or
// a runtime whose allocator is not cudaMalloc and that must account for
// every byte it hands out.  For them this entry point keeps its working
// memory (the exp values, the per-row normalisers, row ids and an error
// word) in one file-scope device array of fixed size.  Every GPU that loads
// this library holds the array until the process exits.
//
// Each call ends by copying the error word to the host and synchronising
// `stream`, so it returns only after its kernels have finished, on the
// error paths too.
//
// The array is shared by every call on a device and keeps what the last call
// left there: the error word is cleared at the start of each call and the
// other parts are fully rewritten before they are read.  Two calls whose
// work overlaps on the GPU (different streams, or different host threads on
// one stream without ordering) race on the array.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/detgpu.h"
#include "dev_math.cuh"
#include "internal.h"

namespace det {
namespace {

constexpr size_t kMaxFloats = DET_NOALLOC_MAX_FLOATS;
constexpr size_t kMaxRows = DET_NOALLOC_MAX_ROWS;
// [0, kMaxFloats)             exp values, row-major n x vocab
// [+0, +kMaxRows)             per-row normaliser Z
// [+kMaxRows, +2*kMaxRows)    row ids 0..n-1 for the shared CDF kernels
// [+2*kMaxRows]               error word; padded to 64 words
constexpr size_t kZOff = kMaxFloats, kRowOff = kZOff + kMaxRows, kErrOff = kRowOff + kMaxRows;
constexpr size_t kWords = kErrOff + 64;

static __device__ __align__(256) uint32_t g_noalloc_scratch[kWords];

// Device address of g_noalloc_scratch per device, taken once with that device
// current.  In host code the array's name is only a host-side stand-in.
std::mutex g_mu;
constexpr int kMaxDevices = 64;
uint32_t* g_scratch_ptr[kMaxDevices] = {};

det_status scratch_for(int dev, uint32_t** out) {
  if (dev < 0 || dev >= kMaxDevices) return DET_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return DET_ERR_CUDA;
    g_scratch_ptr[dev] = static_cast<uint32_t*>(p);
  }
  *out = g_scratch_ptr[dev];
  return DET_OK;
}

// row ids for the shared CDF kernels, and the reference's symbol check
// (symbol < vocab + tail, det-coder cdf.rs:150-152) on the device
__global__ void noalloc_rows_kernel(const uint32_t* __restrict__ symbols, int n, uint32_t alphabet,
                                    uint32_t* __restrict__ rows, uint32_t* err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  rows[i] = (uint32_t)i;
  if (symbols[i] >= alphabet) atomicOr(err, ERRF_SYMBOL);
}

}  // namespace
}  // namespace det

using namespace det;

extern "C" det_status det_symbol_ranges_noalloc(const float* logits, uint32_t n, uint32_t vocab,
                                                const uint32_t* symbols, int byte_escapes, det_symbol_range* out,
                                                void* stream) {
  if (n == 0) return DET_OK;
  if (!logits || !symbols || !out) return DET_ERR_INVALID_ARGUMENT;
  if (vocab == 0) return DET_ERR_CDF_EMPTY;
  const uint32_t tail = byte_escapes ? 256u : 0u;
  if ((uint64_t)vocab + tail > (1u << 18)) return DET_ERR_CDF_TOO_MANY_SYMBOLS;
  if (n > kMaxRows || (uint64_t)n * vocab > kMaxFloats) return DET_ERR_SCRATCH_LIMIT;
  int cnt = 0, dev = 0;
  if (cudaGetDeviceCount(&cnt) != cudaSuccess || cnt == 0) return DET_ERR_NO_DEVICE;
  if (cudaGetDevice(&dev) != cudaSuccess) return DET_ERR_CUDA;
  uint32_t* scratch = nullptr;
  if (det_status st = scratch_for(dev, &scratch)) return st;
  float* e = reinterpret_cast<float*>(scratch);
  float* z = reinterpret_cast<float*>(scratch + kZOff);
  uint32_t* rows = scratch + kRowOff;
  uint32_t* err = scratch + kErrOff;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const Launch L{s, err, nullptr};
  if (cudaMemsetAsync(err, 0, sizeof(uint32_t), s) != cudaSuccess) return DET_ERR_CUDA;
  // once work is enqueued, a failure still waits for the stream, so that no
  // kernel of this call writes the array or `out` after the status returns
  auto fail = [s]() {
    cudaStreamSynchronize(s);
    return DET_ERR_CUDA;
  };
  noalloc_rows_kernel<<<(n + 255) / 256, 256, 0, s>>>(symbols, (int)n, vocab + tail, rows, err);
  if (cudaGetLastError() != cudaSuccess) return fail();
  if (launch_cdf_prepare(L, logits, (int)vocab, rows, (int)n, e, z) != cudaSuccess) return fail();
  // (cum, freq, total) as three u64 per row is the det_symbol_range layout:
  // freq < 2^32 leaves the `reserved` word zero
  if (launch_cdf_ranges(L, e, z, (int)vocab, (int)tail, rows, symbols, (int)n, reinterpret_cast<uint64_t*>(out)) !=
      cudaSuccess)
    return fail();
  uint32_t f = 0;
  if (cudaMemcpyAsync(&f, err, sizeof(f), cudaMemcpyDeviceToHost, s) != cudaSuccess) return fail();
  if (cudaStreamSynchronize(s) != cudaSuccess) return DET_ERR_CUDA;
  if (f & ERRF_SYMBOL) return DET_ERR_CDF_SYMBOL_OUT_OF_RANGE;
  if (f & ERRF_CDF_NONFINITE) return DET_ERR_CDF_NONFINITE_LOGIT;
  if (f & ERRF_CDF_TOTAL) return DET_ERR_CDF_TOTAL_TOO_LARGE;
  if (f) return DET_ERR_CUDA;
  return DET_OK;
}
