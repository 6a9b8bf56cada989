// exchange.cu -- the all-gather of row-sharded tensor parallelism.
//
// After a sharded GEMV each part holds a column slice of a [T][ld] f32
// activation (its rows of the matrix are the activation's columns).  A part
// then pulls every other part's slice straight out of that part's device
// memory -- peer loads over NVLink when the parts sit on different GPUs, plain
// loads when they share one -- into its own full-width copy.  Every write is
// to the puller's own memory, so parts never write into each other.
//
// Ordering is the host's: each part records an event after its producing
// launch, and a part's gather launch waits (cudaStreamWaitEvent) on every
// other part's event.  No kernel waits on another, so no wait can spin.
// The loads are ld.global.cv (fetch again, never a cached copy): a slice is
// rewritten by its owner between layers.
#include <algorithm>

#include "dev_math.cuh"
#include "internal.h"

namespace det {
namespace {

constexpr int GX_THREADS = 256;

// blockIdx.y: the source slice; blocks along x stride over its T x n values
__global__ void __launch_bounds__(GX_THREADS)
    gather_cols_kernel(GatherPlan g, float* __restrict__ dst, int ld_dst, int T) {
  pdl_enter();
  const GatherSrc sc = g.s[blockIdx.y];
  const long long stride = (long long)gridDim.x * GX_THREADS;
  const long long first = (long long)blockIdx.x * GX_THREADS + threadIdx.x;
  const bool v4 = ((sc.ld | sc.col0 | sc.n | ld_dst) & 3) == 0 &&
                  ((reinterpret_cast<uintptr_t>(sc.src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0;
  if (v4) {
    const int n4 = sc.n >> 2;
    const long long total = (long long)T * n4;
    for (long long i = first; i < total; i += stride) {
      const int p = (int)(i / n4), c = (int)(i - (long long)p * n4);
      const float4 v = __ldcv(reinterpret_cast<const float4*>(sc.src + (size_t)p * sc.ld) + c);
      reinterpret_cast<float4*>(dst + (size_t)p * ld_dst + sc.col0)[c] = v;
    }
  } else {
    const long long total = (long long)T * sc.n;
    for (long long i = first; i < total; i += stride) {
      const int p = (int)(i / sc.n), c = (int)(i - (long long)p * sc.n);
      dst[(size_t)p * ld_dst + sc.col0 + c] = __ldcv(sc.src + (size_t)p * sc.ld + c);
    }
  }
}

}  // namespace

cudaError_t launch_gather_cols(const Launch& L, const GatherPlan& g, float* dst, int ld_dst, int T) {
  if (g.n <= 0 || T <= 0) return cudaSuccess;
  if (g.n > kMaxTpParts) return cudaErrorInvalidValue;
  int maxn = 0;
  for (int i = 0; i < g.n; i++) maxn = std::max(maxn, g.s[i].n);
  // one float4 per thread per pass; at most one block per SM per slice
  const long long units = (long long)T * ((maxn + 3) / 4);
  const int bx = (int)std::min<long long>(std::max<long long>((units + GX_THREADS - 1) / GX_THREADS, 1), 148);
  const cudaError_t e = launch_k(L, gather_cols_kernel, dim3(bx, g.n), dim3(GX_THREADS), 0, g, dst, ld_dst, T);
  if (e != cudaSuccess) return e;
  if (L.launches) ++*L.launches;
  return cudaGetLastError();
}

}  // namespace det
