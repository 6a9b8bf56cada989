// exchange.cu -- the all-gather of row-sharded tensor parallelism.
//
// After a sharded GEMV each part holds a column slice of a [T][ld] f32
// activation (its rows of the matrix are the activation's columns).  A part
// then pulls every other part's slice straight out of that part's device
// memory -- peer loads over NVLink when the parts sit on different GPUs, plain
// loads when they share one -- into its own full-width copy.  Every write is
// to the puller's own memory, so parts never write into each other's data.
//
// Two ways to order a pull after the producers:
//  * gather_cols_kernel: the host orders it -- each part records an event
//    after its producing launch and the gathering launch waits on the other
//    parts' events (cudaStreamWaitEvent).  No kernel waits on another; this
//    is the form for parts that share a GPU.
//  * tp_exchange_kernel: parts on distinct GPUs run their own streams and
//    order themselves.  Exchange k of forward e signals by storing the
//    counter e * nx + k + 1 (release, system scope) into its slot of every
//    peer's flag array, then waits until every peer's slot in its own array
//    has reached that value (acquire, system scope) and pulls.  The wait is
//    bounded by the global timer: on timeout the kernel sets ERRF_TIMEOUT and
//    skips the pull, so a missing peer ends in an error status, not a hang;
//    later exchanges of the same forward see the flag and do not wait again.
// The loads are ld.global.cv (fetch again, never a cached copy): a slice is
// rewritten by its owner between layers.
#include <algorithm>

#include "../../include/detgpu.h"
#include "dev_math.cuh"
#include "internal.h"

namespace det {
namespace {

constexpr int GX_THREADS = 256;
constexpr unsigned long long kTpWaitNs = 2000000000ull;  // 2 s

DI unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
DI void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
DI unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// this CTA's share of source blockIdx.y of the plan
DI void pull_slice(const GatherPlan& g, float* __restrict__ dst, int ld_dst, int T) {
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

// blockIdx.y: the source slice; blocks along x stride over its T x n values
__global__ void __launch_bounds__(GX_THREADS)
    gather_cols_kernel(GatherPlan g, float* __restrict__ dst, int ld_dst, int T) {
  pdl_enter();
  pull_slice(g, dst, ld_dst, T);
}

__global__ void __launch_bounds__(GX_THREADS)
    tp_exchange_kernel(TpFlags f, const unsigned long long* __restrict__ epoch, int k, int nx, unsigned wait_mask,
                       GatherPlan g, float* __restrict__ dst, int ld_dst, int T, uint32_t* err) {
  pdl_enter();  // the producing launch has completed: its slice is in this GPU's memory
  __shared__ int timed_out;
  const unsigned long long target = *epoch * (unsigned long long)nx + (unsigned long long)k + 1ull;
  if (threadIdx.x == 0) {
    // an earlier exchange of this forward already gave up: fail fast, so a
    // missing peer costs one bounded wait per forward, not one per exchange
    timed_out = (*reinterpret_cast<volatile uint32_t*>(err) & ERRF_TIMEOUT) ? 1 : 0;
    if (blockIdx.x == 0 && blockIdx.y == 0)
      for (int q = 0; q < f.parts; q++)
        if (f.peer[q]) st_release_sys(f.peer[q], target);
    unsigned long long t0 = 0;
    for (int q = 0; q < f.parts && !timed_out; q++) {
      if (!(wait_mask >> q & 1u)) continue;
      for (unsigned it = 0; ld_acquire_sys(f.mine + q) < target; it++) {
        if (it == 0 && t0 == 0) t0 = gtimer();
        else if ((it & 255u) == 0 && gtimer() - t0 > kTpWaitNs) {
          timed_out = 1;
          atomicOr(err, ERRF_TIMEOUT);
          break;
        }
      }
    }
  }
  __syncthreads();
  if (timed_out || g.n == 0) return;
  pull_slice(g, dst, ld_dst, T);
}

__global__ void tp_epoch_kernel(unsigned long long* epoch) {
  pdl_enter();
  if (threadIdx.x == 0) *epoch += 1ull;
}

int gather_blocks_x(const GatherPlan& g, int T) {
  int maxn = 0;
  for (int i = 0; i < g.n; i++) maxn = std::max(maxn, g.s[i].n);
  // one float4 per thread per pass; at most one block per SM per slice
  const long long units = (long long)T * ((maxn + 3) / 4);
  return (int)std::min<long long>(std::max<long long>((units + GX_THREADS - 1) / GX_THREADS, 1), 148);
}

}  // namespace

cudaError_t launch_gather_cols(const Launch& L, const GatherPlan& g, float* dst, int ld_dst, int T) {
  if (g.n <= 0 || T <= 0) return cudaSuccess;
  if (g.n > kMaxTpParts) return cudaErrorInvalidValue;
  const cudaError_t e =
      launch_k(L, gather_cols_kernel, dim3(gather_blocks_x(g, T), g.n), dim3(GX_THREADS), 0, g, dst, ld_dst, T);
  if (e != cudaSuccess) return e;
  if (L.launches) ++*L.launches;
  return cudaGetLastError();
}

cudaError_t launch_tp_exchange(const Launch& L, const TpFlags& f, const unsigned long long* epoch, int k, int nx,
                               unsigned wait_mask, const GatherPlan& g, float* dst, int ld_dst, int T) {
  if (g.n < 0 || g.n > kMaxTpParts || f.parts > kMaxTpParts) return cudaErrorInvalidValue;
  const dim3 grid(g.n > 0 ? gather_blocks_x(g, T) : 1, g.n > 0 ? g.n : 1);
  const cudaError_t e = launch_k(L, tp_exchange_kernel, grid, dim3(GX_THREADS), 0, f, epoch, k, nx, wait_mask, g,
                                 dst, ld_dst, T, L.err);
  if (e != cudaSuccess) return e;
  if (L.launches) ++*L.launches;
  return cudaGetLastError();
}

cudaError_t launch_tp_epoch(const Launch& L, unsigned long long* epoch) {
  const cudaError_t e = launch_k(L, tp_epoch_kernel, 1, 32, 0, epoch);
  if (e != cudaSuccess) return e;
  if (L.launches) ++*L.launches;
  return cudaGetLastError();
}

}  // namespace det

extern "C" det_status det_tp_exchange_timeout_selftest(int device) {
  using namespace det;
  int cnt = 0;
  if (cudaGetDeviceCount(&cnt) != cudaSuccess || cnt == 0) return DET_ERR_NO_DEVICE;
  if (device < 0 || device >= cnt) return DET_ERR_INVALID_ARGUMENT;
  if (cudaSetDevice(device) != cudaSuccess) return DET_ERR_CUDA;
  // [0, 2): this part's counters (slot 1 is the absent peer's), [2]: epoch,
  // [3]: error word
  unsigned long long* mem = nullptr;
  if (cudaMalloc(&mem, 4 * sizeof(unsigned long long)) != cudaSuccess) return DET_ERR_DEVICE_OOM;
  cudaError_t e = cudaMemset(mem, 0, 4 * sizeof(unsigned long long));
  TpFlags f{};
  f.parts = 2;
  f.mine = mem;  // peer[0], peer[1] stay null: nobody is signalled
  uint32_t* err = reinterpret_cast<uint32_t*>(mem + 3);
  Launch L{nullptr, err, nullptr};
  GatherPlan g;  // no data
  if (e == cudaSuccess) e = launch_tp_exchange(L, f, mem + 2, 0, 1, 1u << 1, g, nullptr, 0, 1);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  uint32_t flag = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&flag, err, 4, cudaMemcpyDeviceToHost);
  cudaFree(mem);
  if (e != cudaSuccess) return DET_ERR_CUDA;
  return (flag & ERRF_TIMEOUT) ? DET_ERR_TIMEOUT : DET_OK;
}
