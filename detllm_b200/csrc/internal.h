// internal.h -- types shared by the host side (host.cpp) and the CUDA kernels
// (kernels.cu) of libdetgpu.so.  Not part of the public ABI.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace det {

// ggml tensor types on this path (det-gguf lib.rs:58-96)
enum : int { GT_F32 = 0, GT_F16 = 1, GT_Q4_0 = 2, GT_Q8_0 = 8, GT_Q4_K = 12, GT_Q6_K = 14 };

// Device error-flag bits (one uint32 per session, OR-ed by kernels)
enum : uint32_t {
  ERRF_NONFINITE = 1u,        // ModelError::NonFinite
  ERRF_CDF_NONFINITE = 2u,    // CdfError::NonFiniteLogit
  ERRF_CDF_TOTAL = 4u,        // CdfError::TotalTooLarge
  ERRF_SHAPE = 8u,            // ModelError::Shape (bad token id etc.)
  ERRF_DECODE = 16u,          // value outside the decoder distribution
  ERRF_TIMEOUT = 32u,         // a bounded device-side wait gave up
  ERRF_SYMBOL = 64u,          // CdfError::SymbolOutOfRange found on the device
};

// A weight matrix in device memory.  Layouts (rows x cols, nb blocks/row):
//   F32  : f[rows][cols]
//   Q8_0 : q int8 [rows][cols], d f16 bits [rows][nb]
//   Q4_0 : q uint8 [rows][cols/2] (GGUF nibble order per 32-block), d [rows][nb]
//   Q4_K : q uint8 [rows][nb][144] (GGUF super-blocks, 16-byte aligned)
//   Q6_K : q uint8 [rows][nb][208] (ql | qh | scales), d [rows][nb]
// Layouts of Q8_0 / Q4_0 matrices:
//   LAYOUT_ROWMAJOR: as above
//   LAYOUT_MMA16   : 16-row tiles of per-block records in m16n8k32 A-fragment
//                    order (gemm.cu documents the record format)
enum : int { LAYOUT_ROWMAJOR = 0, LAYOUT_MMA16 = 1 };

struct DevMatrix {
  int type = GT_F32;
  int layout = LAYOUT_ROWMAJOR;
  int rows = 0, cols = 0, nb = 0;
  const void* q = nullptr;
  const uint16_t* d = nullptr;
  const float* f = nullptr;
  // tensor-core records of the chunk GEMM, or null: Q6_K (gemm_q6k_tc.cu),
  // Q8_0 / Q4_0 in LAYOUT_MMA16 (gemm_q8_tc.cu)
  const uint8_t* tc = nullptr;
};

// Quantised activations for `T` positions of length K (row stride K).
struct DevActs {
  const float* x = nullptr;    // f32 [T][K]
  const float* qa_d = nullptr; // Q8A scales, q8a_slot order (dev_math.cuh)
  const int8_t* qa_q = nullptr;// Q8A quants, q8a_elem order, 64-position groups
  const float* qk_d = nullptr; // Q8_K scales [T][K/256]
  const int8_t* qk_q = nullptr;// Q8_K quants [T][K]
  const uint8_t* qk_p = nullptr;// Q8_K in the class-permuted records of gemm_q6k_tc.cu, or null
};

// epilogue modes of a GEMV/GEMM
enum : int { EPI_STORE = 0, EPI_BIAS = 1, EPI_RESIDUAL = 2 };

// Output of a GEMM over a matrix that is several matrices stored back to
// back (q|k|v, gate|up): rows [sum of earlier rows, + rows) of the launch go
// to out[p * ld + r] with their own epilogue.  All but the last segment
// hold a multiple of 16 rows.
constexpr int kMaxOutSegs = 3;
struct OutSeg {
  int rows = 0;
  float* out = nullptr;
  int ld = 0;
  int epi = 0;
  const float* bias = nullptr;
};
struct OutSegs {
  OutSeg s[kMaxOutSegs];
  int n = 0;
  // 1.0, passed at run time: the GEMM writes its exact adds as fma(x, one,
  // acc), which the compiler must not be able to simplify
  float one = 1.0f;
};

struct Launch {
  cudaStream_t stream;
  uint32_t* err;        // device error flag
  uint64_t* launches;   // host counter of kernels launched
  // launch with programmatic stream serialization (see launch_k); used for
  // short forwards, where launch latency dominates
  bool pdl = false;
};

// Launch `kern` on L.stream, with programmatic stream serialization when
// L.pdl (the kernel may then start before its predecessor finishes; every
// kernel calls pdl_wait() first, see dev_math.cuh).  DETGPU_NO_PDL=1 turns
// the attribute off everywhere.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
cudaError_t launch_k(const Launch& L, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = L.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = L.pdl && pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Raises the dynamic shared-memory cap of `kern` on the current device to at
// least `bytes` (a no-op at 48 KiB or less) and never lowers it: a CUDA graph
// captured earlier may hold a launch of the same kernel that needs more than
// the launch at hand, and whatever replays that launch on its own (a
// profiler's node-by-node replay) checks it against the current cap.
cudaError_t raise_smem_cap(const void* kern, size_t bytes);
// SMs of the current device (read once: one part per node)
int device_sms();

// ---- launchers (kernels.cu) ------------------------------------------------
cudaError_t launch_rope_table(const Launch& L, float* cos_t, float* sin_t, int positions, int half, int rope_dim,
                              float rope_base);
cudaError_t launch_embed(const Launch& L, const DevMatrix& m, const uint32_t* tokens, int T, float* x);
// qd / qq non-null and n % 32 == 0: also writes the Q8A quantisation of h
cudaError_t launch_rmsnorm(const Launch& L, const float* x, const float* w, int n, float eps, int T, float* h,
                           float* qd = nullptr, int8_t* qq = nullptr);
cudaError_t launch_quant_q8a(const Launch& L, const float* x, int K, int T, float* qd, int8_t* qq);
// qp non-null: also writes the class-permuted records gemm_q6k_tc.cu reads
cudaError_t launch_quant_q8k(const Launch& L, const float* x, int K, int T, float* qd, int8_t* qq,
                             uint8_t* qp = nullptr);
// Q4_K matrix, chunk of T > 16 positions (gemm_kq.cu)
cudaError_t launch_gemm_q4k(const Launch& L, const DevMatrix& m, const DevActs& a, int T, float* out, int out_ld,
                            int epi, const float* bias);
// up to three Q4_K matrices of equal width that read the same activation
// (q / k / v, gate / up), chunk of T > 16 positions, one launch
cudaError_t launch_gemm_q4k_segs(const Launch& L, const DevMatrix* const* m, int n, const DevActs& a, int T,
                                 float* const* out, const int* out_ld, const int* epi, const float* const* bias);
// Q6_K matrix, chunk of T > 16 positions, on int8 tensor cores
// (gemm_q6k_tc.cu): needs m.tc (q6k_tc_repack at load) and a.qk_p
size_t q6k_tc_bytes(int rows, int nb);
size_t q6k_tc_act_bytes(int T, int K);
size_t q6k_tc_row_offset(int r0, int nb);  // r0 a multiple of 64
cudaError_t launch_q6k_tc_repack(cudaStream_t st, const DevMatrix& m, uint8_t* out);
cudaError_t launch_gemm_q6k_tc(const Launch& L, const DevMatrix& m, const DevActs& a, int T, float* out, int out_ld,
                               int epi, const float* bias);
// Q4_K / Q6_K matrix, one position (gemm_kq.cu); supported: every Q6_K, and
// Q4_K rows of up to 64 super-blocks (K <= 16384)
bool kq_decode_supported(const DevMatrix& m);
cudaError_t launch_gemv_kq_decode(const Launch& L, const DevMatrix& m, const DevActs& a, float* out, int epi,
                                  const float* bias);
// up to three Q4_K (or three Q6_K) matrices of equal width that read the same
// activation (q / k / v, gate / up), one position, one launch
struct KqSeg {
  const uint8_t* q;
  const uint16_t* d;
  int rows, cta0;
  float* out;
  int epi;
  const float* bias;
};
struct KqSegs {
  KqSeg s[3];
  int nb;
  float one = 1.0f;  // passed at run time (see OutSegs::one)
};
cudaError_t launch_gemv_kq_decode_segs(const Launch& L, const DevMatrix* const* m, int n, const DevActs& a,
                                       float* const* out, const int* epi, const float* const* bias);
// Q8_0 / Q4_0 chunk GEMM on tcgen05 tensor cores (gemm_q8_tc.cu): needs the
// matrix's tensor-core copy in m.tc (q8_tc_repack at load)
size_t q8_tc_bytes(int rows, int nb);
cudaError_t launch_q8_tc_repack(cudaStream_t st, const DevMatrix& m, uint8_t* out);
cudaError_t launch_gemm_q8_tc(const Launch& L, const DevMatrix& m, const DevActs& a, int T, const OutSegs& o);
// the process-wide choice of det_set_q8_tensor_cores (gemm.cu): models loaded
// while it is on get tensor-core copies, and chunk GEMMs use them while it is
bool q8_tensor_cores();
// LAYOUT_MMA16 Q8_0 / Q4_0 matrix with per-segment outputs (gemm.cu)
cudaError_t launch_gemm_mma16(const Launch& L, const DevMatrix& m, const DevActs& a, int T, const OutSegs& o);
cudaError_t launch_gemv(const Launch& L, const DevMatrix& m, const DevActs& a, int T, float* out, int out_ld,
                        int epi, const float* bias);
cudaError_t launch_rope_store(const Launch& L, float* q, float* k, const float* v, int T, const int* pos0, int n_head,
                              int n_head_kv, int head_dim, int rope_dim, int pairing, const float* cos_t,
                              const float* sin_t, float* kc, float* vc, int n_ctx);
cudaError_t launch_attention(const Launch& L, const float* q, const float* kc, const float* vc, int T, const int* pos0,
                             int n_head, int n_head_kv, int head_dim, int n_ctx, float scale, float* out,
                             float* score_scratch);
// tiled three-kernel attention (attention.cu) for head_dim 64 / 128
bool attention_tiled_supported(int n_head, int n_head_kv, int head_dim);
size_t attention_tiled_scratch_floats(int T, int n_head, int n_ctx);
cudaError_t launch_attention_tiled(const Launch& L, const float* q, const float* kc, const float* vc, int T,
                                   const int* pos0, int n_head, int n_head_kv, int head_dim, int n_ctx, float scale,
                                   float* out, float* S);
// floats of global score scratch launch_attention needs (0: scores stay in smem)
size_t attention_scratch_floats(int T, int n_head, int n_head_kv, int hd, int n_ctx);
// qd / qq non-null and n % 32 == 0: also writes the Q8A quantisation of out
cudaError_t launch_swiglu(const Launch& L, const float* g, const float* u, float* out, int n, int T,
                          float* qd = nullptr, int8_t* qq = nullptr);
cudaError_t launch_cdf_prepare(const Launch& L, const float* logits, int V, const uint32_t* rows, int nrows,
                               float* e, float* z);
cudaError_t launch_cdf_ranges(const Launch& L, const float* e, const float* z, int V, int tail,
                              const uint32_t* rows, const uint32_t* symbols, int n, uint64_t* out3);
cudaError_t launch_expf(cudaStream_t st, const float* x, float* y, long long n);
// GGUF tensor bytes (in device memory) -> device layouts (repack.cu); a
// non-finite scale or value sets ERRF_NONFINITE in *err
cudaError_t launch_repack_mma16(const uint8_t* raw, int q8, int rows, int nb, uint8_t* recs, uint32_t* err);
cudaError_t launch_check_q4k(const uint8_t* blocks, long long nblk, uint32_t* err);
cudaError_t launch_split_q6k(const uint8_t* raw, long long nblk, uint8_t* q, uint16_t* d, uint32_t* err);
cudaError_t launch_dense_f32(const uint8_t* raw, int f16, long long n, float* out, uint32_t* err);
// one warp, n pairs of dependent f32 adds, clock cycles into *cycles
cudaError_t launch_add_chain(const float* x, float* out, long long* cycles, int n);
// Row-sharded tensor parallelism (exchange.cu): copy column slices of
// [T][ld] f32 activations that live on other parts (peer memory) into `dst`:
// dst[p * ld_dst + col0 + c] = src[p * ld + c] for c < n, for every source.
constexpr int kMaxTpParts = 8;
struct GatherSrc {
  const float* src;
  int ld, col0, n;
};
struct GatherPlan {
  GatherSrc s[kMaxTpParts];
  int n = 0;
};
cudaError_t launch_gather_cols(const Launch& L, const GatherPlan& g, float* dst, int ld_dst, int T);
// Parts on distinct GPUs order their exchanges themselves (exchange.cu):
// `peer[q]` is this part's counter slot in part q's flag array (null for
// q == self), `mine` this part's own array, one slot per part.
struct TpFlags {
  unsigned long long* peer[kMaxTpParts];
  const unsigned long long* mine;
  int parts;
};
// signal exchange k of the current forward (counter *epoch * nx + k + 1),
// wait (bounded) for the parts in wait_mask, then pull `g` into dst
cudaError_t launch_tp_exchange(const Launch& L, const TpFlags& f, const unsigned long long* epoch, int k, int nx,
                               unsigned wait_mask, const GatherPlan& g, float* dst, int ld_dst, int T);
// *epoch += 1 (the start of a forward)
cudaError_t launch_tp_epoch(const Launch& L, unsigned long long* epoch);
// The decompress loop's device state (one per session in device memory): the
// range decoder (det-coder range.rs:88-178), the window's token count, the
// bytes produced so far, and the symbols one batch of steps decoded.
constexpr int kRcMaxBatch = 64;
enum : uint32_t { RC_RUNNING = 0, RC_DONE = 1, RC_WINDOW_FULL = 2, RC_FAILED = 3 };
struct RcState {
  unsigned long long low, code, range;  // RangeDecoder
  unsigned long long pos, len;          // payload cursor and length
  unsigned long long bytes, orig_len;   // output bytes so far / in the file
  uint32_t status, error;               // RC_*, and the det_status of RC_FAILED
  uint32_t count, max_count;            // symbols this batch / steps allowed this batch
  uint32_t clen, n_ctx, tail, pad;      // tokens in the window, window size, escapes (256 or 0)
  uint32_t syms[kRcMaxBatch];
};
// one decode step (rc_step_kernel): next symbol under logits row 0's CDF
// (cdf_prepare of row 0 must precede it), range decoder advance, and the
// token / position of the next one-position forward
cudaError_t launch_rc_step(const Launch& L, RcState* S, const float* e, const float* z, int V, const uint8_t* payload,
                           const uint16_t* piece_len, uint32_t* tok, int* pos);
cudaError_t launch_decoder_lookup(const Launch& L, const float* e, const float* z, int V, int tail, uint32_t row,
                                  const uint64_t* value, uint64_t* out4);

// ---- one-position forward as one persistent kernel (decode_fused.cu) -------
// A LAYOUT_MMA16 matrix (Q8_0 or Q4_0) as the fused kernel reads it.
struct FdMat {
  const uint8_t* q = nullptr;
  int type = 0, rows = 0, nb = 0;
};
// one layer's weights (device array of L entries)
struct FdLayer {
  FdMat qkv, o, gu, down;
  const float *attn_norm = nullptr, *ffn_norm = nullptr, *bq = nullptr, *bk = nullptr, *bv = nullptr;
};
struct FdParams {
  const FdLayer* layers = nullptr;
  int L = 0;
  FdMat out;
  const float* out_norm = nullptr;
  int d = 0, dff = 0, nh = 0, nkv = 0, hd = 0, half = 0, pairing = 0, n_ctx = 0, s_ld = 0, vocab = 0;
  float eps = 0.0f, scale = 0.0f;
  const int* pos = nullptr;
  const float *cos_t = nullptr, *sin_t = nullptr;
  float *x = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *S = nullptr, *attn = nullptr;
  float *gate = nullptr, *up = nullptr, *logits = nullptr, *kc = nullptr, *vc = nullptr;
  uint32_t* err = nullptr;
  unsigned* sync = nullptr;  // [0] grid-barrier arrivals, [1] abort; zeroed before each launch
  // shared-memory plan (fused_decode_plan): ring slots, largest K / 32, scratch floats
  int ns = 0, nbmax = 0, scratch = 0;
};
// fills p->ns / nbmax / scratch for these shapes on the current device;
// false when the fused kernel does not apply (the per-op kernels run instead)
bool fused_decode_plan(int d, int dff, int nh, int nkv, int hd, int s_ld, FdParams* p);
int fused_decode_smem(const FdParams& p);
// sets the kernel's shared-memory limit on the current device and returns
// the grid (one CTA per SM); once per session, before its first launch
cudaError_t fused_decode_prepare(const FdParams& p, int* grid);
// cooperative launch (every CTA resident: the kernel has grid barriers)
cudaError_t launch_decode_fused(const Launch& L, const FdParams& p, int grid);

}  // namespace det
