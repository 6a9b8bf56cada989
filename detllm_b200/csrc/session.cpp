// session.cpp -- det_session: device workspace, KV cache and RoPE table of one
// context window, the chunked teacher-forced forward, and the logits -> CDF
// entry points.
//
// The layer sequence follows forward_one_with_workspace
// (crates/det-model/src/lib.rs:1249-1400); a chunk of n tokens runs every op
// for all n positions before the next op, which leaves each position's
// arithmetic unchanged (each reduction stays within one position).
#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "host_common.h"

using namespace det;

bool det::g_profiling = false;

namespace det {
void free_session_impl(det_session* s);

// The model's cached session (created on first use, replaced when a caller
// needs a different window or chunk size).  Released by det_model_free.
det_status session_acquire(det_model* m, uint32_t n_ctx, uint32_t max_chunk, det_session** out) {
  det_session* c = m->cached;
  if (c && c->n_ctx == (int)n_ctx && c->max_chunk == (int)std::min(max_chunk, n_ctx)) {
    *out = c;
    return DET_OK;
  }
  if (c) {
    m->cached = nullptr;
    free_session_impl(c);
  }
  det_status st = det_session_create(m, n_ctx, max_chunk, out);
  if (!st) m->cached = *out;
  return st;
}

void session_release_cached(det_model* m) {
  if (m->cached) {
    det_session* c = m->cached;
    m->cached = nullptr;
    free_session_impl(c);
  }
}
det_status cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return DET_OK;
  if (e == cudaErrorMemoryAllocation) return DET_ERR_DEVICE_OOM;
  return DET_ERR_CUDA;
}
}  // namespace det

namespace {

template <typename T>
det_status dalloc(det_session* s, T** p, size_t count) {
  void* q = nullptr;
  const cudaError_t e = cudaMalloc(&q, std::max<size_t>(count * sizeof(T), 256));
  if (e != cudaSuccess) return cuda_status(e);
  s->allocations.push_back(q);
  *p = static_cast<T*>(q);
  return DET_OK;
}

template <typename T>
det_status halloc(det_session* s, T** p, size_t count) {
  void* q = nullptr;
  if (cudaMallocHost(&q, std::max<size_t>(count * sizeof(T), 64)) != cudaSuccess) return DET_ERR_ALLOC;
  *p = static_cast<T*>(q);
  return DET_OK;
}

bool needs_q8a(int type) { return type == GT_Q8_0 || type == GT_Q4_0 || type == GT_Q4_K; }

void add_stats(det_stats* a, const det_stats& b) {
  a->forward_ms += b.forward_ms;
  a->cdf_ms += b.cdf_ms;
  a->launches += b.launches;
  a->h2d_bytes += b.h2d_bytes;
  a->d2h_bytes += b.d2h_bytes;
  a->tokens += b.tokens;
  a->gemm_ms += b.gemm_ms;
  a->gemm_launches += b.gemm_launches;
  a->gemm_bytes += b.gemm_bytes;
  a->gemm_weight_bytes += b.gemm_weight_bytes;
}

void add_prof(ProfTags* a, const ProfTags& b) {
  for (int i = 0; i < PT_COUNT; i++) {
    a->ms[i] += b.ms[i];
    a->n[i] += b.n[i];
  }
}

// launches whose time and algorithmic bytes go into the GEMM statistics (the
// fused one-position forward counts as one: it streams every weight matrix)
bool is_gemm_tag(int tag) {
  return tag == PT_GEMM_QKV || tag == PT_GEMM_O || tag == PT_GEMM_GATE_UP || tag == PT_GEMM_DOWN ||
         tag == PT_GEMM_OUT || tag == PT_FUSED;
}

const char* const kProfTagNames[PT_COUNT] = {"embed",  "rmsnorm",       "quantise", "gemm_qkv", "rope_store",
                                             "attention", "gemm_o",     "gemm_gate_up", "swiglu", "gemm_down",
                                             "gemm_output", "cdf",      "decode_fused"};

void free_session(det_session* s) {
  if (!s) return;
  cudaSetDevice(s->m->device);
  if (s->stream) cudaStreamSynchronize(s->stream);
  // a tensor-parallel session's graphs hold the other parts' launches
  for (auto& g : s->graphs)
    if (g.exec) cudaGraphExecDestroy(g.exec);
  s->graphs.clear();
  if (s->tp) tp_session_release(s);
  cudaSetDevice(s->m->device);
  det_model* owner = s->owner ? s->owner : s->m;
  {
    std::lock_guard<std::recursive_mutex> lk(owner->mu);
    add_stats(&owner->agg, s->stats);
    add_prof(&owner->prof_agg, s->prof);
  }
  for (cudaEvent_t e : s->prof_events) cudaEventDestroy(e);
  for (void* p : s->allocations) cudaFree(p);
  if (s->graph_dev1.exec) cudaGraphExecDestroy(s->graph_dev1.exec);
  for (void* p : {(void*)s->h_tokens, (void*)s->h_rows, (void*)s->h_syms, (void*)s->h_err, (void*)s->h_out,
                  (void*)s->h_value, (void*)s->h_pos, (void*)s->h_rc})
    if (p) cudaFreeHost(p);
  for (auto& e : s->ev)
    if (e) cudaEventDestroy(e);
  if (s->stream) cudaStreamDestroy(s->stream);
  delete s;
}

}  // namespace

void det::free_session_impl(det_session* s) { free_session(s); }

namespace {

Launch launch_of(det_session* s) { return Launch{s->stream, s->d_err, &s->stats.launches}; }

// Reads and clears the device error flag (synchronises the stream), and
// resolves pending profile events.  A tensor-parallel session reads the
// other parts' flags first.
det_status take_error(det_session* s, bool cdf) {
  const det_status part_st = s->tp ? tp_take_part_errors(s) : DET_OK;
  cudaSetDevice(s->m->device);
  cudaError_t e = cudaMemcpyAsync(s->h_err, s->d_err, 4, cudaMemcpyDeviceToHost, s->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  if (e != cudaSuccess) return cuda_status(e);
  for (size_t i = 0; i < s->prof_pending.size(); i++) {
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, s->prof_events[2 * i], s->prof_events[2 * i + 1]) == cudaSuccess) {
      const ProfEntry& pe = s->prof_pending[i];
      s->prof.ms[pe.tag] += ms;
      s->prof.n[pe.tag]++;
      if (is_gemm_tag(pe.tag)) {
        s->stats.gemm_ms += ms;
        s->stats.gemm_launches++;
        s->stats.gemm_bytes += pe.bytes;
        s->stats.gemm_weight_bytes += pe.wbytes;
      }
    }
  }
  s->prof_pending.clear();
  const uint32_t f = *s->h_err;
  if (f) cudaMemsetAsync(s->d_err, 0, 4, s->stream);
  if (f & ERRF_SHAPE) return DET_ERR_SHAPE;
  if (f & ERRF_NONFINITE) return DET_ERR_NONFINITE;
  if (cdf && (f & ERRF_CDF_NONFINITE)) return DET_ERR_CDF_NONFINITE_LOGIT;
  if (cdf && (f & ERRF_CDF_TOTAL)) return DET_ERR_CDF_TOTAL_TOO_LARGE;
  if (f & ERRF_DECODE) return DET_ERR_DECODE;
  if (f & ERRF_TIMEOUT) return DET_ERR_TIMEOUT;
  if (f) return DET_ERR_CUDA;
  return part_st;
}

#define CK(expr)                                   \
  do {                                             \
    const cudaError_t e_ = (expr);                 \
    if (e_ != cudaSuccess) return cuda_status(e_); \
  } while (0)

}  // namespace

det_status det::session_take_error(det_session* s, bool cdf) { return take_error(s, cdf); }

namespace {

double bytes_per_weight(int type) {
  switch (type) {
    case GT_Q8_0: return 34.0 / 32.0;
    case GT_Q4_0: return 18.0 / 32.0;
    case GT_Q4_K: return 144.0 / 256.0;
    case GT_Q6_K: return 210.0 / 256.0;
    default: return 4.0;
  }
}

// A launch with optional event timing (det_set_profiling); `launch`
// enqueues it.  `bytes` / `wbytes`: algorithmic bytes of a weight GEMM.
template <typename F>
cudaError_t timed(det_session* s, int tag, double bytes, double wbytes, F&& launch) {
  if (!g_profiling) return launch();
  const size_t i = s->prof_pending.size();
  while (s->prof_events.size() < 2 * (i + 1)) {
    cudaEvent_t ev;
    cudaError_t e = cudaEventCreate(&ev);
    if (e != cudaSuccess) return e;
    s->prof_events.push_back(ev);
  }
  cudaError_t e = cudaEventRecord(s->prof_events[2 * i], s->stream);
  if (e == cudaSuccess) e = launch();
  if (e == cudaSuccess) e = cudaEventRecord(s->prof_events[2 * i + 1], s->stream);
  s->prof_pending.push_back(ProfEntry{tag, bytes, wbytes});
  return e;
}

// A weight GEMV/GEMM launch: algorithmic bytes are the weights, the
// quantised activations and the outputs (read + write for residual outputs).
template <typename F>
cudaError_t timed_gemm(det_session* s, int tag, const DevMatrix& W, int T, double out_bytes_per_pos, F&& launch) {
  const double wbytes = (double)W.rows * W.cols * bytes_per_weight(W.type);
  const double abytes = (double)T * W.cols *
                        (W.type == GT_Q6_K ? 1.0 + 4.0 / 256.0 : (W.type == GT_F32 ? 4.0 : 1.0 + 4.0 / 32.0));
  return timed(s, tag, wbytes + abytes + (double)T * out_bytes_per_pos, wbytes, launch);
}

cudaError_t gemv(det_session* s, int tag, const Launch& L, const DevMatrix& W, const DevActs& a, int T, float* out,
                 int ld, int epi, const float* bias) {
  return timed_gemm(s, tag, W, T, W.rows * (epi == EPI_RESIDUAL ? 8.0 : 4.0),
                    [&] { return launch_gemv(L, W, a, T, out, ld, epi, bias); });
}

// one launch over a fused (back-to-back) matrix
cudaError_t gemm_fused(det_session* s, int tag, const Launch& L, const DevMatrix& W, const DevActs& a, int T,
                       const OutSegs& o) {
  double ob = 0;
  for (int k = 0; k < o.n; k++) ob += o.s[k].rows * (o.s[k].epi == EPI_RESIDUAL ? 8.0 : 4.0);
  return timed_gemm(s, tag, W, T, ob, [&] { return launch_gemm_mma16(L, W, a, T, o); });
}

// Q4_K matrices of one width that read the same activation, as one chunk
// launch (T > 16)
bool q4k_chunk_fusable(const DevMatrix* const* m, int n) {
  for (int i = 0; i < n; i++)
    if (m[i]->type != GT_Q4_K || m[i]->nb != m[0]->nb || m[i]->rows == 0) return false;
  return true;
}

// one chunk launch over q4k_chunk_fusable matrices
cudaError_t gemm_q4k_segs(det_session* s, int tag, const Launch& L, const DevMatrix* const* m, int n, const DevActs& a,
                          int T, float* const* out, const int* ld, const int* epi, const float* const* bias) {
  double wb = 0, ob = 0;
  for (int i = 0; i < n; i++) {
    wb += (double)m[i]->rows * m[i]->cols * bytes_per_weight(m[i]->type);
    ob += (double)T * m[i]->rows * (epi[i] == EPI_RESIDUAL ? 8.0 : 4.0);
  }
  const double ab = (double)T * m[0]->cols * (1.0 + 4.0 / 32.0);
  return timed(s, tag, wb + ab + ob, wb, [&] { return launch_gemm_q4k_segs(L, m, n, a, T, out, ld, epi, bias); });
}

// Matrices that read the same activation (q / k / v, gate / up) and can run
// as one one-position launch: Q4_K or Q6_K, all of one type and width.
bool kq_fusable(const DevMatrix* const* m, int n) {
  for (int i = 0; i < n; i++)
    if (!kq_decode_supported(*m[i]) || m[i]->type != m[0]->type || m[i]->nb != m[0]->nb || m[i]->rows == 0)
      return false;
  return true;
}

// one launch over kq_fusable matrices, one position
cudaError_t gemv_segs(det_session* s, int tag, const Launch& L, const DevMatrix* const* m, int n, const DevActs& a,
                      float* const* out, const int* epi, const float* const* bias) {
  double wb = 0, ob = 0;
  for (int i = 0; i < n; i++) {
    wb += (double)m[i]->rows * m[i]->cols * bytes_per_weight(m[i]->type);
    ob += m[i]->rows * (epi[i] == EPI_RESIDUAL ? 8.0 : 4.0);
  }
  const double ab = (double)m[0]->cols * (m[0]->type == GT_Q6_K ? 1.0 + 4.0 / 256.0 : 1.0 + 4.0 / 32.0);
  return timed(s, tag, wb + ab + ob, wb, [&] { return launch_gemv_kq_decode_segs(L, m, n, a, out, epi, bias); });
}

// quantise `x` (T x K) for a matrix of type `type` into the session buffers
cudaError_t quantise_for(det_session* s, const Launch& L, int type, const float* x, int K, int T, DevActs* a,
                         int* have) {
  a->x = x;
  if (needs_q8a(type) && !(*have & 1)) {
    cudaError_t e = timed(s, PT_QUANT, 0, 0, [&] { return launch_quant_q8a(L, x, K, T, s->qa_d, s->qa_q); });
    if (e != cudaSuccess) return e;
    *have |= 1;
  }
  if (type == GT_Q6_K && !(*have & 2)) {
    uint8_t* qp = T > 16 ? s->qk_p : nullptr;
    cudaError_t e = timed(s, PT_QUANT, 0, 0, [&] { return launch_quant_q8k(L, x, K, T, s->qk_d, s->qk_q, qp); });
    if (e != cudaSuccess) return e;
    *have |= 2;
  }
  a->qa_d = s->qa_d;
  a->qa_q = s->qa_q;
  a->qk_d = s->qk_d;
  a->qk_q = s->qk_q;
  a->qk_p = T > 16 ? s->qk_p : nullptr;
  return cudaSuccess;
}

// RMSNorm of x into s->h; when `q8a` (a consumer reads Q8A and K % 32 == 0)
// the same launch writes the Q8A quantisation of h and marks it present
cudaError_t norm(det_session* s, const Launch& L, const float* w, int K, int T, bool q8a, int* have) {
  const ModelCfg& c = s->m->cfg;
  q8a = q8a && K % 32 == 0;
  cudaError_t e = timed(s, PT_NORM, 0, 0, [&] {
    return q8a ? launch_rmsnorm(L, s->x, w, K, c.eps, T, s->h, s->qa_d, s->qa_q)
               : launch_rmsnorm(L, s->x, w, K, c.eps, T, s->h);
  });
  if (q8a) *have |= 1;
  return e;
}

}  // namespace

// ---- the forward, in the stages a row-sharded (tensor-parallel) forward
// exchanges slices between (tp.cpp).  A single-device session runs them back
// to back; a part of a tensor-parallel session computes its own rows of
// wo / gate / up / down / lm_head (TpShard) and its own KV heads. --------------
namespace det {

static int shard_d0(const det_session* s) { return s->m->shard ? s->m->shard->d0 : 0; }

det_status fwd_embed(det_session* s, const Launch& L, int T) {
  CK(timed(s, PT_EMBED, 0, 0, [&] { return launch_embed(L, s->m->tok_embd, s->d_tokens, T, s->x); }));
  return DET_OK;
}

// attention block of layer l up to the attention output s->attn
det_status fwd_attention(det_session* s, const Launch& L, int l, int T) {
  det_model* m = s->m;
  const ModelCfg& c = m->cfg;
  const LayerDev& W = m->layers[(size_t)l];
  const int* pos0 = s->d_pos;
  const int qd = c.nh * c.hd, kvd = c.nkv * c.hd;
  const size_t kv_layer = (size_t)c.nkv * s->n_ctx * c.hd;
  DevActs a;
  int have = 0;
  CK(norm(s, L, W.attn_norm, c.d, T, needs_q8a(W.wq.type) || needs_q8a(W.wk.type) || needs_q8a(W.wv.type), &have));
  // one Q8A of h shared by q/k/v (:1284-1292); Q8_K recomputed per Q6_K
  // matrix in the reference gives the same blocks, so it is made once too
  CK(quantise_for(s, L, W.wq.type, s->h, c.d, T, &a, &have));
  CK(quantise_for(s, L, W.wk.type, s->h, c.d, T, &a, &have));
  CK(quantise_for(s, L, W.wv.type, s->h, c.d, T, &a, &have));
  if (W.wqkv.rows) {
    OutSegs o;
    o.n = 3;
    o.s[0] = OutSeg{W.wq.rows, s->q, qd, W.bq ? EPI_BIAS : EPI_STORE, W.bq};
    o.s[1] = OutSeg{W.wk.rows, s->k, kvd, W.bk ? EPI_BIAS : EPI_STORE, W.bk};
    o.s[2] = OutSeg{W.wv.rows, s->v, kvd, W.bv ? EPI_BIAS : EPI_STORE, W.bv};
    CK(gemm_fused(s, PT_GEMM_QKV, L, W.wqkv, a, T, o));
  } else if (const DevMatrix* mq[3] = {&W.wq, &W.wk, &W.wv}; T == 1 && kq_fusable(mq, 3)) {
    float* const oo[3] = {s->q, s->k, s->v};
    const int ee[3] = {W.bq ? EPI_BIAS : EPI_STORE, W.bk ? EPI_BIAS : EPI_STORE, W.bv ? EPI_BIAS : EPI_STORE};
    const float* const bb[3] = {W.bq, W.bk, W.bv};
    CK(gemv_segs(s, PT_GEMM_QKV, L, mq, 3, a, oo, ee, bb));
  } else if (T > 16 && q4k_chunk_fusable(mq, 3)) {
    float* const oo[3] = {s->q, s->k, s->v};
    const int ll[3] = {qd, kvd, kvd};
    const int ee[3] = {W.bq ? EPI_BIAS : EPI_STORE, W.bk ? EPI_BIAS : EPI_STORE, W.bv ? EPI_BIAS : EPI_STORE};
    const float* const bb[3] = {W.bq, W.bk, W.bv};
    CK(gemm_q4k_segs(s, PT_GEMM_QKV, L, mq, 3, a, T, oo, ll, ee, bb));
  } else {
    CK(gemv(s, PT_GEMM_QKV, L, W.wq, a, T, s->q, qd, W.bq ? EPI_BIAS : EPI_STORE, W.bq));
    CK(gemv(s, PT_GEMM_QKV, L, W.wk, a, T, s->k, kvd, W.bk ? EPI_BIAS : EPI_STORE, W.bk));
    CK(gemv(s, PT_GEMM_QKV, L, W.wv, a, T, s->v, kvd, W.bv ? EPI_BIAS : EPI_STORE, W.bv));
  }
  float* kc = s->kc + (size_t)l * kv_layer;
  float* vc = s->vc + (size_t)l * kv_layer;
  CK(timed(s, PT_ROPE, 0, 0, [&] {
    return launch_rope_store(L, s->q, s->k, s->v, T, pos0, c.nh, c.nkv, c.hd, c.rope_dim, c.pairing, s->rope_cos,
                             s->rope_sin, kc, vc, s->n_ctx);
  }));
  CK(timed(s, PT_ATTENTION, 0, 0, [&] {
    return launch_attention(L, s->q, kc, vc, T, pos0, c.nh, c.nkv, c.hd, s->n_ctx, c.attn_scale, s->attn,
                            s->score_scratch);
  }));
  return DET_OK;
}

// x[:, d0 + r] += (attn . wo^T)[:, r] for this part's rows r of wo
det_status fwd_attn_out(det_session* s, const Launch& L, int l, int T, const float* attn) {
  const LayerDev& W = s->m->layers[(size_t)l];
  if (!W.wo.rows) return DET_OK;
  DevActs a;
  int have = 0;
  CK(quantise_for(s, L, W.wo.type, attn, W.wo.cols, T, &a, &have));
  CK(gemv(s, PT_GEMM_O, L, W.wo, a, T, s->x + shard_d0(s), s->m->cfg.d, EPI_RESIDUAL, nullptr));
  return DET_OK;
}

// RMSNorm, this part's rows of gate / up, SwiGLU -> s->ff; *have: which
// quantisations of s->ff the launch left in the session buffers
det_status fwd_ffn_in(det_session* s, const Launch& L, int l, int T, int* have_out) {
  const ModelCfg& c = s->m->cfg;
  const LayerDev& W = s->m->layers[(size_t)l];
  *have_out = 0;
  if (!W.gate.rows) return DET_OK;
  DevActs a;
  int have = 0;
  CK(norm(s, L, W.ffn_norm, c.d, T, needs_q8a(W.gate.type) || needs_q8a(W.up.type), &have));
  CK(quantise_for(s, L, W.gate.type, s->h, c.d, T, &a, &have));
  CK(quantise_for(s, L, W.up.type, s->h, c.d, T, &a, &have));
  if (W.wgu.rows) {
    OutSegs o;
    o.n = 2;
    o.s[0] = OutSeg{W.gate.rows, s->gate, c.dff, EPI_STORE, nullptr};
    o.s[1] = OutSeg{W.up.rows, s->up, c.dff, EPI_STORE, nullptr};
    CK(gemm_fused(s, PT_GEMM_GATE_UP, L, W.wgu, a, T, o));
  } else if (const DevMatrix* mg[2] = {&W.gate, &W.up}; T == 1 && kq_fusable(mg, 2)) {
    float* const oo[2] = {s->gate, s->up};
    const int ee[2] = {EPI_STORE, EPI_STORE};
    const float* const bb[2] = {nullptr, nullptr};
    CK(gemv_segs(s, PT_GEMM_GATE_UP, L, mg, 2, a, oo, ee, bb));
  } else if (T > 16 && q4k_chunk_fusable(mg, 2)) {
    float* const oo[2] = {s->gate, s->up};
    const int ll[2] = {c.dff, c.dff}, ee[2] = {EPI_STORE, EPI_STORE};
    const float* const bb[2] = {nullptr, nullptr};
    CK(gemm_q4k_segs(s, PT_GEMM_GATE_UP, L, mg, 2, a, T, oo, ll, ee, bb));
  } else {
    CK(gemv(s, PT_GEMM_GATE_UP, L, W.gate, a, T, s->gate, c.dff, EPI_STORE, nullptr));
    CK(gemv(s, PT_GEMM_GATE_UP, L, W.up, a, T, s->up, c.dff, EPI_STORE, nullptr));
  }
  // swiglu also quantises its output to Q8A when the down matrix reads it
  // (a single device: a tensor-parallel part holds only a slice of the row)
  const bool ff_q8a = !s->m->shard && needs_q8a(W.down.type) && c.dff % 32 == 0;
  CK(timed(s, PT_SWIGLU, 0, 0, [&] {
    return ff_q8a ? launch_swiglu(L, s->gate, s->up, s->ff, c.dff, T, s->qa_d, s->qa_q)
                  : launch_swiglu(L, s->gate, s->up, s->ff, c.dff, T);
  }));
  if (ff_q8a) *have_out |= 1;
  return DET_OK;
}

// x[:, d0 + r] += (ff . down^T)[:, r] for this part's rows r of down
det_status fwd_ffn_out(det_session* s, const Launch& L, int l, int T, const float* ff, int have) {
  const LayerDev& W = s->m->layers[(size_t)l];
  if (!W.down.rows) return DET_OK;
  DevActs a;
  CK(quantise_for(s, L, W.down.type, ff, W.down.cols, T, &a, &have));
  CK(gemv(s, PT_GEMM_DOWN, L, W.down, a, T, s->x + shard_d0(s), s->m->cfg.d, EPI_RESIDUAL, nullptr));
  return DET_OK;
}

// final RMSNorm and this part's lm_head rows -> s->logits[:, v0 + r]
det_status fwd_head(det_session* s, const Launch& L, int T) {
  det_model* m = s->m;
  if (!m->output.rows) return DET_OK;
  DevActs a;
  int have = 0;
  CK(norm(s, L, m->output_norm, m->cfg.d, T, needs_q8a(m->output.type), &have));
  CK(quantise_for(s, L, m->output.type, s->h, m->cfg.d, T, &a, &have));
  const int v0 = m->shard ? m->shard->v0 : 0;
  CK(gemv(s, PT_GEMM_OUT, L, m->output, a, T, s->logits + v0, m->vocab, EPI_STORE, nullptr));
  return DET_OK;
}

}  // namespace det

namespace {

// DETGPU_FUSED_DECODE=1 runs one-position forwards through decode_fused.cu
// where it applies; unset or 0 keeps the per-op kernels
bool fused_decode_enabled() {
  static const int on = [] {
    const char* e = std::getenv("DETGPU_FUSED_DECODE");
    return e && *e && *e != '0' ? 1 : 0;
  }();
  return on != 0;
}

FdMat fd_mat(const DevMatrix& m) {
  FdMat f;
  f.q = static_cast<const uint8_t*>(m.q);
  f.type = m.type;
  f.rows = m.rows;
  f.nb = m.nb;
  return f;
}

// Whether this session's one-position forwards run as one persistent kernel
// (decode_fused.cu).  It applies to a single-device model whose q|k|v and
// gate|up are fused and whose every weight matrix, lm_head included, is
// Q8_0 / Q4_0 in the MMA16 tile layout, with head_dim 64 or 128.  The first
// call builds the kernel's layer table; it runs outside any graph capture
// (run_forward checks it before capturing).
bool fused_decode_ready(det_session* s) {
  if (s->fd_state) return s->fd_state > 0;
  s->fd_state = -1;
  det_model* m = s->m;
  const ModelCfg& c = m->cfg;
  if (!fused_decode_enabled() || s->tp || m->shard || m->tp) return false;
  if (!attention_tiled_supported(c.nh, c.nkv, c.hd) || !s->score_scratch) return false;
  if (m->output.layout != LAYOUT_MMA16 || !m->output_norm || m->output.cols != c.d) return false;
  std::vector<FdLayer> ly((size_t)c.L);
  double wb = (double)m->output.rows * m->output.cols * bytes_per_weight(m->output.type);
  for (int l = 0; l < c.L; l++) {
    const LayerDev& W = m->layers[(size_t)l];
    if (!W.wqkv.rows || !W.wgu.rows || W.wo.layout != LAYOUT_MMA16 || W.down.layout != LAYOUT_MMA16) return false;
    FdLayer& f = ly[(size_t)l];
    f.qkv = fd_mat(W.wqkv);
    f.o = fd_mat(W.wo);
    f.gu = fd_mat(W.wgu);
    f.down = fd_mat(W.down);
    f.attn_norm = W.attn_norm;
    f.ffn_norm = W.ffn_norm;
    f.bq = W.bq;
    f.bk = W.bk;
    f.bv = W.bv;
    for (const DevMatrix* d : {&W.wqkv, &W.wo, &W.wgu, &W.down})
      wb += (double)d->rows * d->cols * bytes_per_weight(d->type);
  }
  FdParams p;
  const int s_ld = (s->n_ctx + 31) & ~31;
  if (!fused_decode_plan(c.d, c.dff, c.nh, c.nkv, c.hd, s_ld, &p)) return false;
  FdLayer* dl = nullptr;
  unsigned* sync = nullptr;
  if (dalloc(s, &dl, ly.size()) || dalloc(s, &sync, 2)) return false;
  if (cudaMemcpy(dl, ly.data(), ly.size() * sizeof(FdLayer), cudaMemcpyHostToDevice) != cudaSuccess) return false;
  int grid = 0;
  if (fused_decode_prepare(p, &grid) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  p.layers = dl;
  p.L = c.L;
  p.out = fd_mat(m->output);
  p.out_norm = m->output_norm;
  p.d = c.d;
  p.dff = c.dff;
  p.nh = c.nh;
  p.nkv = c.nkv;
  p.hd = c.hd;
  p.half = c.rope_dim / 2;
  p.pairing = c.pairing;
  p.n_ctx = s->n_ctx;
  p.s_ld = s_ld;
  p.vocab = m->vocab;
  p.eps = c.eps;
  p.scale = c.attn_scale;
  p.pos = s->d_pos;
  p.cos_t = s->rope_cos;
  p.sin_t = s->rope_sin;
  p.x = s->x;
  p.q = s->q;
  p.k = s->k;
  p.v = s->v;
  p.S = s->score_scratch;
  p.attn = s->attn;
  p.gate = s->gate;
  p.up = s->up;
  p.logits = s->logits;
  p.kc = s->kc;
  p.vc = s->vc;
  p.err = s->d_err;
  p.sync = sync;
  s->fd = p;
  s->fd_grid = grid;
  s->fd_wbytes = wb;
  s->fd_state = 1;
  return true;
}

// The one-position forward through decode_fused.cu: the embedding row, then
// one launch for every layer and the lm_head.  Algorithmic bytes: the
// weights plus the KV rows the attention reads (K and V of positions
// 0..pos in every layer).
det_status forward_fused(det_session* s, const Launch& L) {
  if (det_status st = fwd_embed(s, L, 1)) return st;
  const ModelCfg& c = s->m->cfg;
  CK(cudaMemsetAsync(s->fd.sync, 0, 2 * sizeof(unsigned), s->stream));
  const double kv = 2.0 * c.L * c.nkv * c.hd * 4.0 * (double)(*s->h_pos + 1);
  CK(timed(s, PT_FUSED, s->fd_wbytes + kv, s->fd_wbytes, [&] { return launch_decode_fused(L, s->fd, s->fd_grid); }));
  return DET_OK;
}

// forward_one_with_workspace for positions pos0 .. pos0+T-1, pos0 = *d_pos
// (tokens and pos0 already on the device)
det_status forward_chunk(det_session* s, int T, uint64_t* launch_counter) {
  Launch L = launch_of(s);
  L.launches = launch_counter;
  if (T == 1 && s->fd_state > 0) return forward_fused(s, L);
  // overlapping launches pays off for one-token (decode) forwards; for
  // chunks it measured slower
  L.pdl = T <= 16;
  if (det_status st = fwd_embed(s, L, T)) return st;
  for (int l = 0; l < s->m->cfg.L; l++) {
    int have = 0;
    if (det_status st = fwd_attention(s, L, l, T)) return st;
    if (det_status st = fwd_attn_out(s, L, l, T, s->attn)) return st;
    if (det_status st = fwd_ffn_in(s, L, l, T, &have)) return st;
    if (det_status st = fwd_ffn_out(s, L, l, T, s->ff, have)) return st;
  }
  return fwd_head(s, L, T);
}

// H2D copies of the chunk's tokens and first position, then the forward
det_status enqueue_forward(det_session* s, int T, uint64_t* launch_counter) {
  CK(cudaMemcpyAsync(s->d_tokens, s->h_tokens, (size_t)T * 4, cudaMemcpyHostToDevice, s->stream));
  CK(cudaMemcpyAsync(s->d_pos, s->h_pos, 4, cudaMemcpyHostToDevice, s->stream));
  return forward_chunk(s, T, launch_counter);
}

bool graphs_enabled() {
  static const int off = [] {
    const char* e = std::getenv("DETGPU_NO_GRAPHS");
    return e && *e && *e != '0' ? 1 : 0;
  }();
  return !off && !g_profiling;
}

// Runs the chunk forward through a CUDA graph captured once per chunk size
// (the kernels read pos0 from device memory, so one graph serves every chunk).
det_status run_forward(det_session* s, int T) {
  if (s->tp) return tp_run_forward(s, T, graphs_enabled());
  // the fused one-position forward is two launches and a memset: no graph
  // (its kernel is a cooperative launch)
  const bool fused = T == 1 && fused_decode_ready(s);
  if (!graphs_enabled() || fused) return enqueue_forward(s, T, &s->stats.launches);
  if ((int)s->graphs.size() <= T) s->graphs.resize((size_t)T + 1);
  det_session::Graph& gr = s->graphs[(size_t)T];
  if (!gr.exec) {
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
    uint64_t count = 0;
    const det_status st = enqueue_forward(s, T, &count);
    const cudaError_t ec = cudaStreamEndCapture(s->stream, &graph);
    if (st) {
      if (graph) cudaGraphDestroy(graph);
      return st;
    }
    CK(ec);
    const cudaError_t ei = cudaGraphInstantiate(&gr.exec, graph, 0);
    cudaGraphDestroy(graph);
    CK(ei);
    gr.kernels = count;
  }
  CK(cudaGraphLaunch(gr.exec, s->stream));
  s->stats.launches += gr.kernels;
  return DET_OK;
}

}  // namespace

det_status det::rc_loop_init(det_session* s) {
  if (s->d_rc) return DET_OK;
  cudaSetDevice(s->m->device);
  det_status st = dalloc(s, &s->d_rc, 1);
  if (!st) st = dalloc(s, &s->d_row0, 1);
  if (!st) st = halloc(s, &s->h_rc, 1);
  if (!st && cudaMemset(s->d_row0, 0, sizeof(uint32_t)) != cudaSuccess) st = DET_ERR_CUDA;
  if (st) s->d_rc = nullptr;
  return st;
}

// forward_one_with_workspace for the one position whose token and position
// a kernel left in s->d_tokens[0] / s->d_pos[0]: the same launches as
// run_forward(s, 1) without the host-to-device copies, in a graph of its own
det_status det::forward_device_inputs(det_session* s) {
  if (s->tp) return DET_ERR_UNSUPPORTED_MODEL_FEATURE;
  const bool fused = fused_decode_ready(s);
  if (!graphs_enabled() || fused) {
    const det_status st = forward_chunk(s, 1, &s->stats.launches);
    s->last_n = 1;
    return st;
  }
  det_session::Graph& gr = s->graph_dev1;
  if (!gr.exec) {
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
    uint64_t count = 0;
    const det_status st = forward_chunk(s, 1, &count);
    const cudaError_t ec = cudaStreamEndCapture(s->stream, &graph);
    if (st) {
      if (graph) cudaGraphDestroy(graph);
      return st;
    }
    CK(ec);
    const cudaError_t ei = cudaGraphInstantiate(&gr.exec, graph, 0);
    cudaGraphDestroy(graph);
    CK(ei);
    gr.kernels = count;
  }
  CK(cudaGraphLaunch(gr.exec, s->stream));
  s->stats.launches += gr.kernels;
  s->last_n = 1;
  return DET_OK;
}

namespace {

// e/z for the listed rows of the last forward (once per row per forward)
det_status prepare_rows(det_session* s, const uint32_t* rows, uint32_t n) {
  std::vector<uint32_t> need;
  for (uint32_t i = 0; i < n; i++)
    if (!s->cdf_ready[rows[i]]) {
      s->cdf_ready[rows[i]] = 1;
      need.push_back(rows[i]);
    }
  if (need.empty()) return DET_OK;
  // staging slots [1024, 2048) of h_rows; the query rows use [0, 1024)
  std::memcpy(s->h_rows + 1024, need.data(), need.size() * 4);
  CK(cudaMemcpyAsync(s->d_rows, s->h_rows + 1024, need.size() * 4, cudaMemcpyHostToDevice, s->stream));
  s->stats.h2d_bytes += need.size() * 4;
  CK(timed(s, PT_CDF, 0, 0, [&] {
    return launch_cdf_prepare(launch_of(s), s->logits, s->m->vocab, s->d_rows, (int)need.size(), s->cdf_e,
                              s->cdf_z);
  }));
  return DET_OK;
}

det_status check_symbols(det_session* s, int tail) {
  const uint64_t V = (uint64_t)s->m->vocab;
  if (V + (uint64_t)tail > (1u << 18)) return DET_ERR_CDF_TOO_MANY_SYMBOLS;
  return DET_OK;
}

// any Q6_K matrix with tensor-core chunk records (then chunks > 16 quantise
// into the permuted Q8_K records too)
bool model_has_q6k_tc(const det_model* m) {
  if (m->output.tc || m->tok_embd.tc) return true;
  for (const LayerDev& L : m->layers)
    for (const DevMatrix* W : {&L.wq, &L.wk, &L.wv, &L.wo, &L.gate, &L.up, &L.down})
      if (W->tc) return true;
  return false;
}

}  // namespace

det_status det::forward_enqueue(det_session* s, const uint32_t* tokens, uint32_t n, uint32_t pos0) {
  if (!s || !tokens) return DET_ERR_INVALID_ARGUMENT;
  if (n == 0 || (int)n > s->max_chunk || (uint64_t)pos0 + n > (uint64_t)s->n_ctx) return DET_ERR_SHAPE;
  det_model* m = s->m;
  for (uint32_t i = 0; i < n; i++)
    if (tokens[i] >= (uint32_t)m->vocab || tokens[i] >= (uint32_t)m->tok_embd.rows) return DET_ERR_SHAPE;
  cudaSetDevice(m->device);
  std::memcpy(s->h_tokens, tokens, n * 4);
  *s->h_pos = (int)pos0;
  s->stats.h2d_bytes += n * 4 + 4;
  CK(cudaEventRecord(s->ev[0], s->stream));
  det_status st = run_forward(s, (int)n);
  if (st) return st;
  CK(cudaEventRecord(s->ev[1], s->stream));
  s->last_n = (int)n;
  s->stats.tokens += n;
  s->fwd_timed = true;
  std::fill(s->cdf_ready.begin(), s->cdf_ready.end(), 0);
  return DET_OK;
}

void det::forward_collect(det_session* s) {
  if (!s->fwd_timed) return;
  float ms = 0.0f;
  if (cudaEventElapsedTime(&ms, s->ev[0], s->ev[1]) == cudaSuccess) s->stats.forward_ms += ms;
  s->fwd_timed = false;
}

extern "C" {

det_status det_session_create(det_model* m, uint32_t n_ctx, uint32_t max_chunk, det_session** out) {
  if (!m || !out) return DET_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  if (m->tp) return tp_session_create(m, n_ctx, max_chunk, out);
  const ModelCfg& c = m->cfg;
  // a tensor-parallel part also holds full-width inputs of wo and down
  const ModelCfg& full = m->shard ? m->shard->full : c;
  // RoPE phases pos * omega stay below 2^20 * pi/2 (the range of the
  // restated rem_pio2) for windows up to 2^20 positions.
  if (n_ctx == 0 || (int)n_ctx > c.ctx || n_ctx > (1u << 20) || max_chunk == 0 || max_chunk > 1024)
    return DET_ERR_SHAPE;
  if (cudaSetDevice(m->device) != cudaSuccess) return DET_ERR_CUDA;
  det_session* s = new (std::nothrow) det_session();
  if (!s) return DET_ERR_ALLOC;
  s->m = m;
  s->owner = m;
  s->n_ctx = (int)n_ctx;
  s->max_chunk = (int)std::min<uint32_t>(max_chunk, n_ctx);
  const size_t T = (size_t)s->max_chunk;
  const size_t qd = (size_t)c.nh * c.hd, kvd = (size_t)c.nkv * c.hd;
  const size_t kmax = std::max({(size_t)c.d, (size_t)c.dff, qd, (size_t)full.dff, (size_t)full.nh * full.hd});
  const size_t kv = (size_t)c.L * c.nkv * n_ctx * c.hd;
  det_status st = DET_OK;
  if (cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) != cudaSuccess) st = DET_ERR_CUDA;
  for (auto& e : s->ev)
    if (!st && cudaEventCreate(&e) != cudaSuccess) st = DET_ERR_CUDA;
  if (!st) st = dalloc(s, &s->x, T * c.d);
  if (!st) st = dalloc(s, &s->h, T * c.d);
  if (!st) st = dalloc(s, &s->tmp, T * c.d);
  if (!st) st = dalloc(s, &s->q, T * qd);
  if (!st) st = dalloc(s, &s->attn, T * qd);
  if (!st) st = dalloc(s, &s->k, T * kvd);
  if (!st) st = dalloc(s, &s->v, T * kvd);
  if (!st) st = dalloc(s, &s->gate, T * c.dff);
  if (!st) st = dalloc(s, &s->up, T * c.dff);
  if (!st) st = dalloc(s, &s->ff, T * c.dff);
  if (!st) st = dalloc(s, &s->logits, T * (size_t)m->vocab);
  if (!st && m->shard) {
    st = dalloc(s, &s->ff_full, T * full.dff);
    if (!st && m->shard->attn_sharded) st = dalloc(s, &s->attn_full, T * (size_t)full.nh * full.hd);
  }
  // Q8A buffers cover whole 64-position groups; the padding positions stay
  // zero so the chunk GEMM may read (and discard) them.
  const size_t Tg = (T + 63) / 64 * 64;
  if (!st) st = dalloc(s, &s->qa_d, Tg * (kmax / 32));
  if (!st) st = dalloc(s, &s->qa_q, Tg * kmax);
  if (!st && (cudaMemset(s->qa_d, 0, Tg * (kmax / 32) * sizeof(float)) != cudaSuccess ||
              cudaMemset(s->qa_q, 0, Tg * kmax) != cudaSuccess))
    st = DET_ERR_CUDA;
  if (!st) st = dalloc(s, &s->qk_d, T * (kmax / 256 + 1));
  if (!st) st = dalloc(s, &s->qk_q, T * kmax + 64);
  if (!st && T > 16 && model_has_q6k_tc(m)) st = dalloc(s, &s->qk_p, q6k_tc_act_bytes((int)T, (int)kmax));
  if (!st) st = dalloc(s, &s->kc, kv);
  if (!st) st = dalloc(s, &s->vc, kv);
  if (!st) st = dalloc(s, &s->rope_cos, (size_t)n_ctx * (c.rope_dim / 2));
  if (!st) st = dalloc(s, &s->rope_sin, (size_t)n_ctx * (c.rope_dim / 2));
  if (!st) {
    const size_t sf = attention_scratch_floats((int)T, c.nh, c.nkv, c.hd, (int)n_ctx);
    if (sf) st = dalloc(s, &s->score_scratch, sf);
  }
  if (!st) st = dalloc(s, &s->cdf_e, T * (size_t)m->vocab);
  if (!st) st = dalloc(s, &s->cdf_z, T);
  if (!st) st = dalloc(s, &s->d_tokens, T);
  if (!st) st = dalloc(s, &s->d_pos, 1);
  if (!st) st = halloc(s, &s->h_pos, 1);
  if (!st) st = dalloc(s, &s->d_rows, 2048);
  if (!st) st = dalloc(s, &s->d_syms, std::max<size_t>(T, 1024) * 4);
  if (!st) st = dalloc(s, &s->d_out, std::max<size_t>(T, 1024) * 4 * 3);
  if (!st) st = dalloc(s, &s->d_value, 8);
  if (!st) st = dalloc(s, &s->d_err, 4);
  if (!st) st = halloc(s, &s->h_tokens, T);
  if (!st) st = halloc(s, &s->h_rows, 2048);
  if (!st) st = halloc(s, &s->h_syms, std::max<size_t>(T, 1024) * 4);
  if (!st) st = halloc(s, &s->h_out, std::max<size_t>(T, 1024) * 4 * 3);
  if (!st) st = halloc(s, &s->h_value, 8);
  if (!st) st = halloc(s, &s->h_err, 4);
  if (!st && cudaMemsetAsync(s->d_err, 0, 4, s->stream) != cudaSuccess) st = DET_ERR_CUDA;
  if (!st) st = cuda_status(cudaMemsetAsync(s->kc, 0, kv * 4, s->stream));
  if (!st) st = cuda_status(cudaMemsetAsync(s->vc, 0, kv * 4, s->stream));
  if (!st)
    st = cuda_status(launch_rope_table(launch_of(s), s->rope_cos, s->rope_sin, (int)n_ctx, c.rope_dim / 2,
                                       c.rope_dim, c.rope_base));
  if (!st) st = take_error(s, false);
  if (st) {
    free_session(s);
    return st;
  }
  s->cdf_ready.assign(T, 0);
  *out = s;
  return DET_OK;
}

void det_session_free(det_session* s) { free_session(s); }

det_status det_session_reset(det_session* s) {
  if (!s) return DET_ERR_INVALID_ARGUMENT;
  if (s->tp)
    if (det_status st = tp_reset(s)) return st;
  cudaSetDevice(s->m->device);
  const ModelCfg& c = s->m->cfg;
  const size_t kv = (size_t)c.L * c.nkv * s->n_ctx * c.hd;
  // KvCache::new is all zeros; a replayed window only reads positions it
  // has written, so clearing is for exact state parity, not correctness.
  CK(cudaMemsetAsync(s->kc, 0, kv * 4, s->stream));
  CK(cudaMemsetAsync(s->vc, 0, kv * 4, s->stream));
  s->last_n = 0;
  return DET_OK;
}

det_status det_forward(det_session* s, const uint32_t* tokens, uint32_t n, uint32_t pos0, float* logits_out) {
  if (det_status st = forward_enqueue(s, tokens, n, pos0)) return st;
  det_model* m = s->m;
  det_status st = DET_OK;
  if (logits_out) {
    const size_t bytes = (size_t)n * m->vocab * 4;
    CK(cudaMemcpyAsync(logits_out, s->logits, bytes, cudaMemcpyDeviceToHost, s->stream));
    s->stats.d2h_bytes += bytes;
  }
  st = take_error(s, false);
  forward_collect(s);
  if (st) s->last_n = 0;
  return st;
}

det_status det_symbol_ranges(det_session* s, const uint32_t* rows, const uint32_t* symbols, uint32_t n,
                             int byte_escapes, det_symbol_range* out) {
  if (!s || (!symbols && n) || (!out && n)) return DET_ERR_INVALID_ARGUMENT;
  if (n == 0) return DET_OK;
  const int tail = byte_escapes ? 256 : 0;
  if (det_status st = check_symbols(s, tail)) return st;
  const uint32_t V = (uint32_t)s->m->vocab;
  cudaSetDevice(s->m->device);
  const uint32_t cap = 1024;
  for (uint32_t base = 0; base < n; base += cap) {
    const uint32_t cnt = std::min(cap, n - base);
    for (uint32_t i = 0; i < cnt; i++) {
      const uint32_t r = rows ? rows[base + i] : base + i;
      if (r >= (uint32_t)s->last_n) return DET_ERR_SHAPE;
      if (symbols[base + i] >= V + (uint32_t)tail) return DET_ERR_CDF_SYMBOL_OUT_OF_RANGE;
      s->h_rows[i] = r;
      s->h_syms[i] = symbols[base + i];
    }
    CK(cudaEventRecord(s->ev[2], s->stream));
    if (det_status st = prepare_rows(s, s->h_rows, cnt)) return st;
    CK(cudaMemcpyAsync(s->d_rows + 1024, s->h_rows, cnt * 4, cudaMemcpyHostToDevice, s->stream));
    CK(cudaMemcpyAsync(s->d_syms, s->h_syms, cnt * 4, cudaMemcpyHostToDevice, s->stream));
    s->stats.h2d_bytes += cnt * 8;
    CK(timed(s, PT_CDF, 0, 0, [&] {
      return launch_cdf_ranges(launch_of(s), s->cdf_e, s->cdf_z, (int)V, tail, s->d_rows + 1024, s->d_syms, (int)cnt,
                              s->d_out);
    }));
    CK(cudaEventRecord(s->ev[3], s->stream));
    CK(cudaMemcpyAsync(s->h_out, s->d_out, cnt * 24, cudaMemcpyDeviceToHost, s->stream));
    s->stats.d2h_bytes += cnt * 24;
    if (det_status st = take_error(s, true)) return st;
    forward_collect(s);  // a forward enqueued without a synchronisation has run
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, s->ev[2], s->ev[3]) == cudaSuccess) s->stats.cdf_ms += ms;
    for (uint32_t i = 0; i < cnt; i++) {
      out[base + i].cum = s->h_out[3 * i];
      out[base + i].freq = (uint32_t)s->h_out[3 * i + 1];
      out[base + i].reserved = 0;
      out[base + i].total = s->h_out[3 * i + 2];
    }
  }
  return DET_OK;
}

det_status det_decoder_total(det_session* s, uint32_t row, int byte_escapes, uint64_t* total) {
  if (!s || !total) return DET_ERR_INVALID_ARGUMENT;
  const uint32_t sym = 0;
  det_symbol_range r;
  det_status st = det_symbol_ranges(s, &row, &sym, 1, byte_escapes, &r);
  if (st) return st;
  *total = r.total;
  return DET_OK;
}

det_status det_decoder_lookup(det_session* s, uint32_t row, int byte_escapes, uint64_t value, uint32_t* symbol,
                              det_symbol_range* out) {
  if (!s || !symbol || !out) return DET_ERR_INVALID_ARGUMENT;
  const int tail = byte_escapes ? 256 : 0;
  if (det_status st = check_symbols(s, tail)) return st;
  if (row >= (uint32_t)s->last_n) return DET_ERR_SHAPE;
  cudaSetDevice(s->m->device);
  if (det_status st = prepare_rows(s, &row, 1)) return st;
  *s->h_value = value;
  CK(cudaMemcpyAsync(s->d_value, s->h_value, 8, cudaMemcpyHostToDevice, s->stream));
  CK(timed(s, PT_CDF, 0, 0, [&] {
    return launch_decoder_lookup(launch_of(s), s->cdf_e, s->cdf_z, s->m->vocab, tail, row, s->d_value, s->d_out);
  }));
  CK(cudaMemcpyAsync(s->h_out, s->d_out, 32, cudaMemcpyDeviceToHost, s->stream));
  s->stats.h2d_bytes += 8;
  s->stats.d2h_bytes += 32;
  if (det_status st = take_error(s, true)) return st;
  if (value >= s->h_out[3]) return DET_ERR_DECODE;
  *symbol = (uint32_t)s->h_out[0];
  out->cum = s->h_out[1];
  out->freq = (uint32_t)s->h_out[2];
  out->reserved = 0;
  out->total = s->h_out[3];
  return DET_OK;
}

det_status det_logits_hash(det_model* m, const uint32_t* tokens, size_t n, uint32_t chunk, uint8_t out[32]) {
  if (!m || !tokens || !out) return DET_ERR_INVALID_ARGUMENT;
  // validate_logits_request (det-model lib.rs:1467-1483)
  if (n == 0 || chunk == 0 || n > (size_t)m->cfg.ctx) return DET_ERR_SHAPE;
  for (size_t i = 0; i < n; i++)
    if (tokens[i] >= (uint32_t)m->tok_embd.rows) return DET_ERR_SHAPE;
  det_session* s;
  const uint32_t T = std::min<uint32_t>(chunk, 256);
  if (det_status st = det_session_create(m, (uint32_t)n, T, &s)) return st;
  std::vector<float> buf((size_t)T * m->vocab);
  Sha256 h;
  det_status st = DET_OK;
  for (size_t p = 0; p < n && !st; p += T) {
    const uint32_t cnt = (uint32_t)std::min<size_t>(T, n - p);
    st = det_forward(s, tokens + p, cnt, (uint32_t)p, buf.data());
    if (!st) h.update(buf.data(), (size_t)cnt * m->vocab * 4);  // little-endian f32 bits
  }
  det_session_free(s);
  if (!st) h.finish(out);
  return st;
}

det_status det_device_expf(int device, const float* x, float* y, size_t n) {
  if ((!x || !y) && n) return DET_ERR_INVALID_ARGUMENT;
  int cnt = 0;
  if (cudaGetDeviceCount(&cnt) != cudaSuccess || cnt == 0) return DET_ERR_NO_DEVICE;
  if (device < 0 || device >= cnt) return DET_ERR_INVALID_ARGUMENT;
  if (n == 0) return DET_OK;
  CK(cudaSetDevice(device));
  float *dx = nullptr, *dy = nullptr;
  const size_t chunk = std::min<size_t>(n, (size_t)1 << 26);
  CK(cudaMalloc(&dx, chunk * 4));
  if (cudaMalloc(&dy, chunk * 4) != cudaSuccess) {
    cudaFree(dx);
    return DET_ERR_DEVICE_OOM;
  }
  cudaError_t e = cudaSuccess;
  for (size_t b = 0; b < n && e == cudaSuccess; b += chunk) {
    const size_t c = std::min(chunk, n - b);
    e = cudaMemcpy(dx, x + b, c * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = launch_expf(nullptr, dx, dy, (long long)c);
    if (e == cudaSuccess) e = cudaMemcpy(y + b, dy, c * 4, cudaMemcpyDeviceToHost);
  }
  cudaFree(dx);
  cudaFree(dy);
  return cuda_status(e);
}

det_status det_add_latency_cycles(int device, double* cycles_per_add) {
  if (!cycles_per_add) return DET_ERR_INVALID_ARGUMENT;
  int cnt = 0;
  if (cudaGetDeviceCount(&cnt) != cudaSuccess || cnt == 0) return DET_ERR_NO_DEVICE;
  if (device < 0 || device >= cnt) return DET_ERR_INVALID_ARGUMENT;
  CK(cudaSetDevice(device));
  void* mem = nullptr;
  CK(cudaMalloc(&mem, 1024));  // 64 inputs (zeros), 32 outputs, the cycle count
  float* x = static_cast<float*>(mem);
  long long* cyc = reinterpret_cast<long long*>(static_cast<char*>(mem) + 768);
  const int n = 4096;
  cudaError_t e = cudaMemset(mem, 0, 1024);
  double best = 0.0;
  for (int rep = 0; rep < 3 && e == cudaSuccess; rep++) {  // the first run also loads the code
    long long c = 0;
    e = launch_add_chain(x, x + 64, cyc, n);
    if (e == cudaSuccess) e = cudaMemcpy(&c, cyc, sizeof c, cudaMemcpyDeviceToHost);
    const double v = (double)c / (2.0 * n);
    if (e == cudaSuccess && (best == 0.0 || v < best)) best = v;
  }
  cudaFree(mem);
  if (e != cudaSuccess) return cuda_status(e);
  *cycles_per_add = best;
  return DET_OK;
}

det_status det_session_gemv_stream(det_session* s, uint32_t reps, double* ms_per_pass, double* bytes_per_pass) {
  if (!s || !ms_per_pass || !bytes_per_pass || reps == 0) return DET_ERR_INVALID_ARGUMENT;
  if (s->tp) return DET_ERR_UNSUPPORTED_MODEL_FEATURE;
  det_model* m = s->m;
  const ModelCfg& c = m->cfg;
  cudaSetDevice(m->device);
  // the weight GEMVs of one single-token forward, outputs into scratch rows
  // (the logits and FFN buffers, which this call invalidates)
  Launch L = launch_of(s);
  uint64_t count = 0;
  L.launches = &count;
  L.pdl = true;
  DevActs a;
  a.x = s->h;
  a.qa_d = s->qa_d;
  a.qa_q = s->qa_q;
  a.qk_d = s->qk_d;
  a.qk_q = s->qk_q;
  double bytes = 0;
  auto add_bytes = [&](const DevMatrix& W) {
    bytes += (double)W.rows * W.cols * bytes_per_weight(W.type) + W.cols * (1.0 + 4.0 / 32.0) + W.rows * 4.0;
  };
  auto enqueue = [&]() -> cudaError_t {
    bytes = 0;
    for (int l = 0; l < c.L; l++) {
      const LayerDev& W = m->layers[(size_t)l];
      cudaError_t e;
      if (W.wqkv.rows) {
        OutSegs o;
        o.n = 1;
        o.s[0] = OutSeg{W.wqkv.rows, s->logits, W.wqkv.rows, EPI_STORE, nullptr};
        e = launch_gemm_mma16(L, W.wqkv, a, 1, o);
        add_bytes(W.wqkv);
      } else if (const DevMatrix* mq[3] = {&W.wq, &W.wk, &W.wv}; kq_fusable(mq, 3)) {
        float* const oo[3] = {s->logits, s->logits + W.wq.rows, s->logits + W.wq.rows + W.wk.rows};
        const int ee[3] = {EPI_STORE, EPI_STORE, EPI_STORE};
        const float* const bb[3] = {nullptr, nullptr, nullptr};
        e = launch_gemv_kq_decode_segs(L, mq, 3, a, oo, ee, bb);
        for (const DevMatrix* Wm : mq) add_bytes(*Wm);
      } else {
        for (const DevMatrix* Wm : {&W.wq, &W.wk, &W.wv}) {
          if ((e = launch_gemv(L, *Wm, a, 1, s->logits, Wm->rows, EPI_STORE, nullptr)) != cudaSuccess) return e;
          add_bytes(*Wm);
        }
      }
      if (e != cudaSuccess) return e;
      if ((e = launch_gemv(L, W.wo, a, 1, s->gate, W.wo.rows, EPI_STORE, nullptr)) != cudaSuccess) return e;
      add_bytes(W.wo);
      if (W.wgu.rows) {
        OutSegs o;
        o.n = 1;
        o.s[0] = OutSeg{W.wgu.rows, s->logits, W.wgu.rows, EPI_STORE, nullptr};
        e = launch_gemm_mma16(L, W.wgu, a, 1, o);
        add_bytes(W.wgu);
      } else if (const DevMatrix* mg[2] = {&W.gate, &W.up}; kq_fusable(mg, 2)) {
        float* const oo[2] = {s->logits, s->logits + W.gate.rows};
        const int ee[2] = {EPI_STORE, EPI_STORE};
        const float* const bb[2] = {nullptr, nullptr};
        e = launch_gemv_kq_decode_segs(L, mg, 2, a, oo, ee, bb);
        for (const DevMatrix* Wm : mg) add_bytes(*Wm);
      } else {
        for (const DevMatrix* Wm : {&W.gate, &W.up}) {
          if ((e = launch_gemv(L, *Wm, a, 1, s->logits, Wm->rows, EPI_STORE, nullptr)) != cudaSuccess) return e;
          add_bytes(*Wm);
        }
      }
      if (e != cudaSuccess) return e;
      if ((e = launch_gemv(L, W.down, a, 1, s->gate, W.down.rows, EPI_STORE, nullptr)) != cudaSuccess) return e;
      add_bytes(W.down);
    }
    add_bytes(m->output);
    return launch_gemv(L, m->output, a, 1, s->logits, m->vocab, EPI_STORE, nullptr);
  };
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  CK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
  const cudaError_t eq = enqueue();
  const cudaError_t ec = cudaStreamEndCapture(s->stream, &graph);
  if (eq != cudaSuccess || ec != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    return cuda_status(eq != cudaSuccess ? eq : ec);
  }
  const cudaError_t ei = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  CK(ei);
  cudaError_t e = cudaGraphLaunch(exec, s->stream);  // warm-up
  if (e == cudaSuccess) e = cudaEventRecord(s->ev[2], s->stream);
  for (uint32_t i = 0; i < reps && e == cudaSuccess; i++) e = cudaGraphLaunch(exec, s->stream);
  if (e == cudaSuccess) e = cudaEventRecord(s->ev[3], s->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  float ms = 0.0f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, s->ev[2], s->ev[3]);
  cudaGraphExecDestroy(exec);
  CK(e);
  s->last_n = 0;  // the logits were overwritten
  std::fill(s->cdf_ready.begin(), s->cdf_ready.end(), 0);
  *ms_per_pass = (double)ms / reps;
  *bytes_per_pass = bytes;
  // the outputs are discarded: clear any flag their values raised
  CK(cudaMemsetAsync(s->d_err, 0, 4, s->stream));
  CK(cudaStreamSynchronize(s->stream));
  return DET_OK;
}

det_status det_session_stats(det_session* s, det_stats* out, int reset) {
  if (!s || !out) return DET_ERR_INVALID_ARGUMENT;
  *out = s->stats;
  if (reset) s->stats = det_stats{};
  return DET_OK;
}

det_status det_model_stats(det_model* m, det_stats* out, int reset) {
  if (!m || !out) return DET_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::recursive_mutex> lk(m->mu);
  *out = m->agg;
  if (m->cached) {  // include the live cached session
    add_stats(out, m->cached->stats);
    if (reset) m->cached->stats = det_stats{};
  }
  if (reset) m->agg = det_stats{};
  return DET_OK;
}

det_status det_model_profile(det_model* m, char* out, size_t cap, int reset) {
  if (!m || (!out && cap)) return DET_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::recursive_mutex> lk(m->mu);
  ProfTags p = m->prof_agg;
  if (m->cached) {
    add_prof(&p, m->cached->prof);
    if (reset) m->cached->prof = ProfTags{};
  }
  if (reset) m->prof_agg = ProfTags{};
  std::string js = "{";
  for (int i = 0; i < PT_COUNT; i++) {
    char buf[128];
    std::snprintf(buf, sizeof buf, "%s\"%s\": [%llu, %.6f]", i ? ", " : "", kProfTagNames[i],
                  (unsigned long long)p.n[i], p.ms[i]);
    js += buf;
  }
  js += "}";
  if (js.size() + 1 > cap) return DET_ERR_INVALID_ARGUMENT;
  std::memcpy(out, js.c_str(), js.size() + 1);
  return DET_OK;
}

det_status det_set_profiling(int enable) {
  g_profiling = enable != 0;
  return DET_OK;
}

}  // extern "C"
