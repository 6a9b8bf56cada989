// tp.cpp -- row-sharded tensor parallelism for single-stream latency.
//
// The reference splits each GEMV's output rows over worker threads
// (gemv_rows_parallel, crates/det-model/src/lib.rs:291-321); every row is
// one reduction, so the split cannot change a result.  Here the split is over
// devices.  Part p of G owns contiguous 64-row slices of the rows of wo,
// ffn_gate, ffn_up, ffn_down and the lm_head and, when head_count_kv % G == 0,
// kv heads [h0, h1) with their query heads, q/k/v rows and KV cache.  Every
// part keeps the whole residual stream and runs the row-wise ops (RMSNorm,
// the activation quantisers, RoPE) itself.  Per layer the parts exchange:
//   attention output (when the heads are sharded), before wo
//   residual x, after wo            (each part adds its rows of wo)
//   SwiGLU output, before ffn_down
//   residual x, after ffn_down
// and after the lm_head the primary part (devices[0], which runs the CDF)
// gathers the logits.  exchange.cu does the copies; this file plans them and
// orders them one of two ways:
//  * parts on distinct GPUs: each part runs its own stream (one CUDA graph
//    per part and chunk size), and each exchange is one kernel that signals
//    the peers through counters in their memory, waits for theirs (bounded)
//    and pulls; with replicated attention a data-free exchange stands in for
//    the attention exchange;
//  * parts sharing a GPU (kernels that wait on one another must never share
//    one): host events order the pulls, and the whole multi-device forward is
//    captured in one CUDA graph per chunk size.  DETGPU_TP_EVENTS=1 selects
//    this form for distinct GPUs too.
//
// Ordering.  A gather waits for every other part's event recorded after
// that part wrote its slice (read-after-write).  A part rewrites a slice
// another part reads only after an exchange that waited for the reader
// (write-after-read): the attention output and the SwiGLU output are
// rewritten a layer later, past two exchanges; x's slice is rewritten by
// down after the SwiGLU exchange and by the next layer's wo after the
// attention exchange -- or, when the attention is replicated and that
// exchange does not exist, after a wait on every part's `done` event of the
// previous layer's last gather.  Eager forwards also wait, on entry, for the
// other parts' last exchange of the previous forward; a graph forward is one
// unit on part 0's stream.  The device-side form keeps the same order: each
// exchange kernel is an all-to-all barrier (it signals, then waits for every
// peer), the replicated-attention barrier takes the place of the `done` wait,
// and det_forward synchronises every part before it returns.
//
// Weights: one replica per distinct device; each part's model (a "shard")
// views its replica's matrices through row offsets and owns only the fused
// q|k|v and gate|up buffers of its slices.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <new>
#include <thread>

#include "host_common.h"

using namespace det;

namespace det {

struct TpModel {
  std::vector<int> devices;          // device of each part
  std::vector<det_model*> replicas;  // one per distinct device; [0] is the caller's model
  std::vector<det_model*> shards;    // one per part
};

struct TpSession {
  std::vector<det_session*> parts;   // [0] is the session the caller holds
  // distinct GPUs: device-side ordering (flag[p]: part p's counters, one per
  // part; epoch[p]: forwards started on part p)
  bool device_sync = false;
  std::vector<unsigned long long*> flag, epoch;
  // per part, recorded at every exchange: [0] eager forwards, [1] inside
  // graph captures (an event recorded in a capture is not waited on outside)
  std::vector<cudaEvent_t> ev[2];
  // per part, recorded after its last gather of a layer (same [0] / [1] split)
  std::vector<cudaEvent_t> done[2];
  std::vector<cudaEvent_t> join;     // per part, end of a captured forward
  cudaEvent_t fork = nullptr;        // start of a captured forward (on part 0)
};

}  // namespace det

namespace {

#define CK(expr)                                   \
  do {                                             \
    const cudaError_t e_ = (expr);                 \
    if (e_ != cudaSuccess) return cuda_status(e_); \
  } while (0)

constexpr int kRowGrain = 64;  // slice boundaries: whole tiles of every GEMM kernel

// boundaries b[0..G] of G contiguous, balanced slices of `rows` rows
std::vector<int> split_rows(int rows, int G) {
  std::vector<int> b((size_t)G + 1);
  const long long tiles = rows / kRowGrain;
  for (int p = 0; p <= G; p++) b[(size_t)p] = (int)(tiles * p / G) * kRowGrain;
  b[(size_t)G] = rows;
  return b;
}

// rows [r0, r1) of a device matrix, in place (r0 a multiple of 16)
DevMatrix row_view(const DevMatrix& M, int r0, int r1) {
  DevMatrix v = M;
  v.rows = r1 - r0;
  const size_t r = (size_t)r0;
  const uint8_t* q = static_cast<const uint8_t*>(M.q);
  switch (M.type) {
    case GT_F32:
      v.f = M.f + r * (size_t)M.cols;
      break;
    case GT_Q8_0:
    case GT_Q4_0:
      if (M.layout == LAYOUT_MMA16) {
        v.q = q + (r / 16) * (size_t)M.nb * (M.type == GT_Q8_0 ? 544 : 288);
        v.tc = nullptr;  // parts run the mma.sync chunk GEMM (the tensor-core copy has 128-row tiles)
      } else {
        v.q = q + r * (size_t)(M.type == GT_Q8_0 ? M.cols : M.cols / 2);
        v.d = M.d + r * (size_t)M.nb;
      }
      break;
    case GT_Q4_K:
      v.q = q + r * (size_t)M.nb * 144;
      break;
    default:  // GT_Q6_K
      v.q = q + r * (size_t)M.nb * 208;
      v.d = M.d + r * (size_t)M.nb;
      if (M.tc) v.tc = M.tc + q6k_tc_row_offset(r0, M.nb);  // r0: a multiple of 64 (kRowGrain)
      break;
  }
  return v;
}

// One LAYOUT_MMA16 buffer holding `parts` back to back (as model.cpp's
// fuse_matrices, but copying views and leaving them in place).  *fused stays
// empty (rows 0) when the parts cannot be fused.
det_status fuse_views(det_model* owner, const DevMatrix* parts, int n, DevMatrix* fused) {
  *fused = DevMatrix();
  int rows = 0;
  for (int i = 0; i < n; i++) {
    const DevMatrix& p = parts[i];
    if (p.layout != LAYOUT_MMA16 || p.type != parts[0].type || p.cols != parts[0].cols || p.rows == 0) return DET_OK;
    if (i + 1 < n && p.rows % 16) return DET_OK;
    rows += p.rows;
  }
  const size_t rec = parts[0].type == GT_Q8_0 ? 544 : 288;
  size_t bytes = 0;
  for (int i = 0; i < n; i++) bytes += (size_t)((parts[i].rows + 15) / 16) * parts[i].nb * rec;
  void* buf = nullptr;
  if (cudaMalloc(&buf, bytes) != cudaSuccess) return DET_ERR_DEVICE_OOM;
  owner->allocations.push_back(buf);
  size_t off = 0;
  for (int i = 0; i < n; i++) {
    const size_t b = (size_t)((parts[i].rows + 15) / 16) * parts[i].nb * rec;
    CK(cudaMemcpy(static_cast<uint8_t*>(buf) + off, parts[i].q, b, cudaMemcpyDeviceToDevice));
    off += b;
  }
  *fused = parts[0];
  fused->rows = rows;
  fused->q = buf;
  return DET_OK;
}

void free_shard(det_model* S) {
  if (!S) return;
  cudaSetDevice(S->device);
  for (void* p : S->allocations) cudaFree(p);
  delete S->shard;
  delete S;
}

// the model of part p: views of replica R's weights
det_status make_shard(det_model* R, int p, int G, bool attn_sharded, det_model** out) {
  *out = nullptr;
  det_model* S = new (std::nothrow) det_model();
  if (!S) return DET_ERR_ALLOC;
  TpShard* sh = new (std::nothrow) TpShard();
  if (!sh) {
    delete S;
    return DET_ERR_ALLOC;
  }
  S->shard = sh;
  const ModelCfg& c = R->cfg;
  S->device = R->device;
  S->cfg = c;
  S->vocab = R->vocab;
  std::memcpy(S->sha, R->sha, 32);
  S->tok_status = R->tok_status;
  S->tok = R->tok;
  S->tok_embd = R->tok_embd;
  S->tied = R->tied;
  S->output_norm = R->output_norm;
  std::memcpy(S->weight_types, R->weight_types, sizeof S->weight_types);
  S->has_bias = R->has_bias;
  sh->part = p;
  sh->parts = G;
  sh->attn_sharded = attn_sharded;
  sh->full = c;
  const std::vector<int> bd = split_rows(c.d, G), bf = split_rows(c.dff, G), bv = split_rows(R->vocab, G);
  sh->d0 = bd[(size_t)p];
  sh->d1 = bd[(size_t)p + 1];
  sh->f0 = bf[(size_t)p];
  sh->f1 = bf[(size_t)p + 1];
  sh->v0 = bv[(size_t)p];
  sh->v1 = bv[(size_t)p + 1];
  sh->h0 = attn_sharded ? c.nkv * p / G : 0;
  sh->h1 = attn_sharded ? c.nkv * (p + 1) / G : c.nkv;
  const int gsz = c.nh / c.nkv;
  S->cfg.nkv = sh->h1 - sh->h0;
  S->cfg.nh = S->cfg.nkv * gsz;
  S->cfg.dff = sh->f1 - sh->f0;
  S->output = row_view(R->output, sh->v0, sh->v1);
  const int q0 = sh->h0 * gsz * c.hd, q1 = sh->h1 * gsz * c.hd, k0 = sh->h0 * c.hd, k1 = sh->h1 * c.hd;
  S->layers.resize(R->layers.size());
  det_status st = DET_OK;
  for (size_t l = 0; l < R->layers.size() && !st; l++) {
    const LayerDev& W = R->layers[l];
    LayerDev& D = S->layers[l];
    D.attn_norm = W.attn_norm;
    D.ffn_norm = W.ffn_norm;
    if (attn_sharded) {
      D.wq = row_view(W.wq, q0, q1);
      D.wk = row_view(W.wk, k0, k1);
      D.wv = row_view(W.wv, k0, k1);
      D.bq = W.bq ? W.bq + q0 : nullptr;
      D.bk = W.bk ? W.bk + k0 : nullptr;
      D.bv = W.bv ? W.bv + k0 : nullptr;
      const DevMatrix qkv[3] = {D.wq, D.wk, D.wv};
      st = fuse_views(S, qkv, 3, &D.wqkv);
    } else {
      D.wq = W.wq;
      D.wk = W.wk;
      D.wv = W.wv;
      D.wqkv = W.wqkv;
      D.bq = W.bq;
      D.bk = W.bk;
      D.bv = W.bv;
    }
    D.wo = row_view(W.wo, sh->d0, sh->d1);
    D.gate = row_view(W.gate, sh->f0, sh->f1);
    D.up = row_view(W.up, sh->f0, sh->f1);
    D.down = row_view(W.down, sh->d0, sh->d1);
    if (!st) {
      const DevMatrix gu[2] = {D.gate, D.up};
      st = fuse_views(S, gu, 2, &D.wgu);
    }
  }
  if (st) {
    free_shard(S);
    return st;
  }
  *out = S;
  return DET_OK;
}

// ---- the forward ------------------------------------------------------------
// X_BARRIER: no data, every part waits for every other (device-side form)
enum XKind { X_ATTN, X_RESID, X_FF, X_LOGITS, X_BARRIER };

det_status set_dev(const det_session* s) { return cuda_status(cudaSetDevice(s->m->device)); }

Launch part_launch(det_session* s, uint64_t* counter) {
  Launch L{s->stream, s->d_err, counter};
  L.pdl = false;
  return L;
}

// The slices part p pulls for an exchange of `kind` into *dst (row stride *ld).
GatherPlan plan_for(TpSession& ts, XKind kind, int p, float** dst, int* ld) {
  const int G = (int)ts.parts.size();
  det_session* sp = ts.parts[(size_t)p];
  GatherPlan g;
  *dst = nullptr;
  *ld = 0;
  for (int q = 0; q < G && kind != X_BARRIER; q++) {
    if ((kind == X_RESID || kind == X_LOGITS) && q == p) continue;
    det_session* sq = ts.parts[(size_t)q];
    const TpShard& sh = *sq->m->shard;
    const ModelCfg& full = sh.full;
    GatherSrc src{nullptr, 0, 0, 0};
    switch (kind) {
      case X_ATTN: {
        const int qd = sq->m->cfg.nh * full.hd;
        src = GatherSrc{sq->attn, qd, sh.h0 * (full.nh / full.nkv) * full.hd, qd};
        *dst = sp->attn_full;
        *ld = full.nh * full.hd;
        break;
      }
      case X_RESID:
        src = GatherSrc{sq->x + sh.d0, full.d, sh.d0, sh.d1 - sh.d0};
        *dst = sp->x;
        *ld = full.d;
        break;
      case X_FF:
        src = GatherSrc{sq->ff, sh.f1 - sh.f0, sh.f0, sh.f1 - sh.f0};
        *dst = sp->ff_full;
        *ld = full.dff;
        break;
      case X_LOGITS:
        src = GatherSrc{sq->logits + sh.v0, sq->m->vocab, sh.v0, sh.v1 - sh.v0};
        *dst = sp->logits;
        *ld = sq->m->vocab;
        break;
      case X_BARRIER:
        break;
    }
    if (src.n > 0) g.s[g.n++] = src;
  }
  return g;
}

// Every part records its event; each part that gathers waits for the
// others' and pulls their slices.  X_RESID / X_LOGITS gather into the buffer
// the slices live in (a part's own slice is already there); X_ATTN / X_FF
// gather every part's local output into a separate full-width buffer.
// `mark_done`: each part then records its `done` event after its gather.
det_status exchange(TpSession& ts, XKind kind, int T, uint64_t* counter, bool capture, bool mark_done = false) {
  const int G = (int)ts.parts.size();
  const std::vector<cudaEvent_t>& ev = ts.ev[capture ? 1 : 0];
  for (int p = 0; p < G; p++) {
    if (det_status st = set_dev(ts.parts[(size_t)p])) return st;
    CK(cudaEventRecord(ev[(size_t)p], ts.parts[(size_t)p]->stream));
  }
  for (int p = 0; p < G; p++) {
    if (kind == X_LOGITS && p) break;
    det_session* sp = ts.parts[(size_t)p];
    if (det_status st = set_dev(sp)) return st;
    for (int q = 0; q < G; q++)
      if (q != p) CK(cudaStreamWaitEvent(sp->stream, ev[(size_t)q], 0));
    float* dst = nullptr;
    int ld = 0;
    const GatherPlan g = plan_for(ts, kind, p, &dst, &ld);
    CK(launch_gather_cols(part_launch(sp, counter), g, dst, ld, T));
    if (mark_done) CK(cudaEventRecord(ts.done[capture ? 1 : 0][(size_t)p], sp->stream));
  }
  return DET_OK;
}

// Enqueues one chunk forward on every part.  `capture`: inside a stream
// capture begun on part 0's stream (the other parts fork from it and join
// back at the end).  Otherwise every part first waits for the other parts'
// last exchange, so no part overwrites a slice another may still be reading.
det_status tp_enqueue(det_session* s0, int T, uint64_t* counter, bool capture) {
  TpSession& ts = *s0->tp;
  const int G = (int)ts.parts.size();
  auto part = [&](int p) { return ts.parts[(size_t)p]; };
  if (capture) {
    if (det_status st = set_dev(s0)) return st;
    CK(cudaEventRecord(ts.fork, s0->stream));
    for (int p = 1; p < G; p++) {
      if (det_status st = set_dev(part(p))) return st;
      CK(cudaStreamWaitEvent(part(p)->stream, ts.fork, 0));
    }
  } else {
    for (int p = 0; p < G; p++) {
      if (det_status st = set_dev(part(p))) return st;
      for (int q = 0; q < G; q++)
        if (q != p) CK(cudaStreamWaitEvent(part(p)->stream, ts.ev[0][(size_t)q], 0));
    }
  }
  for (int p = 0; p < G; p++) {
    det_session* s = part(p);
    if (det_status st = set_dev(s)) return st;
    CK(cudaMemcpyAsync(s->d_tokens, s->h_tokens, (size_t)T * 4, cudaMemcpyHostToDevice, s->stream));
    CK(cudaMemcpyAsync(s->d_pos, s->h_pos, 4, cudaMemcpyHostToDevice, s->stream));
    if (det_status st = fwd_embed(s, part_launch(s, counter), T)) return st;
  }
  const bool attn_sharded = s0->m->shard->attn_sharded;
  const int L = s0->m->cfg.L;
  for (int l = 0; l < L; l++) {
    for (int p = 0; p < G; p++) {
      if (det_status st = set_dev(part(p))) return st;
      if (det_status st = fwd_attention(part(p), part_launch(part(p), counter), l, T)) return st;
    }
    if (attn_sharded)
      if (det_status st = exchange(ts, X_ATTN, T, counter, capture)) return st;
    for (int p = 0; p < G; p++) {
      det_session* s = part(p);
      if (det_status st = set_dev(s)) return st;
      // wo adds into this part's slice of x, which the others read in the
      // previous layer's last gather.  With sharded heads the attention
      // exchange already ordered that; with replicated attention nothing
      // else does.
      if (!attn_sharded && l > 0)
        for (int q = 0; q < G; q++)
          if (q != p) CK(cudaStreamWaitEvent(s->stream, ts.done[capture ? 1 : 0][(size_t)q], 0));
      if (det_status st = fwd_attn_out(s, part_launch(s, counter), l, T, attn_sharded ? s->attn_full : s->attn))
        return st;
    }
    if (det_status st = exchange(ts, X_RESID, T, counter, capture)) return st;
    for (int p = 0; p < G; p++) {
      int have = 0;
      if (det_status st = set_dev(part(p))) return st;
      if (det_status st = fwd_ffn_in(part(p), part_launch(part(p), counter), l, T, &have)) return st;
    }
    if (det_status st = exchange(ts, X_FF, T, counter, capture)) return st;
    for (int p = 0; p < G; p++) {
      det_session* s = part(p);
      if (det_status st = set_dev(s)) return st;
      if (det_status st = fwd_ffn_out(s, part_launch(s, counter), l, T, s->ff_full, 0)) return st;
    }
    if (det_status st = exchange(ts, X_RESID, T, counter, capture, !attn_sharded)) return st;
  }
  for (int p = 0; p < G; p++) {
    if (det_status st = set_dev(part(p))) return st;
    if (det_status st = fwd_head(part(p), part_launch(part(p), counter), T)) return st;
  }
  if (det_status st = exchange(ts, X_LOGITS, T, counter, capture)) return st;
  if (capture) {
    for (int p = 1; p < G; p++) {
      if (det_status st = set_dev(part(p))) return st;
      CK(cudaEventRecord(ts.join[(size_t)p], part(p)->stream));
      if (det_status st = set_dev(s0)) return st;
      CK(cudaStreamWaitEvent(s0->stream, ts.join[(size_t)p], 0));
    }
  }
  return set_dev(s0);
}

// ---- distinct GPUs: one stream per part, device-side exchanges ---------------
// exchange k (0-based, nx per forward) of part p
det_status exchange_device(TpSession& ts, int p, XKind kind, int k, int nx, int T, const Launch& L) {
  const int G = (int)ts.parts.size();
  TpFlags f{};
  f.parts = G;
  f.mine = ts.flag[(size_t)p];
  unsigned wait = 0;
  for (int q = 0; q < G; q++) {
    f.peer[q] = q == p ? nullptr : ts.flag[(size_t)q] + p;
    if (q != p) wait |= 1u << q;
  }
  // logits: the other parts only signal; part 0 waits and pulls
  if (kind == X_LOGITS && p != 0) wait = 0;
  float* dst = nullptr;
  int ld = 0;
  GatherPlan g;
  if (!(kind == X_LOGITS && p != 0)) g = plan_for(ts, kind, p, &dst, &ld);
  CK(launch_tp_exchange(L, f, ts.epoch[(size_t)p], k, nx, wait, g, dst, ld, T));
  return DET_OK;
}

// one chunk forward of part p on its own stream
det_status tp_enqueue_part(TpSession& ts, int p, int T, uint64_t* counter) {
  det_session* s = ts.parts[(size_t)p];
  if (det_status st = set_dev(s)) return st;
  Launch L{s->stream, s->d_err, counter};
  L.pdl = T <= 16;  // as on one device
  CK(cudaMemcpyAsync(s->d_tokens, s->h_tokens, (size_t)T * 4, cudaMemcpyHostToDevice, s->stream));
  CK(cudaMemcpyAsync(s->d_pos, s->h_pos, 4, cudaMemcpyHostToDevice, s->stream));
  CK(launch_tp_epoch(L, ts.epoch[(size_t)p]));
  if (det_status st = fwd_embed(s, L, T)) return st;
  const bool attn_sharded = s->m->shard->attn_sharded;
  const int nl = s->m->cfg.L, nx = 4 * nl + 1;
  int k = 0;
  for (int l = 0; l < nl; l++) {
    if (det_status st = fwd_attention(s, L, l, T)) return st;
    // replicated attention: a barrier in its place keeps wo from rewriting
    // this part's slice of x before the others have pulled it
    if (det_status st = exchange_device(ts, p, attn_sharded ? X_ATTN : X_BARRIER, k++, nx, T, L)) return st;
    if (det_status st = fwd_attn_out(s, L, l, T, attn_sharded ? s->attn_full : s->attn)) return st;
    if (det_status st = exchange_device(ts, p, X_RESID, k++, nx, T, L)) return st;
    int have = 0;
    if (det_status st = fwd_ffn_in(s, L, l, T, &have)) return st;
    if (det_status st = exchange_device(ts, p, X_FF, k++, nx, T, L)) return st;
    if (det_status st = fwd_ffn_out(s, L, l, T, s->ff_full, 0)) return st;
    if (det_status st = exchange_device(ts, p, X_RESID, k++, nx, T, L)) return st;
  }
  if (det_status st = fwd_head(s, L, T)) return st;
  return exchange_device(ts, p, X_LOGITS, k++, nx, T, L);
}

det_status tp_run_device(det_session* s0, int T, bool graphs) {
  TpSession& ts = *s0->tp;
  const int G = (int)ts.parts.size();
  if (!graphs) {
    for (int p = 0; p < G; p++)
      if (det_status st = tp_enqueue_part(ts, p, T, &s0->stats.launches)) return st;
    return set_dev(s0);
  }
  for (int p = 0; p < G; p++) {
    det_session* s = ts.parts[(size_t)p];
    if ((int)s->graphs.size() <= T) s->graphs.resize((size_t)T + 1);
    det_session::Graph& gr = s->graphs[(size_t)T];
    if (gr.exec) continue;
    if (det_status st = set_dev(s)) return st;
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
    uint64_t count = 0;
    const det_status st = tp_enqueue_part(ts, p, T, &count);
    cudaSetDevice(s->m->device);
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
  for (int p = 0; p < G; p++) {
    det_session* s = ts.parts[(size_t)p];
    if (det_status st = set_dev(s)) return st;
    CK(cudaGraphLaunch(s->graphs[(size_t)T].exec, s->stream));
    s0->stats.launches += s->graphs[(size_t)T].kernels;
  }
  return set_dev(s0);
}

bool tp_force_events() {
  static const int on = [] {
    const char* e = std::getenv("DETGPU_TP_EVENTS");
    return e && *e && *e != '0' ? 1 : 0;
  }();
  return on != 0;
}

void destroy_events(TpSession* ts) {
  for (size_t p = 0; p < ts->parts.size(); p++) {
    if (ts->parts[p]) cudaSetDevice(ts->parts[p]->m->device);
    for (auto* set : {&ts->ev[0], &ts->ev[1], &ts->done[0], &ts->done[1]})
      if (p < set->size() && (*set)[p]) cudaEventDestroy((*set)[p]);
    if (p < ts->join.size() && ts->join[p]) cudaEventDestroy(ts->join[p]);
  }
  if (ts->fork && ts->parts[0]) {
    cudaSetDevice(ts->parts[0]->m->device);
    cudaEventDestroy(ts->fork);
  }
}

}  // namespace

// ---- hooks called by model.cpp / session.cpp --------------------------------
namespace det {

void tp_model_free(det_model* m) {
  TpModel* tm = m->tp;
  if (!tm) return;
  m->tp = nullptr;
  for (det_model* S : tm->shards) free_shard(S);
  for (size_t i = 1; i < tm->replicas.size(); i++) det_model_free(tm->replicas[i]);
  delete tm;
}

det_status tp_session_create(det_model* m, uint32_t n_ctx, uint32_t max_chunk, det_session** out) {
  TpModel& tm = *m->tp;
  const int G = (int)tm.shards.size();
  TpSession* ts = new (std::nothrow) TpSession();
  if (!ts) return DET_ERR_ALLOC;
  ts->parts.assign((size_t)G, nullptr);
  ts->ev[0].assign((size_t)G, nullptr);
  ts->ev[1].assign((size_t)G, nullptr);
  ts->done[0].assign((size_t)G, nullptr);
  ts->done[1].assign((size_t)G, nullptr);
  ts->join.assign((size_t)G, nullptr);
  det_status st = DET_OK;
  for (int p = 0; p < G && !st; p++) st = det_session_create(tm.shards[(size_t)p], n_ctx, max_chunk, &ts->parts[(size_t)p]);
  for (int p = 0; p < G && !st; p++) {
    if (cudaSetDevice(tm.devices[(size_t)p]) != cudaSuccess ||
        cudaEventCreateWithFlags(&ts->ev[0][(size_t)p], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ts->ev[1][(size_t)p], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ts->done[0][(size_t)p], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ts->done[1][(size_t)p], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ts->join[(size_t)p], cudaEventDisableTiming) != cudaSuccess)
      st = DET_ERR_CUDA;
  }
  if (!st && (cudaSetDevice(tm.devices[0]) != cudaSuccess ||
              cudaEventCreateWithFlags(&ts->fork, cudaEventDisableTiming) != cudaSuccess))
    st = DET_ERR_CUDA;
  // one part per GPU: exchanges ordered on the devices
  bool distinct = G > 1 && !tp_force_events();
  for (int p = 0; p < G && distinct; p++)
    for (int q = 0; q < p; q++)
      if (tm.devices[(size_t)p] == tm.devices[(size_t)q]) distinct = false;
  if (!st && distinct) {
    ts->device_sync = true;
    ts->flag.assign((size_t)G, nullptr);
    ts->epoch.assign((size_t)G, nullptr);
    for (int p = 0; p < G && !st; p++) {
      void *f = nullptr, *e = nullptr;
      if (cudaSetDevice(tm.devices[(size_t)p]) != cudaSuccess || cudaMalloc(&f, (size_t)G * 8) != cudaSuccess ||
          cudaMalloc(&e, 8) != cudaSuccess || cudaMemset(f, 0, (size_t)G * 8) != cudaSuccess ||
          cudaMemset(e, 0, 8) != cudaSuccess) {
        st = DET_ERR_DEVICE_OOM;
        if (f) cudaFree(f);
        if (e) cudaFree(e);
        break;
      }
      ts->flag[(size_t)p] = static_cast<unsigned long long*>(f);
      ts->epoch[(size_t)p] = static_cast<unsigned long long*>(e);
    }
  }
  if (st) {
    destroy_events(ts);
    for (size_t p = 0; p < ts->flag.size(); p++) {
      cudaSetDevice(tm.devices[p]);
      if (ts->flag[p]) cudaFree(ts->flag[p]);
      if (ts->epoch[p]) cudaFree(ts->epoch[p]);
    }
    for (det_session* s : ts->parts)
      if (s) det_session_free(s);
    delete ts;
    return st;
  }
  det_session* s0 = ts->parts[0];
  s0->tp = ts;
  s0->owner = m;
  *out = s0;
  return DET_OK;
}

void tp_session_release(det_session* s) {
  TpSession* ts = s->tp;
  if (!ts) return;
  s->tp = nullptr;
  for (size_t p = 1; p < ts->parts.size(); p++) {
    cudaSetDevice(ts->parts[p]->m->device);
    cudaStreamSynchronize(ts->parts[p]->stream);
  }
  destroy_events(ts);
  for (size_t p = 0; p < ts->flag.size(); p++) {
    cudaSetDevice(ts->parts[p]->m->device);
    if (ts->flag[p]) cudaFree(ts->flag[p]);
    if (ts->epoch[p]) cudaFree(ts->epoch[p]);
  }
  for (size_t p = 1; p < ts->parts.size(); p++) det_session_free(ts->parts[p]);
  delete ts;
}

det_status tp_take_part_errors(det_session* s) {
  det_status first = DET_OK;
  for (size_t p = 1; p < s->tp->parts.size(); p++) {
    const det_status st = session_take_error(s->tp->parts[p], false);
    if (st && !first) first = st;
  }
  return first;
}

det_status tp_reset(det_session* s) {
  for (size_t p = 1; p < s->tp->parts.size(); p++)
    if (det_status st = det_session_reset(s->tp->parts[p])) return st;
  return DET_OK;
}

// The chunk forward on every part: eagerly, or through one multi-device CUDA
// graph per chunk size held by the primary session.
det_status tp_run_forward(det_session* s0, int T, bool graphs) {
  TpSession& ts = *s0->tp;
  for (size_t p = 1; p < ts.parts.size(); p++) {
    std::memcpy(ts.parts[p]->h_tokens, s0->h_tokens, (size_t)T * 4);
    *ts.parts[p]->h_pos = *s0->h_pos;
  }
  if (ts.device_sync) return tp_run_device(s0, T, graphs);
  if (!graphs) return tp_enqueue(s0, T, &s0->stats.launches, false);
  if ((int)s0->graphs.size() <= T) s0->graphs.resize((size_t)T + 1);
  det_session::Graph& gr = s0->graphs[(size_t)T];
  if (!gr.exec) {
    if (det_status st = set_dev(s0)) return st;
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(s0->stream, cudaStreamCaptureModeThreadLocal));
    uint64_t count = 0;
    const det_status st = tp_enqueue(s0, T, &count, true);
    cudaSetDevice(s0->m->device);
    const cudaError_t ec = cudaStreamEndCapture(s0->stream, &graph);
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
  if (det_status st = set_dev(s0)) return st;
  CK(cudaGraphLaunch(gr.exec, s0->stream));
  s0->stats.launches += gr.kernels;
  return DET_OK;
}

}  // namespace det

extern "C" det_status det_model_load_tp(const uint8_t* gguf, size_t len, const int* devices, int n, det_model** out) {
  if (!gguf || !devices || !out || n < 1 || n > kMaxTpParts) return DET_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  int cnt = 0;
  if (cudaGetDeviceCount(&cnt) != cudaSuccess || cnt == 0) return DET_ERR_NO_DEVICE;
  std::vector<int> uniq;
  for (int i = 0; i < n; i++) {
    if (devices[i] < 0 || devices[i] >= cnt) return DET_ERR_INVALID_ARGUMENT;
    if (std::find(uniq.begin(), uniq.end(), devices[i]) == uniq.end()) uniq.push_back(devices[i]);
  }
  // every pair of distinct devices reads each other's memory
  for (int a : uniq)
    for (int b : uniq) {
      if (a == b) continue;
      int ok = 0;
      if (cudaDeviceCanAccessPeer(&ok, a, b) != cudaSuccess || !ok) return DET_ERR_COLLECTIVE;
      if (cudaSetDevice(a) != cudaSuccess) return DET_ERR_CUDA;
      const cudaError_t e = cudaDeviceEnablePeerAccess(b, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
      else if (e != cudaSuccess) return DET_ERR_COLLECTIVE;
    }
  TpModel* tm = new (std::nothrow) TpModel();
  if (!tm) return DET_ERR_ALLOC;
  // one host thread per device uploads its replica
  std::vector<det_model*> reps(uniq.size(), nullptr);
  std::vector<det_status> rst(uniq.size(), DET_OK);
  {
    std::vector<std::thread> th;
    for (size_t i = 0; i < uniq.size(); i++)
      th.emplace_back([&, i] { rst[i] = det_model_load(gguf, len, uniq[i], &reps[i]); });
    for (auto& t : th) t.join();
  }
  det_status st = DET_OK;
  for (size_t i = 0; i < uniq.size(); i++) {
    if (reps[i]) tm->replicas.push_back(reps[i]);
    if (rst[i] && !st) st = rst[i];
  }
  if (!st) {
    const ModelCfg& c = tm->replicas[0]->cfg;
    // heads are sharded when they divide evenly and every part's q/k/v rows
    // start on a 16-row tile of the tensor-core weight layout
    const bool attn_sharded = c.nkv % n == 0 && (c.nkv / n) * c.hd % 16 == 0;
    tm->devices.assign(devices, devices + n);
    for (int p = 0; p < n && !st; p++) {
      const size_t r = (size_t)(std::find(uniq.begin(), uniq.end(), devices[p]) - uniq.begin());
      det_model* S = nullptr;
      if (cudaSetDevice(devices[p]) != cudaSuccess) st = DET_ERR_CUDA;
      if (!st) st = make_shard(tm->replicas[r], p, n, attn_sharded, &S);
      if (!st) tm->shards.push_back(S);
    }
  }
  if (st) {
    for (det_model* S : tm->shards) free_shard(S);
    for (det_model* r : tm->replicas) det_model_free(r);
    delete tm;
    return st;
  }
  det_model* m = tm->replicas[0];
  m->tp = tm;
  *out = m;
  return DET_OK;
}
