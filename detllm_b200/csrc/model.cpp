// model.cpp -- det_model_load: GGUF -> validated model in device memory.
//
// Mirrors F32Llama::from_gguf (crates/det-model/src/lib.rs:1035-1140),
// LlamaConfig::from_gguf (:1498-1596) and the per-type tensor readers
// (:1650-1953), including their error order, then repacks each weight matrix
// into the device layout documented in internal.h: a tensor's bytes go to the
// device as stored in the file and repack.cu's kernels write the layout (and
// check the scales) there.  The tokenizer
// (byte fallback, byte-level BPE or SentencePiece) is read by
// det::Tokenizer::from_gguf in tokenizer.cpp, following Tokenizer::from_gguf
// (crates/det-token/src/lib.rs:86-132); its status is kept and reported
// when compress/decompress need the tokenizer.
#include <cmath>
#include <cstdio>
#include <cstdlib>

#include <thread>

#include "host_common.h"

using namespace det;

namespace {

int map_gg(int e) {
  if (e == GG_METADATA_NOT_FOUND) return DET_ERR_MISSING_METADATA;
  return DET_ERR_GGUF;
}

bool finite_f(float x) {
  uint32_t b;
  std::memcpy(&b, &x, 4);
  return (b & 0x7f800000u) != 0x7f800000u;
}

uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
bool f16_finite(uint16_t b) { return (b & 0x7c00) != 0x7c00; }

// f16_to_f32 (det-num f16.rs:6-34)
float f16_to_f32(uint16_t bits) {
  const uint32_t sign = ((uint32_t)bits & 0x8000u) << 16;
  const uint32_t exp = (bits >> 10) & 0x1f, frac = bits & 0x3ffu;
  uint32_t out;
  if (exp == 0) {
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
  } else if (exp == 0x1f) {
    out = sign | 0x7f800000u | (frac << 13);
  } else {
    out = sign | ((exp - 15 + 127) << 23) | (frac << 13);
  }
  float r;
  std::memcpy(&r, &out, 4);
  return r;
}

struct Loader {
  det_model* m;
  const Gguf& g;
  // device staging of one tensor's GGUF bytes (grown as needed) and the
  // repack kernels' error word
  uint8_t* stage = nullptr;
  size_t stage_cap = 0;
  uint32_t* d_err = nullptr;

  Loader(det_model* m_, const Gguf& g_) : m(m_), g(g_) {}
  Loader(const Loader&) = delete;
  Loader& operator=(const Loader&) = delete;
  ~Loader() {
    if (stage) cudaFree(stage);
    if (d_err) cudaFree(d_err);
  }

  det_status ensure_err() {
    if (d_err) return DET_OK;
    if (cudaMalloc(&d_err, 4) != cudaSuccess) return DET_ERR_DEVICE_OOM;
    return cudaMemset(d_err, 0, 4) == cudaSuccess ? DET_OK : DET_ERR_CUDA;
  }
  // the tensor's bytes, as stored in the file, in device memory
  det_status staged(const uint8_t* data, size_t len, const uint8_t** dev) {
    if (det_status st = ensure_err()) return st;
    if (len > stage_cap) {
      if (stage) cudaFree(stage);
      stage = nullptr;
      stage_cap = 0;
      if (cudaMalloc(&stage, len) != cudaSuccess) return DET_ERR_DEVICE_OOM;
      stage_cap = len;
    }
    if (len && cudaMemcpy(stage, data, len, cudaMemcpyHostToDevice) != cudaSuccess) return DET_ERR_CUDA;
    *dev = stage;
    return DET_OK;
  }
  // waits for the repack kernels; a non-finite scale or value fails the load
  det_status repack_status() {
    uint32_t f = 0;
    if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(&f, d_err, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
      return DET_ERR_CUDA;
    if (f & ERRF_NONFINITE) return DET_ERR_NONFINITE;
    return f ? DET_ERR_CUDA : DET_OK;
  }
  det_status alloc(size_t bytes, void** p) {
    *p = nullptr;
    if (cudaMalloc(p, bytes ? bytes : 16) != cudaSuccess) return DET_ERR_DEVICE_OOM;
    m->allocations.push_back(*p);
    return DET_OK;
  }

  det_status upload(const void* host, size_t bytes, void** dev) {
    void* p = nullptr;
    if (cudaMalloc(&p, bytes ? bytes : 16) != cudaSuccess) return DET_ERR_DEVICE_OOM;
    m->allocations.push_back(p);
    if (bytes && cudaMemcpy(p, host, bytes, cudaMemcpyHostToDevice) != cudaSuccess) return DET_ERR_CUDA;
    *dev = p;
    return DET_OK;
  }

  // read_dense_tensor_as_f32 (:1720-1776)
  det_status dense_f32(const GgufTensor& t, std::vector<float>* out) {
    const uint8_t* data;
    size_t len;
    if (g.tensor_bytes(t.name, &data, &len)) return DET_ERR_GGUF;
    uint64_t n;
    if (Gguf::element_count(t, &n)) return DET_ERR_SHAPE;
    out->resize((size_t)n);
    if (t.type == GT_F32) {
      if (len != n * 4) return DET_ERR_SHAPE;
      std::memcpy(out->data(), data, len);
      for (float v : *out)
        if (!finite_f(v)) return DET_ERR_NONFINITE;
    } else if (t.type == GT_F16) {
      if (len != n * 2) return DET_ERR_SHAPE;
      for (uint64_t i = 0; i < n; i++) {
        const uint16_t b = rd16(data + 2 * i);
        if (!f16_finite(b)) return DET_ERR_NONFINITE;
        (*out)[i] = f16_to_f32(b);
      }
    } else {
      return DET_ERR_UNSUPPORTED_TENSOR_TYPE;
    }
    return DET_OK;
  }

  // read_f32_vector / read_optional_f32_vector (:1656-1681)
  det_status vector(const std::string& name, size_t len, float** dev, bool optional) {
    const GgufTensor* t;
    const int e = g.tensor(name, &t);
    if (e == GG_TENSOR_NOT_FOUND && optional) {
      *dev = nullptr;
      return DET_OK;
    }
    if (e) return DET_ERR_GGUF;
    if (t->dims.size() != 1 || t->dims[0] != len) return DET_ERR_SHAPE;
    std::vector<float> v;
    if (det_status st = dense_f32(*t, &v)) return st;
    void* p;
    if (det_status st = upload(v.data(), v.size() * 4, &p)) return st;
    *dev = static_cast<float*>(p);
    return DET_OK;
  }

  // read_weight_matrix (:1778-1810) + read_q8/q4/q4k/q6k_matrix (:1812-1953)
  det_status matrix(const std::string& name, size_t rows, size_t cols, DevMatrix* out, uint32_t* src_type) {
    const GgufTensor* t;
    if (g.tensor(name, &t)) return DET_ERR_GGUF;
    if (t->dims.size() != 2 || t->dims[0] != cols || t->dims[1] != rows) return DET_ERR_SHAPE;
    *src_type = t->type;
    out->rows = (int)rows;
    out->cols = (int)cols;
    if (t->type == GT_F32 || t->type == GT_F16) {
      const uint8_t* data;
      size_t len;
      uint64_t n;
      if (g.tensor_bytes(t->name, &data, &len)) return DET_ERR_GGUF;
      if (Gguf::element_count(*t, &n)) return DET_ERR_SHAPE;
      const bool f16 = t->type == GT_F16;
      if (len != n * (f16 ? 2 : 4)) return DET_ERR_SHAPE;
      if (rows == 0 || cols == 0) return DET_ERR_SHAPE;
      const uint8_t* raw;
      if (det_status st = staged(data, len, &raw)) return st;
      void* p;
      if (det_status st = alloc((size_t)n * 4, &p)) return st;
      if (launch_dense_f32(raw, f16 ? 1 : 0, (long long)n, static_cast<float*>(p), d_err) != cudaSuccess)
        return DET_ERR_CUDA;
      if (det_status st = repack_status()) return st;
      out->type = GT_F32;
      out->f = static_cast<float*>(p);
      m->weight_bytes += (size_t)n * 4;
      return DET_OK;
    }
    size_t bk, tb;
    switch (t->type) {
      case GT_Q8_0: bk = 32; tb = 34; break;
      case GT_Q4_0: bk = 32; tb = 18; break;
      case GT_Q4_K: bk = 256; tb = 144; break;
      case GT_Q6_K: bk = 256; tb = 210; break;
      default: return DET_ERR_UNSUPPORTED_TENSOR_TYPE;
    }
    if (cols % bk) return DET_ERR_SHAPE;
    const size_t nb = cols / bk, nblk = rows * nb;
    const uint8_t* data;
    size_t len;
    if (g.tensor_bytes(name, &data, &len)) return DET_ERR_GGUF;
    if (len != nblk * tb) return DET_ERR_SHAPE;
    out->type = t->type;
    out->nb = (int)nb;
    if (rows == 0 || cols == 0) return DET_ERR_SHAPE;
    void* p;
    if (t->type == GT_Q4_K) {  // the blocks as stored: copied straight into place, then checked
      if (det_status st = alloc(len, &p)) return st;
      if (cudaMemcpy(p, data, len, cudaMemcpyHostToDevice) != cudaSuccess) return DET_ERR_CUDA;
      if (det_status st = ensure_err()) return st;
      if (launch_check_q4k(static_cast<const uint8_t*>(p), (long long)nblk, d_err) != cudaSuccess)
        return DET_ERR_CUDA;
      if (det_status st = repack_status()) return st;
      out->q = p;
      m->weight_bytes += len;
      return DET_OK;
    }
    const uint8_t* raw;
    if (det_status st = staged(data, len, &raw)) return st;
    if (t->type == GT_Q8_0 || t->type == GT_Q4_0) {
      // tensor-core tile records (gemm.cu): one record per (16-row tile, block)
      const bool q8 = t->type == GT_Q8_0;
      const size_t rb = q8 ? 544 : 288, tiles = (rows + 15) / 16;
      if (det_status st = alloc(tiles * nb * rb, &p)) return st;
      if (launch_repack_mma16(raw, q8 ? 1 : 0, (int)rows, (int)nb, static_cast<uint8_t*>(p), d_err) != cudaSuccess)
        return DET_ERR_CUDA;
      if (det_status st = repack_status()) return st;
      out->q = p;
      out->layout = LAYOUT_MMA16;
      m->weight_bytes += tiles * nb * rb;
      return DET_OK;
    }
    // Q6_K: ql | qh | scales kept together (208 B), d split out
    void* pd;
    if (det_status st = alloc(nblk * 208, &p)) return st;
    if (det_status st = alloc(nblk * 2, &pd)) return st;
    if (launch_split_q6k(raw, (long long)nblk, static_cast<uint8_t*>(p), static_cast<uint16_t*>(pd), d_err) !=
        cudaSuccess)
      return DET_ERR_CUDA;
    if (det_status st = repack_status()) return st;
    out->q = p;
    out->d = static_cast<const uint16_t*>(pd);
    m->weight_bytes += nblk * 210;
    // the tensor-core chunk GEMM's records, built on the device from the
    // split blocks (gemm_q6k_tc.cu)
    const size_t tb_bytes = q6k_tc_bytes((int)rows, (int)nb);
    void* tcp;
    if (det_status st = alloc(tb_bytes, &tcp)) return st;
    if (launch_q6k_tc_repack(nullptr, *out, static_cast<uint8_t*>(tcp)) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess)
      return DET_ERR_CUDA;
    out->tc = static_cast<const uint8_t*>(tcp);
    m->weight_bytes += tb_bytes;
    return DET_OK;
  }
};

// Store matrices that read the same activations (q/k/v, gate/up) back to back
// as one LAYOUT_MMA16 matrix so one launch covers them; each part's `q` then
// points into the fused buffer.  Leaves *fused empty (rows 0) when the parts
// cannot be fused: other types or layouts, different widths, or a part other
// than the last whose rows are not a multiple of 16.
det_status fuse_matrices(det_model* m, DevMatrix* const* parts, int n, DevMatrix* fused) {
  *fused = DevMatrix();
  size_t bytes = 0;
  int rows = 0;
  for (int i = 0; i < n; i++) {
    const DevMatrix& p = *parts[i];
    if (p.layout != LAYOUT_MMA16 || p.type != parts[0]->type || p.cols != parts[0]->cols) return DET_OK;
    if (i + 1 < n && p.rows % 16) return DET_OK;
    rows += p.rows;
  }
  const size_t rec = parts[0]->type == GT_Q8_0 ? 544 : 288;
  for (int i = 0; i < n; i++) bytes += (size_t)((parts[i]->rows + 15) / 16) * parts[i]->nb * rec;
  void* buf = nullptr;
  if (cudaMalloc(&buf, bytes) != cudaSuccess) return DET_ERR_DEVICE_OOM;
  m->allocations.push_back(buf);
  size_t off = 0;
  for (int i = 0; i < n; i++) {
    DevMatrix& p = *parts[i];
    const size_t b = (size_t)((p.rows + 15) / 16) * p.nb * rec;
    uint8_t* dst = static_cast<uint8_t*>(buf) + off;
    if (cudaMemcpy(dst, p.q, b, cudaMemcpyDeviceToDevice) != cudaSuccess) return DET_ERR_CUDA;
    void* old = const_cast<void*>(p.q);
    for (auto& a : m->allocations)
      if (a == old) a = nullptr;
    cudaFree(old);
    p.q = dst;
    off += b;
  }
  *fused = *parts[0];
  fused->rows = rows;
  fused->q = buf;
  return DET_OK;
}

// the tensor-core copy (gemm_q8_tc.cu) of a LAYOUT_MMA16 matrix that chunk
// GEMMs read, built on the device from its records
det_status build_q8_tc(det_model* m, DevMatrix* M) {
  // the copy doubles the matrix's footprint: only when the tcgen05 kernel is chosen
  if (!M->rows || M->layout != LAYOUT_MMA16 || M->tc || !q8_tensor_cores()) return DET_OK;
  const size_t bytes = q8_tc_bytes(M->rows, M->nb);
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return DET_ERR_DEVICE_OOM;
  m->allocations.push_back(p);
  if (launch_q8_tc_repack(nullptr, *M, static_cast<uint8_t*>(p)) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess)
    return DET_ERR_CUDA;
  M->tc = static_cast<const uint8_t*>(p);
  m->weight_bytes += bytes;
  return DET_OK;
}

// optional metadata helpers (det-model lib.rs:1566-1645)
det_status opt_u32(const Gguf& g, const std::string& k, uint32_t* v, bool* present) {
  const int e = g.get_u32(k, v);
  *present = e == GG_OK;
  if (e == GG_METADATA_NOT_FOUND || e == GG_OK) return DET_OK;
  return map_gg(e);
}
det_status opt_f32(const Gguf& g, const std::string& k, float* v, bool* present) {
  const int e = g.get_f32(k, v);
  *present = e == GG_OK;
  if (e == GG_METADATA_NOT_FOUND || e == GG_OK) return DET_OK;
  return map_gg(e);
}
det_status opt_bool(const Gguf& g, const std::string& k, bool* v, bool* present) {
  const GgufValue* x = g.find(k);
  *present = x != nullptr;
  if (!x) return DET_OK;
  if (x->type != GV_BOOL) return DET_ERR_GGUF;
  *v = x->bits != 0;
  return DET_OK;
}
det_status reject_nonzero_f32(const Gguf& g, const std::string& k) {
  const GgufValue* x = g.find(k);
  if (!x) return DET_OK;
  if (x->type != GV_F32 && x->type != GV_F64) return DET_ERR_GGUF;
  if (!std::isfinite(x->real)) return DET_ERR_SHAPE;
  if (x->real != 0.0) return DET_ERR_UNSUPPORTED_MODEL_FEATURE;
  return DET_OK;
}

det_status config_from_gguf(const Gguf& g, ModelCfg* c) {
  const GgufValue* arch = g.find("general.architecture");
  if (!arch) return DET_ERR_MISSING_METADATA;
  if (arch->type != GV_STRING) return DET_ERR_GGUF;
  std::string pre;
  if (arch->str == "llama") { pre = "llama"; c->pairing = DET_ROPE_ADJACENT; }
  else if (arch->str == "qwen2") { pre = "qwen2"; c->pairing = DET_ROPE_SPLIT_HALF; }
  else return DET_ERR_UNSUPPORTED_ARCHITECTURE;
  auto K = [&](const char* s) { return pre + "." + s; };
  uint32_t v;
  bool pr, b;
  float f;
  det_status st;
  if (int e = g.get_u32(K("attention.head_count"), &v)) return map_gg(e);
  c->nh = (int)v;
  if ((st = opt_u32(g, K("attention.head_count_kv"), &v, &pr))) return st;
  c->nkv = pr ? (int)v : c->nh;
  if (int e = g.get_u32(K("embedding_length"), &v)) return map_gg(e);
  c->d = (int)v;
  if (c->nh == 0 || c->d % c->nh) return DET_ERR_SHAPE;
  if ((st = opt_u32(g, K("embedding_length_out"), &v, &pr))) return st;
  if (pr && (int)v != c->d) return DET_ERR_UNSUPPORTED_MODEL_FEATURE;
  if ((st = opt_bool(g, K("attention.causal"), &b, &pr))) return st;
  if (pr && !b) return DET_ERR_UNSUPPORTED_MODEL_FEATURE;
  if (const GgufValue* rs = g.find(K("rope.scaling.type"))) {
    if (rs->type != GV_STRING) return DET_ERR_GGUF;
    if (rs->str != "none") return DET_ERR_UNSUPPORTED_ROPE_SCALING;
  }
  if ((st = opt_bool(g, K("use_parallel_residual"), &b, &pr))) return st;
  if (pr && b) return DET_ERR_UNSUPPORTED_MODEL_FEATURE;
  if ((st = opt_u32(g, K("attention.sliding_window"), &v, &pr))) return st;
  if (pr && v != 0) return DET_ERR_UNSUPPORTED_MODEL_FEATURE;
  for (const char* z : {"attention.max_alibi_bias", "attention.clamp_kqv", "attention.value_scale",
                        "attn_logit_softcapping", "final_logit_softcapping", "logit_scale", "embedding_scale",
                        "residual_scale"})
    if ((st = reject_nonzero_f32(g, K(z)))) return st;
  c->hd = c->d / c->nh;
  for (const char* lk : {"attention.key_length", "attention.value_length"}) {
    if ((st = opt_u32(g, K(lk), &v, &pr))) return st;
    if (pr && (int)v != c->hd) return DET_ERR_UNSUPPORTED_HEAD_LENGTH;
  }
  if ((st = opt_f32(g, K("attention.scale"), &f, &pr))) return st;
  // default_attention_scale (:1647-1649): 1 / sqrt(head_dim as f32)
  c->attn_scale = pr ? f : 1.0f / std::sqrt((float)c->hd);
  if (int e = g.get_u32(K("block_count"), &v)) return map_gg(e);
  c->L = (int)v;
  if (int e = g.get_u32(K("feed_forward_length"), &v)) return map_gg(e);
  c->dff = (int)v;
  if (int e = g.get_f32(K("attention.layer_norm_rms_epsilon"), &f)) return map_gg(e);
  c->eps = f;
  if ((st = opt_f32(g, K("rope.freq_base"), &f, &pr))) return st;
  c->rope_base = pr ? f : 10000.0f;
  if ((st = opt_u32(g, K("rope.dimension_count"), &v, &pr))) return st;
  c->rope_dim = pr ? (int)v : c->hd;
  if (int e = g.get_u32(K("context_length"), &v)) return map_gg(e);
  c->ctx = (int)v;
  if (c->L == 0 || c->d == 0 || c->dff == 0 || c->nh == 0 || c->nkv == 0 || c->ctx == 0 || c->nh % c->nkv ||
      c->rope_dim == 0 || c->rope_dim % 2 || !finite_f(c->eps) || c->eps <= 0.0f || !finite_f(c->attn_scale) ||
      c->attn_scale <= 0.0f || !finite_f(c->rope_base) || c->rope_base <= 0.0f || c->rope_dim > c->hd)
    return DET_ERR_SHAPE;
  return DET_OK;
}

// vocab_size (det-model lib.rs:1620-1648)
det_status vocab_size(const Gguf& g, size_t* out) {
  const GgufValue* arch = g.find("general.architecture");
  if (!arch) return DET_ERR_MISSING_METADATA;
  if (arch->type != GV_STRING) return DET_ERR_GGUF;
  for (const std::string& k : {arch->str + ".vocab_size", std::string("llama.vocab_size")}) {
    uint32_t v;
    const int e = g.get_u32(k, &v);
    if (e == GG_OK) { *out = v; return DET_OK; }
    if (e != GG_METADATA_NOT_FOUND) return map_gg(e);
  }
  if (const GgufValue* toks = g.find("tokenizer.ggml.tokens")) {
    if (toks->type != GV_ARRAY || toks->elem_type != GV_STRING) return DET_ERR_GGUF;
    *out = toks->strs.size();
    return DET_OK;
  }
  const GgufTensor* t;
  if (g.tensor("token_embd.weight", &t)) return DET_ERR_GGUF;
  if (t->dims.size() == 2) { *out = (size_t)t->dims[1]; return DET_OK; }
  return DET_ERR_MISSING_METADATA;
}

void free_model(det_model* m) {
  if (!m) return;
  int cur;
  if (cudaGetDevice(&cur) == cudaSuccess && cur != m->device) cudaSetDevice(m->device);
  session_release_cached(m);
  tp_model_free(m);  // the other replicas and the per-part views
  cudaSetDevice(m->device);
  for (void* p : m->allocations) cudaFree(p);
  delete m;
}

det_status load_impl(const uint8_t* bytes, size_t len, det_model* m) {
  // the file hash (the DTLZ header's model SHA-256) on a second thread, while
  // this one parses, repacks and uploads; joined on every return path
  struct Hasher {
    std::thread t;
    ~Hasher() {
      if (t.joinable()) t.join();
    }
  } hasher;
  hasher.t = std::thread([bytes, len, m] {
    Sha256 h;
    h.update(bytes, len);
    h.finish(m->sha);
  });
  Gguf g;
  if (g.parse(bytes, len)) return DET_ERR_GGUF;
  m->tok_status = m->tok.from_gguf(g);
  ModelCfg& c = m->cfg;
  if (det_status st = config_from_gguf(g, &c)) return st;
  size_t V;
  if (det_status st = vocab_size(g, &V)) return st;
  Loader ld(m, g);
  const size_t hd = (size_t)c.hd;
  if (det_status st = ld.matrix("token_embd.weight", V, c.d, &m->tok_embd, &m->weight_types[0])) return st;
  m->layers.resize((size_t)c.L);
  for (int l = 0; l < c.L; l++) {
    LayerDev& L = m->layers[(size_t)l];
    const std::string p = "blk." + std::to_string(l) + ".";
    uint32_t ty[7];
    det_status st;
    if ((st = ld.vector(p + "attn_norm.weight", c.d, &L.attn_norm, false))) return st;
    if ((st = ld.matrix(p + "attn_q.weight", c.nh * hd, c.d, &L.wq, &ty[0]))) return st;
    if ((st = ld.vector(p + "attn_q.bias", c.nh * hd, &L.bq, true))) return st;
    if ((st = ld.matrix(p + "attn_k.weight", c.nkv * hd, c.d, &L.wk, &ty[1]))) return st;
    if ((st = ld.vector(p + "attn_k.bias", c.nkv * hd, &L.bk, true))) return st;
    if ((st = ld.matrix(p + "attn_v.weight", c.nkv * hd, c.d, &L.wv, &ty[2]))) return st;
    if ((st = ld.vector(p + "attn_v.bias", c.nkv * hd, &L.bv, true))) return st;
    if ((st = ld.matrix(p + "attn_output.weight", c.d, c.nh * hd, &L.wo, &ty[3]))) return st;
    if ((st = ld.vector(p + "ffn_norm.weight", c.d, &L.ffn_norm, false))) return st;
    if ((st = ld.matrix(p + "ffn_gate.weight", c.dff, c.d, &L.gate, &ty[4]))) return st;
    if ((st = ld.matrix(p + "ffn_up.weight", c.dff, c.d, &L.up, &ty[5]))) return st;
    if ((st = ld.matrix(p + "ffn_down.weight", c.d, c.dff, &L.down, &ty[6]))) return st;
    DevMatrix* qkv[3] = {&L.wq, &L.wk, &L.wv};
    if ((st = fuse_matrices(m, qkv, 3, &L.wqkv))) return st;
    DevMatrix* gu[2] = {&L.gate, &L.up};
    if ((st = fuse_matrices(m, gu, 2, &L.wgu))) return st;
    if (l == 0) {
      for (int i = 0; i < 7; i++) m->weight_types[1 + i] = ty[i];
      m->has_bias = L.bq != nullptr;
    }
  }
  if (det_status st = ld.vector("output_norm.weight", c.d, &m->output_norm, false)) return st;
  const GgufTensor* t;
  const int e = g.tensor("output.weight", &t);
  if (e == GG_OK) {
    if (det_status st = ld.matrix("output.weight", V, c.d, &m->output, &m->weight_types[8])) return st;
  } else if (e == GG_TENSOR_NOT_FOUND) {
    m->output = m->tok_embd;  // tied embeddings (:1127-1131)
    m->weight_types[8] = m->weight_types[0];
    m->tied = true;
  } else {
    return DET_ERR_GGUF;
  }
  m->vocab = (int)V;
  // tensor-core copies of the Q8_0 / Q4_0 matrices the chunk GEMMs read (the
  // fused q|k|v and gate|up where they exist, else their parts)
  for (LayerDev& L : m->layers) {
    det_status st;
    if (L.wqkv.rows) {
      if ((st = build_q8_tc(m, &L.wqkv))) return st;
    } else {
      for (DevMatrix* W : {&L.wq, &L.wk, &L.wv})
        if ((st = build_q8_tc(m, W))) return st;
    }
    if (L.wgu.rows) {
      if ((st = build_q8_tc(m, &L.wgu))) return st;
    } else {
      for (DevMatrix* W : {&L.gate, &L.up})
        if ((st = build_q8_tc(m, W))) return st;
    }
    for (DevMatrix* W : {&L.wo, &L.down})
      if ((st = build_q8_tc(m, W))) return st;
  }
  if (det_status st = build_q8_tc(m, &m->output)) return st;
  return DET_OK;
}

}  // namespace

extern "C" {

const char* det_status_string(det_status s) {
  switch (s) {
    case DET_OK: return "ok";
    case DET_ERR_SHAPE: return "shape";
    case DET_ERR_NONFINITE: return "non-finite value";
    case DET_ERR_UNSUPPORTED_ARCHITECTURE: return "unsupported architecture";
    case DET_ERR_UNSUPPORTED_HEAD_LENGTH: return "unsupported attention head length";
    case DET_ERR_UNSUPPORTED_MODEL_FEATURE: return "unsupported model feature";
    case DET_ERR_UNSUPPORTED_ROPE_SCALING: return "unsupported rope scaling";
    case DET_ERR_MISSING_METADATA: return "missing metadata";
    case DET_ERR_GGUF: return "gguf";
    case DET_ERR_UNSUPPORTED_TENSOR_TYPE: return "unsupported tensor type";
    case DET_ERR_CDF_EMPTY: return "cdf: empty";
    case DET_ERR_CDF_MALFORMED: return "cdf: malformed";
    case DET_ERR_CDF_NONFINITE_LOGIT: return "cdf: non-finite logit";
    case DET_ERR_CDF_SYMBOL_OUT_OF_RANGE: return "cdf: symbol out of range";
    case DET_ERR_CDF_TOO_MANY_SYMBOLS: return "cdf: too many symbols";
    case DET_ERR_CDF_TOTAL_TOO_LARGE: return "cdf: total too large";
    case DET_ERR_RANGE_INVALID_FREQUENCY: return "range coder: invalid frequency";
    case DET_ERR_RANGE_UNEXPECTED_EOF: return "range coder: unexpected end of payload";
    case DET_ERR_FILE_TOO_SHORT: return "dtlz: too short";
    case DET_ERR_FILE_BAD_MAGIC: return "dtlz: bad magic";
    case DET_ERR_FILE_UNSUPPORTED_VERSION: return "dtlz: unsupported version";
    case DET_ERR_FILE_UNSUPPORTED_FLAGS: return "dtlz: unsupported flags";
    case DET_ERR_FILE_INVALID_CONTEXT: return "dtlz: invalid context";
    case DET_ERR_FILE_INVALID_OVERLAP: return "dtlz: invalid overlap";
    case DET_ERR_TOKENIZER: return "tokenizer";
    case DET_ERR_WINDOW: return "invalid context window";
    case DET_ERR_MODEL_HASH_MISMATCH: return "model SHA-256 does not match the DTLZ header";
    case DET_ERR_NONCANONICAL: return "DTLZ payload is not the canonical encoding";
    case DET_ERR_VOCAB_MISMATCH: return "tokenizer / model vocabulary mismatch";
    case DET_ERR_DECODE: return "decoder value outside the distribution";
    case DET_ERR_ALLOC: return "host allocation failed";
    case DET_ERR_INVALID_ARGUMENT: return "invalid argument";
    case DET_ERR_CUDA: return "CUDA error";
    case DET_ERR_NO_DEVICE: return "no CUDA device";
    case DET_ERR_DEVICE_OOM: return "device out of memory";
    case DET_ERR_TIMEOUT: return "timed out";
    case DET_ERR_COLLECTIVE: return "collective failed";
    case DET_ERR_SCRATCH_LIMIT: return "request exceeds the fixed scratch array";
    default: return "unknown status";
  }
}

det_status det_device_count(int* count) {
  if (!count) return DET_ERR_INVALID_ARGUMENT;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) n = 0;
  *count = n;
  return DET_OK;
}

det_status det_model_load(const uint8_t* gguf, size_t len, int device, det_model** out) {
  if (!gguf || !out) return DET_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return DET_ERR_NO_DEVICE;
  if (device < 0 || device >= n) return DET_ERR_INVALID_ARGUMENT;
  if (cudaSetDevice(device) != cudaSuccess) return DET_ERR_CUDA;
  det_model* m = new (std::nothrow) det_model();
  if (!m) return DET_ERR_ALLOC;
  m->device = device;
  const det_status st = load_impl(gguf, len, m);
  if (st) {
    free_model(m);
    return st;
  }
  *out = m;
  return DET_OK;
}

void det_model_free(det_model* m) { free_model(m); }

det_status det_model_info(const det_model* m, det_config* o) {
  if (!m || !o) return DET_ERR_INVALID_ARGUMENT;
  const ModelCfg& c = m->cfg;
  std::memset(o, 0, sizeof *o);
  o->block_count = (uint32_t)c.L;
  o->embedding_length = (uint32_t)c.d;
  o->feed_forward_length = (uint32_t)c.dff;
  o->head_count = (uint32_t)c.nh;
  o->head_count_kv = (uint32_t)c.nkv;
  o->head_dim = (uint32_t)c.hd;
  o->rope_dimension_count = (uint32_t)c.rope_dim;
  o->rope_pairing = (uint32_t)c.pairing;
  o->context_length = (uint32_t)c.ctx;
  o->vocab = (uint32_t)m->vocab;
  o->rms_epsilon = c.eps;
  o->attention_scale = c.attn_scale;
  o->rope_freq_base = c.rope_base;
  for (int i = 0; i < 9; i++) o->weight_types[i] = m->weight_types[i];
  o->has_qkv_bias = m->has_bias ? 1u : 0u;
  o->tied_output = m->tied ? 1u : 0u;
  return DET_OK;
}

det_status det_model_sha256(const det_model* m, uint8_t out[32]) {
  if (!m || !out) return DET_ERR_INVALID_ARGUMENT;
  std::memcpy(out, m->sha, 32);
  return DET_OK;
}

void det_free(void* p) { std::free(p); }

}  // extern "C"
