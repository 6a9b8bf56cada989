// host_common.h -- host-side structures of libdetgpu.so (not public ABI).
#pragma once

#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/detgpu.h"
#include "internal.h"

namespace det {

// ---- SHA-256 (FIPS 180-4); the logits hash and the model file hash -------
class Sha256 {
 public:
  Sha256();
  void update(const void* data, size_t len);
  void finish(uint8_t out[32]);

 private:
  void block(const uint8_t* p);
  void blocks(const uint8_t* p, size_t n);  // SHA extensions where the CPU has them
  uint32_t st_[8];
  uint64_t len_ = 0;
  uint8_t buf_[64];
  size_t n_ = 0;
};

// ---- 64-bit range coder: RangeEncoder / RangeDecoder
// (crates/det-coder/src/range.rs:11-178) ------------------------------------
class RangeEncoder {
 public:
  det_status encode(uint64_t cum, uint64_t freq, uint64_t total);
  std::vector<uint8_t> finish();

 private:
  uint64_t low_ = 0, range_ = ~0ull;
  std::vector<uint8_t> out_;
};

class RangeDecoder {
 public:
  det_status init(const uint8_t* data, size_t len);
  det_status decode_freq(uint64_t total, uint64_t* value);
  det_status advance(uint64_t cum, uint64_t freq, uint64_t total);

 private:
  det_status next_byte(uint8_t* b);
  uint64_t low_ = 0, code_ = 0, range_ = ~0ull;
  bool pending_ = false;
  uint64_t pend_range_ = 0, pend_total_ = 0;
  const uint8_t* in_ = nullptr;
  size_t len_ = 0, pos_ = 0;
};

// ---- GGUF reader (crates/det-gguf/src/lib.rs:156-528) ---------------------
enum GgufErr : int {
  GG_OK = 0, GG_BAD_MAGIC, GG_UNSUPPORTED_VERSION, GG_TRUNCATED, GG_UNSUPPORTED_VALUE_TYPE, GG_INVALID_UTF8,
  GG_INVALID_TENSOR_OFFSET, GG_INVALID_TENSOR_SHAPE, GG_TENSOR_NOT_FOUND, GG_METADATA_NOT_FOUND,
  GG_DUPLICATE_METADATA_KEY, GG_DUPLICATE_TENSOR_NAME, GG_INVALID_BOOL, GG_METADATA_TYPE_MISMATCH,
  GG_UNSUPPORTED_TENSOR_TYPE
};

enum GgufValueType : uint32_t {
  GV_U8 = 0, GV_I8, GV_U16, GV_I16, GV_U32, GV_I32, GV_F32, GV_BOOL, GV_STRING, GV_ARRAY, GV_U64, GV_I64, GV_F64
};

struct GgufValue {
  uint32_t type = 0, elem_type = 0;
  uint64_t bits = 0;       // scalar payload
  double real = 0.0;       // F32/F64 payload
  std::string str;         // GV_STRING
  std::vector<std::string> strs;  // string arrays
  const uint8_t* raw = nullptr;   // other arrays: little-endian payload
  uint64_t count = 0;
};

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t type = 0;
  uint64_t offset = 0;
};

class Gguf {
 public:
  int parse(const uint8_t* bytes, size_t len);
  const GgufValue* find(const std::string& key) const;
  int get_u32(const std::string& key, uint32_t* out) const;
  int get_f32(const std::string& key, float* out) const;
  int tensor(const std::string& name, const GgufTensor** out) const;
  int tensor_bytes(const std::string& name, const uint8_t** data, size_t* len) const;
  static int type_size(uint32_t type, uint64_t* bytes_per_block, uint64_t* block);
  static int element_count(const GgufTensor& t, uint64_t* n);

  std::vector<std::pair<std::string, GgufValue>> kv;
  std::vector<GgufTensor> tensors;
  size_t data_offset = 0;

 private:
  const uint8_t* bytes_ = nullptr;
  size_t len_ = 0;
};

// ---- tokenizers (tokenizer.cpp; det-token lib.rs:85-850) -------------------
struct Tokenizer {
  enum Kind : int { BYTE_FALLBACK = 0, BPE = 1, SPM = 2 };
  Kind kind = BYTE_FALLBACK;
  size_t vocab = 0;
  int32_t byte_to_token[256];       // the single-byte token of each byte, -1 if none emittable
  std::vector<std::string> bytes;   // token_to_bytes
  std::vector<char> has_bytes;      // byte fallback: only the "<0xHH>" tokens have bytes
  std::unordered_map<uint64_t, std::pair<uint64_t, uint32_t>> merges;  // (left, right) -> (rank, merged)
  std::unordered_map<std::string, uint32_t> pieces;  // SentencePiece multi-byte pieces -> token
  size_t max_piece_len = 1;

  det_status from_gguf(const Gguf& g);
  det_status tokenize(const uint8_t* in, size_t n, std::vector<uint32_t>* out) const;
  det_status codec_symbols(const uint8_t* in, size_t n, std::vector<uint32_t>* out) const;
  det_status symbol_bytes(uint32_t symbol, bool escapes, std::string* piece) const;
};

// ---- model ------------------------------------------------------------------
struct LayerDev {
  DevMatrix wq, wk, wv, wo, gate, up, down;
  // q|k|v and gate|up stored back to back (rows == 0: not fused)
  DevMatrix wqkv, wgu;
  float *attn_norm = nullptr, *ffn_norm = nullptr, *bq = nullptr, *bk = nullptr, *bv = nullptr;
};

struct ModelCfg {
  int L = 0, d = 0, dff = 0, nh = 0, nkv = 0, hd = 0, rope_dim = 0, ctx = 0, pairing = 0;
  float eps = 0, attn_scale = 0, rope_base = 0;
};

}  // namespace det

namespace det {
// Device-time profile of one forward (det_set_profiling): an event pair
// around every launch, grouped by what the launch computes.
enum ProfTag : int {
  PT_EMBED,
  PT_NORM,
  PT_QUANT,
  PT_GEMM_QKV,
  PT_ROPE,
  PT_ATTENTION,
  PT_GEMM_O,
  PT_GEMM_GATE_UP,
  PT_SWIGLU,
  PT_GEMM_DOWN,
  PT_GEMM_OUT,
  PT_CDF,
  PT_FUSED,  // the one-position forward as one persistent kernel (decode_fused.cu)
  PT_COUNT
};
struct ProfTags {
  double ms[PT_COUNT] = {};
  uint64_t n[PT_COUNT] = {};
};
struct ProfEntry {
  int tag;
  double bytes, wbytes;  // algorithmic bytes of a weight GEMM (0 otherwise)
};

// Row-sharded tensor parallelism (tp.cpp).  Part p of a G-part model owns
// rows [d0, d1) of wo and down, [f0, f1) of gate and up and [v0, v1) of the
// lm_head: contiguous slices on 64-row boundaries, so every output row is
// the same reduction as on one device.  When the KV heads divide evenly
// (head_count_kv % G == 0) it also owns kv heads [h0, h1) with their query
// heads, q/k/v rows and KV cache; otherwise every part runs the whole
// attention block.
struct TpShard {
  int part = 0, parts = 1;
  bool attn_sharded = false;
  int d0 = 0, d1 = 0, f0 = 0, f1 = 0, v0 = 0, v1 = 0, h0 = 0, h1 = 0;
  ModelCfg full;  // the unsharded configuration
};
struct TpModel;
struct TpSession;
}  // namespace det

struct det_model {
  int device = 0;
  det::ModelCfg cfg;
  int vocab = 0;
  uint8_t sha[32];
  // the codec's tokenizer (tokenizer.cpp); tok_status: its construction error
  det_status tok_status = DET_OK;
  det::Tokenizer tok;
  det::DevMatrix tok_embd, output;
  bool tied = false;
  std::vector<det::LayerDev> layers;
  float* output_norm = nullptr;
  std::vector<void*> allocations;
  uint32_t weight_types[9] = {0};
  bool has_bias = false;
  size_t weight_bytes = 0;  // device bytes of all weight matrices
  det_stats agg{};          // stats of finished sessions
  det::ProfTags prof_agg;   // per-kernel profile of finished sessions
  // session reused by the model-level codec entry points (compress,
  // decompress, encode symbols) so repeated calls skip allocation, RoPE
  // table and graph capture
  det_session* cached = nullptr;
  // serialises those entry points (they share `cached`) and guards the
  // statistics aggregates: callers may use one model from several host
  // threads, as the reference's immutable model allows; their codec calls
  // then run one after another
  std::recursive_mutex mu;
  // tensor parallelism: `tp` on the model det_model_load_tp returns (its
  // sessions are tensor-parallel); `shard` on the per-part models that view
  // the replicas' weights (cfg then holds this part's head and FFN counts)
  det::TpModel* tp = nullptr;
  det::TpShard* shard = nullptr;
  // bytes of every codec symbol (tokens, then the 256 byte escapes) for the
  // decompress loop on the device; built on first use
  uint16_t* piece_len = nullptr;
  size_t max_piece = 1;
};


struct det_session {
  det_model* m = nullptr;
  det_model* owner = nullptr;  // the model whose statistics this session adds to
  int n_ctx = 0, max_chunk = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
  // activations [max_chunk][*]
  float *x = nullptr, *h = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr, *tmp = nullptr;
  float *gate = nullptr, *up = nullptr, *ff = nullptr, *logits = nullptr;
  float* qa_d = nullptr;
  int8_t* qa_q = nullptr;
  float* qk_d = nullptr;
  int8_t* qk_q = nullptr;
  uint8_t* qk_p = nullptr;  // Q8_K records of the tensor-core Q6_K chunk GEMM (chunks > 16)
  float *kc = nullptr, *vc = nullptr, *rope_cos = nullptr, *rope_sin = nullptr, *score_scratch = nullptr;
  float *cdf_e = nullptr, *cdf_z = nullptr;
  uint32_t *d_tokens = nullptr, *d_rows = nullptr, *d_syms = nullptr, *d_err = nullptr;
  uint64_t *d_out = nullptr, *d_value = nullptr;
  int* d_pos = nullptr;  // first position of the current chunk (read by RoPE / attention)
  // pinned staging
  uint32_t *h_tokens = nullptr, *h_rows = nullptr, *h_syms = nullptr, *h_err = nullptr;
  uint64_t *h_out = nullptr, *h_value = nullptr;
  int* h_pos = nullptr;
  // one CUDA graph per chunk size: copies of tokens / pos0 + the whole forward
  struct Graph {
    cudaGraphExec_t exec = nullptr;
    uint64_t kernels = 0;
  };
  std::vector<Graph> graphs;  // indexed by chunk size
  int last_n = 0;
  bool fwd_timed = false;  // a forward whose device time forward_collect has not added yet
  std::vector<uint8_t> cdf_ready;
  det_stats stats{};
  std::vector<void*> allocations;
  // profiling: event pairs around launches, resolved at the next sync
  std::vector<cudaEvent_t> prof_events;
  std::vector<det::ProfEntry> prof_pending;
  det::ProfTags prof;
  // tensor parallelism: the gathered attention output / SwiGLU output of a
  // part (full width), and on the session returned to the caller, the parts
  float *attn_full = nullptr, *ff_full = nullptr;
  det::TpSession* tp = nullptr;
  // one-position forward as one persistent kernel (decode_fused.cu):
  // fd_state 0 = not yet checked, 1 = in use, -1 = the per-op kernels run
  int fd_state = 0;
  det::FdParams fd;
  int fd_grid = 0;
  double fd_wbytes = 0;  // weight bytes one fused forward streams
  // the decompress loop on the device (codec.cpp): its state, a pinned copy,
  // row id 0 for the CDF of the one-position logits, and the one-position
  // forward that reads its token and position from device memory
  det::RcState* d_rc = nullptr;
  det::RcState* h_rc = nullptr;
  uint32_t* d_row0 = nullptr;
  Graph graph_dev1;
};

namespace det {
extern bool g_profiling;
det_status cuda_status(cudaError_t e);
// reads and clears a session's device error flag (synchronises its stream)
det_status session_take_error(det_session* s, bool cdf);
// the decompress loop on the device: allocates the session's RcState (once)
det_status rc_loop_init(det_session* s);
// det_forward split in two for the codec's pipeline: the forward enqueued
// without a synchronisation (its errors surface at the next take_error), and
// its device time added once the stream has passed it
det_status forward_enqueue(det_session* s, const uint32_t* tokens, uint32_t n, uint32_t pos0);
void forward_collect(det_session* s);
// a one-position forward whose token and position are already in device
// memory (s->d_tokens[0], s->d_pos[0]), e.g. written by rc_step_kernel
det_status forward_device_inputs(det_session* s);
// forward stages (session.cpp); `have` carries which quantisations of the
// FFN activation the SwiGLU launch already wrote
det_status fwd_embed(det_session* s, const Launch& L, int T);
det_status fwd_attention(det_session* s, const Launch& L, int l, int T);
det_status fwd_attn_out(det_session* s, const Launch& L, int l, int T, const float* attn);
det_status fwd_ffn_in(det_session* s, const Launch& L, int l, int T, int* have);
det_status fwd_ffn_out(det_session* s, const Launch& L, int l, int T, const float* ff, int have);
det_status fwd_head(det_session* s, const Launch& L, int T);
// tensor parallelism (tp.cpp)
void tp_model_free(det_model* m);
det_status tp_session_create(det_model* m, uint32_t n_ctx, uint32_t max_chunk, det_session** out);
void tp_session_release(det_session* s);  // frees the other parts of a primary session
det_status tp_run_forward(det_session* s, int T, bool graphs);
det_status tp_reset(det_session* s);
det_status tp_take_part_errors(det_session* s);  // error flags of the parts other than the primary
// model-owned session for the model-level entry points (not re-entrant)
det_status session_acquire(det_model* m, uint32_t n_ctx, uint32_t max_chunk, det_session** out);
void session_release_cached(det_model* m);
}
