// codec.cpp -- compress / decompress on the device forward.
//
// Reproduces det-cli's windowed codec (crates/det-cli/src/main.rs:433-855):
// a fixed window of n_ctx positions, overlap n_ctx/4, KV reset and replay of
// the overlap tokens at positions 0.. when the window fills, the uniform CDF
// while the window is empty, byte escapes that do not advance the model, the
// 56-byte DTLZ header (crates/det-coder/src/file.rs) and the canonical
// re-encode check of decompress.
//
// Encode is teacher-forced, so the whole schedule is known up front: the
// symbols are mapped to (window, logits position) pairs, each window's tokens
// run through the device in chunks of up to `encode_chunk()` positions, and the
// ranges of all symbols whose logits a chunk produced come back in one call.
// The range coder consumes them in symbol order, so the payload is the same
// byte stream the one-token-at-a-time reference produces.  Positions whose
// logits no symbol uses (the last token of a full window, overlap tokens of a
// window nobody reads from) are skipped; that changes no output.
#include <algorithm>
#include <cstdlib>

#include <atomic>

#include "host_common.h"

using namespace det;

namespace {

// Positions per forward launch sequence: larger chunks give the GEMMs and
// attention more parallel work per weight pass.  DETGPU_CHUNK, or
// det_set_encode_chunk, overrides the default (16 .. 1024); the output bytes
// do not depend on it.
uint32_t env_chunk() {
  const char* e = std::getenv("DETGPU_CHUNK");
  const long v = e ? std::strtol(e, nullptr, 10) : 0;
  return v >= 16 && v <= 1024 ? (uint32_t)v : 1024u;
}
std::atomic<uint32_t> g_chunk{0};  // 0: not read yet
uint32_t encode_chunk() {
  uint32_t c = g_chunk.load(std::memory_order_relaxed);
  if (!c) {
    uint32_t want = env_chunk(), zero = 0;
    g_chunk.compare_exchange_strong(zero, want);
    c = g_chunk.load(std::memory_order_relaxed);
  }
  return c;
}
constexpr uint32_t kEscapes = 256;

// next_window_start (det-cli main.rs:772-778)
size_t next_window_start(size_t pos, size_t ws, size_t n_ctx, size_t overlap) {
  const size_t d = pos > ws ? pos - ws : 0;
  if (d >= n_ctx) return pos > overlap ? pos - overlap : 0;
  return ws;
}

// validate_window (det-cli main.rs:810-826)
det_status validate_window(size_t n_ctx, size_t overlap, size_t model_ctx) {
  if (n_ctx == 0 || n_ctx > model_ctx || overlap >= n_ctx) return DET_ERR_WINDOW;
  return DET_OK;
}

struct SymbolPlan {
  int32_t window;  // -1: uniform CDF (empty context)
  int32_t pos;     // logits position within the window
};

struct WindowPlan {
  size_t start;   // token index of position 0
  size_t needed;  // positions that must be forwarded (max logits pos + 1)
};

// Encode the symbol stream (encode_symbols_with_model, main.rs:523-552).
det_status encode_impl(det_model* m, const uint32_t* sym, size_t n, uint32_t n_ctx, uint32_t overlap, int escapes,
                       std::vector<uint8_t>* payload) {
  if (det_status st = validate_window(n_ctx, overlap, (size_t)m->cfg.ctx)) return st;
  const uint32_t V = (uint32_t)m->vocab;
  const uint32_t tail = escapes ? kEscapes : 0;
  if ((uint64_t)V + tail > (1u << 18)) return DET_ERR_CDF_TOO_MANY_SYMBOLS;
  const uint64_t symbols_total = (uint64_t)V + tail;
  // ---- plan: replay the reference state machine on indices only
  std::vector<uint32_t> tokens;
  std::vector<SymbolPlan> plan(n);
  std::vector<WindowPlan> windows;
  windows.push_back({0, 0});
  size_t ws = 0, clen = 0;
  for (size_t i = 0; i < n; i++) {
    const size_t pos = tokens.size();
    const size_t nws = next_window_start(pos, ws, n_ctx, overlap);
    if (nws != ws) {  // replay (main.rs:691-701)
      ws = nws;
      clen = pos - ws;
      windows.push_back({ws, 0});
    }
    const uint32_t s = sym[i];
    if (clen == 0) {
      if (s >= symbols_total) return DET_ERR_CDF_SYMBOL_OUT_OF_RANGE;
      plan[i] = {-1, 0};
    } else {
      if (s >= symbols_total) return DET_ERR_CDF_SYMBOL_OUT_OF_RANGE;
      plan[i] = {(int32_t)windows.size() - 1, (int32_t)(clen - 1)};
      WindowPlan& w = windows.back();
      w.needed = std::max(w.needed, clen);
    }
    if (escapes && s >= V) continue;
    if (s >= V) return DET_ERR_CDF_SYMBOL_OUT_OF_RANGE;
    tokens.push_back(s);
    clen++;
  }
  // ---- execute window by window, chunk by chunk
  RangeEncoder enc;
  size_t next = 0;  // next symbol to encode
  auto drain_uniform = [&]() -> det_status {
    while (next < n && plan[next].window < 0) {
      if (det_status st = enc.encode(sym[next], 1, symbols_total)) return st;
      next++;
    }
    return DET_OK;
  };
  if (det_status st = drain_uniform()) return st;
  det_session* s = nullptr;
  bool need_device = false;
  for (const auto& w : windows)
    if (w.needed) need_device = true;
  if (need_device)
    if (det_status st = session_acquire(m, n_ctx, encode_chunk(), &s)) return st;
  // the forwards as one list of chunks: window, first position, length
  struct Chunk {
    size_t wi, p0;
    uint32_t cnt;
  };
  std::vector<Chunk> chunks;
  if (s)
    for (size_t wi = 0; wi < windows.size(); wi++)
      for (size_t p0 = 0; p0 < windows[wi].needed; p0 += (size_t)s->max_chunk)
        chunks.push_back({wi, p0, (uint32_t)std::min<size_t>((size_t)s->max_chunk, windows[wi].needed - p0)});
  // Chunk k + 1 is enqueued as soon as chunk k's ranges are on the host, so
  // the host range-codes chunk k while the device runs chunk k + 1 (the
  // ranges call is the synchronisation point, and a forward's errors surface
  // there).  A window after the first starts from a cleared KV cache.
  // Tensor-parallel sessions forward synchronously (their forward spans
  // several devices).
  auto enqueue = [&](size_t k) -> det_status {
    const Chunk& c = chunks[k];
    if (c.p0 == 0 && c.wi > 0)
      if (det_status st = det_session_reset(s)) return st;
    const uint32_t* tk = tokens.data() + windows[c.wi].start + c.p0;
    return s->tp ? det_forward(s, tk, c.cnt, (uint32_t)c.p0, nullptr) : forward_enqueue(s, tk, c.cnt, (uint32_t)c.p0);
  };
  std::vector<uint32_t> rows, qsym;
  std::vector<det_symbol_range> ranges;
  det_status st = chunks.empty() ? DET_OK : enqueue(0);
  for (size_t k = 0; k < chunks.size() && !st; k++) {
    const Chunk& c = chunks[k];
    rows.clear();
    qsym.clear();
    size_t j = next;
    for (; j < n; j++) {
      const SymbolPlan& sp = plan[j];
      if (sp.window < 0) {
        // a uniform symbol after a device window can only follow a window
        // with no tokens, which cannot happen mid-stream
        break;
      }
      if ((size_t)sp.window != c.wi || (size_t)sp.pos >= c.p0 + c.cnt) break;
      rows.push_back((uint32_t)(sp.pos - c.p0));
      qsym.push_back(sym[j]);
    }
    ranges.resize(rows.size());
    if (!rows.empty()) {
      st = det_symbol_ranges(s, rows.data(), qsym.data(), (uint32_t)rows.size(), escapes, ranges.data());
    } else {  // no symbol reads this chunk's logits: still check its forward
      st = session_take_error(s, false);
      forward_collect(s);
    }
    if (!st && k + 1 < chunks.size()) st = enqueue(k + 1);
    for (size_t q = 0; q < rows.size() && !st; q++) st = enc.encode(ranges[q].cum, ranges[q].freq, ranges[q].total);
    next = j;
    if (!st) st = drain_uniform();
  }
  if (st && s) {  // leave the session idle for its next user
    cudaSetDevice(m->device);
    cudaStreamSynchronize(s->stream);
    session_take_error(s, false);
    forward_collect(s);
    s->last_n = 0;
  }
  if (st) return st;
  if (next != n) return DET_ERR_WINDOW;
  *payload = enc.finish();
  return DET_OK;
}

det_status copy_out(const std::vector<uint8_t>& v, uint8_t** out, size_t* out_len) {
  uint8_t* p = static_cast<uint8_t*>(std::malloc(v.size() ? v.size() : 1));
  if (!p) return DET_ERR_ALLOC;
  if (!v.empty()) std::memcpy(p, v.data(), v.size());
  *out = p;
  *out_len = v.size();
  return DET_OK;
}

// LoadedModel checks (det-cli main.rs:954-1008)
det_status codec_model_checks(det_model* m) {
  if (m->tok_status) return m->tok_status;
  if (m->tok.vocab != (size_t)m->vocab) return DET_ERR_VOCAB_MISMATCH;
  if ((uint64_t)m->vocab + kEscapes > (1u << 18)) return DET_ERR_CDF_TOO_MANY_SYMBOLS;
  return DET_OK;
}

void put_le(uint8_t* p, uint64_t v, int n) {
  for (int i = 0; i < n; i++) p[i] = (uint8_t)(v >> (8 * i));
}
uint64_t get_le(const uint8_t* p, int n) {
  uint64_t v = 0;
  for (int i = n - 1; i >= 0; i--) v = (v << 8) | p[i];
  return v;
}

// bytes of every codec symbol on the device, for the decompress loop (once
// per model): token pieces, then 1 for each byte escape; 0 marks a symbol
// without bytes (det-token lib.rs:182-196)
det_status ensure_piece_len(det_model* m) {
  if (m->piece_len) return DET_OK;
  const size_t n = (size_t)m->vocab + kEscapes;
  std::vector<uint16_t> len(n);
  std::string piece;
  size_t mx = 1;
  for (size_t i = 0; i < n; i++) {
    const bool ok = m->tok.symbol_bytes((uint32_t)i, true, &piece) == DET_OK;
    len[i] = ok ? (uint16_t)std::min<size_t>(piece.size(), 65535) : 0;
    if (ok) mx = std::max(mx, piece.size());
  }
  void* p = nullptr;
  cudaSetDevice(m->device);
  if (cudaMalloc(&p, n * sizeof(uint16_t)) != cudaSuccess) return DET_ERR_DEVICE_OOM;
  m->allocations.push_back(p);
  if (cudaMemcpy(p, len.data(), n * sizeof(uint16_t), cudaMemcpyHostToDevice) != cudaSuccess) return DET_ERR_CUDA;
  m->piece_len = static_cast<uint16_t*>(p);
  m->max_piece = mx;
  return DET_OK;
}

// decode_bytes_with_model (det-cli main.rs:585-630) with the symbol loop on
// the device: per step, the CDF of the last logits row, the range decoder's
// decode_freq / symbol search / advance (rc_step_kernel) and the next
// one-position forward, whose token and position the step kernel writes.
// The host enqueues a batch of steps and synchronises once per batch, not
// per symbol; it maps the batch's symbols to bytes and replays the overlap
// when a window is full, as the host loop does.  Symbols and bytes are those
// of the host loop: every step computes the same ranges on the same logits.
det_status decode_on_device(det_model* m, det_session* s, const uint8_t* payload, size_t plen, uint64_t orig_len,
                            uint32_t n_ctx, uint32_t overlap, int escapes, std::vector<uint8_t>* bytes,
                            std::vector<uint32_t>* syms) {
  if (plen < 8) return DET_ERR_RANGE_UNEXPECTED_EOF;  // RangeDecoder::new reads 8 bytes
  if (det_status st = ensure_piece_len(m)) return st;
  if (det_status st = rc_loop_init(s)) return st;
  cudaSetDevice(m->device);
  const uint32_t V = (uint32_t)m->vocab;
  struct DevBuf {
    uint8_t* p = nullptr;
    ~DevBuf() {
      if (p) cudaFree(p);
    }
  } pay;
  if (cudaMalloc(&pay.p, plen) != cudaSuccess) return DET_ERR_DEVICE_OOM;
  RcState& H = *s->h_rc;
  std::memset(&H, 0, sizeof(H));
  H.low = 0;
  H.range = ~0ull;
  for (int i = 0; i < 8; i++) H.code = (H.code << 8) | payload[i];
  H.pos = 8;
  H.len = plen;
  H.orig_len = orig_len;
  H.n_ctx = n_ctx;
  H.tail = escapes ? kEscapes : 0;
  // before any forward: finite logits for the (unused) CDF of an empty
  // window, and token 0 at position 0 for the recomputing forwards
  if (cudaMemcpyAsync(pay.p, payload, plen, cudaMemcpyHostToDevice, s->stream) != cudaSuccess ||
      cudaMemsetAsync(s->logits, 0, (size_t)V * sizeof(float), s->stream) != cudaSuccess ||
      cudaMemsetAsync(s->d_tokens, 0, sizeof(uint32_t), s->stream) != cudaSuccess ||
      cudaMemsetAsync(s->d_pos, 0, sizeof(int), s->stream) != cudaSuccess)
    return DET_ERR_CUDA;
  s->stats.h2d_bytes += plen;
  const Launch L{s->stream, s->d_err, &s->stats.launches};
  std::vector<uint32_t> ctx;
  std::string piece;
  size_t ws = 0;
  uint32_t clen = 0;
  while (bytes->size() < orig_len) {
    // steps this batch: no more symbols than the remaining bytes can hold,
    // no more tokens than the window has room for
    const uint64_t remaining = orig_len - bytes->size();
    uint32_t B = (uint32_t)std::min<uint64_t>(kRcMaxBatch, std::max<uint64_t>(1, remaining / m->max_piece));
    B = std::min<uint32_t>(B, std::max<uint32_t>(1, n_ctx - clen));
    H.count = 0;
    H.max_count = B;
    H.status = RC_RUNNING;
    H.clen = clen;
    if (cudaMemcpyAsync(s->d_rc, &H, sizeof(RcState), cudaMemcpyHostToDevice, s->stream) != cudaSuccess)
      return DET_ERR_CUDA;
    if (cudaEventRecord(s->ev[0], s->stream) != cudaSuccess) return DET_ERR_CUDA;
    for (uint32_t b = 0; b < B; b++) {
      if (launch_cdf_prepare(L, s->logits, (int)V, s->d_row0, 1, s->cdf_e, s->cdf_z) != cudaSuccess ||
          launch_rc_step(L, s->d_rc, s->cdf_e, s->cdf_z, (int)V, pay.p, m->piece_len, s->d_tokens, s->d_pos) !=
              cudaSuccess)
        return DET_ERR_CUDA;
      if (det_status st = forward_device_inputs(s)) return st;
    }
    if (cudaEventRecord(s->ev[1], s->stream) != cudaSuccess ||
        cudaMemcpyAsync(&H, s->d_rc, sizeof(RcState), cudaMemcpyDeviceToHost, s->stream) != cudaSuccess)
      return DET_ERR_CUDA;
    s->stats.h2d_bytes += sizeof(RcState);
    s->stats.d2h_bytes += sizeof(RcState);
    if (det_status st = session_take_error(s, true)) return st;
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, s->ev[0], s->ev[1]) == cudaSuccess) s->stats.forward_ms += ms;
    for (uint32_t i = 0; i < H.count; i++) {
      const uint32_t symbol = H.syms[i];
      if (det_status st = m->tok.symbol_bytes(symbol, escapes != 0, &piece)) return st;
      bytes->insert(bytes->end(), piece.begin(), piece.end());
      syms->push_back(symbol);
      if (escapes && symbol >= V) continue;
      ctx.push_back(symbol);
      s->stats.tokens++;
    }
    clen = H.clen;
    if (H.status == RC_FAILED) return (det_status)H.error;
    if (H.status == RC_DONE) break;
    if (H.status == RC_WINDOW_FULL) {  // replay the overlap as chunked prefill
      const size_t pos = ctx.size();
      ws = next_window_start(pos, ws, n_ctx, overlap);
      clen = 0;
      if (det_status st = det_session_reset(s)) return st;
      for (size_t p = ws; p < pos; p += (size_t)s->max_chunk) {
        const uint32_t cnt = (uint32_t)std::min<size_t>((size_t)s->max_chunk, pos - p);
        if (det_status st = det_forward(s, ctx.data() + p, cnt, clen, nullptr)) return st;
        clen += cnt;
      }
      // the last replayed position once more as a one-position forward: its
      // logits go to row 0 and its token and position to the buffers the
      // steps' forwards read (bit-identical to the chunk's last row)
      if (clen) {
        if (det_status st = det_forward(s, &ctx.back(), 1, clen - 1, nullptr)) return st;
      } else if (cudaMemsetAsync(s->d_tokens, 0, sizeof(uint32_t), s->stream) != cudaSuccess ||
                 cudaMemsetAsync(s->d_pos, 0, sizeof(int), s->stream) != cudaSuccess) {
        return DET_ERR_CUDA;
      }
    }
  }
  return DET_OK;
}

}  // namespace

extern "C" {

det_status det_set_encode_chunk(uint32_t chunk, uint32_t* previous) {
  if (chunk != 0 && (chunk < 16 || chunk > 1024)) return DET_ERR_INVALID_ARGUMENT;
  const uint32_t prev = encode_chunk();
  g_chunk.store(chunk ? chunk : env_chunk(), std::memory_order_relaxed);
  if (previous) *previous = prev;
  return DET_OK;
}

det_status det_encode_symbols(det_model* m, const uint32_t* symbols, size_t n, uint32_t n_ctx, uint32_t overlap,
                              int byte_escapes, uint8_t** out, size_t* out_len) {
  if (!m || (!symbols && n) || !out || !out_len) return DET_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::recursive_mutex> lk(m->mu);  // the model's cached session
  std::vector<uint8_t> payload;
  if (det_status st = encode_impl(m, symbols, n, n_ctx, overlap, byte_escapes, &payload)) return st;
  return copy_out(payload, out, out_len);
}

// compress (det-cli main.rs:433-463)
det_status det_compress(det_model* m, const uint8_t* input, size_t len, uint32_t n_ctx, uint8_t** out,
                        size_t* out_len) {
  if (!m || (!input && len) || !out || !out_len) return DET_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::recursive_mutex> lk(m->mu);  // the model's cached session
  if (det_status st = codec_model_checks(m)) return st;
  std::vector<uint32_t> sym;  // codec_symbols (det-token lib.rs:150-180)
  sym.reserve(len);
  if (det_status st = m->tok.codec_symbols(input, len, &sym)) return st;
  const uint32_t ctx = n_ctx ? n_ctx : (uint32_t)m->cfg.ctx;
  const uint32_t overlap = ctx / 4;
  std::vector<uint8_t> payload;
  if (det_status st = encode_impl(m, sym.data(), sym.size(), ctx, overlap, 1, &payload)) return st;
  std::vector<uint8_t> file(56 + payload.size());
  std::memcpy(file.data(), "DTLZ", 4);  // DtlzHeader::encode (file.rs:28-38)
  put_le(&file[4], 1, 2);
  put_le(&file[6], 1, 2);  // FLAG_BYTE_ESCAPES
  std::memcpy(&file[8], m->sha, 32);
  put_le(&file[40], ctx, 4);
  put_le(&file[44], overlap, 4);
  put_le(&file[48], len, 8);
  std::memcpy(&file[56], payload.data(), payload.size());
  return copy_out(file, out, out_len);
}

// decompress (det-cli main.rs:465-511) with decode_bytes_with_model
// (:585-630): one symbol at a time (the next token depends on the decoded
// one), then the canonical re-encode through the chunked encoder.
det_status det_decompress(det_model* m, const uint8_t* dtlz, size_t len, uint8_t** out, size_t* out_len) {
  if (!m || (!dtlz && len) || !out || !out_len) return DET_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::recursive_mutex> lk(m->mu);  // the model's cached session and piece table
  // DtlzHeader::decode (file.rs:58-90)
  if (len < 56) return DET_ERR_FILE_TOO_SHORT;
  if (std::memcmp(dtlz, "DTLZ", 4) != 0) return DET_ERR_FILE_BAD_MAGIC;
  if (get_le(dtlz + 4, 2) != 1) return DET_ERR_FILE_UNSUPPORTED_VERSION;
  const uint32_t flags = (uint32_t)get_le(dtlz + 6, 2);
  if (flags & ~1u) return DET_ERR_FILE_UNSUPPORTED_FLAGS;
  const uint32_t n_ctx = (uint32_t)get_le(dtlz + 40, 4), overlap = (uint32_t)get_le(dtlz + 44, 4);
  const uint64_t orig_len = get_le(dtlz + 48, 8);
  if (n_ctx == 0) return DET_ERR_FILE_INVALID_CONTEXT;
  if (overlap >= n_ctx) return DET_ERR_FILE_INVALID_OVERLAP;
  if (det_status st = codec_model_checks(m)) return st;
  if (std::memcmp(m->sha, dtlz + 8, 32) != 0) return DET_ERR_MODEL_HASH_MISMATCH;
  if (det_status st = validate_window(n_ctx, overlap, (size_t)m->cfg.ctx)) return st;
  const int escapes = (flags & 1) != 0;
  const uint32_t V = (uint32_t)m->vocab, tail = escapes ? kEscapes : 0;
  const uint64_t symbols_total = (uint64_t)V + tail;
  const uint8_t* payload = dtlz + 56;
  const size_t plen = len - 56;
  RangeDecoder dec;
  if (det_status st = dec.init(payload, plen)) return st;
  det_session* s = nullptr;
  if (det_status st = session_acquire(m, n_ctx, encode_chunk(), &s)) return st;
  if (det_status st = det_session_reset(s)) return st;
  std::vector<uint8_t> bytes;
  std::vector<uint32_t> ctx, syms;
  std::string piece;
  size_t ws = 0, clen = 0;
  uint32_t last_row = 0;
  det_status st = DET_OK;
  // one session on one device: the symbol loop runs on the device; a
  // tensor-parallel session (parts on several devices) keeps the host loop
  if (!s->tp) st = decode_on_device(m, s, payload, plen, orig_len, n_ctx, overlap, escapes, &bytes, &syms);
  while (s->tp && !st && bytes.size() < orig_len) {
    const size_t pos = ctx.size();
    const size_t nws = next_window_start(pos, ws, n_ctx, overlap);
    if (nws != ws) {  // replay the overlap as chunked prefill
      ws = nws;
      clen = 0;
      st = det_session_reset(s);
      for (size_t p = ws; p < pos && !st; p += (size_t)s->max_chunk) {
        const uint32_t cnt = (uint32_t)std::min<size_t>((size_t)s->max_chunk, pos - p);
        st = det_forward(s, ctx.data() + p, cnt, (uint32_t)clen, nullptr);
        clen += cnt;
        last_row = cnt - 1;
      }
      if (st) break;
    }
    uint32_t symbol;
    if (clen == 0) {  // uniform CDF (decode_symbol, main.rs:813-827)
      uint64_t value;
      if ((st = dec.decode_freq(symbols_total, &value))) break;
      symbol = (uint32_t)value;
      if ((st = dec.advance(value, 1, symbols_total))) break;
    } else {
      uint64_t total, value;
      det_symbol_range r;
      if ((st = det_decoder_total(s, last_row, escapes, &total))) break;
      if ((st = dec.decode_freq(total, &value))) break;
      if ((st = det_decoder_lookup(s, last_row, escapes, value, &symbol, &r))) break;
      if ((st = dec.advance(r.cum, r.freq, r.total))) break;
    }
    // decode_codec_symbol / detokenize_bytes (det-token lib.rs:182-196); a
    // symbol without bytes is an error (det-cli main.rs:614-616)
    if ((st = m->tok.symbol_bytes(symbol, escapes != 0, &piece))) break;
    if (piece.empty()) { st = DET_ERR_TOKENIZER; break; }
    bytes.insert(bytes.end(), piece.begin(), piece.end());
    syms.push_back(symbol);
    if (escapes && symbol >= V) continue;
    ctx.push_back(symbol);
    if (clen >= n_ctx) { st = DET_ERR_WINDOW; break; }
    st = det_forward(s, &symbol, 1, (uint32_t)clen, nullptr);
    clen++;
    last_row = 0;
  }
  if (st) return st;
  std::vector<uint8_t> canon;
  if ((st = encode_impl(m, syms.data(), syms.size(), n_ctx, overlap, escapes, &canon))) return st;
  if (canon.size() != plen || std::memcmp(canon.data(), payload, plen) != 0) return DET_ERR_NONCANONICAL;
  bytes.resize((size_t)orig_len);
  return copy_out(bytes, out, out_len);
}

}  // extern "C"
