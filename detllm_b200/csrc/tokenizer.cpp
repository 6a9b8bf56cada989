// tokenizer.cpp -- the codec's tokenizers, selected from GGUF metadata:
// byte fallback, byte-level BPE and SentencePiece (crates/det-token/src/
// lib.rs:85-850), and the codec symbol stream with byte escapes.  Host code:
// the model keeps one Tokenizer, compress tokenizes the input with it and
// decompress turns each decoded symbol back into its bytes.
#include <algorithm>
#include <cstring>
#include <queue>

#include "host_common.h"

namespace det {

namespace {

// canonical_byte_fallback_token (lib.rs:841-848): "<0xHH>", HH parsed like
// u8::from_str_radix(_, 16) (an optional leading '+')
int byte_fallback_of(const std::string& s) {
  if (s.size() != 6 || s[0] != '<' || s[1] != '0' || s[2] != 'x' || s[5] != '>') return -1;
  const char* h = s.c_str() + 3;
  const int start = h[0] == '+' ? 1 : 0;
  if (start == 1 && h[1] == '+') return -1;
  int v = 0;
  for (int i = start; i < 2; i++) {
    const char c = h[i];
    int dgt;
    if (c >= '0' && c <= '9') dgt = c - '0';
    else if (c >= 'a' && c <= 'f') dgt = c - 'a' + 10;
    else if (c >= 'A' && c <= 'F') dgt = c - 'A' + 10;
    else return -1;
    v = v * 16 + dgt;
  }
  return v;
}

// the byte a GPT-2 byte-unicode code point stands for, or -1
// (gpt2_char_to_byte, lib.rs:821-839): printable bytes map to themselves,
// the other 68 to code points 256.. in byte order
int gpt2_byte(uint32_t cp) {
  static const auto table = [] {
    std::vector<int> t(256 + 68, -1);
    auto printable = [](int b) { return (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255); };
    int n = 0;
    for (int b = 0; b < 256; b++) {
      if (printable(b)) t[(size_t)b] = b;
      else t[(size_t)(256 + n++)] = b;
    }
    return t;
  }();
  return cp < table.size() ? table[cp] : -1;
}

// token_piece_bytes (lib.rs:797-811): byte fallback token, else a GPT-2
// byte-unicode string, else "▁rest" -> " rest", else the UTF-8 bytes
std::string piece_bytes(const std::string& s) {
  const int b = byte_fallback_of(s);
  if (b >= 0) return std::string(1, (char)b);
  std::string out;
  bool ok = true;
  for (size_t i = 0; i < s.size() && ok;) {
    const uint8_t c = (uint8_t)s[i];
    const int extra = c < 0x80 ? 0 : c >= 0xF0 ? 3 : c >= 0xE0 ? 2 : 1;
    uint32_t cp = extra ? (c & (0x3Fu >> extra)) : c;
    for (int k = 1; k <= extra && i + k < s.size(); k++) cp = (cp << 6) | ((uint8_t)s[i + k] & 0x3Fu);
    i += 1 + extra;
    const int v = gpt2_byte(cp);
    if (v < 0) ok = false;
    else out.push_back((char)v);
  }
  if (ok) return out;
  if (s.size() >= 3 && (uint8_t)s[0] == 0xE2 && (uint8_t)s[1] == 0x96 && (uint8_t)s[2] == 0x81)
    return " " + s.substr(3);
  return s;
}

int emittable_type(int64_t t) {  // token_type_is_emittable (lib.rs:704-710)
  if (t == 1 || t == 4 || t == 6) return 1;
  if (t == 2 || t == 3 || t == 5) return 0;
  return -1;
}

uint64_t pair_key(uint32_t l, uint32_t r) { return (uint64_t)l << 32 | r; }

}  // namespace

// Tokenizer::from_gguf (lib.rs:86-132) and the three constructors
// (:258-304, :343-407, :520-566)
det_status Tokenizer::from_gguf(const Gguf& g) {
  *this = Tokenizer();
  const GgufValue* toks = g.find("tokenizer.ggml.tokens");
  if (!toks || toks->type != GV_ARRAY || toks->elem_type != GV_STRING) return DET_ERR_TOKENIZER;
  const size_t V = toks->strs.size();
  vocab = V;
  std::vector<int> emit;  // empty: every token emittable
  if (const GgufValue* tt = g.find("tokenizer.ggml.token_type")) {
    if (tt->type != GV_ARRAY || (tt->elem_type != GV_I32 && tt->elem_type != GV_U32) || tt->count != V)
      return DET_ERR_TOKENIZER;
    emit.resize(V);
    for (size_t i = 0; i < V; i++) {
      uint32_t raw;
      std::memcpy(&raw, tt->raw + 4 * i, 4);
      emit[i] = emittable_type(tt->elem_type == GV_I32 ? (int64_t)(int32_t)raw : (int64_t)raw);
      if (emit[i] < 0) return DET_ERR_TOKENIZER;
    }
  }
  auto emittable = [&](size_t i) { return emit.empty() || emit[i] != 0; };
  const GgufValue* merges = g.find("tokenizer.ggml.merges");
  if (merges && (merges->type != GV_ARRAY || merges->elem_type != GV_STRING)) return DET_ERR_TOKENIZER;
  const GgufValue* model = g.find("tokenizer.ggml.model");
  if (model && model->type != GV_STRING) return DET_ERR_TOKENIZER;
  const GgufValue* scores = g.find("tokenizer.ggml.scores");
  if (model) {
    if (model->str == "gpt2") kind = BPE;
    else if (model->str == "llama" || model->str == "spm" || model->str == "sentencepiece") kind = SPM;
    else return DET_ERR_TOKENIZER;  // UnsupportedTokenizerModel
  } else if (merges && !merges->strs.empty()) {
    kind = BPE;
  } else if (scores) {
    if (scores->type != GV_ARRAY || scores->elem_type != GV_F32) return DET_ERR_TOKENIZER;
    kind = SPM;
  } else {
    kind = BYTE_FALLBACK;
  }
  for (int b = 0; b < 256; b++) byte_to_token[b] = -1;
  bytes.assign(V, std::string());
  has_bytes.assign(V, kind != BYTE_FALLBACK);
  if (kind != BYTE_FALLBACK)
    for (size_t i = 0; i < V; i++) bytes[i] = piece_bytes(toks->strs[i]);

  // every byte needs exactly one "<0xHH>" token (byte fallback, and the
  // fallback of SentencePiece); non-emittable ones stay out of the table
  auto byte_fallback = [&](bool record) -> det_status {
    bool seen[256] = {false};
    for (size_t i = 0; i < V; i++) {
      const int b = byte_fallback_of(toks->strs[i]);
      if (b < 0) continue;
      if (seen[b]) return DET_ERR_TOKENIZER;  // DuplicateByteFallback
      seen[b] = true;
      if (record) {
        bytes[i] = std::string(1, (char)b);
        has_bytes[i] = 1;
      }
      if (emittable(i)) byte_to_token[b] = (int32_t)i;
    }
    for (bool s : seen)
      if (!s) return DET_ERR_TOKENIZER;  // IncompleteByteFallback
    return DET_OK;
  };

  if (kind == BYTE_FALLBACK) return byte_fallback(true);

  if (kind == SPM) {
    std::vector<float> sc(V, 0.0f);
    if (scores) {  // optional_gguf_scores (:646-664)
      if (scores->type != GV_ARRAY || scores->elem_type != GV_F32 || scores->count != V) return DET_ERR_TOKENIZER;
      for (size_t i = 0; i < V; i++) {
        uint32_t bits;
        std::memcpy(&bits, scores->raw + 4 * i, 4);
        if ((bits & 0x7f800000u) == 0x7f800000u) return DET_ERR_TOKENIZER;  // NonFiniteScore
        std::memcpy(&sc[i], &bits, 4);
      }
    }
    if (det_status st = byte_fallback(false)) return st;
    // per distinct multi-byte piece: a later token replaces the kept one
    // only with a strictly higher score (equal scores keep the lower id)
    std::unordered_map<std::string, std::pair<uint32_t, float>> best;
    for (size_t i = 0; i < V; i++) {
      if (bytes[i].size() <= 1 || !emittable(i)) continue;
      max_piece_len = std::max(max_piece_len, bytes[i].size());
      auto it = best.find(bytes[i]);
      if (it == best.end()) best.emplace(bytes[i], std::make_pair((uint32_t)i, sc[i]));
      else if (sc[i] > it->second.second) it->second = std::make_pair((uint32_t)i, sc[i]);
    }
    for (auto& kv : best) pieces.emplace(kv.first, kv.second.first);
    return DET_OK;
  }

  // byte-level BPE: single-byte pieces seed the byte table, every emittable
  // piece must be unique, merges resolve through the pieces' bytes
  std::unordered_map<std::string, uint32_t> by_bytes;
  for (size_t i = 0; i < V; i++) {
    if (!emittable(i)) continue;
    if (bytes[i].size() == 1) {
      const uint8_t b = (uint8_t)bytes[i][0];
      if (byte_to_token[b] >= 0) return DET_ERR_TOKENIZER;  // DuplicateByteFallback
      byte_to_token[b] = (int32_t)i;
    }
    if (!by_bytes.emplace(bytes[i], (uint32_t)i).second) return DET_ERR_TOKENIZER;  // DuplicateTokenBytes
  }
  const size_t nm = merges ? merges->strs.size() : 0;
  for (size_t r = 0; r < nm; r++) {
    const std::string& m = merges->strs[r];  // parse_merge (:772-786)
    const size_t sp = m.find(' ');
    if (sp == std::string::npos || sp == 0 || sp + 1 == m.size() || m.find(' ', sp + 1) != std::string::npos)
      return DET_ERR_TOKENIZER;  // InvalidMerge
    const std::string lb = piece_bytes(m.substr(0, sp)), rb = piece_bytes(m.substr(sp + 1));
    const auto li = by_bytes.find(lb), ri = by_bytes.find(rb), mi = by_bytes.find(lb + rb);
    if (li == by_bytes.end() || ri == by_bytes.end() || mi == by_bytes.end()) {
      if (!emit.empty()) continue;
      return DET_ERR_TOKENIZER;  // MissingTokenBytes / MissingMergeToken
    }
    if (!this->merges.emplace(pair_key(li->second, ri->second), std::make_pair((uint64_t)r, mi->second)).second)
      return DET_ERR_TOKENIZER;  // DuplicateMerge
  }
  return DET_OK;
}

// tokenize_bytes of the selected tokenizer (lib.rs:306-312, 409-476, 568-604)
det_status Tokenizer::tokenize(const uint8_t* in, size_t n, std::vector<uint32_t>* out) const {
  if (kind == SPM) {  // longest multi-byte piece at each position, else the byte token
    std::string key;
    for (size_t pos = 0; pos < n;) {
      const size_t max_end = std::min(n, pos + max_piece_len);
      int64_t best = -1;
      size_t best_len = 0;
      for (size_t end = pos + 2; end <= max_end; end++) {
        key.assign(reinterpret_cast<const char*>(in + pos), end - pos);
        const auto it = pieces.find(key);
        if (it != pieces.end()) {
          best = it->second;
          best_len = end - pos;
        }
      }
      if (best >= 0) {
        out->push_back((uint32_t)best);
        pos += best_len;
      } else {
        if (byte_to_token[in[pos]] < 0) return DET_ERR_TOKENIZER;  // MissingByteFallback
        out->push_back((uint32_t)byte_to_token[in[pos]]);
        pos++;
      }
    }
    return DET_OK;
  }
  const size_t base = out->size();
  for (size_t i = 0; i < n; i++) {
    if (byte_to_token[in[i]] < 0) return DET_ERR_TOKENIZER;  // MissingByteFallback
    out->push_back((uint32_t)byte_to_token[in[i]]);
  }
  if (kind == BYTE_FALLBACK || n < 2) return DET_OK;
  // BPE: apply the lowest-rank merge, leftmost first, until none applies.
  // Candidates (rank, left index, merged id) come off a min-heap; stale
  // ones (a side already merged away, or the pair changed) are skipped.
  uint32_t* ids = out->data() + base;
  std::vector<int64_t> prev(n), next(n);
  std::vector<char> alive(n, 1);
  for (size_t i = 0; i < n; i++) {
    prev[i] = (int64_t)i - 1;
    next[i] = i + 1 < n ? (int64_t)i + 1 : -1;
  }
  using Cand = std::tuple<uint64_t, size_t, uint32_t>;
  std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> heap;
  auto push = [&](size_t left, int64_t right) {
    if (right < 0) return;
    const auto it = merges.find(pair_key(ids[left], ids[(size_t)right]));
    if (it != merges.end()) heap.emplace(it->second.first, left, it->second.second);
  };
  for (size_t i = 0; i + 1 < n; i++) push(i, (int64_t)i + 1);
  while (!heap.empty()) {
    const auto [rank, index, merged] = heap.top();
    heap.pop();
    if (!alive[index]) continue;
    const int64_t right = next[index];
    if (right < 0 || !alive[(size_t)right]) continue;
    const auto it = merges.find(pair_key(ids[index], ids[(size_t)right]));
    if (it == merges.end() || it->second.first != rank || it->second.second != merged) continue;
    ids[index] = merged;
    alive[(size_t)right] = 0;
    next[index] = next[(size_t)right];
    if (next[index] >= 0) prev[(size_t)next[index]] = (int64_t)index;
    if (prev[index] >= 0) push((size_t)prev[index], (int64_t)index);
    push(index, next[index]);
  }
  size_t k = base;
  for (int64_t i = 0; i >= 0; i = next[(size_t)i])
    if (alive[(size_t)i]) (*out)[k++] = ids[i];
  out->resize(k);
  return DET_OK;
}

// codec_symbol_stream / codec_symbols (lib.rs:150-180): runs of bytes that
// have a single-byte token are tokenized; any other byte is escaped as
// vocab + byte
det_status Tokenizer::codec_symbols(const uint8_t* in, size_t n, std::vector<uint32_t>* out) const {
  for (size_t pos = 0; pos < n;) {
    if (byte_to_token[in[pos]] < 0) {
      out->push_back((uint32_t)(vocab + in[pos]));
      pos++;
      continue;
    }
    const size_t start = pos++;
    while (pos < n && byte_to_token[in[pos]] >= 0) pos++;
    if (det_status st = tokenize(in + start, pos - start, out)) return st;
  }
  return DET_OK;
}

// decode_codec_symbol (lib.rs:182-196): a token's bytes (a byte-fallback
// tokenizer knows its byte tokens only), or the escaped byte
det_status Tokenizer::symbol_bytes(uint32_t symbol, bool escapes, std::string* piece) const {
  if (symbol < vocab) {
    if (!has_bytes[symbol]) return DET_ERR_TOKENIZER;  // InvalidToken
    *piece = bytes[symbol];
    return DET_OK;
  }
  if (escapes && symbol < vocab + 256) {
    *piece = std::string(1, (char)(symbol - vocab));
    return DET_OK;
  }
  return DET_ERR_TOKENIZER;
}

}  // namespace det

// ---- host-only entry points (no device needed) --------------------------------
namespace {
det_status tokenizer_of(const uint8_t* gguf, size_t len, det::Tokenizer* t) {
  det::Gguf g;
  if (g.parse(gguf, len)) return DET_ERR_GGUF;
  return t->from_gguf(g);
}

det_status copy_u32(const std::vector<uint32_t>& v, uint32_t** out, size_t* n) {
  uint32_t* p = static_cast<uint32_t*>(std::malloc(std::max<size_t>(v.size(), 1) * 4));
  if (!p) return DET_ERR_ALLOC;
  if (!v.empty()) std::memcpy(p, v.data(), v.size() * 4);
  *out = p;
  *n = v.size();
  return DET_OK;
}
}  // namespace

extern "C" {

det_status det_tokenizer_kind(const uint8_t* gguf, size_t len, int* kind) {
  if (!gguf || !kind) return DET_ERR_INVALID_ARGUMENT;
  det::Tokenizer t;
  if (det_status st = tokenizer_of(gguf, len, &t)) return st;
  *kind = (int)t.kind;
  return DET_OK;
}

det_status det_tokenize(const uint8_t* gguf, size_t len, const uint8_t* input, size_t n, int codec, uint32_t** out,
                        size_t* out_n) {
  if (!gguf || (!input && n) || !out || !out_n) return DET_ERR_INVALID_ARGUMENT;
  det::Tokenizer t;
  if (det_status st = tokenizer_of(gguf, len, &t)) return st;
  std::vector<uint32_t> v;
  if (det_status st = codec ? t.codec_symbols(input, n, &v) : t.tokenize(input, n, &v)) return st;
  return copy_u32(v, out, out_n);
}

det_status det_detokenize(const uint8_t* gguf, size_t len, const uint32_t* symbols, size_t n, int byte_escapes,
                          uint8_t** out, size_t* out_n) {
  if (!gguf || (!symbols && n) || !out || !out_n) return DET_ERR_INVALID_ARGUMENT;
  det::Tokenizer t;
  if (det_status st = tokenizer_of(gguf, len, &t)) return st;
  std::string bytes, piece;
  for (size_t i = 0; i < n; i++) {
    if (det_status st = t.symbol_bytes(symbols[i], byte_escapes != 0, &piece)) return st;
    bytes += piece;
  }
  uint8_t* p = static_cast<uint8_t*>(std::malloc(std::max<size_t>(bytes.size(), 1)));
  if (!p) return DET_ERR_ALLOC;
  std::memcpy(p, bytes.data(), bytes.size());
  *out = p;
  *out_n = bytes.size();
  return DET_OK;
}

}  // extern "C"
