// host_util.cpp -- SHA-256, the range coder and the GGUF reader of
// libdetgpu.so (host side).
#include <algorithm>
#include <cstdlib>

#if defined(__x86_64__)
#include <cpuid.h>
#include <immintrin.h>
#endif

#include "host_common.h"

namespace det {

// ---- SHA-256 -------------------------------------------------------------------
static const uint32_t kSha[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

static inline uint32_t ror(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

Sha256::Sha256() {
  static const uint32_t iv[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                                 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  std::memcpy(st_, iv, sizeof iv);
}

void Sha256::block(const uint8_t* p) {
  uint32_t w[64];
  for (int i = 0; i < 16; i++) w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
  for (int i = 16; i < 64; i++) {
    const uint32_t s0 = ror(w[i - 15], 7) ^ ror(w[i - 15], 18) ^ (w[i - 15] >> 3);
    const uint32_t s1 = ror(w[i - 2], 17) ^ ror(w[i - 2], 19) ^ (w[i - 2] >> 10);
    w[i] = w[i - 16] + s0 + w[i - 7] + s1;
  }
  uint32_t a = st_[0], b = st_[1], c = st_[2], d = st_[3], e = st_[4], f = st_[5], g = st_[6], h = st_[7];
  for (int i = 0; i < 64; i++) {
    const uint32_t t1 = h + (ror(e, 6) ^ ror(e, 11) ^ ror(e, 25)) + ((e & f) ^ (~e & g)) + kSha[i] + w[i];
    const uint32_t t2 = (ror(a, 2) ^ ror(a, 13) ^ ror(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
    h = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
  }
  st_[0] += a; st_[1] += b; st_[2] += c; st_[3] += d; st_[4] += e; st_[5] += f; st_[6] += g; st_[7] += h;
}

#if defined(__x86_64__)
// n 64-byte blocks with the x86 SHA extensions (Intel's SHA-256 instruction
// set: sha256rnds2 runs two rounds on the state packed as ABEF / CDGH,
// sha256msg1 / sha256msg2 extend the message schedule four words at a time)
__attribute__((target("sha,sse4.1,ssse3"))) static void sha256_blocks_ni(uint32_t st[8], const uint8_t* p,
                                                                          size_t n) {
  const __m128i bswap = _mm_set_epi64x(0x0c0d0e0f08090a0bLL, 0x0405060700010203LL);
  __m128i t = _mm_shuffle_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(st)), 0xB1);  // b a d c
  __m128i s1 = _mm_shuffle_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(st + 4)), 0x1B);  // h g f e
  __m128i s0 = _mm_alignr_epi8(t, s1, 8);  // f e b a (ABEF)
  s1 = _mm_blend_epi16(s1, t, 0xF0);       // h g d c (CDGH)
  for (; n; n--, p += 64) {
    const __m128i save0 = s0, save1 = s1;
    __m128i m[16];
    for (int g = 0; g < 4; g++)
      m[g] = _mm_shuffle_epi8(_mm_loadu_si128(reinterpret_cast<const __m128i*>(p + 16 * g)), bswap);
    for (int g = 4; g < 16; g++)  // W[t..t+3] from W[t-16..t-1]
      m[g] = _mm_sha256msg2_epu32(
          _mm_add_epi32(_mm_sha256msg1_epu32(m[g - 4], m[g - 3]), _mm_alignr_epi8(m[g - 1], m[g - 2], 4)), m[g - 1]);
    for (int g = 0; g < 16; g++) {
      __m128i k = _mm_add_epi32(m[g], _mm_loadu_si128(reinterpret_cast<const __m128i*>(kSha + 4 * g)));
      s1 = _mm_sha256rnds2_epu32(s1, s0, k);
      k = _mm_shuffle_epi32(k, 0x0E);
      s0 = _mm_sha256rnds2_epu32(s0, s1, k);
    }
    s0 = _mm_add_epi32(s0, save0);
    s1 = _mm_add_epi32(s1, save1);
  }
  t = _mm_shuffle_epi32(s0, 0x1B);    // a b e f
  s1 = _mm_shuffle_epi32(s1, 0xB1);   // g h c d
  s0 = _mm_blend_epi16(t, s1, 0xF0);  // a b c d
  s1 = _mm_alignr_epi8(s1, t, 8);     // e f g h
  _mm_storeu_si128(reinterpret_cast<__m128i*>(st), s0);
  _mm_storeu_si128(reinterpret_cast<__m128i*>(st + 4), s1);
}

static bool cpu_has_sha() {
  static const bool has = [] {
    unsigned a, b, c, d;
    if (!__get_cpuid_count(7, 0, &a, &b, &c, &d)) return false;
    return ((b >> 29) & 1u) != 0;  // CPUID.(EAX=7, ECX=0):EBX.SHA
  }();
  return has;
}
#endif

void Sha256::blocks(const uint8_t* p, size_t n) {
#if defined(__x86_64__)
  if (cpu_has_sha()) {
    sha256_blocks_ni(st_, p, n);
    return;
  }
#endif
  for (; n; n--, p += 64) block(p);
}

void Sha256::update(const void* data, size_t len) {
  const uint8_t* p = static_cast<const uint8_t*>(data);
  len_ += len;
  while (len) {
    if (n_ == 0 && len >= 64) {
      const size_t nb = len / 64;
      blocks(p, nb);
      p += 64 * nb;
      len -= 64 * nb;
      continue;
    }
    const size_t k = std::min(len, 64 - n_);
    std::memcpy(buf_ + n_, p, k);
    n_ += k;
    p += k;
    len -= k;
    if (n_ == 64) {
      block(buf_);
      n_ = 0;
    }
  }
}

void Sha256::finish(uint8_t out[32]) {
  const uint64_t bits = len_ * 8;
  buf_[n_++] = 0x80;
  if (n_ > 56) {
    std::memset(buf_ + n_, 0, 64 - n_);
    block(buf_);
    n_ = 0;
  }
  std::memset(buf_ + n_, 0, 56 - n_);
  for (int i = 0; i < 8; i++) buf_[56 + i] = (uint8_t)(bits >> (56 - 8 * i));
  block(buf_);
  for (int i = 0; i < 8; i++)
    for (int k = 0; k < 4; k++) out[4 * i + k] = (uint8_t)(st_[i] >> (24 - 8 * k));
}

// ---- range coder (range.rs) ---------------------------------------------------
static constexpr uint64_t kTop = 1ull << 56, kBottom = 1ull << 48;

static det_status validate_range(uint64_t cum, uint64_t freq, uint64_t total) {
  const uint64_t end = cum + freq;
  if (end < cum || freq == 0 || total == 0 || total >= (1ull << 31) || end > total)
    return DET_ERR_RANGE_INVALID_FREQUENCY;
  return DET_OK;
}

// normalize_step (range.rs:169-178)
static bool renorm_needed(uint64_t low, uint64_t* range) {
  if ((low ^ (low + *range)) < kTop) return true;
  if (*range < kBottom) {
    *range = (0 - low) & (kBottom - 1);
    return true;
  }
  return false;
}

det_status RangeEncoder::encode(uint64_t cum, uint64_t freq, uint64_t total) {
  const det_status st = validate_range(cum, freq, total);
  if (st) return st;
  range_ /= total;
  low_ += range_ * cum;
  range_ *= freq;
  while (renorm_needed(low_, &range_)) {
    out_.push_back((uint8_t)(low_ >> 56));
    low_ <<= 8;
    range_ <<= 8;
  }
  return DET_OK;
}

std::vector<uint8_t> RangeEncoder::finish() {
  for (int i = 0; i < 8; i++) {
    out_.push_back((uint8_t)(low_ >> 56));
    low_ <<= 8;
  }
  return std::move(out_);
}

det_status RangeDecoder::next_byte(uint8_t* b) {
  if (pos_ >= len_) return DET_ERR_RANGE_UNEXPECTED_EOF;
  *b = in_[pos_++];
  return DET_OK;
}

det_status RangeDecoder::init(const uint8_t* data, size_t len) {
  in_ = data;
  len_ = len;
  pos_ = 0;
  low_ = code_ = 0;
  range_ = ~0ull;
  pending_ = false;
  for (int i = 0; i < 8; i++) {
    uint8_t b;
    const det_status st = next_byte(&b);
    if (st) return st;
    code_ = (code_ << 8) | b;
  }
  return DET_OK;
}

det_status RangeDecoder::decode_freq(uint64_t total, uint64_t* value) {
  if (pending_ || total == 0 || total >= (1ull << 31)) return DET_ERR_RANGE_INVALID_FREQUENCY;
  const uint64_t r = range_ / total;
  if (r == 0) return DET_ERR_RANGE_INVALID_FREQUENCY;
  const uint64_t v = (code_ - low_) / r;
  if (v >= total) return DET_ERR_RANGE_INVALID_FREQUENCY;
  pending_ = true;
  pend_range_ = r;
  pend_total_ = total;
  *value = v;
  return DET_OK;
}

det_status RangeDecoder::advance(uint64_t cum, uint64_t freq, uint64_t total) {
  det_status st = validate_range(cum, freq, total);
  if (st) return st;
  if (!pending_ || pend_total_ != total) return DET_ERR_RANGE_INVALID_FREQUENCY;
  pending_ = false;
  range_ = pend_range_;
  low_ += range_ * cum;
  range_ *= freq;
  while (renorm_needed(low_, &range_)) {
    uint8_t b;
    if ((st = next_byte(&b))) return st;
    code_ = (code_ << 8) | b;
    low_ <<= 8;
    range_ <<= 8;
  }
  return DET_OK;
}

// ---- GGUF -----------------------------------------------------------------------
namespace {
struct Cursor {
  const uint8_t* p;
  size_t len, pos = 0;
  int take(size_t n, const uint8_t** out) {
    if (n > len - pos) return GG_TRUNCATED;
    *out = p + pos;
    pos += n;
    return GG_OK;
  }
  template <typename U>
  int le(U* v) {
    const uint8_t* b;
    if (int e = take(sizeof(U), &b)) return e;
    U x = 0;
    for (int i = (int)sizeof(U) - 1; i >= 0; i--) x = (U)((x << 8) | (U)b[i]);
    *v = x;
    return GG_OK;
  }
  int need(uint64_t n, size_t each) {
    if (each && n > (uint64_t)((len - pos) / each)) return GG_TRUNCATED;
    return GG_OK;
  }
};

// str::from_utf8 validity
bool valid_utf8(const uint8_t* s, size_t n) {
  for (size_t i = 0; i < n;) {
    const uint8_t c = s[i];
    if (c < 0x80) { i++; continue; }
    int k;
    uint32_t cp;
    if (c >= 0xc2 && c <= 0xdf) { k = 1; cp = c & 0x1f; }
    else if (c >= 0xe0 && c <= 0xef) { k = 2; cp = c & 0x0f; }
    else if (c >= 0xf0 && c <= 0xf4) { k = 3; cp = c & 0x07; }
    else return false;
    if (i + k >= n) return false;
    for (int j = 1; j <= k; j++) {
      if ((s[i + j] & 0xc0) != 0x80) return false;
      cp = (cp << 6) | (s[i + j] & 0x3f);
    }
    if (k == 2 && (cp < 0x800 || (cp >= 0xd800 && cp <= 0xdfff))) return false;
    if (k == 3 && (cp < 0x10000 || cp > 0x10ffff)) return false;
    i += (size_t)k + 1;
  }
  return true;
}

int read_string(Cursor& c, std::string* out) {
  uint64_t n;
  if (int e = c.le(&n)) return e;
  const uint8_t* b;
  if (n > c.len) return GG_TRUNCATED;
  if (int e = c.take((size_t)n, &b)) return e;
  if (!valid_utf8(b, (size_t)n)) return GG_INVALID_UTF8;
  out->assign(reinterpret_cast<const char*>(b), (size_t)n);
  return GG_OK;
}

int elem_bytes(uint32_t t, size_t* n) {
  switch (t) {
    case GV_U8: case GV_I8: case GV_BOOL: *n = 1; return GG_OK;
    case GV_U16: case GV_I16: *n = 2; return GG_OK;
    case GV_U32: case GV_I32: case GV_F32: *n = 4; return GG_OK;
    case GV_STRING: case GV_U64: case GV_I64: case GV_F64: *n = 8; return GG_OK;
    default: return GG_UNSUPPORTED_VALUE_TYPE;
  }
}

int read_value(Cursor& c, GgufValue* v) {
  if (int e = c.le(&v->type)) return e;
  switch (v->type) {
    case GV_U8: case GV_I8: { uint8_t x = 0; int e = c.le(&x); v->bits = x; return e; }
    case GV_U16: case GV_I16: { uint16_t x = 0; int e = c.le(&x); v->bits = x; return e; }
    case GV_U32: case GV_I32: { uint32_t x = 0; int e = c.le(&x); v->bits = x; return e; }
    case GV_F32: {
      uint32_t x = 0;
      int e = c.le(&x);
      float f;
      std::memcpy(&f, &x, 4);
      v->bits = x;
      v->real = f;
      return e;
    }
    case GV_BOOL: {
      uint8_t x;
      if (int e = c.le(&x)) return e;
      if (x > 1) return GG_INVALID_BOOL;
      v->bits = x;
      return GG_OK;
    }
    case GV_STRING: return read_string(c, &v->str);
    case GV_U64: case GV_I64: return c.le(&v->bits);
    case GV_F64: {
      int e = c.le(&v->bits);
      std::memcpy(&v->real, &v->bits, 8);
      return e;
    }
    case GV_ARRAY: {
      if (int e = c.le(&v->elem_type)) return e;
      if (int e = c.le(&v->count)) return e;
      size_t each;
      if (int e = elem_bytes(v->elem_type, &each)) return e;
      if (int e = c.need(v->count, each)) return e;
      if (v->elem_type == GV_STRING) {
        v->strs.resize((size_t)v->count);
        for (auto& s : v->strs)
          if (int e = read_string(c, &s)) return e;
        return GG_OK;
      }
      const uint8_t* b;
      if (int e = c.take((size_t)v->count * each, &b)) return e;
      if (v->elem_type == GV_BOOL)
        for (uint64_t i = 0; i < v->count; i++)
          if (b[i] > 1) return GG_INVALID_BOOL;
      v->raw = b;
      return GG_OK;
    }
    default: return GG_UNSUPPORTED_VALUE_TYPE;
  }
}
}  // namespace

int Gguf::type_size(uint32_t t, uint64_t* bytes, uint64_t* block) {
  static const struct { uint32_t t; uint64_t b, k; } tab[] = {
      {0, 4, 1}, {1, 2, 1}, {2, 18, 32}, {3, 20, 32}, {6, 22, 32}, {7, 24, 32}, {8, 34, 32},
      {9, 40, 32}, {10, 84, 256}, {11, 110, 256}, {12, 144, 256}, {13, 176, 256}, {14, 210, 256}, {15, 292, 256}};
  for (const auto& e : tab)
    if (e.t == t) {
      *bytes = e.b;
      *block = e.k;
      return GG_OK;
    }
  return GG_UNSUPPORTED_TENSOR_TYPE;
}

int Gguf::element_count(const GgufTensor& t, uint64_t* n) {
  if (t.dims.empty()) return GG_INVALID_TENSOR_SHAPE;
  uint64_t c = 1;
  for (uint64_t d : t.dims) {
    if (d == 0 || c > ~0ull / d) return GG_INVALID_TENSOR_SHAPE;
    c *= d;
  }
  *n = c;
  return GG_OK;
}

static int encoded_len(const GgufTensor& t, uint64_t* len) {
  uint64_t n, tb, bk;
  if (int e = Gguf::element_count(t, &n)) return e;
  if (Gguf::type_size(t.type, &tb, &bk)) return GG_UNSUPPORTED_TENSOR_TYPE;
  if (n % bk || n / bk > ~0ull / tb) return GG_INVALID_TENSOR_SHAPE;
  *len = n / bk * tb;
  return GG_OK;
}

// parse_inner (det-gguf lib.rs:164-228) with validate_tensor_data_layout
int Gguf::parse(const uint8_t* bytes, size_t len) {
  bytes_ = bytes;
  len_ = len;
  Cursor c{bytes, len};
  const uint8_t* magic;
  if (int e = c.take(4, &magic)) return e;
  if (std::memcmp(magic, "GGUF", 4) != 0) return GG_BAD_MAGIC;
  uint32_t version;
  if (int e = c.le(&version)) return e;
  if (version != 2 && version != 3) return GG_UNSUPPORTED_VERSION;
  uint64_t n_tensors, n_kv;
  if (int e = c.le(&n_tensors)) return e;
  if (int e = c.le(&n_kv)) return e;
  if (int e = c.need(n_kv, 12)) return e;
  kv.reserve((size_t)n_kv);
  for (uint64_t i = 0; i < n_kv; i++) {
    std::string key;
    if (int e = read_string(c, &key)) return e;
    GgufValue v;
    if (int e = read_value(c, &v)) return e;
    if (find(key)) return GG_DUPLICATE_METADATA_KEY;
    kv.emplace_back(std::move(key), std::move(v));
  }
  if (int e = c.need(n_tensors, 24)) return e;
  tensors.reserve((size_t)n_tensors);
  for (uint64_t i = 0; i < n_tensors; i++) {
    GgufTensor t;
    if (int e = read_string(c, &t.name)) return e;
    uint32_t nd;
    if (int e = c.le(&nd)) return e;
    if (int e = c.need(nd, 8)) return e;
    t.dims.resize(nd);
    for (auto& d : t.dims)
      if (int e = c.le(&d)) return e;
    if (int e = c.le(&t.type)) return e;
    if (int e = c.le(&t.offset)) return e;
    for (const auto& o : tensors)
      if (o.name == t.name) return GG_DUPLICATE_TENSOR_NAME;
    tensors.push_back(std::move(t));
  }
  data_offset = (c.pos + 31) & ~(size_t)31;
  if (data_offset > len) return GG_TRUNCATED;
  std::vector<std::pair<uint64_t, uint64_t>> ranges;
  for (const auto& t : tensors) {
    uint64_t el;
    if (int e = encoded_len(t, &el)) return e;
    const uint64_t s = data_offset + t.offset;
    if (s < t.offset || s + el < s) return GG_INVALID_TENSOR_OFFSET;
    if (s + el > len) return GG_TRUNCATED;
    ranges.emplace_back(s, s + el);
  }
  std::sort(ranges.begin(), ranges.end());
  for (size_t i = 1; i < ranges.size(); i++)
    if (ranges[i - 1].second > ranges[i].first) return GG_INVALID_TENSOR_OFFSET;
  return GG_OK;
}

const GgufValue* Gguf::find(const std::string& key) const {
  for (const auto& e : kv)
    if (e.first == key) return &e.second;
  return nullptr;
}

int Gguf::get_u32(const std::string& key, uint32_t* out) const {
  const GgufValue* v = find(key);
  if (!v) return GG_METADATA_NOT_FOUND;
  if (v->type == GV_U32) { *out = (uint32_t)v->bits; return GG_OK; }
  if (v->type == GV_U64 && v->bits <= 0xffffffffull) { *out = (uint32_t)v->bits; return GG_OK; }
  return GG_METADATA_TYPE_MISMATCH;
}

int Gguf::get_f32(const std::string& key, float* out) const {
  const GgufValue* v = find(key);
  if (!v) return GG_METADATA_NOT_FOUND;
  if (v->type == GV_F32 || v->type == GV_F64) { *out = (float)v->real; return GG_OK; }
  return GG_METADATA_TYPE_MISMATCH;
}

int Gguf::tensor(const std::string& name, const GgufTensor** out) const {
  for (const auto& t : tensors)
    if (t.name == name) { *out = &t; return GG_OK; }
  return GG_TENSOR_NOT_FOUND;
}

int Gguf::tensor_bytes(const std::string& name, const uint8_t** data, size_t* len) const {
  const GgufTensor* t;
  if (int e = tensor(name, &t)) return e;
  uint64_t el;
  if (int e = encoded_len(*t, &el)) return e;
  *data = bytes_ + data_offset + t->offset;
  *len = (size_t)el;
  return GG_OK;
}

}  // namespace det
