/*
 * oracle/ref_coder.c -- det-coder restated in C (TEST INFRASTRUCTURE, see
 * ref.h): logits -> integer CDF (crates/det-coder/src/cdf.rs:52-425) and the
 * 64-bit range coder (crates/det-coder/src/range.rs:1-178).
 */
#include <math.h>
#include <stdlib.h>

#include "ref.h"
#include "ref_internal.h"
#include "ref_coder.h"

#define CDF_M 16777216.0f
#define MAX_SYMBOLS (1u << 18)
#define BYTE_ESCAPES 256u

/* max over finite logits (cdf.rs:74-83) and the exp fill (cdf.rs:281-300) */
static int exp_fill(const float* logits, size_t n, float* e) {
    float mx = -INFINITY;
    for (size_t i = 0; i < n; i++) {
        if (!isfinite_f(logits[i])) return REF_ERR_CDF_NONFINITE_LOGIT;
        if (logits[i] > mx) mx = logits[i];
    }
    for (size_t i = 0; i < n; i++) {
        float t = logits[i] - mx;
        e[i] = ref_expf(t > -88.0f ? t : -88.0f);
    }
    return REF_OK;
}

/* f_i = ((e_i / Z) * 2^24) as u32 + 1 (cdf.rs:85-93) */
static inline uint32_t freq_of(float e, float z) {
    float p = e / z;
    return f32_as_u32(p * CDF_M) + 1u;
}

/* cdf.rs:52-94 */
int ref_logits_to_cdf(const float* logits, size_t n, uint32_t* freq, uint64_t* cum, uint64_t* total) {
    if (n == 0) return REF_ERR_CDF_EMPTY;
    if (n > MAX_SYMBOLS) return REF_ERR_CDF_TOO_MANY_SYMBOLS;
    float* e = (float*)malloc(sizeof(float) * n);
    if (!e) return REF_ERR_ALLOC;
    int st = exp_fill(logits, n, e);
    if (st) { free(e); return st; }
    float z = ref_sum_f32(e, n);
    uint64_t t = 0;
    for (size_t i = 0; i < n; i++) {
        uint32_t f = freq_of(e[i], z);
        cum[i] = t;
        freq[i] = f;
        t += f;
    }
    free(e);
    if (t >= (1ull << 31)) return REF_ERR_CDF_TOTAL_TOO_LARGE;
    *total = t;
    return REF_OK;
}

/* cdf.rs:138-199 */
int ref_logits_to_symbol_range(const float* logits, size_t n, size_t symbol, int byte_escapes,
                               ref_symbol_range* out) {
    size_t tail = byte_escapes ? BYTE_ESCAPES : 0;
    if (n == 0) return REF_ERR_CDF_EMPTY;
    if (n + tail > MAX_SYMBOLS) return REF_ERR_CDF_TOO_MANY_SYMBOLS;
    if (symbol >= n + tail) return REF_ERR_CDF_SYMBOL_OUT_OF_RANGE;
    float* e = (float*)malloc(sizeof(float) * n);
    if (!e) return REF_ERR_ALLOC;
    int st = exp_fill(logits, n, e);
    if (st) { free(e); return st; }
    float z = ref_sum_f32(e, n);
    uint64_t total = 0, cum = 0;
    uint32_t fr = 0;
    for (size_t i = 0; i < n; i++) {
        uint32_t f = freq_of(e[i], z);
        if (i == symbol) { cum = total; fr = f; }
        total += f;
    }
    free(e);
    if (symbol >= n) { cum = total + (symbol - n); fr = 1; }
    total += tail;
    if (total >= (1ull << 31)) return REF_ERR_CDF_TOTAL_TOO_LARGE;
    out->cum = cum;
    out->freq = fr;
    out->pad = 0;
    out->total = total;
    return REF_OK;
}

/* cdf.rs:201-245: frequencies + total */
int coder_decoder_freqs(const float* logits, size_t n, size_t tail, uint32_t* freq, uint64_t* total) {
    if (n == 0) return REF_ERR_CDF_EMPTY;
    if (n + tail > MAX_SYMBOLS) return REF_ERR_CDF_TOO_MANY_SYMBOLS;
    float* e = (float*)malloc(sizeof(float) * n);
    if (!e) return REF_ERR_ALLOC;
    int st = exp_fill(logits, n, e);
    if (st) { free(e); return st; }
    float z = ref_sum_f32(e, n);
    uint64_t t = 0;
    for (size_t i = 0; i < n; i++) {
        freq[i] = freq_of(e[i], z);
        t += freq[i];
    }
    free(e);
    t += tail;
    if (t >= (1ull << 31)) return REF_ERR_CDF_TOTAL_TOO_LARGE;
    *total = t;
    return REF_OK;
}

/* logits_to_decoder_distribution_impl + DecoderDistribution::total (det-coder cdf.rs:201-245, 388) */
int ref_decoder_total(const float* logits, size_t n, int byte_escapes, uint64_t* total) {
    uint32_t* f = (uint32_t*)malloc(sizeof(uint32_t) * (n ? n : 1));
    if (!f) return REF_ERR_ALLOC;
    int st = coder_decoder_freqs(logits, n, byte_escapes ? BYTE_ESCAPES : 0, f, total);
    free(f);
    return st;
}

/* DecoderDistribution::symbol_range (cdf.rs:392-425): linear scan */
int decoder_lookup_freqs(const uint32_t* freq, size_t n, size_t tail, uint64_t total, uint64_t value,
                         uint32_t* symbol, ref_symbol_range* out) {
    if (value >= total) return REF_ERR_DECODE;
    uint64_t cum = 0;
    for (size_t i = 0; i < n; i++) {
        uint64_t next = cum + freq[i];
        if (value < next) {
            *symbol = (uint32_t)i;
            out->cum = cum;
            out->freq = freq[i];
            out->total = total;
            out->pad = 0;
            return REF_OK;
        }
        cum = next;
    }
    uint64_t off = value - cum;
    if (off < tail) {
        *symbol = (uint32_t)(n + off);
        out->cum = value;
        out->freq = 1;
        out->total = total;
        out->pad = 0;
        return REF_OK;
    }
    return REF_ERR_DECODE;
}

int ref_decoder_lookup(const float* logits, size_t n, int byte_escapes, uint64_t value, uint32_t* symbol,
                       ref_symbol_range* out) {
    size_t tail = byte_escapes ? BYTE_ESCAPES : 0;
    uint32_t* f = (uint32_t*)malloc(sizeof(uint32_t) * (n ? n : 1));
    if (!f) return REF_ERR_ALLOC;
    uint64_t total;
    int st = coder_decoder_freqs(logits, n, tail, f, &total);
    if (!st) st = decoder_lookup_freqs(f, n, tail, total, value, symbol, out);
    free(f);
    return st;
}

/* ---- range coder: range.rs:11-178 -------------------------------------------- */
#define RC_TOP (1ull << 56)
#define RC_BOTTOM (1ull << 48)

static int rc_validate(uint64_t cum, uint64_t freq, uint64_t total) {
    uint64_t end = cum + freq;
    if (end < cum) return REF_ERR_RANGE_INVALID_FREQUENCY;
    if (freq == 0 || total == 0 || total >= (1ull << 31) || end > total) return REF_ERR_RANGE_INVALID_FREQUENCY;
    return REF_OK;
}

/* normalize_step (range.rs:169-178) */
static int rc_norm_step(uint64_t low, uint64_t* range) {
    if ((low ^ (low + *range)) < RC_TOP) return 1;
    if (*range < RC_BOTTOM) {
        *range = (0 - low) & (RC_BOTTOM - 1);
        return 1;
    }
    return 0;
}

int rc_enc_push(rc_enc* e, uint8_t b) {
    if (e->len == e->cap) {
        size_t nc = e->cap ? e->cap * 2 : 256;
        uint8_t* p = (uint8_t*)realloc(e->out, nc);
        if (!p) return REF_ERR_ALLOC;
        e->out = p;
        e->cap = nc;
    }
    e->out[e->len++] = b;
    return REF_OK;
}

void rc_enc_init(rc_enc* e) {
    e->low = 0;
    e->range = UINT64_MAX;
    e->out = NULL;
    e->len = e->cap = 0;
}

/* RangeEncoder::encode (range.rs:58-65) */
int rc_enc_encode(rc_enc* e, uint64_t cum, uint64_t freq, uint64_t total) {
    int st = rc_validate(cum, freq, total);
    if (st) return st;
    e->range /= total;
    e->low += e->range * cum;
    e->range *= freq;
    while (rc_norm_step(e->low, &e->range)) {
        if ((st = rc_enc_push(e, (uint8_t)(e->low >> 56)))) return st;
        e->low <<= 8;
        e->range <<= 8;
    }
    return REF_OK;
}

/* RangeEncoder::finish (range.rs:67-73) */
int rc_enc_finish(rc_enc* e) {
    for (int i = 0; i < 8; i++) {
        int st = rc_enc_push(e, (uint8_t)(e->low >> 56));
        if (st) return st;
        e->low <<= 8;
    }
    return REF_OK;
}

/* RangeDecoder::new (range.rs:96-108) */
int rc_dec_init(rc_dec* d, const uint8_t* in, size_t len) {
    d->low = 0;
    d->code = 0;
    d->range = UINT64_MAX;
    d->pending = 0;
    d->in = in;
    d->len = len;
    d->pos = 0;
    for (int i = 0; i < 8; i++) {
        if (d->pos >= d->len) return REF_ERR_RANGE_UNEXPECTED_EOF;
        d->code = (d->code << 8) | d->in[d->pos++];
    }
    return REF_OK;
}

/* RangeDecoder::decode_freq (range.rs:110-127) */
int rc_dec_decode_freq(rc_dec* d, uint64_t total, uint64_t* value) {
    if (d->pending) return REF_ERR_RANGE_INVALID_FREQUENCY;
    if (total == 0 || total >= (1ull << 31)) return REF_ERR_RANGE_INVALID_FREQUENCY;
    uint64_t r = d->range / total;
    if (r == 0) return REF_ERR_RANGE_INVALID_FREQUENCY;
    uint64_t v = (d->code - d->low) / r;
    if (v >= total) return REF_ERR_RANGE_INVALID_FREQUENCY;
    d->pending = 1;
    d->pend_range = r;
    d->pend_total = total;
    *value = v;
    return REF_OK;
}

/* RangeDecoder::advance (range.rs:129-151) */
int rc_dec_advance(rc_dec* d, uint64_t cum, uint64_t freq, uint64_t total) {
    int st = rc_validate(cum, freq, total);
    if (st) return st;
    if (!d->pending) return REF_ERR_RANGE_INVALID_FREQUENCY;
    if (d->pend_total != total) return REF_ERR_RANGE_INVALID_FREQUENCY;
    d->pending = 0;
    d->range = d->pend_range;
    d->low += d->range * cum;
    d->range *= freq;
    while (rc_norm_step(d->low, &d->range)) {
        if (d->pos >= d->len) return REF_ERR_RANGE_UNEXPECTED_EOF;
        d->code = (d->code << 8) | d->in[d->pos++];
        d->low <<= 8;
        d->range <<= 8;
    }
    return REF_OK;
}

int ref_range_encode(const uint64_t* cum, const uint64_t* freq, const uint64_t* total, size_t n, uint8_t* out,
                     size_t cap, size_t* out_len) {
    rc_enc e;
    rc_enc_init(&e);
    int st = REF_OK;
    for (size_t i = 0; i < n && !st; i++) st = rc_enc_encode(&e, cum[i], freq[i], total[i]);
    if (!st) st = rc_enc_finish(&e);
    if (!st) {
        *out_len = e.len;
        if (e.len <= cap) memcpy(out, e.out, e.len);
    }
    free(e.out);
    return st;
}
