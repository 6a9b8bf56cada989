/*
 * oracle/ref_codec.c -- the compress/decompress driver of the CPU oracle
 * (TEST INFRASTRUCTURE, see ref.h).
 *
 * Follows crates/det-cli/src/main.rs:433-855 (LoadedModel, windowed model
 * state, encode/decode loops, canonical re-encode) and crates/det-coder/src/
 * file.rs:1-90 (DTLZ header); the tokenizers are ref_token.c.
 */
#include <stdlib.h>

#include "ref.h"
#include "ref_coder.h"
#include "ref_internal.h"
#include "ref_model.h"
#include "ref_token.h"

#define BYTE_ESCAPES 256u
#define MAX_SYMBOLS (1u << 18)

/* ---- windowed model state: det-cli main.rs:632-778 ---------------------------- */
typedef struct {
    ref_state st;
    size_t window_start, context_len, n_ctx, symbols; /* uniform CDF size */
    int escapes;
} wstate;

/* next_window_start (det-cli main.rs:772-778) */
static size_t next_window_start(size_t pos, size_t ws, size_t n_ctx, size_t overlap) {
    size_t d = pos > ws ? pos - ws : 0;
    if (d >= n_ctx) return pos > overlap ? pos - overlap : 0;
    return ws;
}

/* exported for the rollover known-answer test (det-cli main.rs:1289-1304) */
size_t ref_next_window_start(size_t pos, size_t ws, size_t n_ctx, size_t overlap) {
    return next_window_start(pos, ws, n_ctx, overlap);
}

static int ws_init(wstate* w, const ref_model* m, size_t n_ctx, int escapes) {
    memset(w, 0, sizeof *w);
    int st = ref_state_init(&w->st, m, n_ctx);
    if (st) return st;
    w->n_ctx = n_ctx;
    w->escapes = escapes;
    w->symbols = m->vocab + (escapes ? BYTE_ESCAPES : 0);
    if (w->symbols > MAX_SYMBOLS) { ref_state_free(&w->st); return REF_ERR_CDF_TOO_MANY_SYMBOLS; }
    return REF_OK;
}

static int ws_advance(wstate* w, size_t token) {
    if (w->context_len >= w->n_ctx) return REF_ERR_WINDOW;
    int st = ref_forward_one(&w->st, token, w->context_len);
    if (st) return st;
    w->context_len++;
    return REF_OK;
}

static int ws_sync(wstate* w, const uint32_t* ctx, size_t pos, size_t overlap) {
    size_t ns = next_window_start(pos, w->window_start, w->n_ctx, overlap);
    if (ns == w->window_start) return REF_OK;
    ref_state_reset_cache(&w->st);
    w->window_start = ns;
    w->context_len = 0;
    for (size_t i = ns; i < pos; i++) {
        int st = ws_advance(w, ctx[i]);
        if (st) return st;
    }
    return REF_OK;
}

/* WindowedModelState::symbol_range (:703-722) */
static int ws_symbol_range(wstate* w, size_t symbol, ref_symbol_range* r) {
    if (w->context_len == 0) {
        if (symbol >= w->symbols) return REF_ERR_CDF_SYMBOL_OUT_OF_RANGE;
        r->cum = symbol;
        r->freq = 1;
        r->pad = 0;
        r->total = w->symbols;
        return REF_OK;
    }
    return ref_logits_to_symbol_range(w->st.logits, w->st.m->vocab, symbol, w->escapes, r);
}

/* WindowedModelState::decode_symbol (:724-751) */
static int ws_decode_symbol(wstate* w, rc_dec* d, uint32_t* symbol) {
    uint64_t value;
    int st;
    if (w->context_len == 0) {
        if ((st = rc_dec_decode_freq(d, w->symbols, &value))) return st;
        *symbol = (uint32_t)value;
        return rc_dec_advance(d, value, 1, w->symbols);
    }
    size_t V = w->st.m->vocab, tail = w->escapes ? BYTE_ESCAPES : 0;
    uint32_t* f = (uint32_t*)malloc(sizeof(uint32_t) * V);
    if (!f) return REF_ERR_ALLOC;
    uint64_t total;
    st = coder_decoder_freqs(w->st.logits, V, tail, f, &total);
    if (!st) st = rc_dec_decode_freq(d, total, &value);
    ref_symbol_range r;
    if (!st) st = decoder_lookup_freqs(f, V, tail, total, value, symbol, &r);
    free(f);
    if (st) return st;
    return rc_dec_advance(d, r.cum, r.freq, r.total);
}

/* validate_window (det-cli main.rs:810-826) */
static int validate_window(size_t n_ctx, size_t overlap, size_t model_ctx) {
    if (n_ctx == 0 || n_ctx > model_ctx || overlap >= n_ctx) return REF_ERR_WINDOW;
    return REF_OK;
}

/* encode_symbols_with_model (:523-552); when ranges != NULL the per-symbol
 * ranges are recorded too */
static int encode_symbols(const ref_model* m, const uint32_t* symbols, size_t n, size_t n_ctx, size_t overlap,
                          int escapes, rc_enc* enc, ref_symbol_range* ranges) {
    int st = validate_window(n_ctx, overlap, m->cfg.ctx);
    if (st) return st;
    wstate w;
    if ((st = ws_init(&w, m, n_ctx, escapes))) return st;
    uint32_t* ctx = (uint32_t*)malloc(sizeof(uint32_t) * (n ? n : 1));
    if (!ctx) { ref_state_free(&w.st); return REF_ERR_ALLOC; }
    size_t clen = 0, V = m->vocab;
    for (size_t i = 0; i < n && !st; i++) {
        uint32_t s = symbols[i];
        if ((st = ws_sync(&w, ctx, clen, overlap))) break;
        ref_symbol_range r;
        if ((st = ws_symbol_range(&w, s, &r))) break;
        if (ranges) ranges[i] = r;
        if (enc && (st = rc_enc_encode(enc, r.cum, r.freq, r.total))) break;
        if (escapes && s >= V) continue;
        if (s >= V) { st = REF_ERR_CDF_SYMBOL_OUT_OF_RANGE; break; }
        ctx[clen++] = s;
        st = ws_advance(&w, s);
    }
    free(ctx);
    ref_state_free(&w.st);
    return st;
}

int ref_encode_symbols(const ref_model* m, const uint32_t* symbols, size_t n, uint32_t n_ctx, uint32_t overlap,
                       int byte_escapes, uint8_t** out, size_t* out_len) {
    rc_enc e;
    rc_enc_init(&e);
    int st = encode_symbols(m, symbols, n, n_ctx, overlap, byte_escapes, &e, NULL);
    if (!st) st = rc_enc_finish(&e);
    if (st) { free(e.out); return st; }
    *out = e.out;
    *out_len = e.len;
    return REF_OK;
}

int ref_symbol_ranges_stream(const ref_model* m, const uint32_t* symbols, size_t n, uint32_t n_ctx,
                             uint32_t overlap, int byte_escapes, ref_symbol_range* out) {
    return encode_symbols(m, symbols, n, n_ctx, overlap, byte_escapes, NULL, out);
}

/* ---- LoadedModel::load (det-cli main.rs:933-1008) ---------------------------- */
typedef struct {
    uint8_t sha[32];
    ref_model* model;
    ref_tok tok;
} loaded_t;

static int load(const uint8_t* bytes, size_t len, loaded_t* L) {
    memset(L, 0, sizeof *L);
    ref_sha256(bytes, len, L->sha);
    gg_file g;
    if (gg_parse(bytes, len, &g)) return REF_ERR_GGUF;
    int st = ref_tok_from_gguf(&g, &L->tok);
    if (!st) st = ref_model_load_gguf(&g, bytes, &L->model);
    gg_free(&g);
    if (st) { ref_tok_free(&L->tok); return st; }
    if (L->tok.vocab != L->model->vocab) st = REF_ERR_VOCAB_MISMATCH;
    else if (L->model->vocab + BYTE_ESCAPES > MAX_SYMBOLS) st = REF_ERR_CDF_TOO_MANY_SYMBOLS;
    if (st) {
        ref_model_free(L->model);
        ref_tok_free(&L->tok);
    }
    return st;
}

static void unload(loaded_t* L) {
    ref_model_free(L->model);
    ref_tok_free(&L->tok);
}

static void put_le(uint8_t* p, uint64_t v, int n) {
    for (int i = 0; i < n; i++) p[i] = (uint8_t)(v >> (8 * i));
}
static uint64_t get_le(const uint8_t* p, int n) {
    uint64_t v = 0;
    for (int i = n - 1; i >= 0; i--) v = (v << 8) | p[i];
    return v;
}

/* compress (det-cli main.rs:433-463) */
int ref_compress(const uint8_t* model_bytes, size_t model_len, const uint8_t* input, size_t in_len, uint32_t n_ctx_opt,
                 uint8_t** out, size_t* out_len) {
    loaded_t L;
    int st = load(model_bytes, model_len, &L);
    if (st) return st;
    uint32_t* sym = NULL;
    size_t nsym = 0;
    if ((st = ref_tok_codec_symbols(&L.tok, input, in_len, &sym, &nsym))) { unload(&L); return st; }
    size_t n_ctx = n_ctx_opt ? n_ctx_opt : L.model->cfg.ctx;
    size_t overlap = n_ctx / 4;
    rc_enc e;
    rc_enc_init(&e);
    st = encode_symbols(L.model, sym, nsym, n_ctx, overlap, 1, &e, NULL);
    if (!st) st = rc_enc_finish(&e);
    free(sym);
    if (st) { free(e.out); unload(&L); return st; }
    /* DtlzHeader::encode (file.rs:28-38) */
    uint8_t* o = (uint8_t*)malloc(56 + e.len);
    if (!o) { free(e.out); unload(&L); return REF_ERR_ALLOC; }
    memcpy(o, "DTLZ", 4);
    put_le(o + 4, 1, 2);
    put_le(o + 6, 1, 2); /* FLAG_BYTE_ESCAPES */
    memcpy(o + 8, L.sha, 32);
    put_le(o + 40, n_ctx, 4);
    put_le(o + 44, overlap, 4);
    put_le(o + 48, in_len, 8);
    memcpy(o + 56, e.out, e.len);
    *out = o;
    *out_len = 56 + e.len;
    free(e.out);
    unload(&L);
    return REF_OK;
}

/* decompress (det-cli main.rs:465-511) with decode_bytes_with_model (:585-630) */
int ref_decompress(const uint8_t* model_bytes, size_t model_len, const uint8_t* dtlz, size_t dtlz_len, uint8_t** out,
                   size_t* out_len) {
    /* DtlzHeader::decode (file.rs:58-90) */
    if (dtlz_len < 56) return REF_ERR_FILE_TOO_SHORT;
    if (memcmp(dtlz, "DTLZ", 4) != 0) return REF_ERR_FILE_BAD_MAGIC;
    if (get_le(dtlz + 4, 2) != 1) return REF_ERR_FILE_UNSUPPORTED_VERSION;
    uint32_t flags = (uint32_t)get_le(dtlz + 6, 2);
    if (flags & ~1u) return REF_ERR_FILE_UNSUPPORTED_FLAGS;
    size_t n_ctx = (size_t)get_le(dtlz + 40, 4), overlap = (size_t)get_le(dtlz + 44, 4);
    uint64_t orig_len = get_le(dtlz + 48, 8);
    if (n_ctx == 0) return REF_ERR_FILE_INVALID_CONTEXT;
    if (overlap >= n_ctx) return REF_ERR_FILE_INVALID_OVERLAP;
    const uint8_t* payload = dtlz + 56;
    size_t plen = dtlz_len - 56;
    loaded_t L;
    int st = load(model_bytes, model_len, &L);
    if (st) return st;
    if (memcmp(L.sha, dtlz + 8, 32) != 0) { unload(&L); return REF_ERR_MODEL_HASH_MISMATCH; }
    if ((st = validate_window(n_ctx, overlap, L.model->cfg.ctx))) { unload(&L); return st; }
    int escapes = (flags & 1) != 0;
    rc_dec d;
    if ((st = rc_dec_init(&d, payload, plen))) { unload(&L); return st; }
    wstate w;
    if ((st = ws_init(&w, L.model, n_ctx, escapes))) { unload(&L); return st; }
    /* the last symbol may run past orig_len by up to one token's bytes */
    size_t maxtok = 1;
    for (size_t i = 0; i < L.tok.vocab; i++)
        if (L.tok.tok_len[i] > (int64_t)maxtok) maxtok = (size_t)L.tok.tok_len[i];
    size_t cap = (size_t)orig_len + maxtok + 16;
    uint8_t* bytes = (uint8_t*)malloc(cap);
    uint32_t* ctx = (uint32_t*)malloc(sizeof(uint32_t) * (cap));
    uint32_t* syms = (uint32_t*)malloc(sizeof(uint32_t) * (cap));
    size_t nb = 0, clen = 0, ns = 0;
    if (!bytes || !ctx || !syms) st = REF_ERR_ALLOC;
    while (!st && nb < orig_len) {
        if ((st = ws_sync(&w, ctx, clen, overlap))) break;
        uint32_t s;
        if ((st = ws_decode_symbol(&w, &d, &s))) break;
        /* decode_codec_symbol (det-token lib.rs:182-196) / detokenize_bytes;
         * a symbol that yields no bytes is an error (main.rs:614-616) */
        uint8_t one;
        const uint8_t* piece;
        size_t plen_sym;
        if ((st = ref_tok_symbol_bytes(&L.tok, s, escapes, &one, &piece, &plen_sym))) break;
        if (plen_sym == 0) { st = REF_ERR_TOKENIZER; break; }
        memcpy(bytes + nb, piece, plen_sym);
        nb += plen_sym;
        syms[ns++] = s;
        if (escapes && s >= L.tok.vocab) continue;
        ctx[clen++] = s;
        st = ws_advance(&w, s);
    }
    ref_state_free(&w.st);
    free(ctx);
    if (!st) {
        rc_enc e;
        rc_enc_init(&e);
        st = encode_symbols(L.model, syms, ns, n_ctx, overlap, escapes, &e, NULL);
        if (!st) st = rc_enc_finish(&e);
        if (!st && (e.len != plen || memcmp(e.out, payload, plen) != 0)) st = REF_ERR_NONCANONICAL;
        free(e.out);
    }
    free(syms);
    unload(&L);
    if (st) { free(bytes); return st; }
    *out = bytes;
    *out_len = (size_t)orig_len;
    return REF_OK;
}

/* ---- tokenizer entry points for the tests: Tokenizer::from_gguf on the GGUF
 * metadata, then tokenize_bytes / codec_symbols / decode_codec_symbol ---- */
static int tok_load(const uint8_t* gguf, size_t len, ref_tok* t) {
    gg_file g;
    if (gg_parse(gguf, len, &g)) return REF_ERR_GGUF;
    const int st = ref_tok_from_gguf(&g, t);
    gg_free(&g);
    return st;
}

int ref_tokenizer_kind(const uint8_t* gguf, size_t len, int* kind) {
    ref_tok t;
    const int st = tok_load(gguf, len, &t);
    if (st) return st;
    *kind = t.kind;
    ref_tok_free(&t);
    return REF_OK;
}

int ref_tokenize(const uint8_t* gguf, size_t len, const uint8_t* in, size_t n, int codec, uint32_t** out,
                 size_t* out_n) {
    ref_tok t;
    int st = tok_load(gguf, len, &t);
    if (st) return st;
    st = codec ? ref_tok_codec_symbols(&t, in, n, out, out_n) : ref_tok_tokenize(&t, in, n, out, out_n);
    ref_tok_free(&t);
    return st;
}

int ref_detokenize(const uint8_t* gguf, size_t len, const uint32_t* syms, size_t n, int escapes, uint8_t** out,
                   size_t* out_n) {
    ref_tok t;
    int st = tok_load(gguf, len, &t);
    if (st) return st;
    size_t total = 0, cap = 64;
    uint8_t* o = (uint8_t*)malloc(cap);
    if (!o) st = REF_ERR_ALLOC;
    for (size_t i = 0; !st && i < n; i++) {
        uint8_t one;
        const uint8_t* p;
        size_t pl;
        if ((st = ref_tok_symbol_bytes(&t, syms[i], escapes, &one, &p, &pl))) break;
        while (total + pl > cap) {
            uint8_t* q = (uint8_t*)realloc(o, cap * 2);
            if (!q) { st = REF_ERR_ALLOC; break; }
            o = q;
            cap *= 2;
        }
        if (st) break;
        memcpy(o + total, p, pl);
        total += pl;
    }
    ref_tok_free(&t);
    if (st) { free(o); return st; }
    *out = o;
    *out_n = total;
    return REF_OK;
}
