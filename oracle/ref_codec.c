/*
 * oracle/ref_codec.c -- the compress/decompress driver of the CPU oracle
 * (TEST INFRASTRUCTURE, see ref.h).
 *
 * Follows crates/det-cli/src/main.rs:433-855 (LoadedModel, windowed model
 * state, encode/decode loops, canonical re-encode), crates/det-token/src/
 * lib.rs:85-326, 619-850 (tokenizer selection, byte-fallback tokenizer,
 * codec symbols) and crates/det-coder/src/file.rs:1-90 (DTLZ header).
 * Only the byte-fallback tokenizer is restated; GGUFs that select the
 * byte-BPE or SentencePiece tokenizers are rejected with REF_ERR_TOKENIZER.
 */
#include <stdlib.h>

#include "ref.h"
#include "ref_coder.h"
#include "ref_internal.h"
#include "ref_model.h"

#define BYTE_ESCAPES 256u
#define MAX_SYMBOLS (1u << 18)

/* ---- byte-fallback tokenizer ------------------------------------------------ */
typedef struct {
    int32_t byte_to_token[256]; /* -1 if absent or not emittable */
    int16_t* token_to_byte;      /* -1 if the token is not a byte-fallback token */
    size_t vocab;
} ref_tokenizer;

/* canonical_byte_fallback_token (det-token lib.rs:841-848): "<0xHH>" where
 * HH parses like u8::from_str_radix(_, 16) (an optional leading '+'). */
static int byte_fallback_of(const gg_str* s) {
    if (s->len != 6) return -1;
    const uint8_t* p = s->ptr;
    if (p[0] != '<' || p[1] != '0' || p[2] != 'x' || p[5] != '>') return -1;
    int v = 0;
    int start = 3;
    if (p[3] == '+') start = 4;
    if (start == 4 && p[4] == '+') return -1;
    for (int i = start; i < 5; i++) {
        int c = p[i], d;
        if (c >= '0' && c <= '9') d = c - '0';
        else if (c >= 'a' && c <= 'f') d = c - 'a' + 10;
        else if (c >= 'A' && c <= 'F') d = c - 'A' + 10;
        else return -1;
        v = v * 16 + d;
    }
    return v;
}

/* token_type_is_emittable (det-token lib.rs:704-710) */
static int token_type_emittable(int64_t t, int* ok) {
    *ok = 1;
    if (t == 1 || t == 4 || t == 6) return 1;
    if (t == 2 || t == 3 || t == 5) return 0;
    *ok = 0;
    return 0;
}

/* Tokenizer::from_gguf (det-token lib.rs:86-132) restricted to the
 * byte-fallback branch, and ByteFallbackTokenizer::from_tokens_and_emit_mask
 * (:256-296). */
static int tokenizer_from_gguf(const gg_file* g, ref_tokenizer* t) {
    memset(t, 0, sizeof *t);
    const gg_kv* toks = gg_find(g, "tokenizer.ggml.tokens");
    if (!toks || toks->type != GV_ARRAY || toks->elem_type != GV_STRING) return REF_ERR_TOKENIZER;
    size_t V = (size_t)toks->count;
    const gg_kv* tt = gg_find(g, "tokenizer.ggml.token_type");
    if (tt) {
        if (tt->type != GV_ARRAY || (tt->elem_type != GV_I32 && tt->elem_type != GV_U32)) return REF_ERR_TOKENIZER;
        if (tt->count != V) return REF_ERR_TOKENIZER;
    }
    const gg_kv* merges = gg_find(g, "tokenizer.ggml.merges");
    if (merges && (merges->type != GV_ARRAY || merges->elem_type != GV_STRING)) return REF_ERR_TOKENIZER;
    const gg_kv* model = gg_find(g, "tokenizer.ggml.model");
    if (model && model->type != GV_STRING) return REF_ERR_TOKENIZER;
    const gg_kv* scores = gg_find(g, "tokenizer.ggml.scores");
    if (scores && (scores->type != GV_ARRAY || scores->elem_type != GV_F32)) return REF_ERR_TOKENIZER;
    /* byte-BPE / SentencePiece selection: not restated (out of scope) */
    if (model || (merges && merges->count > 0) || scores) return REF_ERR_TOKENIZER;
    int* emit = NULL;
    if (tt) {
        emit = (int*)malloc(sizeof(int) * (V ? V : 1));
        if (!emit) return REF_ERR_ALLOC;
        for (size_t i = 0; i < V; i++) {
            uint32_t raw = (uint32_t)tt->arr[4 * i] | ((uint32_t)tt->arr[4 * i + 1] << 8) |
                           ((uint32_t)tt->arr[4 * i + 2] << 16) | ((uint32_t)tt->arr[4 * i + 3] << 24);
            int64_t v = tt->elem_type == GV_I32 ? (int64_t)(int32_t)raw : (int64_t)raw;
            int ok;
            emit[i] = token_type_emittable(v, &ok);
            if (!ok) { free(emit); return REF_ERR_TOKENIZER; }
        }
    }
    int seen[256];
    for (int b = 0; b < 256; b++) { seen[b] = 0; t->byte_to_token[b] = -1; }
    t->vocab = V;
    t->token_to_byte = (int16_t*)malloc(sizeof(int16_t) * (V ? V : 1));
    if (!t->token_to_byte) { free(emit); return REF_ERR_ALLOC; }
    for (size_t i = 0; i < V; i++) t->token_to_byte[i] = -1;
    for (size_t i = 0; i < V; i++) {
        int b = byte_fallback_of(&toks->strs[i]);
        if (b < 0) continue;
        if (seen[b]) { free(emit); free(t->token_to_byte); t->token_to_byte = NULL; return REF_ERR_TOKENIZER; }
        seen[b] = 1;
        t->token_to_byte[i] = (int16_t)b;
        if (!emit || emit[i]) t->byte_to_token[b] = (int32_t)i;
    }
    free(emit);
    for (int b = 0; b < 256; b++)
        if (!seen[b]) { free(t->token_to_byte); t->token_to_byte = NULL; return REF_ERR_TOKENIZER; }
    return REF_OK;
}

/* Tokenizer::codec_symbols (det-token lib.rs:150-180) for byte fallback */
static void codec_symbols(const ref_tokenizer* t, const uint8_t* in, size_t n, size_t V, uint32_t* out) {
    for (size_t i = 0; i < n; i++) {
        int32_t tok = t->byte_to_token[in[i]];
        out[i] = tok >= 0 ? (uint32_t)tok : (uint32_t)(V + in[i]);
    }
}

/* ---- windowed model state: det-cli main.rs:632-778 ---------------------------- */
typedef struct {
    ref_state st;
    size_t window_start, context_len, n_ctx, symbols; /* uniform CDF size */
    int escapes;
} wstate;

static size_t next_window_start(size_t pos, size_t ws, size_t n_ctx, size_t overlap) {
    size_t d = pos > ws ? pos - ws : 0;
    if (d >= n_ctx) return pos > overlap ? pos - overlap : 0;
    return ws;
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
    ref_tokenizer tok;
} loaded_t;

static int load(const uint8_t* bytes, size_t len, loaded_t* L) {
    memset(L, 0, sizeof *L);
    ref_sha256(bytes, len, L->sha);
    gg_file g;
    if (gg_parse(bytes, len, &g)) return REF_ERR_GGUF;
    int st = tokenizer_from_gguf(&g, &L->tok);
    if (!st) st = ref_model_load_gguf(&g, bytes, &L->model);
    gg_free(&g);
    if (st) { free(L->tok.token_to_byte); return st; }
    if (L->tok.vocab != L->model->vocab) st = REF_ERR_VOCAB_MISMATCH;
    else if (L->model->vocab + BYTE_ESCAPES > MAX_SYMBOLS) st = REF_ERR_CDF_TOO_MANY_SYMBOLS;
    if (st) {
        ref_model_free(L->model);
        free(L->tok.token_to_byte);
    }
    return st;
}

static void unload(loaded_t* L) {
    ref_model_free(L->model);
    free(L->tok.token_to_byte);
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
    size_t V = L.model->vocab;
    uint32_t* sym = (uint32_t*)malloc(sizeof(uint32_t) * (in_len ? in_len : 1));
    if (!sym) { unload(&L); return REF_ERR_ALLOC; }
    codec_symbols(&L.tok, input, in_len, V, sym);
    size_t n_ctx = n_ctx_opt ? n_ctx_opt : L.model->cfg.ctx;
    size_t overlap = n_ctx / 4;
    rc_enc e;
    rc_enc_init(&e);
    st = encode_symbols(L.model, sym, in_len, n_ctx, overlap, 1, &e, NULL);
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
    size_t V = L.model->vocab;
    rc_dec d;
    if ((st = rc_dec_init(&d, payload, plen))) { unload(&L); return st; }
    wstate w;
    if ((st = ws_init(&w, L.model, n_ctx, escapes))) { unload(&L); return st; }
    size_t cap = (size_t)orig_len + 16;
    uint8_t* bytes = (uint8_t*)malloc(cap);
    uint32_t* ctx = (uint32_t*)malloc(sizeof(uint32_t) * (cap));
    uint32_t* syms = (uint32_t*)malloc(sizeof(uint32_t) * (cap));
    size_t nb = 0, clen = 0, ns = 0;
    if (!bytes || !ctx || !syms) st = REF_ERR_ALLOC;
    while (!st && nb < orig_len) {
        if ((st = ws_sync(&w, ctx, clen, overlap))) break;
        uint32_t s;
        if ((st = ws_decode_symbol(&w, &d, &s))) break;
        /* decode_codec_symbol (det-token lib.rs:182-199) / detokenize_bytes */
        int byte;
        if (s < V) {
            byte = L.tok.token_to_byte[s];
            if (byte < 0) { st = REF_ERR_TOKENIZER; break; }
        } else if (escapes && s < V + BYTE_ESCAPES) {
            byte = (int)(s - V);
        } else {
            st = REF_ERR_TOKENIZER;
            break;
        }
        bytes[nb++] = (uint8_t)byte;
        syms[ns++] = s;
        if (escapes && s >= V) continue;
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
