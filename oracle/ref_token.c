/*
 * oracle/ref_token.c -- tokenizers of the CPU oracle (TEST INFRASTRUCTURE,
 * see ref.h).
 *
 * Restates crates/det-token/src/lib.rs:
 *   Tokenizer::from_gguf            :86-132  (selection by tokenizer.ggml.model,
 *                                             merges and scores)
 *   ByteFallbackTokenizer           :228-326
 *   ByteBpeTokenizer                :328-503 (merges applied lowest rank first,
 *                                             then leftmost, through a heap)
 *   SentencePieceTokenizer          :505-617 (longest piece, byte fallback)
 *   codec_symbol_stream             :161-180 (byte escapes for bytes without a
 *                                             single-byte token)
 *   decode_codec_symbol             :182-196
 *   token_piece_bytes and helpers   :619-848
 * Every construction error of the reference maps to REF_ERR_TOKENIZER.
 */
#include <stdlib.h>
#include <string.h>

#include "ref.h"
#include "ref_token.h"

/* canonical_byte_fallback_token (lib.rs:841-848): "<0xHH>" where HH parses
 * like u8::from_str_radix(_, 16) (an optional leading '+') */
static int byte_fallback_of(const uint8_t* p, size_t n) {
    if (n != 6) return -1;
    if (p[0] != '<' || p[1] != '0' || p[2] != 'x' || p[5] != '>') return -1;
    int v = 0, start = p[3] == '+' ? 4 : 3;
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

/* token_type_is_emittable (lib.rs:704-710): 1 / 0, or -1 for an invalid type */
static int token_type_emittable(int64_t t) {
    if (t == 1 || t == 4 || t == 6) return 1;
    if (t == 2 || t == 3 || t == 5) return 0;
    return -1;
}

static int gpt2_printable(uint32_t b) { return (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255); }

/* gpt2_char_to_byte (lib.rs:821-839): printable bytes stand for themselves;
 * the other 68 byte values map to code points 256, 257, ... in byte order */
static int gpt2_char_to_byte(uint32_t code) {
    if (gpt2_printable(code)) return (int)code;
    uint32_t n = 0;
    for (uint32_t b = 0; b <= 255; b++) {
        if (gpt2_printable(b)) continue;
        if (code == 256 + n) return (int)b;
        n++;
    }
    return -1;
}

/* one code point of a UTF-8 string (GGUF strings are validated UTF-8) */
static uint32_t utf8_next(const uint8_t* s, size_t n, size_t* i) {
    const uint8_t c = s[*i];
    if (c < 0x80) {
        (*i)++;
        return c;
    }
    const int extra = c >= 0xF0 ? 3 : c >= 0xE0 ? 2 : 1;
    uint32_t cp = c & (0x3Fu >> extra);
    for (int k = 1; k <= extra && *i + k < n; k++) cp = (cp << 6) | (s[*i + k] & 0x3Fu);
    *i += 1 + extra;
    return cp;
}

/* token_piece_bytes (lib.rs:797-811) into out (room for n bytes): a byte
 * fallback token, else a GPT-2 byte-unicode string, else "▁rest" -> " rest",
 * else the UTF-8 bytes */
static size_t piece_bytes(const uint8_t* s, size_t n, uint8_t* out) {
    const int b = byte_fallback_of(s, n);
    if (b >= 0) {
        out[0] = (uint8_t)b;
        return 1;
    }
    size_t i = 0, k = 0;
    int ok = 1;
    while (i < n) {
        const int v = gpt2_char_to_byte(utf8_next(s, n, &i));
        if (v < 0) {
            ok = 0;
            break;
        }
        out[k++] = (uint8_t)v;
    }
    if (ok) return k;
    if (n >= 3 && s[0] == 0xE2 && s[1] == 0x96 && s[2] == 0x81) {
        out[0] = ' ';
        memcpy(out + 1, s + 3, n - 3);
        return n - 2;
    }
    memcpy(out, s, n);
    return n;
}

static int bytes_cmp(const uint8_t* a, size_t an, const uint8_t* b, size_t bn) {
    const size_t m = an < bn ? an : bn;
    const int c = m ? memcmp(a, b, m) : 0;
    if (c) return c;
    return an < bn ? -1 : an > bn ? 1 : 0;
}

/* (bytes, id) of the emittable tokens, sorted by bytes: bytes_to_token */
typedef struct {
    const uint8_t* b;
    size_t n;
    uint32_t id;
    float score;
} bt_entry;

static int bt_cmp(const void* x, const void* y) {
    const bt_entry* a = (const bt_entry*)x;
    const bt_entry* b = (const bt_entry*)y;
    const int c = bytes_cmp(a->b, a->n, b->b, b->n);
    if (c) return c;
    return a->id < b->id ? -1 : a->id > b->id ? 1 : 0;
}

static const bt_entry* bt_find(const bt_entry* e, size_t n, const uint8_t* b, size_t bn) {
    size_t lo = 0, hi = n;
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        const int c = bytes_cmp(e[mid].b, e[mid].n, b, bn);
        if (c < 0) lo = mid + 1;
        else hi = mid;
    }
    return lo < n && bytes_cmp(e[lo].b, e[lo].n, b, bn) == 0 ? &e[lo] : NULL;
}

static int merge_cmp(const void* x, const void* y) {
    const ref_merge* a = (const ref_merge*)x;
    const ref_merge* b = (const ref_merge*)y;
    if (a->left != b->left) return a->left < b->left ? -1 : 1;
    if (a->right != b->right) return a->right < b->right ? -1 : 1;
    return a->rank < b->rank ? -1 : a->rank > b->rank ? 1 : 0;
}

static const ref_merge* merge_find(const ref_tok* t, uint32_t l, uint32_t r) {
    size_t lo = 0, hi = t->n_merges;
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        const ref_merge* m = &t->merges[mid];
        if (m->left < l || (m->left == l && m->right < r)) lo = mid + 1;
        else hi = mid;
    }
    return lo < t->n_merges && t->merges[lo].left == l && t->merges[lo].right == r ? &t->merges[lo] : NULL;
}

void ref_tok_free(ref_tok* t) {
    free(t->pool);
    free(t->off);
    free(t->tok_len);
    free(t->merges);
    free(t->pieces);
    memset(t, 0, sizeof *t);
}

static int fail(ref_tok* t, void* a, void* b, int st) {
    free(a);
    free(b);
    ref_tok_free(t);
    return st;
}

/* ByteFallbackTokenizer::from_tokens_and_emit_mask (lib.rs:258-304): every
 * byte needs exactly one "<0xHH>" token; emittable ones go into the byte
 * table.  token_len_out (tok_len) is 1 for byte tokens when `set_lens`. */
static int byte_fallback_build(ref_tok* t, const gg_kv* toks, const int* emit, int set_lens) {
    int seen[256];
    for (int b = 0; b < 256; b++) seen[b] = 0;
    for (size_t i = 0; i < t->vocab; i++) {
        const int b = byte_fallback_of(toks->strs[i].ptr, (size_t)toks->strs[i].len);
        if (b < 0) continue;
        if (seen[b]) return REF_ERR_TOKENIZER; /* DuplicateByteFallback */
        seen[b] = 1;
        if (set_lens) {
            t->pool[t->off[i]] = (uint8_t)b;
            t->tok_len[i] = 1;
        }
        if (!emit || emit[i]) t->byte_to_token[b] = (int32_t)i;
    }
    for (int b = 0; b < 256; b++)
        if (!seen[b]) return REF_ERR_TOKENIZER; /* IncompleteByteFallback */
    return REF_OK;
}

int ref_tok_from_gguf(const gg_file* g, ref_tok* t) {
    memset(t, 0, sizeof *t);
    for (int b = 0; b < 256; b++) t->byte_to_token[b] = -1;
    /* gguf_tokens (:619-626) */
    const gg_kv* toks = gg_find(g, "tokenizer.ggml.tokens");
    if (!toks || toks->type != GV_ARRAY || toks->elem_type != GV_STRING) return REF_ERR_TOKENIZER;
    const size_t V = (size_t)toks->count;
    t->vocab = V;
    /* optional_gguf_emit_mask (:666-695) */
    int* emit = NULL;
    const gg_kv* tt = gg_find(g, "tokenizer.ggml.token_type");
    if (tt) {
        if (tt->type != GV_ARRAY || (tt->elem_type != GV_I32 && tt->elem_type != GV_U32) || tt->count != V)
            return REF_ERR_TOKENIZER;
        emit = (int*)malloc(sizeof(int) * (V ? V : 1));
        if (!emit) return REF_ERR_ALLOC;
        for (size_t i = 0; i < V; i++) {
            const uint32_t raw = (uint32_t)tt->arr[4 * i] | ((uint32_t)tt->arr[4 * i + 1] << 8) |
                                 ((uint32_t)tt->arr[4 * i + 2] << 16) | ((uint32_t)tt->arr[4 * i + 3] << 24);
            const int64_t v = tt->elem_type == GV_I32 ? (int64_t)(int32_t)raw : (int64_t)raw;
            emit[i] = token_type_emittable(v);
            if (emit[i] < 0) return fail(t, emit, NULL, REF_ERR_TOKENIZER);
        }
    }
    /* optional merges / model (:628-644) */
    const gg_kv* merges = gg_find(g, "tokenizer.ggml.merges");
    if (merges && (merges->type != GV_ARRAY || merges->elem_type != GV_STRING)) return fail(t, emit, NULL, REF_ERR_TOKENIZER);
    const gg_kv* model = gg_find(g, "tokenizer.ggml.model");
    if (model && model->type != GV_STRING) return fail(t, emit, NULL, REF_ERR_TOKENIZER);
    const gg_kv* scores = gg_find(g, "tokenizer.ggml.scores");
    int kind;
    if (model) {
        const gg_str* m = &model->s;
        if (m->len == 4 && !memcmp(m->ptr, "gpt2", 4)) kind = REF_TOK_BPE;
        else if ((m->len == 5 && !memcmp(m->ptr, "llama", 5)) || (m->len == 3 && !memcmp(m->ptr, "spm", 3)) ||
                 (m->len == 13 && !memcmp(m->ptr, "sentencepiece", 13)))
            kind = REF_TOK_SPM;
        else return fail(t, emit, NULL, REF_ERR_TOKENIZER); /* UnsupportedTokenizerModel */
    } else if (merges && merges->count > 0) {
        kind = REF_TOK_BPE;
    } else if (scores) {
        if (scores->type != GV_ARRAY || scores->elem_type != GV_F32) return fail(t, emit, NULL, REF_ERR_TOKENIZER);
        kind = REF_TOK_SPM;
    } else {
        kind = REF_TOK_BYTE_FALLBACK;
    }
    t->kind = kind;
    /* optional_gguf_scores (:646-664) for SentencePiece */
    const float* sc = NULL;
    float* sc_buf = NULL;
    if (kind == REF_TOK_SPM && scores) {
        if (scores->type != GV_ARRAY || scores->elem_type != GV_F32 || scores->count != V)
            return fail(t, emit, NULL, REF_ERR_TOKENIZER); /* MetadataType / ScoresLength */
        sc_buf = (float*)malloc(sizeof(float) * (V ? V : 1));
        if (!sc_buf) return fail(t, emit, NULL, REF_ERR_ALLOC);
        for (size_t i = 0; i < V; i++) {
            memcpy(&sc_buf[i], scores->arr + 4 * i, 4);
            uint32_t bits;
            memcpy(&bits, &sc_buf[i], 4);
            if ((bits & 0x7f800000u) == 0x7f800000u) return fail(t, emit, sc_buf, REF_ERR_TOKENIZER); /* NonFiniteScore */
        }
        sc = sc_buf;
    }
    /* token_to_bytes */
    size_t total = 0;
    for (size_t i = 0; i < V; i++) total += (size_t)toks->strs[i].len;
    t->pool = (uint8_t*)malloc(total ? total : 1);
    t->off = (size_t*)malloc(sizeof(size_t) * (V ? V : 1));
    t->tok_len = (int64_t*)malloc(sizeof(int64_t) * (V ? V : 1));
    if (!t->pool || !t->off || !t->tok_len) return fail(t, emit, sc_buf, REF_ERR_ALLOC);
    size_t o = 0;
    for (size_t i = 0; i < V; i++) {
        t->off[i] = o;
        if (kind == REF_TOK_BYTE_FALLBACK) {
            t->tok_len[i] = -1;
        } else {
            t->tok_len[i] = (int64_t)piece_bytes(toks->strs[i].ptr, (size_t)toks->strs[i].len, t->pool + o);
        }
        o += (size_t)toks->strs[i].len;
    }
    int st = REF_OK;
    if (kind == REF_TOK_BYTE_FALLBACK) {
        st = byte_fallback_build(t, toks, emit, 1);
    } else if (kind == REF_TOK_SPM) {
        /* SentencePieceTokenizer::from_tokens_scores_and_emit_mask (:520-566) */
        st = byte_fallback_build(t, toks, emit, 0);
        bt_entry* e = NULL;
        size_t ne = 0;
        if (!st) {
            e = (bt_entry*)malloc(sizeof(bt_entry) * (V ? V : 1));
            if (!e) st = REF_ERR_ALLOC;
        }
        for (size_t i = 0; !st && i < V; i++) {
            if (t->tok_len[i] > 1 && (!emit || emit[i])) {
                e[ne].b = t->pool + t->off[i];
                e[ne].n = (size_t)t->tok_len[i];
                e[ne].id = (uint32_t)i;
                e[ne].score = sc ? sc[i] : 0.0f;
                ne++;
                if ((size_t)t->tok_len[i] > t->max_piece_len) t->max_piece_len = (size_t)t->tok_len[i];
            }
        }
        if (t->max_piece_len < 1) t->max_piece_len = 1;
        if (!st) {
            /* per distinct bytes: the highest score, the lowest id among equal
             * scores (a later token replaces the kept one only with a strictly
             * higher score) */
            qsort(e, ne, sizeof *e, bt_cmp);
            t->pieces = (ref_piece*)malloc(sizeof(ref_piece) * (ne ? ne : 1));
            if (!t->pieces) st = REF_ERR_ALLOC;
            for (size_t i = 0; !st && i < ne;) {
                size_t j = i, best = i;
                while (j < ne && bytes_cmp(e[j].b, e[j].n, e[i].b, e[i].n) == 0) {
                    if (e[j].score > e[best].score) best = j;
                    j++;
                }
                ref_piece* pc = &t->pieces[t->n_pieces++];
                pc->bytes = e[best].b;
                pc->len = e[best].n;
                pc->id = e[best].id;
                pc->score = e[best].score;
                i = j;
            }
        }
        free(e);
    } else {
        /* ByteBpeTokenizer::from_tokens_merges_and_emit_mask (:343-407) */
        bt_entry* e = (bt_entry*)malloc(sizeof(bt_entry) * (V ? V : 1));
        size_t ne = 0;
        if (!e) st = REF_ERR_ALLOC;
        for (size_t i = 0; !st && i < V; i++) {
            if (emit && !emit[i]) continue;
            const uint8_t* b = t->pool + t->off[i];
            const size_t n = (size_t)t->tok_len[i];
            if (n == 1) {
                if (t->byte_to_token[b[0]] >= 0) st = REF_ERR_TOKENIZER; /* DuplicateByteFallback */
                t->byte_to_token[b[0]] = (int32_t)i;
            }
            e[ne].b = b;
            e[ne].n = n;
            e[ne].id = (uint32_t)i;
            e[ne].score = 0.0f;
            ne++;
        }
        if (!st) {
            qsort(e, ne, sizeof *e, bt_cmp);
            for (size_t i = 1; i < ne && !st; i++)
                if (bytes_cmp(e[i].b, e[i].n, e[i - 1].b, e[i - 1].n) == 0) st = REF_ERR_TOKENIZER; /* DuplicateTokenBytes */
        }
        const size_t nm = merges ? (size_t)merges->count : 0;
        uint8_t* buf = NULL;
        if (!st && nm) {
            t->merges = (ref_merge*)malloc(sizeof(ref_merge) * nm);
            size_t mx = 0;
            for (size_t r = 0; r < nm; r++)
                if ((size_t)merges->strs[r].len > mx) mx = (size_t)merges->strs[r].len;
            buf = (uint8_t*)malloc(2 * mx + 2);
            if (!t->merges || !buf) st = REF_ERR_ALLOC;
        }
        for (size_t r = 0; !st && r < nm; r++) {
            /* parse_merge (:772-786): exactly two non-empty parts split on ' ' */
            const uint8_t* s = merges->strs[r].ptr;
            const size_t n = (size_t)merges->strs[r].len;
            size_t sp = 0, spaces = 0;
            for (size_t k = 0; k < n; k++)
                if (s[k] == ' ') {
                    if (!spaces) sp = k;
                    spaces++;
                }
            if (spaces != 1 || sp == 0 || sp + 1 == n) {
                st = REF_ERR_TOKENIZER; /* InvalidMerge */
                break;
            }
            uint8_t* lb = buf;
            const size_t ln = piece_bytes(s, sp, lb);
            uint8_t* rb = buf + ln;
            const size_t rn = piece_bytes(s + sp + 1, n - sp - 1, rb);
            const bt_entry* le = bt_find(e, ne, lb, ln);
            const bt_entry* re = bt_find(e, ne, rb, rn);
            const bt_entry* me = bt_find(e, ne, lb, ln + rn); /* left bytes then right bytes, contiguous in buf */
            if (!le || !re || !me) {
                if (emit) continue;
                st = REF_ERR_TOKENIZER; /* MissingTokenBytes / MissingMergeToken */
                break;
            }
            ref_merge* m = &t->merges[t->n_merges++];
            m->left = le->id;
            m->right = re->id;
            m->merged = me->id;
            m->rank = r;
        }
        free(buf);
        if (!st && t->n_merges) {
            qsort(t->merges, t->n_merges, sizeof(ref_merge), merge_cmp);
            for (size_t i = 1; i < t->n_merges; i++)
                if (t->merges[i].left == t->merges[i - 1].left && t->merges[i].right == t->merges[i - 1].right)
                    st = REF_ERR_TOKENIZER; /* DuplicateMerge */
        }
        free(e);
    }
    free(emit);
    free(sc_buf);
    if (st) ref_tok_free(t);
    return st;
}

/* min-heap of BPE merge candidates ordered by (rank, left index, merged id):
 * the BinaryHeap<Reverse<(rank, index, merged_id)>> of lib.rs:420-470 */
typedef struct {
    uint64_t rank;
    size_t index;
    uint32_t merged;
} hent;

static int hless(const hent* a, const hent* b) {
    if (a->rank != b->rank) return a->rank < b->rank;
    if (a->index != b->index) return a->index < b->index;
    return a->merged < b->merged;
}

typedef struct {
    hent* v;
    size_t n, cap;
} heap_t;

static int heap_push(heap_t* h, hent e) {
    if (h->n == h->cap) {
        const size_t cap = h->cap ? 2 * h->cap : 64;
        hent* v = (hent*)realloc(h->v, cap * sizeof(hent));
        if (!v) return REF_ERR_ALLOC;
        h->v = v;
        h->cap = cap;
    }
    size_t i = h->n++;
    h->v[i] = e;
    while (i > 0) {
        const size_t p = (i - 1) / 2;
        if (!hless(&h->v[i], &h->v[p])) break;
        const hent tmp = h->v[i];
        h->v[i] = h->v[p];
        h->v[p] = tmp;
        i = p;
    }
    return REF_OK;
}

static hent heap_pop(heap_t* h) {
    const hent top = h->v[0];
    h->v[0] = h->v[--h->n];
    size_t i = 0;
    for (;;) {
        const size_t l = 2 * i + 1, r = l + 1;
        size_t m = i;
        if (l < h->n && hless(&h->v[l], &h->v[m])) m = l;
        if (r < h->n && hless(&h->v[r], &h->v[m])) m = r;
        if (m == i) break;
        const hent tmp = h->v[i];
        h->v[i] = h->v[m];
        h->v[m] = tmp;
        i = m;
    }
    return top;
}

/* push_bpe_pair (lib.rs:491-503) */
static int push_pair(const ref_tok* t, heap_t* h, const uint32_t* ids, size_t left, long right) {
    if (right < 0) return REF_OK;
    const ref_merge* m = merge_find(t, ids[left], ids[right]);
    if (!m) return REF_OK;
    hent e = {m->rank, left, m->merged};
    return heap_push(h, e);
}

/* ByteBpeTokenizer::tokenize_bytes (lib.rs:409-476) */
static int bpe_tokenize(const ref_tok* t, const uint8_t* in, size_t n, uint32_t* out, size_t* out_n) {
    for (size_t i = 0; i < n; i++) {
        if (t->byte_to_token[in[i]] < 0) return REF_ERR_TOKENIZER; /* MissingByteFallback */
        out[i] = (uint32_t)t->byte_to_token[in[i]];
    }
    if (n < 2) {
        *out_n = n;
        return REF_OK;
    }
    long* prev = (long*)malloc(sizeof(long) * n);
    long* next = (long*)malloc(sizeof(long) * n);
    char* alive = (char*)malloc(n);
    heap_t h = {NULL, 0, 0};
    int st = prev && next && alive ? REF_OK : REF_ERR_ALLOC;
    for (size_t i = 0; !st && i < n; i++) {
        prev[i] = i == 0 ? -1 : (long)i - 1;
        next[i] = i + 1 == n ? -1 : (long)i + 1;
        alive[i] = 1;
    }
    for (size_t i = 0; !st && i + 1 < n; i++) st = push_pair(t, &h, out, i, (long)i + 1);
    while (!st && h.n) {
        const hent e = heap_pop(&h);
        if (!alive[e.index]) continue;
        const long right = next[e.index];
        if (right < 0 || !alive[right]) continue;
        const ref_merge* m = merge_find(t, out[e.index], out[right]);
        if (!m || m->rank != e.rank || m->merged != e.merged) continue;
        out[e.index] = e.merged;
        alive[right] = 0;
        const long after = next[right];
        next[e.index] = after;
        if (after >= 0) prev[after] = (long)e.index;
        if (prev[e.index] >= 0) st = push_pair(t, &h, out, (size_t)prev[e.index], (long)e.index);
        if (!st) st = push_pair(t, &h, out, e.index, next[e.index]);
    }
    size_t k = 0;
    for (long i = 0; !st && i >= 0; i = next[i])
        if (alive[i]) out[k++] = out[i];
    *out_n = k;
    free(prev);
    free(next);
    free(alive);
    free(h.v);
    return st;
}

/* SentencePieceTokenizer::tokenize_bytes (lib.rs:568-604): at each position
 * the longest multi-byte piece, else the byte-fallback token */
static int spm_tokenize(const ref_tok* t, const uint8_t* in, size_t n, uint32_t* out, size_t* out_n) {
    size_t pos = 0, k = 0;
    while (pos < n) {
        const size_t max_end = n < pos + t->max_piece_len ? n : pos + t->max_piece_len;
        const ref_piece* best = NULL;
        for (size_t end = pos + 1; end <= max_end; end++) {
            size_t lo = 0, hi = t->n_pieces;
            while (lo < hi) {
                const size_t mid = (lo + hi) / 2;
                if (bytes_cmp(t->pieces[mid].bytes, t->pieces[mid].len, in + pos, end - pos) < 0) lo = mid + 1;
                else hi = mid;
            }
            if (lo < t->n_pieces && bytes_cmp(t->pieces[lo].bytes, t->pieces[lo].len, in + pos, end - pos) == 0)
                best = &t->pieces[lo]; /* a longer match always wins */
        }
        if (best) {
            out[k++] = best->id;
            pos += best->len;
        } else {
            if (t->byte_to_token[in[pos]] < 0) return REF_ERR_TOKENIZER; /* MissingByteFallback */
            out[k++] = (uint32_t)t->byte_to_token[in[pos]];
            pos++;
        }
    }
    *out_n = k;
    return REF_OK;
}

static int tokenize_into(const ref_tok* t, const uint8_t* in, size_t n, uint32_t* out, size_t* out_n) {
    if (t->kind == REF_TOK_BPE) return bpe_tokenize(t, in, n, out, out_n);
    if (t->kind == REF_TOK_SPM) return spm_tokenize(t, in, n, out, out_n);
    for (size_t i = 0; i < n; i++) { /* ByteFallbackTokenizer::tokenize_bytes (:306-312) */
        if (t->byte_to_token[in[i]] < 0) return REF_ERR_TOKENIZER;
        out[i] = (uint32_t)t->byte_to_token[in[i]];
    }
    *out_n = n;
    return REF_OK;
}

int ref_tok_tokenize(const ref_tok* t, const uint8_t* in, size_t n, uint32_t** out, size_t* out_n) {
    uint32_t* o = (uint32_t*)malloc(sizeof(uint32_t) * (n ? n : 1));
    if (!o) return REF_ERR_ALLOC;
    const int st = tokenize_into(t, in, n, o, out_n);
    if (st) {
        free(o);
        return st;
    }
    *out = o;
    return REF_OK;
}

int ref_tok_codec_symbols(const ref_tok* t, const uint8_t* in, size_t n, uint32_t** out, size_t* out_n) {
    uint32_t* o = (uint32_t*)malloc(sizeof(uint32_t) * (n ? n : 1));
    if (!o) return REF_ERR_ALLOC;
    size_t k = 0, pos = 0;
    while (pos < n) {
        if (t->byte_to_token[in[pos]] < 0) { /* ByteEscape */
            o[k++] = (uint32_t)(t->vocab + in[pos]);
            pos++;
            continue;
        }
        const size_t start = pos++;
        while (pos < n && t->byte_to_token[in[pos]] >= 0) pos++;
        size_t m = 0;
        const int st = tokenize_into(t, in + start, pos - start, o + k, &m);
        if (st) {
            free(o);
            return st;
        }
        k += m;
    }
    *out = o;
    *out_n = k;
    return REF_OK;
}

int ref_tok_symbol_bytes(const ref_tok* t, uint32_t symbol, int escapes, uint8_t* scratch, const uint8_t** bytes,
                         size_t* len) {
    if (symbol < t->vocab) {
        /* token_to_bytes; a byte-fallback tokenizer knows its byte tokens only */
        if (t->tok_len[symbol] < 0) return REF_ERR_TOKENIZER; /* InvalidToken */
        *bytes = t->pool + t->off[symbol];
        *len = (size_t)t->tok_len[symbol];
        return REF_OK;
    }
    if (escapes && symbol < t->vocab + 256) {
        scratch[0] = (uint8_t)(symbol - t->vocab);
        *bytes = scratch;
        *len = 1;
        return REF_OK;
    }
    return REF_ERR_TOKENIZER;
}
