/*
 * oracle/ref_fixture.c -- regenerates the reference's fixture GGUF files
 * byte for byte (TEST INFRASTRUCTURE, see ref.h).  Follows
 * xtask/src/main.rs:4765-5120 (tiny_f32_gguf, tiny_qmix_gguf, encode_gguf,
 * push_tensor / push_vector / push_q8_tensor / push_q4_tensor).
 */
#include <stdio.h>
#include <stdlib.h>

#include "ref.h"
#include "ref_internal.h"

typedef struct {
    uint8_t* p;
    size_t len, cap;
} buf_t;

static void bput(buf_t* b, const void* d, size_t n) {
    if (b->len + n > b->cap) {
        size_t nc = b->cap ? b->cap : 1024;
        while (nc < b->len + n) nc *= 2;
        b->p = (uint8_t*)realloc(b->p, nc);
        b->cap = nc;
    }
    memcpy(b->p + b->len, d, n);
    b->len += n;
}
static void bu8(buf_t* b, uint8_t v) { bput(b, &v, 1); }
static void bu32(buf_t* b, uint32_t v) {
    uint8_t x[4] = {(uint8_t)v, (uint8_t)(v >> 8), (uint8_t)(v >> 16), (uint8_t)(v >> 24)};
    bput(b, x, 4);
}
static void bu64(buf_t* b, uint64_t v) {
    uint8_t x[8];
    for (int i = 0; i < 8; i++) x[i] = (uint8_t)(v >> (8 * i));
    bput(b, x, 8);
}
static void bstr(buf_t* b, const char* s) {
    bu64(b, strlen(s));
    bput(b, s, strlen(s));
}

typedef struct {
    char name[64];
    uint32_t ndim;
    uint64_t dims[2];
    uint32_t ty;
    uint64_t offset;
} tspec;

typedef struct {
    tspec t[16];
    int n;
    buf_t data;
} fx;

static void push_tensor(fx* f, const char* name, size_t rows, size_t cols, float scale) {
    tspec* t = &f->t[f->n++];
    snprintf(t->name, sizeof t->name, "%s", name);
    t->ndim = 2;
    t->dims[0] = cols;
    t->dims[1] = rows;
    t->ty = 0;
    t->offset = f->data.len;
    for (size_t i = 0; i < rows * cols; i++) {
        float v = ((float)(i % 13) - 6.0f) * scale;
        bu32(&f->data, f2u(v));
    }
}

static void push_vector(fx* f, const char* name, size_t len, float value) {
    tspec* t = &f->t[f->n++];
    snprintf(t->name, sizeof t->name, "%s", name);
    t->ndim = 1;
    t->dims[0] = len;
    t->ty = 0;
    t->offset = f->data.len;
    for (size_t i = 0; i < len; i++) bu32(&f->data, f2u(value));
}

static void push_q8(fx* f, const char* name, size_t rows, size_t cols, uint16_t scale, int8_t q) {
    tspec* t = &f->t[f->n++];
    snprintf(t->name, sizeof t->name, "%s", name);
    t->ndim = 2;
    t->dims[0] = cols;
    t->dims[1] = rows;
    t->ty = 8;
    t->offset = f->data.len;
    for (size_t i = 0; i < rows * (cols / 32); i++) {
        bu8(&f->data, (uint8_t)scale);
        bu8(&f->data, (uint8_t)(scale >> 8));
        for (int j = 0; j < 32; j++) bu8(&f->data, (uint8_t)q);
    }
}

static void push_q4(fx* f, const char* name, size_t rows, size_t cols, uint16_t scale, uint8_t packed) {
    tspec* t = &f->t[f->n++];
    snprintf(t->name, sizeof t->name, "%s", name);
    t->ndim = 2;
    t->dims[0] = cols;
    t->dims[1] = rows;
    t->ty = 2;
    t->offset = f->data.len;
    for (size_t i = 0; i < rows * (cols / 32); i++) {
        bu8(&f->data, (uint8_t)scale);
        bu8(&f->data, (uint8_t)(scale >> 8));
        for (int j = 0; j < 16; j++) bu8(&f->data, packed);
    }
}

static void meta_u32(buf_t* b, const char* k, uint32_t v) { bstr(b, k); bu32(b, 4); bu32(b, v); }
static void meta_f32(buf_t* b, const char* k, float v) { bstr(b, k); bu32(b, 6); bu32(b, f2u(v)); }

/* encode_gguf (xtask :4939-4984) */
static void encode_gguf(fx* f, uint32_t vocab, uint32_t d, uint32_t dff, uint32_t nh, uint32_t nkv, uint32_t ctx,
                        buf_t* out) {
    bput(out, "GGUF", 4);
    bu32(out, 3);
    bu64(out, (uint64_t)f->n);
    bu64(out, 12);
    bstr(out, "general.architecture");
    bu32(out, 8);
    bstr(out, "llama");
    meta_u32(out, "llama.block_count", 1);
    meta_u32(out, "llama.embedding_length", d);
    meta_u32(out, "llama.feed_forward_length", dff);
    meta_u32(out, "llama.attention.head_count", nh);
    meta_u32(out, "llama.attention.head_count_kv", nkv);
    meta_f32(out, "llama.attention.layer_norm_rms_epsilon", 1e-5f);
    meta_f32(out, "llama.rope.freq_base", 10000.0f);
    meta_u32(out, "llama.rope.dimension_count", d / nh);
    meta_u32(out, "llama.context_length", ctx);
    meta_u32(out, "llama.vocab_size", vocab);
    bstr(out, "tokenizer.ggml.tokens");
    bu32(out, 9);
    bu32(out, 8);
    bu64(out, 256);
    for (int b = 0; b < 256; b++) {
        char s[8];
        snprintf(s, sizeof s, "<0x%02X>", b);
        bstr(out, s);
    }
    for (int i = 0; i < f->n; i++) {
        bstr(out, f->t[i].name);
        bu32(out, f->t[i].ndim);
        for (uint32_t k = 0; k < f->t[i].ndim; k++) bu64(out, f->t[i].dims[k]);
        bu32(out, f->t[i].ty);
        bu64(out, f->t[i].offset);
    }
    while (out->len % 32) bu8(out, 0);
    bput(out, f->data.p, f->data.len);
}

size_t ref_fixture_gguf(int which, uint8_t* out, size_t cap) {
    fx f;
    memset(&f, 0, sizeof f);
    buf_t o = {0, 0, 0};
    if (which == 0) { /* tiny_f32_gguf (xtask :4765-4843) */
        push_tensor(&f, "token_embd.weight", 256, 4, 0.001f);
        push_vector(&f, "blk.0.attn_norm.weight", 4, 1.0f);
        push_tensor(&f, "blk.0.attn_q.weight", 4, 4, 0.002f);
        push_tensor(&f, "blk.0.attn_k.weight", 2, 4, -0.0015f);
        push_tensor(&f, "blk.0.attn_v.weight", 2, 4, 0.0025f);
        push_tensor(&f, "blk.0.attn_output.weight", 4, 4, -0.002f);
        push_vector(&f, "blk.0.ffn_norm.weight", 4, 1.0f);
        push_tensor(&f, "blk.0.ffn_gate.weight", 6, 4, 0.003f);
        push_tensor(&f, "blk.0.ffn_up.weight", 6, 4, -0.0025f);
        push_tensor(&f, "blk.0.ffn_down.weight", 4, 6, 0.0018f);
        push_vector(&f, "output_norm.weight", 4, 1.0f);
        push_tensor(&f, "output.weight", 256, 4, 0.0022f);
        encode_gguf(&f, 256, 4, 6, 2, 1, 16, &o);
    } else { /* tiny_qmix_gguf (xtask :4845-4937) */
        push_q8(&f, "token_embd.weight", 256, 32, 0x3c00, 2);
        push_vector(&f, "blk.0.attn_norm.weight", 32, 1.0f);
        push_q8(&f, "blk.0.attn_q.weight", 32, 32, 0x3c00, 1);
        push_q4(&f, "blk.0.attn_k.weight", 16, 32, 0x3c00, 0x99);
        push_q8(&f, "blk.0.attn_v.weight", 16, 32, 0x3c00, -1);
        push_q4(&f, "blk.0.attn_output.weight", 32, 32, 0x3c00, 0x99);
        push_vector(&f, "blk.0.ffn_norm.weight", 32, 1.0f);
        push_q8(&f, "blk.0.ffn_gate.weight", 32, 32, 0x3c00, 2);
        push_q4(&f, "blk.0.ffn_up.weight", 32, 32, 0x3c00, 0x99);
        push_q8(&f, "blk.0.ffn_down.weight", 32, 32, 0x3c00, -2);
        push_vector(&f, "output_norm.weight", 32, 1.0f);
        encode_gguf(&f, 256, 32, 32, 2, 1, 16, &o);
    }
    size_t n = o.len;
    if (out && n <= cap) memcpy(out, o.p, n);
    free(o.p);
    free(f.data.p);
    return n;
}
