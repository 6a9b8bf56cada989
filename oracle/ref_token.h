/*
 * oracle/ref_token.h -- tokenizers of the CPU oracle (TEST INFRASTRUCTURE,
 * see ref.h).  Follows crates/det-token/src/lib.rs:85-850: the GGUF
 * tokenizer selection, the byte-fallback, byte-BPE and SentencePiece
 * tokenizers, and the codec symbol stream with byte escapes.
 */
#ifndef DETLLM_ORACLE_REF_TOKEN_H
#define DETLLM_ORACLE_REF_TOKEN_H

#include <stddef.h>
#include <stdint.h>

#include "ref_gguf.h"

enum { REF_TOK_BYTE_FALLBACK = 0, REF_TOK_BPE = 1, REF_TOK_SPM = 2 };

typedef struct {
    uint32_t left, right, merged;
    uint64_t rank;
} ref_merge;

typedef struct {
    const uint8_t* bytes;
    size_t len;
    uint32_t id;
    float score;
} ref_piece;

typedef struct {
    int kind;
    size_t vocab;
    /* the single-byte token emitted for each byte value, -1 if none (for
     * SentencePiece: its byte-fallback tokenizer's table) */
    int32_t byte_to_token[256];
    /* token_to_bytes: bytes of token i at pool + off[i], tok_len[i] long;
     * tok_len[i] < 0: the token has no bytes (a byte-fallback tokenizer's
     * non-byte tokens) */
    uint8_t* pool;
    size_t* off;
    int64_t* tok_len;
    ref_merge* merges; /* byte-BPE, sorted by (left, right) */
    size_t n_merges;
    ref_piece* pieces; /* SentencePiece multi-byte pieces, sorted by bytes */
    size_t n_pieces, max_piece_len;
} ref_tok;

/* Tokenizer::from_gguf (det-token lib.rs:86-132); REF_OK or REF_ERR_TOKENIZER */
int ref_tok_from_gguf(const gg_file* g, ref_tok* t);
void ref_tok_free(ref_tok* t);
/* tokenize_bytes of the selected tokenizer; *out malloc'd */
int ref_tok_tokenize(const ref_tok* t, const uint8_t* in, size_t n, uint32_t** out, size_t* out_n);
/* codec_symbols (lib.rs:150-180): tokens, and V + byte for byte escapes */
int ref_tok_codec_symbols(const ref_tok* t, const uint8_t* in, size_t n, uint32_t** out, size_t* out_n);
/* decode_codec_symbol (lib.rs:182-196): the bytes of one codec symbol
 * (escapes: symbols V..V+255 are bytes), at *bytes / *len (pointing into the
 * tokenizer or at `scratch`); REF_ERR_TOKENIZER for an invalid symbol or a
 * token without bytes */
int ref_tok_symbol_bytes(const ref_tok* t, uint32_t symbol, int escapes, uint8_t* scratch, const uint8_t** bytes,
                         size_t* len);

#endif
