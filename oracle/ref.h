/*
 * oracle/ref.h -- CPU restatement of the detllm reference CPU path.
 *
 * TEST INFRASTRUCTURE ONLY.  This oracle is the parity checker for the
 * B200 library (libdetgpu.so).  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product
 * path never links, calls or executes anything under oracle/.
 *
 * Parity pin: the restatement reproduces every golden vector the reference
 * repository holds for this path (fixture logits hashes, the det-num and CLI
 * runtime canaries, quant-kernel-hash, the byte streams of both fixture GGUF
 * files, and the codec smoke sizes); tests/test_oracle_golden.py checks them.
 *
 * Every function names the reference file:line it follows.  The reference is
 * Rust (no cargo in this image), so it cannot be compiled here; this C code is
 * built with -ffp-contract=off and no fast-math so that each f32/f64 operation
 * is one IEEE-754 round-to-nearest-even operation, exactly as in the Rust.
 */
#ifndef DETLLM_ORACLE_REF_H
#define DETLLM_ORACLE_REF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: identical numbering to include/detgpu.h. */
enum {
    REF_OK = 0,
    /* ModelError (crates/det-model/src/lib.rs:48-59), in declaration order */
    REF_ERR_SHAPE = 1,
    REF_ERR_NONFINITE = 2,
    REF_ERR_UNSUPPORTED_ARCH = 3,
    REF_ERR_UNSUPPORTED_HEAD_LEN = 4,
    REF_ERR_UNSUPPORTED_FEATURE = 5,
    REF_ERR_UNSUPPORTED_ROPE_SCALING = 6,
    REF_ERR_MISSING_METADATA = 7,
    REF_ERR_GGUF = 8,
    REF_ERR_UNSUPPORTED_TENSOR_TYPE = 9,
    REF_ERR_THREAD = 10,
    /* CdfError (crates/det-coder/src/cdf.rs:10-17) */
    REF_ERR_CDF_EMPTY = 32,
    REF_ERR_CDF_MALFORMED = 33,
    REF_ERR_CDF_NONFINITE_LOGIT = 34,
    REF_ERR_CDF_SYMBOL_OUT_OF_RANGE = 35,
    REF_ERR_CDF_TOO_MANY_SYMBOLS = 36,
    REF_ERR_CDF_TOTAL_TOO_LARGE = 37,
    /* RangeError (crates/det-coder/src/range.rs:4-8) */
    REF_ERR_RANGE_INVALID_FREQUENCY = 40,
    REF_ERR_RANGE_UNEXPECTED_EOF = 41,
    /* FileError (crates/det-coder/src/file.rs:17-25) */
    REF_ERR_FILE_TOO_SHORT = 48,
    REF_ERR_FILE_BAD_MAGIC = 49,
    REF_ERR_FILE_UNSUPPORTED_VERSION = 50,
    REF_ERR_FILE_UNSUPPORTED_FLAGS = 51,
    REF_ERR_FILE_INVALID_CONTEXT = 52,
    REF_ERR_FILE_INVALID_OVERLAP = 53,
    /* codec driver (crates/det-cli/src/main.rs:433-855) */
    REF_ERR_TOKENIZER = 56,
    REF_ERR_WINDOW = 57,
    REF_ERR_MODEL_HASH_MISMATCH = 58,
    REF_ERR_NONCANONICAL = 59,
    REF_ERR_VOCAB_MISMATCH = 60,
    REF_ERR_DECODE = 61,
    REF_ERR_ALLOC = 62,
};

/* ---- det-num ---------------------------------------------------------- */
float ref_expf(float x);                 /* det-num/src/vendored_libm/expf.rs:33-106 */
void ref_expf_batch(const float* x, float* y, size_t n);
float ref_silu(float x);                 /* det-num/src/math.rs:30-34 */
double ref_exp_f64(double x);            /* vendored_libm/exp.rs */
double ref_ln_f64(double x);             /* vendored_libm/log.rs */
double ref_sin_f64(double x);            /* vendored_libm/sin.rs */
double ref_cos_f64(double x);            /* vendored_libm/cos.rs */
float ref_dot_f32(const float* x, const float* y, size_t n);   /* reduce.rs:2-11 */
float ref_sum_f32(const float* x, size_t n);                   /* reduce.rs:14-22 */
float ref_sum_squares_f32(const float* x, size_t n);           /* reduce.rs:25-33 */
float ref_f16_to_f32(uint16_t bits);     /* det-num/src/f16.rs:6-34 */
int32_t ref_round_ties_even_i32(float x);/* det-num/src/round.rs:2-20 */
void ref_sha256(const uint8_t* data, size_t len, uint8_t out[32]);
void ref_canary_hash(uint8_t out[32]);   /* det-num/src/canary.rs:26-53 */

typedef struct { uint32_t state[8]; uint64_t len; uint8_t buf[64]; size_t buf_len; } ref_sha256_ctx;
void ref_sha256_init(ref_sha256_ctx* c);
void ref_sha256_update(ref_sha256_ctx* c, const uint8_t* data, size_t len);
void ref_sha256_final(ref_sha256_ctx* c, uint8_t out[32]);

/* ---- det-quant --------------------------------------------------------- */
typedef struct { float d; int8_t q[32]; } ref_q8a_block;          /* Q8ABlock / Q8_0Block */
typedef struct { float d; uint8_t qs[16]; } ref_q4_0_block;        /* Q4_0Block */
typedef struct { float d, dmin; uint8_t scales[12]; uint8_t qs[128]; } ref_q4k_block;
typedef struct { float d; uint8_t ql[128]; uint8_t qh[64]; int8_t scales[16]; } ref_q6k_block;
typedef struct { float d; int8_t q[256]; int16_t bsums[16]; } ref_q8k_block;

int ref_quantize_q8a(const float* x, size_t n, ref_q8a_block* out);   /* det-quant :67-80 */
int ref_quantize_q8k(const float* x, size_t n, ref_q8k_block* out);   /* det-quant :92-105 */
float ref_dot_q8_0_q8a_block(const ref_q8a_block* w, const ref_q8a_block* a);
float ref_dot_q4_0_q8a_block(const ref_q4_0_block* w, const ref_q8a_block* a);
int ref_dot_q8_0_q8a(const ref_q8a_block* w, const ref_q8a_block* a, size_t nb, float* out);
int ref_dot_q4_0_q8a(const ref_q4_0_block* w, const ref_q8a_block* a, size_t nb, float* out);
/* the same per-row results as ref_dot_q4_k_q8a / ref_dot_q6_k_q8k for n <=
 * REF_ROW_GROUP consecutive rows (ref_quant.c explains the equivalence) */
#define REF_ROW_GROUP 32
void ref_q8a_dequant(const ref_q8a_block* a, size_t nblocks, float* act);
int ref_dot_q4_k_rows(const ref_q4k_block* w, size_t nb, size_t n, const float* act, float* out);
int ref_dot_q6_k_rows(const ref_q6k_block* w, size_t nb, size_t n, const ref_q8k_block* a, float* out);
/* 1: the GEMV takes the one-row functions for every row (tests compare the two) */
void ref_set_rowwise_gemv(int on);
int ref_dot_q4_k_q8a(const ref_q4k_block* w, const ref_q8a_block* a, size_t nb, float* out);
int ref_dot_q6_k_q8a(const ref_q6k_block* w, const ref_q8a_block* a, size_t nb, float* out);
int ref_dot_q6_k_q8k(const ref_q6k_block* w, const ref_q8k_block* a, size_t nb, float* out);
float ref_q4_k_value(const ref_q4k_block* w, size_t index);
float ref_q6_k_value(const ref_q6k_block* w, size_t index);

/* Flat-array helpers for ctypes callers: quantize a vector into split
 * (scale, quants) arrays.  Returns a status code. */
int ref_quantize_q8a_flat(const float* x, size_t n, float* d, int8_t* q);
int ref_quantize_q8k_flat(const float* x, size_t n, float* d, int8_t* q, int16_t* bsums);

/* ---- canaries / quant-kernel-hash (det-cli/src/main.rs:146-388) -------- */
int ref_runtime_canary_hash(uint8_t out[32]);
int ref_quant_kernel_hash(uint8_t out[32]);

/* ---- fixture generator (xtask/src/main.rs:4765-5120) ------------------- */
/* which: 0 = tiny-f32.gguf, 1 = tiny-qmix.gguf.  Returns bytes written, or
 * the required size when cap is too small. */
size_t ref_fixture_gguf(int which, uint8_t* out, size_t cap);

/* ---- det-model ----------------------------------------------------------- */
typedef struct ref_model ref_model;
typedef struct {
    uint32_t block_count, embedding_length, feed_forward_length;
    uint32_t head_count, head_count_kv, head_dim;
    uint32_t rope_dimension_count, rope_pairing; /* 0 adjacent, 1 split-half */
    uint32_t context_length, vocab;
    float rms_epsilon, attention_scale, rope_freq_base;
    uint32_t weight_types[9]; /* ggml type of token_embd, q, k, v, o, gate, up, down, output */
    uint32_t has_qkv_bias, tied_output;
} ref_model_info;

void ref_set_threads(int threads);

/* Tokenizers (ref_token.c; det-token lib.rs:85-850) on a GGUF's metadata:
 * the selected kind (0 byte fallback, 1 byte-BPE, 2 SentencePiece),
 * tokenize_bytes (codec = 0) or codec_symbols with byte escapes (codec = 1),
 * and the bytes of a symbol sequence (decode_codec_symbol).  *out is
 * malloc'd (ref_free). */
int ref_tokenizer_kind(const uint8_t* gguf, size_t len, int* kind);
int ref_tokenize(const uint8_t* gguf, size_t len, const uint8_t* in, size_t n, int codec, uint32_t** out,
                 size_t* out_n);
int ref_detokenize(const uint8_t* gguf, size_t len, const uint32_t* syms, size_t n, int escapes, uint8_t** out,
                   size_t* out_n);
int ref_model_load(const uint8_t* gguf, size_t len, ref_model** out);
void ref_model_free(ref_model* m);
int ref_model_get_info(const ref_model* m, ref_model_info* info);
/* logits for tokens[0..n) at positions 0..n-1 (teacher forced), n*V floats */
int ref_logits(const ref_model* m, const uint32_t* tokens, size_t n, float* out);
/* det-model lib.rs:1406-1418 */
int ref_logits_hash(const ref_model* m, const uint32_t* tokens, size_t n, size_t chunk, uint8_t out[32]);
/* RoPE tables (det-model lib.rs:813-846): positions x (rope_dim/2) floats each */
int ref_rope_tables(const ref_model* m, size_t positions, float* cos_out, float* sin_out);

/* ---- det-coder ------------------------------------------------------------ */
typedef struct { uint64_t cum; uint32_t freq; uint32_t pad; uint64_t total; } ref_symbol_range;
int ref_logits_to_symbol_range(const float* logits, size_t n, size_t symbol, int byte_escapes,
                               ref_symbol_range* out);                          /* cdf.rs:138-199 */
int ref_decoder_total(const float* logits, size_t n, int byte_escapes, uint64_t* total);
int ref_decoder_lookup(const float* logits, size_t n, int byte_escapes, uint64_t value,
                       uint32_t* symbol, ref_symbol_range* out);                /* cdf.rs:201-245,392-425 */
int ref_logits_to_cdf(const float* logits, size_t n, uint32_t* freq, uint64_t* cum, uint64_t* total);

/* range coder (range.rs) exposed for tests */
int ref_range_encode(const uint64_t* cum, const uint64_t* freq, const uint64_t* total, size_t n,
                     uint8_t* out, size_t cap, size_t* out_len);

/* ---- codec driver (det-cli main.rs:433-855) ------------------------------- */
/* compress(model bytes, input) -> DTLZ bytes.  n_ctx == 0 uses context_length.
 * *out is malloc'd; free with ref_free. */
int ref_compress(const uint8_t* model_bytes, size_t model_len, const uint8_t* input, size_t in_len,
                 uint32_t n_ctx, uint8_t** out, size_t* out_len);
int ref_decompress(const uint8_t* model_bytes, size_t model_len, const uint8_t* dtlz, size_t dtlz_len,
                   uint8_t** out, size_t* out_len);
/* Encode an explicit codec-symbol stream (symbols >= V are byte escapes) and
 * return the range-coder payload (no header). */
int ref_encode_symbols(const ref_model* m, const uint32_t* symbols, size_t n, uint32_t n_ctx,
                       uint32_t overlap, int byte_escapes, uint8_t** out, size_t* out_len);
/* RoPE rotation of one position's `heads` x hd values with a table row of
 * `half` cos / sin entries (pairing 0 adjacent, 1 split-half), and
 * softmax_in_place; exported for the det-model op-order tests. */
int ref_rope_rotate(float* x, size_t heads, size_t hd, size_t half, int pairing, const float* cs_row,
                    const float* sn_row);
int ref_softmax(float* x, size_t n);
/* rmsnorm (det-model :2053-2073) */
int ref_rmsnorm(const float* x, const float* w, size_t n, float eps, float* out);
/* det-cli next_window_start (main.rs:772-778): the window's first token
 * index after the token at `pos` is appended to a window starting at `ws`. */
size_t ref_next_window_start(size_t pos, size_t ws, size_t n_ctx, size_t overlap);
/* Per-symbol ranges of that stream (what the device boundary returns). */
int ref_symbol_ranges_stream(const ref_model* m, const uint32_t* symbols, size_t n, uint32_t n_ctx,
                             uint32_t overlap, int byte_escapes, ref_symbol_range* out);
void ref_free(void* p);

#ifdef __cplusplus
}
#endif
#endif
