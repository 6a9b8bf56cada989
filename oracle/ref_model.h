/*
 * oracle/ref_model.h -- model internals shared by the CPU oracle's forward
 * (ref_model.c) and codec driver (ref_codec.c).  TEST INFRASTRUCTURE, see
 * ref.h.  Mirrors crates/det-model/src/lib.rs:26-170.
 */
#ifndef DETLLM_ORACLE_REF_MODEL_H
#define DETLLM_ORACLE_REF_MODEL_H

#include "ref.h"
#include "ref_gguf.h"

typedef struct {
    uint32_t type; /* GT_F32 (F32/F16 load as F32), GT_Q8_0, GT_Q4_0, GT_Q4_K, GT_Q6_K */
    uint32_t src_type; /* ggml type in the file */
    size_t rows, cols, blocks_per_row;
    void* data; /* float[rows*cols] or block array */
    int owned;
} ref_matrix;

typedef struct {
    float* attn_norm;
    ref_matrix wq, wk, wv, wo, w_gate, w_up, w_down;
    float *q_bias, *k_bias, *v_bias;
    float* ffn_norm;
} ref_layer;

typedef struct {
    size_t block_count, d, d_ff, n_head, n_head_kv, head_dim, rope_dim, ctx;
    int pairing; /* 0 adjacent (llama), 1 split-half (qwen2) */
    float eps, attn_scale, rope_base;
} ref_config;

struct ref_model {
    ref_config cfg;
    ref_matrix tok_embd;
    ref_layer* layers;
    float* output_norm;
    ref_matrix output;
    int tied;
    size_t vocab; /* output rows */
    /* tokenizer table (byte fallback), filled by the codec loader */
};

/* Window/forward state: det-cli main.rs:632-770 (rope, cache, workspace) */
typedef struct {
    const ref_model* m;
    size_t n_ctx, positions;
    float *rope_cos, *rope_sin;
    float *kcache, *vcache; /* [L][Hkv][n_ctx][hd] */
    float *x, *h, *q, *k, *v, *attn, *scores, *probs, *tmp_d, *gate, *up, *ff;
    ref_q8a_block* q8a;
    ref_q8k_block* q8k;
    float* logits;
} ref_state;

int ref_state_init(ref_state* s, const ref_model* m, size_t n_ctx);
void ref_state_free(ref_state* s);
void ref_state_reset_cache(ref_state* s);
/* det-model lib.rs:1249-1400 */
int ref_forward_one(ref_state* s, size_t token, size_t pos);
int ref_model_load_gguf(const gg_file* g, const uint8_t* bytes, ref_model** out);
int map_gguf_error(int gg);

#endif
