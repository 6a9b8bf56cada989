/*
 * oracle/ref_coder.h -- range coder state of the CPU oracle (TEST
 * INFRASTRUCTURE, see ref.h).  Mirrors crates/det-coder/src/range.rs.
 */
#ifndef DETLLM_ORACLE_REF_CODER_H
#define DETLLM_ORACLE_REF_CODER_H

#include <stddef.h>
#include <stdint.h>

#include "ref.h"

typedef struct {
    uint64_t low, range;
    uint8_t* out;
    size_t len, cap;
} rc_enc;

typedef struct {
    uint64_t low, code, range;
    int pending;
    uint64_t pend_range, pend_total;
    const uint8_t* in;
    size_t len, pos;
} rc_dec;

void rc_enc_init(rc_enc* e);
int rc_enc_encode(rc_enc* e, uint64_t cum, uint64_t freq, uint64_t total);
int rc_enc_finish(rc_enc* e);
int rc_enc_push(rc_enc* e, uint8_t b);
int rc_dec_init(rc_dec* d, const uint8_t* in, size_t len);
int rc_dec_decode_freq(rc_dec* d, uint64_t total, uint64_t* value);
int rc_dec_advance(rc_dec* d, uint64_t cum, uint64_t freq, uint64_t total);

int coder_decoder_freqs(const float* logits, size_t n, size_t tail, uint32_t* freq, uint64_t* total);
int decoder_lookup_freqs(const uint32_t* freq, size_t n, size_t tail, uint64_t total, uint64_t value,
                         uint32_t* symbol, ref_symbol_range* out);

#endif
