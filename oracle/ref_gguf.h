/*
 * oracle/ref_gguf.h -- GGUF v2/v3 reader of the CPU oracle (TEST
 * INFRASTRUCTURE, see ref.h).  Follows crates/det-gguf/src/lib.rs:156-528.
 */
#ifndef DETLLM_ORACLE_REF_GGUF_H
#define DETLLM_ORACLE_REF_GGUF_H

#include <stddef.h>
#include <stdint.h>

enum {
    GG_OK = 0,
    GG_BAD_MAGIC = 1, GG_UNSUPPORTED_VERSION, GG_TRUNCATED, GG_UNSUPPORTED_VALUE_TYPE,
    GG_INVALID_UTF8, GG_INVALID_TENSOR_OFFSET, GG_INVALID_TENSOR_SHAPE, GG_TENSOR_NOT_FOUND,
    GG_METADATA_NOT_FOUND, GG_DUPLICATE_METADATA_KEY, GG_DUPLICATE_TENSOR_NAME, GG_INVALID_BOOL,
    GG_METADATA_TYPE_MISMATCH, GG_UNSUPPORTED_TENSOR_TYPE, GG_ALLOC
};

/* metadata value types (GGUF spec) */
enum { GV_U8 = 0, GV_I8, GV_U16, GV_I16, GV_U32, GV_I32, GV_F32, GV_BOOL, GV_STRING, GV_ARRAY,
       GV_U64, GV_I64, GV_F64 };

/* ggml tensor types used on this path */
enum { GT_F32 = 0, GT_F16 = 1, GT_Q4_0 = 2, GT_Q8_0 = 8, GT_Q4_K = 12, GT_Q6_K = 14 };

typedef struct {
    const uint8_t* ptr;
    uint64_t len;
} gg_str;

typedef struct {
    char* key;
    uint32_t type;      /* GV_* */
    uint32_t elem_type; /* for GV_ARRAY */
    uint64_t count;     /* array length or string length */
    uint64_t u;         /* integer payload (bit pattern) */
    double f;           /* F32 / F64 payload */
    gg_str s;           /* GV_STRING */
    const uint8_t* arr; /* raw little-endian array payload (non-string arrays) */
    gg_str* strs;       /* string array elements */
} gg_kv;

typedef struct {
    char* name;
    uint32_t ndim;
    uint64_t* dims;
    uint32_t ty;
    uint64_t offset;
} gg_tensor;

typedef struct {
    uint32_t version;
    size_t n_kv;
    gg_kv* kv;
    size_t n_tensors;
    gg_tensor* tensors;
    size_t data_offset;
    size_t file_len;
} gg_file;

int gg_parse(const uint8_t* bytes, size_t len, gg_file* out);
int ref_gguf_parse_status(const uint8_t* bytes, size_t len);
void gg_free(gg_file* f);
const gg_kv* gg_find(const gg_file* f, const char* key);
int gg_u32(const gg_file* f, const char* key, uint32_t* out);
int gg_f32(const gg_file* f, const char* key, float* out);
int gg_str_eq(const gg_file* f, const char* key, const char* want, int* eq); /* GG_OK + eq */
int gg_find_tensor(const gg_file* f, const char* name, const gg_tensor** out);
int gg_tensor_data(const gg_file* f, const uint8_t* bytes, const char* name, const uint8_t** data, size_t* len);
int gg_element_count(const gg_tensor* t, uint64_t* n);
int gg_type_size(uint32_t ty, uint64_t* type_size, uint64_t* block_size);

#endif
