/*
 * oracle/ref_gguf.c -- GGUF v2/v3 reader of the CPU oracle (TEST
 * INFRASTRUCTURE, see ref.h).  Follows crates/det-gguf/src/lib.rs:156-528:
 * 32-byte aligned data section, duplicate-key / duplicate-name rejection,
 * UTF-8 validated strings, tensor ranges checked against the file and for
 * overlap.
 */
#include "ref_gguf.h"

#include <stdlib.h>
#include <string.h>

typedef struct {
    const uint8_t* b;
    size_t len, pos;
} rd;

static int rd_exact(rd* r, size_t n, const uint8_t** out) {
    if (n > r->len - r->pos) return GG_TRUNCATED;
    *out = r->b + r->pos;
    r->pos += n;
    return GG_OK;
}
static int rd_u8(rd* r, uint8_t* v) {
    const uint8_t* p;
    int st = rd_exact(r, 1, &p);
    if (!st) *v = p[0];
    return st;
}
static int rd_u16(rd* r, uint16_t* v) {
    const uint8_t* p;
    int st = rd_exact(r, 2, &p);
    if (!st) *v = (uint16_t)(p[0] | (p[1] << 8));
    return st;
}
static int rd_u32(rd* r, uint32_t* v) {
    const uint8_t* p;
    int st = rd_exact(r, 4, &p);
    if (!st) *v = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
    return st;
}
static int rd_u64(rd* r, uint64_t* v) {
    const uint8_t* p;
    int st = rd_exact(r, 8, &p);
    if (!st) {
        uint64_t x = 0;
        for (int i = 7; i >= 0; i--) x = (x << 8) | p[i];
        *v = x;
    }
    return st;
}
static int ensure_count(rd* r, uint64_t n, size_t min_bytes) {
    if (min_bytes && n > (uint64_t)(SIZE_MAX / min_bytes)) return GG_TRUNCATED;
    size_t need = (size_t)n * min_bytes;
    if (need > r->len - r->pos) return GG_TRUNCATED;
    return GG_OK;
}

/* str::from_utf8 acceptance: well-formed UTF-8, no overlongs, no surrogates */
static int utf8_ok(const uint8_t* s, size_t n) {
    size_t i = 0;
    while (i < n) {
        uint8_t c = s[i];
        if (c < 0x80) { i++; continue; }
        size_t k;
        uint32_t cp;
        if (c >= 0xc2 && c <= 0xdf) { k = 1; cp = c & 0x1f; }
        else if (c >= 0xe0 && c <= 0xef) { k = 2; cp = c & 0x0f; }
        else if (c >= 0xf0 && c <= 0xf4) { k = 3; cp = c & 0x07; }
        else return 0;
        if (i + k >= n) return 0;
        for (size_t j = 1; j <= k; j++) {
            uint8_t d = s[i + j];
            if ((d & 0xc0) != 0x80) return 0;
            cp = (cp << 6) | (d & 0x3f);
        }
        if (k == 2 && (cp < 0x800 || (cp >= 0xd800 && cp <= 0xdfff))) return 0;
        if (k == 3 && (cp < 0x10000 || cp > 0x10ffff)) return 0;
        i += k + 1;
    }
    return 1;
}

static int rd_string(rd* r, gg_str* out) {
    uint64_t n;
    int st = rd_u64(r, &n);
    if (st) return st;
    if (n > SIZE_MAX) return GG_TRUNCATED;
    const uint8_t* p;
    st = rd_exact(r, (size_t)n, &p);
    if (st) return st;
    if (!utf8_ok(p, (size_t)n)) return GG_INVALID_UTF8;
    out->ptr = p;
    out->len = n;
    return GG_OK;
}

static char* dup_str(gg_str s) {
    char* c = (char*)malloc((size_t)s.len + 1);
    if (!c) return NULL;
    memcpy(c, s.ptr, (size_t)s.len);
    c[s.len] = 0;
    return c;
}

static int elem_size(uint32_t t, size_t* sz) {
    switch (t) {
        case GV_U8: case GV_I8: case GV_BOOL: *sz = 1; return GG_OK;
        case GV_U16: case GV_I16: *sz = 2; return GG_OK;
        case GV_U32: case GV_I32: case GV_F32: *sz = 4; return GG_OK;
        case GV_STRING: case GV_U64: case GV_I64: case GV_F64: *sz = 8; return GG_OK;
        default: return GG_UNSUPPORTED_VALUE_TYPE;
    }
}

/* det-gguf lib.rs:372-475 */
static int read_value(rd* r, gg_kv* kv) {
    uint32_t ty;
    int st = rd_u32(r, &ty);
    if (st) return st;
    kv->type = ty;
    switch (ty) {
        case GV_U8: case GV_I8: { uint8_t v = 0; st = rd_u8(r, &v); kv->u = v; return st; }
        case GV_U16: case GV_I16: { uint16_t v = 0; st = rd_u16(r, &v); kv->u = v; return st; }
        case GV_U32: case GV_I32: { uint32_t v = 0; st = rd_u32(r, &v); kv->u = v; return st; }
        case GV_F32: {
            uint32_t v = 0;
            st = rd_u32(r, &v);
            float f;
            memcpy(&f, &v, 4);
            kv->u = v;
            kv->f = f;
            return st;
        }
        case GV_BOOL: {
            uint8_t v = 0;
            st = rd_u8(r, &v);
            if (st) return st;
            if (v > 1) return GG_INVALID_BOOL;
            kv->u = v;
            return GG_OK;
        }
        case GV_STRING: return rd_string(r, &kv->s);
        case GV_U64: case GV_I64: return rd_u64(r, &kv->u);
        case GV_F64: {
            st = rd_u64(r, &kv->u);
            memcpy(&kv->f, &kv->u, 8);
            return st;
        }
        case GV_ARRAY: {
            uint32_t et;
            uint64_t n;
            if ((st = rd_u32(r, &et))) return st;
            if ((st = rd_u64(r, &n))) return st;
            size_t esz;
            if ((st = elem_size(et, &esz))) return st;
            if ((st = ensure_count(r, n, esz))) return st;
            kv->elem_type = et;
            kv->count = n;
            if (et == GV_STRING) {
                kv->strs = (gg_str*)calloc(n ? (size_t)n : 1, sizeof(gg_str));
                if (!kv->strs) return GG_ALLOC;
                for (uint64_t i = 0; i < n; i++)
                    if ((st = rd_string(r, &kv->strs[i]))) return st;
                return GG_OK;
            }
            const uint8_t* p;
            if ((st = rd_exact(r, (size_t)n * esz, &p))) return st;
            if (et == GV_BOOL)
                for (uint64_t i = 0; i < n; i++)
                    if (p[i] > 1) return GG_INVALID_BOOL;
            kv->arr = p;
            return GG_OK;
        }
        default: return GG_UNSUPPORTED_VALUE_TYPE;
    }
}

int gg_type_size(uint32_t ty, uint64_t* ts, uint64_t* bs) {
    switch (ty) {
        case 0: *ts = 4; *bs = 1; return GG_OK;
        case 1: *ts = 2; *bs = 1; return GG_OK;
        case 2: *ts = 18; *bs = 32; return GG_OK;
        case 3: *ts = 20; *bs = 32; return GG_OK;
        case 6: *ts = 22; *bs = 32; return GG_OK;
        case 7: *ts = 24; *bs = 32; return GG_OK;
        case 8: *ts = 34; *bs = 32; return GG_OK;
        case 9: *ts = 40; *bs = 32; return GG_OK;
        case 10: *ts = 84; *bs = 256; return GG_OK;
        case 11: *ts = 110; *bs = 256; return GG_OK;
        case 12: *ts = 144; *bs = 256; return GG_OK;
        case 13: *ts = 176; *bs = 256; return GG_OK;
        case 14: *ts = 210; *bs = 256; return GG_OK;
        case 15: *ts = 292; *bs = 256; return GG_OK;
        default: return GG_UNSUPPORTED_TENSOR_TYPE;
    }
}

/* det-gguf lib.rs:341-352 */
int gg_element_count(const gg_tensor* t, uint64_t* n) {
    if (t->ndim == 0) return GG_INVALID_TENSOR_SHAPE;
    uint64_t c = 1;
    for (uint32_t i = 0; i < t->ndim; i++) {
        uint64_t d = t->dims[i];
        if (d == 0) return GG_INVALID_TENSOR_SHAPE;
        if (c > UINT64_MAX / d) return GG_INVALID_TENSOR_SHAPE;
        c *= d;
    }
    *n = c;
    return GG_OK;
}

/* det-gguf lib.rs:354-371 */
static int encoded_len(const gg_tensor* t, uint64_t* len) {
    uint64_t n, ts, bs;
    int st = gg_element_count(t, &n);
    if (st) return st;
    if (gg_type_size(t->ty, &ts, &bs)) return GG_UNSUPPORTED_TENSOR_TYPE;
    if (n % bs) return GG_INVALID_TENSOR_SHAPE;
    if ((n / bs) > UINT64_MAX / ts) return GG_INVALID_TENSOR_SHAPE;
    *len = (n / bs) * ts;
    return GG_OK;
}

typedef struct { uint64_t s, e; } range_t;
static int cmp_range(const void* a, const void* b) {
    const range_t* x = (const range_t*)a;
    const range_t* y = (const range_t*)b;
    return x->s < y->s ? -1 : (x->s > y->s ? 1 : 0);
}

/* det-gguf lib.rs:164-258 */
int gg_parse(const uint8_t* bytes, size_t len, gg_file* f) {
    memset(f, 0, sizeof *f);
    rd r = {bytes, len, 0};
    const uint8_t* magic;
    int st = rd_exact(&r, 4, &magic);
    if (st) return st;
    if (memcmp(magic, "GGUF", 4) != 0) return GG_BAD_MAGIC;
    if ((st = rd_u32(&r, &f->version))) return st;
    if (f->version != 2 && f->version != 3) return GG_UNSUPPORTED_VERSION;
    uint64_t n_tensors, n_kv;
    if ((st = rd_u64(&r, &n_tensors))) return st;
    if ((st = rd_u64(&r, &n_kv))) return st;
    /* each metadata entry needs at least 12 bytes (key length + type) */
    if ((st = ensure_count(&r, n_kv, 12))) return st;
    f->kv = (gg_kv*)calloc(n_kv ? (size_t)n_kv : 1, sizeof(gg_kv));
    if (!f->kv) return GG_ALLOC;
    for (uint64_t i = 0; i < n_kv; i++) {
        gg_str key;
        if ((st = rd_string(&r, &key))) { gg_free(f); return st; }
        gg_kv* kv = &f->kv[f->n_kv];
        kv->key = dup_str(key);
        f->n_kv++;
        if (!kv->key) { gg_free(f); return GG_ALLOC; }
        if ((st = read_value(&r, kv))) { gg_free(f); return st; }
        for (size_t j = 0; j + 1 < f->n_kv; j++)
            if (strcmp(f->kv[j].key, kv->key) == 0) { gg_free(f); return GG_DUPLICATE_METADATA_KEY; }
    }
    if ((st = ensure_count(&r, n_tensors, 24))) { gg_free(f); return st; }
    f->tensors = (gg_tensor*)calloc(n_tensors ? (size_t)n_tensors : 1, sizeof(gg_tensor));
    if (!f->tensors) { gg_free(f); return GG_ALLOC; }
    for (uint64_t i = 0; i < n_tensors; i++) {
        gg_tensor* t = &f->tensors[f->n_tensors];
        gg_str name;
        if ((st = rd_string(&r, &name))) { gg_free(f); return st; }
        t->name = dup_str(name);
        f->n_tensors++;
        if (!t->name) { gg_free(f); return GG_ALLOC; }
        if ((st = rd_u32(&r, &t->ndim))) { gg_free(f); return st; }
        if ((st = ensure_count(&r, t->ndim, 8))) { gg_free(f); return st; }
        t->dims = (uint64_t*)calloc(t->ndim ? t->ndim : 1, sizeof(uint64_t));
        if (!t->dims) { gg_free(f); return GG_ALLOC; }
        for (uint32_t d = 0; d < t->ndim; d++)
            if ((st = rd_u64(&r, &t->dims[d]))) { gg_free(f); return st; }
        if ((st = rd_u32(&r, &t->ty))) { gg_free(f); return st; }
        if ((st = rd_u64(&r, &t->offset))) { gg_free(f); return st; }
        for (size_t j = 0; j + 1 < f->n_tensors; j++)
            if (strcmp(f->tensors[j].name, t->name) == 0) { gg_free(f); return GG_DUPLICATE_TENSOR_NAME; }
    }
    size_t data_offset = (r.pos + 31) & ~(size_t)31;
    if (data_offset > len) { gg_free(f); return GG_TRUNCATED; }
    f->data_offset = data_offset;
    f->file_len = len;
    /* det-gguf lib.rs:231-258 */
    range_t* ranges = (range_t*)malloc(sizeof(range_t) * (f->n_tensors ? f->n_tensors : 1));
    if (!ranges) { gg_free(f); return GG_ALLOC; }
    for (size_t i = 0; i < f->n_tensors; i++) {
        uint64_t el;
        if ((st = encoded_len(&f->tensors[i], &el))) { free(ranges); gg_free(f); return st; }
        uint64_t s = (uint64_t)data_offset + f->tensors[i].offset;
        if (s < f->tensors[i].offset) { free(ranges); gg_free(f); return GG_INVALID_TENSOR_OFFSET; }
        uint64_t e = s + el;
        if (e < s) { free(ranges); gg_free(f); return GG_INVALID_TENSOR_OFFSET; }
        if (e > len) { free(ranges); gg_free(f); return GG_TRUNCATED; }
        ranges[i].s = s;
        ranges[i].e = e;
    }
    qsort(ranges, f->n_tensors, sizeof(range_t), cmp_range);
    for (size_t i = 0; i + 1 < f->n_tensors; i++)
        if (ranges[i].e > ranges[i + 1].s) { free(ranges); gg_free(f); return GG_INVALID_TENSOR_OFFSET; }
    free(ranges);
    return GG_OK;
}

void gg_free(gg_file* f) {
    for (size_t i = 0; i < f->n_kv; i++) {
        free(f->kv[i].key);
        free(f->kv[i].strs);
    }
    free(f->kv);
    for (size_t i = 0; i < f->n_tensors; i++) {
        free(f->tensors[i].name);
        free(f->tensors[i].dims);
    }
    free(f->tensors);
    memset(f, 0, sizeof *f);
}

/* Gguf::metadata_value (det-gguf lib.rs:278-281) */
const gg_kv* gg_find(const gg_file* f, const char* key) {
    for (size_t i = 0; i < f->n_kv; i++)
        if (strcmp(f->kv[i].key, key) == 0) return &f->kv[i];
    return NULL;
}

/* det-gguf lib.rs:291-297 */
int gg_u32(const gg_file* f, const char* key, uint32_t* out) {
    const gg_kv* kv = gg_find(f, key);
    if (!kv) return GG_METADATA_NOT_FOUND;
    if (kv->type == GV_U32) { *out = (uint32_t)kv->u; return GG_OK; }
    if (kv->type == GV_U64) {
        if (kv->u > UINT32_MAX) return GG_METADATA_TYPE_MISMATCH;
        *out = (uint32_t)kv->u;
        return GG_OK;
    }
    return GG_METADATA_TYPE_MISMATCH;
}

/* det-gguf lib.rs:299-305 */
int gg_f32(const gg_file* f, const char* key, float* out) {
    const gg_kv* kv = gg_find(f, key);
    if (!kv) return GG_METADATA_NOT_FOUND;
    if (kv->type == GV_F32 || kv->type == GV_F64) { *out = (float)kv->f; return GG_OK; }
    return GG_METADATA_TYPE_MISMATCH;
}

int gg_str_eq(const gg_file* f, const char* key, const char* want, int* eq) {
    const gg_kv* kv = gg_find(f, key);
    if (!kv) return GG_METADATA_NOT_FOUND;
    if (kv->type != GV_STRING) return GG_METADATA_TYPE_MISMATCH;
    size_t n = strlen(want);
    *eq = (kv->s.len == n && memcmp(kv->s.ptr, want, n) == 0);
    return GG_OK;
}

/* Gguf::tensor (det-gguf lib.rs:305-313): a duplicate name is an error */
int gg_find_tensor(const gg_file* f, const char* name, const gg_tensor** out) {
    for (size_t i = 0; i < f->n_tensors; i++)
        if (strcmp(f->tensors[i].name, name) == 0) { *out = &f->tensors[i]; return GG_OK; }
    return GG_TENSOR_NOT_FOUND;
}

/* Gguf::tensor_data (det-gguf lib.rs:314-338) */
int gg_tensor_data(const gg_file* f, const uint8_t* bytes, const char* name, const uint8_t** data, size_t* len) {
    const gg_tensor* t;
    int st = gg_find_tensor(f, name, &t);
    if (st) return st;
    uint64_t el;
    if ((st = encoded_len(t, &el))) return st;
    uint64_t s = (uint64_t)f->data_offset + t->offset, e = s + el;
    if (s < t->offset || e < s) return GG_INVALID_TENSOR_OFFSET;
    if (e > f->file_len) return GG_TRUNCATED;
    *data = bytes + s;
    *len = (size_t)el;
    return GG_OK;
}

/* gg_parse's status for a whole file (exported for the parser tests that
 * restate det-gguf lib.rs:586-730) */
int ref_gguf_parse_status(const uint8_t* bytes, size_t len) {
    gg_file f;
    int st = gg_parse(bytes, len, &f);
    if (!st) gg_free(&f);
    return st;
}
