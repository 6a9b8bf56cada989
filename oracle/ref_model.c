/*
 * oracle/ref_model.c -- det-model restated in C (TEST INFRASTRUCTURE, see
 * ref.h).  Follows crates/det-model/src/lib.rs: GGUF loading (:1035-1140,
 * :1498-1565, :1778-1953), the per-token forward (:1249-1400), RMSNorm
 * (:2053-2073), RoPE (:813-846, :2011-2051), attention (:2175-2418), SwiGLU
 * (:2420-2434), and the row-partitioned GEMV (:244-345) on a pthread pool.
 */
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <unistd.h>

#include "ref.h"
#include "ref_internal.h"
#include "ref_model.h"

/* ---- thread pool: det-model lib.rs:291-345 (contiguous row chunks) ------ */
typedef struct {
    pthread_t* th;
    int n; /* workers besides the caller */
    pthread_mutex_t mu;
    pthread_cond_t cv_start, cv_done;
    unsigned long gen;
    int pending;
    ref_range_fn fn;
    void* ctx;
    size_t total, chunk;
    int quit;
} pool_t;

static pool_t g_pool;
static int g_pool_up = 0;
static int g_threads = 0;
static pthread_mutex_t g_pool_init = PTHREAD_MUTEX_INITIALIZER;

typedef struct { int idx; } worker_arg;

static void* worker_main(void* p) {
    int idx = ((worker_arg*)p)->idx;
    free(p);
    unsigned long seen = 0;
    pthread_mutex_lock(&g_pool.mu);
    for (;;) {
        while (g_pool.gen == seen && !g_pool.quit) pthread_cond_wait(&g_pool.cv_start, &g_pool.mu);
        if (g_pool.quit) break;
        seen = g_pool.gen;
        ref_range_fn fn = g_pool.fn;
        void* ctx = g_pool.ctx;
        size_t b = (size_t)(idx + 1) * g_pool.chunk;
        size_t e = b + g_pool.chunk;
        if (e > g_pool.total) e = g_pool.total;
        pthread_mutex_unlock(&g_pool.mu);
        if (b < e) fn(ctx, b, e);
        pthread_mutex_lock(&g_pool.mu);
        if (--g_pool.pending == 0) pthread_cond_signal(&g_pool.cv_done);
    }
    pthread_mutex_unlock(&g_pool.mu);
    return NULL;
}

static void pool_stop(void) {
    if (!g_pool_up) return;
    pthread_mutex_lock(&g_pool.mu);
    g_pool.quit = 1;
    pthread_cond_broadcast(&g_pool.cv_start);
    pthread_mutex_unlock(&g_pool.mu);
    for (int i = 0; i < g_pool.n; i++) pthread_join(g_pool.th[i], NULL);
    free(g_pool.th);
    pthread_mutex_destroy(&g_pool.mu);
    pthread_cond_destroy(&g_pool.cv_start);
    pthread_cond_destroy(&g_pool.cv_done);
    g_pool_up = 0;
}

int ref_thread_count(void) {
    if (g_threads > 0) return g_threads;
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

void ref_set_threads(int threads) {
    pthread_mutex_lock(&g_pool_init);
    pool_stop();
    g_threads = threads > 0 ? threads : 0;
    pthread_mutex_unlock(&g_pool_init);
}

static void pool_start(int workers) {
    memset(&g_pool, 0, sizeof g_pool);
    pthread_mutex_init(&g_pool.mu, NULL);
    pthread_cond_init(&g_pool.cv_start, NULL);
    pthread_cond_init(&g_pool.cv_done, NULL);
    g_pool.th = (pthread_t*)calloc(workers > 0 ? (size_t)workers : 1, sizeof(pthread_t));
    for (int i = 0; i < workers; i++) {
        worker_arg* a = (worker_arg*)malloc(sizeof *a);
        a->idx = i;
        if (pthread_create(&g_pool.th[i], NULL, worker_main, a) != 0) {
            free(a);
            break;
        }
        g_pool.n++;
    }
    g_pool_up = 1;
}

void ref_parallel_for(size_t n, ref_range_fn fn, void* ctx) {
    int threads = ref_thread_count();
    if ((size_t)threads > n) threads = (int)(n ? n : 1);
    if (threads <= 1 || n < 2) {
        fn(ctx, 0, n);
        return;
    }
    pthread_mutex_lock(&g_pool_init);
    int want = ref_thread_count() - 1;
    if (!g_pool_up || g_pool.n != want) {
        pool_stop();
        pool_start(want);
    }
    size_t chunk = (n + (size_t)threads - 1) / (size_t)threads;
    size_t workers_needed = (n + chunk - 1) / chunk - 1; /* chunks beyond the caller's */
    if ((int)workers_needed > g_pool.n) workers_needed = (size_t)g_pool.n;
    pthread_mutex_lock(&g_pool.mu);
    g_pool.fn = fn;
    g_pool.ctx = ctx;
    g_pool.total = n;
    g_pool.chunk = chunk;
    g_pool.pending = g_pool.n;
    g_pool.gen++;
    pthread_cond_broadcast(&g_pool.cv_start);
    pthread_mutex_unlock(&g_pool.mu);
    fn(ctx, 0, chunk < n ? chunk : n);
    /* any chunk a missing worker could not take runs here */
    for (size_t c = (size_t)g_pool.n + 1; c * chunk < n; c++) {
        size_t e = (c + 1) * chunk;
        fn(ctx, c * chunk, e < n ? e : n);
    }
    pthread_mutex_lock(&g_pool.mu);
    while (g_pool.pending > 0) pthread_cond_wait(&g_pool.cv_done, &g_pool.mu);
    pthread_mutex_unlock(&g_pool.mu);
    pthread_mutex_unlock(&g_pool_init);
    (void)workers_needed;
}

/* ---- small helpers -------------------------------------------------------- */
static int finite_slice(const float* x, size_t n) {
    for (size_t i = 0; i < n; i++)
        if (!isfinite_f(x[i])) return 0;
    return 1;
}

int map_gguf_error(int gg) {
    if (gg == GG_METADATA_NOT_FOUND) return REF_ERR_MISSING_METADATA;
    if (gg == GG_ALLOC) return REF_ERR_ALLOC;
    return REF_ERR_GGUF;
}

/* det-model lib.rs:2053-2073 */
int ref_rmsnorm(const float* x, const float* w, size_t n, float eps, float* out) {
    if (n == 0) return REF_ERR_SHAPE;
    if (!finite_slice(x, n) || !finite_slice(w, n) || !isfinite_f(eps)) return REF_ERR_NONFINITE;
    float ss = ref_sum_squares_f32(x, n);
    float m = ss / (float)n;
    float r = 1.0f / sqrtf(m + eps);
    if (!isfinite_f(r)) return REF_ERR_NONFINITE;
    for (size_t i = 0; i < n; i++) {
        out[i] = (x[i] * r) * w[i];
        if (!isfinite_f(out[i])) return REF_ERR_NONFINITE;
    }
    return REF_OK;
}

/* ---- GEMV: det-model lib.rs:445-655 ------------------------------------------ */
typedef struct {
    const ref_matrix* m;
    const float* x;
    const ref_q8a_block* qa;
    const ref_q8k_block* qk;
    const float* act; /* Q4_K: a.d * a.q per element (row-independent) */
    float* out;
    volatile int err;
} gemv_ctx;

static int g_rowwise = 0;
void ref_set_rowwise_gemv(int on) { g_rowwise = on; }

static void gemv_range(void* p, size_t b, size_t e) {
    gemv_ctx* c = (gemv_ctx*)p;
    const ref_matrix* m = c->m;
    if (!g_rowwise && (m->type == GT_Q4_K || m->type == GT_Q6_K)) {
        /* REF_ROW_GROUP rows at a time, same per-row results (ref_quant.c) */
        for (size_t r = b; r < e && !c->err; r += REF_ROW_GROUP) {
            size_t n = e - r < REF_ROW_GROUP ? e - r : REF_ROW_GROUP;
            int st = m->type == GT_Q4_K
                         ? ref_dot_q4_k_rows((const ref_q4k_block*)m->data + r * m->blocks_per_row,
                                             m->blocks_per_row, n, c->act, c->out + r)
                         : ref_dot_q6_k_rows((const ref_q6k_block*)m->data + r * m->blocks_per_row,
                                             m->blocks_per_row, n, c->qk, c->out + r);
            if (st != REF_OK) {
                c->err = st;
                return;
            }
        }
        return;
    }
    for (size_t r = b; r < e && !c->err; r++) {
        float v = 0.0f;
        int st = REF_OK;
        switch (m->type) {
            case GT_F32: v = ref_dot_f32((const float*)m->data + r * m->cols, c->x, m->cols); break;
            case GT_Q8_0:
                st = ref_dot_q8_0_q8a((const ref_q8a_block*)m->data + r * m->blocks_per_row, c->qa,
                                      m->blocks_per_row, &v);
                break;
            case GT_Q4_0:
                st = ref_dot_q4_0_q8a((const ref_q4_0_block*)m->data + r * m->blocks_per_row, c->qa,
                                      m->blocks_per_row, &v);
                break;
            case GT_Q4_K:
                st = ref_dot_q4_k_q8a((const ref_q4k_block*)m->data + r * m->blocks_per_row, c->qa,
                                      m->blocks_per_row, &v);
                break;
            case GT_Q6_K:
                st = ref_dot_q6_k_q8k((const ref_q6k_block*)m->data + r * m->blocks_per_row, c->qk,
                                      m->blocks_per_row, &v);
                break;
        }
        if (st != REF_OK || !isfinite_f(v)) {
            c->err = st ? st : REF_ERR_NONFINITE;
            return;
        }
        c->out[r] = v;
    }
}

/* WeightMatrix::needs_q8a (det-model lib.rs:488-490) */
static int needs_q8a(const ref_matrix* m) {
    return m->type == GT_Q8_0 || m->type == GT_Q4_0 || m->type == GT_Q4_K;
}

/* gemv_with_optional_q8a_and_q8k_scratch (:550-606) when qa is given,
 * gemv_with_quant_scratch (:608-655) otherwise */
static int gemv(const ref_matrix* m, const float* x, const ref_q8a_block* shared_qa, ref_q8a_block* qa_scratch,
                ref_q8k_block* qk_scratch, float* out) {
    if (!finite_slice(x, m->cols)) return REF_ERR_NONFINITE;
    gemv_ctx c = {m, x, NULL, NULL, NULL, out, 0};
    float* act = NULL;
    if (needs_q8a(m)) {
        if (shared_qa) {
            c.qa = shared_qa;
        } else {
            int st = ref_quantize_q8a(x, m->cols, qa_scratch);
            if (st) return st;
            c.qa = qa_scratch;
        }
        if (m->type == GT_Q4_K && !g_rowwise) {
            act = (float*)malloc(m->cols * sizeof(float));
            if (!act) return REF_ERR_SHAPE;
            ref_q8a_dequant(c.qa, m->cols / 32, act);
            c.act = act;
        }
    } else if (m->type == GT_Q6_K) {
        int st = ref_quantize_q8k(x, m->cols, qk_scratch);
        if (st) return st;
        c.qk = qk_scratch;
    }
    ref_parallel_for(m->rows, gemv_range, &c);
    free(act);
    return c.err;
}

/* write_row_validated (:667-746): embedding row dequantisation */
static int write_row(const ref_matrix* m, size_t row, float* out) {
    size_t K = m->cols;
    switch (m->type) {
        case GT_F32: memcpy(out, (const float*)m->data + row * K, K * sizeof(float)); return REF_OK;
        case GT_Q8_0: {
            const ref_q8a_block* b = (const ref_q8a_block*)m->data + row * m->blocks_per_row;
            for (size_t i = 0; i < K; i++) {
                out[i] = b[i / 32].d * (float)b[i / 32].q[i % 32];
                if (!isfinite_f(out[i])) return REF_ERR_NONFINITE;
            }
            return REF_OK;
        }
        case GT_Q4_0: {
            const ref_q4_0_block* b = (const ref_q4_0_block*)m->data + row * m->blocks_per_row;
            for (size_t i = 0; i < K; i++) {
                const ref_q4_0_block* bb = &b[i / 32];
                size_t j = i % 32;
                uint8_t nib = j < 16 ? (bb->qs[j] & 0x0f) : (bb->qs[j - 16] >> 4);
                out[i] = bb->d * (float)((int)nib - 8);
                if (!isfinite_f(out[i])) return REF_ERR_NONFINITE;
            }
            return REF_OK;
        }
        case GT_Q4_K: {
            const ref_q4k_block* b = (const ref_q4k_block*)m->data + row * m->blocks_per_row;
            for (size_t i = 0; i < K; i++) {
                out[i] = ref_q4_k_value(&b[i / 256], i % 256);
                if (!isfinite_f(out[i])) return REF_ERR_NONFINITE;
            }
            return REF_OK;
        }
        case GT_Q6_K: {
            const ref_q6k_block* b = (const ref_q6k_block*)m->data + row * m->blocks_per_row;
            for (size_t i = 0; i < K; i++) {
                out[i] = ref_q6_k_value(&b[i / 256], i % 256);
                if (!isfinite_f(out[i])) return REF_ERR_NONFINITE;
            }
            return REF_OK;
        }
    }
    return REF_ERR_SHAPE;
}

/* ---- layer ops ------------------------------------------------------------------ */
/* add_optional_bias (:1982-1998), residual_add (:1967-1980) */
static int add_into(float* x, const float* b, size_t n) {
    if (!b) return REF_OK;
    if (!finite_slice(x, n) || !finite_slice(b, n)) return REF_ERR_NONFINITE;
    for (size_t i = 0; i < n; i++) {
        x[i] += b[i];
        if (!isfinite_f(x[i])) return REF_ERR_NONFINITE;
    }
    return REF_OK;
}

/* apply_rope (:2011-2051): the `half` rotation pairs of each of `heads`
 * heads of hd values (adjacent (2j, 2j+1) for pairing 0, split-half
 * (j, j+half) for pairing 1) with one position's table row; values past
 * the rotary pairs are left as they are */
static int rope_rotate(float* x, size_t heads, size_t hd, size_t half, int pairing, const float* cs_row,
                       const float* sn_row) {
    if (!finite_slice(x, heads * hd)) return REF_ERR_NONFINITE;
    for (size_t h = 0; h < heads; h++) {
        size_t base = h * hd;
        for (size_t j = 0; j < half; j++) {
            size_t a, b;
            if (pairing == 0) {
                a = base + 2 * j;
                b = a + 1;
            } else {
                a = base + j;
                b = base + j + half;
            }
            float x0 = x[a], x1 = x[b];
            float cs = cs_row[j], sn = sn_row[j];
            x[a] = x0 * cs - x1 * sn;
            x[b] = x0 * sn + x1 * cs;
            if (!isfinite_f(x[a]) || !isfinite_f(x[b])) return REF_ERR_NONFINITE;
        }
    }
    return REF_OK;
}

static int apply_rope(float* x, size_t heads, size_t hd, const ref_state* s, size_t pos) {
    const ref_config* c = &s->m->cfg;
    size_t half = c->rope_dim / 2;
    return rope_rotate(x, heads, hd, half, c->pairing, s->rope_cos + pos * half, s->rope_sin + pos * half);
}

/* exported for the op-order known answers (det-model :2752-2821) */
int ref_rope_rotate(float* x, size_t heads, size_t hd, size_t half, int pairing, const float* cs_row,
                    const float* sn_row) {
    if (hd == 0 || 2 * half > hd) return REF_ERR_SHAPE;
    return rope_rotate(x, heads, hd, half, pairing, cs_row, sn_row);
}

static inline float max_f(float a, float b) { return a > b ? a : (b != b ? a : b); }

/* softmax_in_place (:2361-2388) */
static int softmax(float* x, size_t n) {
    if (n == 0) return REF_ERR_SHAPE;
    float mx = -INFINITY;
    for (size_t i = 0; i < n; i++) {
        if (!isfinite_f(x[i])) return REF_ERR_NONFINITE;
        if (x[i] > mx) mx = x[i];
    }
    for (size_t i = 0; i < n; i++) {
        float t = x[i] - mx;
        x[i] = ref_expf(t > -88.0f ? t : -88.0f);
    }
    float z = ref_sum_f32(x, n);
    if (!isfinite_f(z) || z == 0.0f) return REF_ERR_NONFINITE;
    for (size_t i = 0; i < n; i++) {
        x[i] /= z;
        if (!isfinite_f(x[i])) return REF_ERR_NONFINITE;
    }
    return REF_OK;
}

/* exported for the op-order known answers (det-model :2462-2469) */
int ref_softmax(float* x, size_t n) { return softmax(x, n); }

/* attention_one_head (:2300-2333) with scores (:2335-2359) and weighted
 * value (:2390-2418) */
typedef struct {
    ref_state* s;
    size_t layer, pos;
    volatile int err;
} attn_ctx;

static void attn_range(void* p, size_t hb, size_t he) {
    attn_ctx* c = (attn_ctx*)p;
    ref_state* s = c->s;
    const ref_config* cfg = &s->m->cfg;
    size_t hd = cfg->head_dim, len = c->pos + 1;
    for (size_t head = hb; head < he && !c->err; head++) {
        size_t kvh = head / (cfg->n_head / cfg->n_head_kv);
        const float* kb = s->kcache + ((c->layer * cfg->n_head_kv + kvh) * s->n_ctx) * hd;
        const float* vb = s->vcache + ((c->layer * cfg->n_head_kv + kvh) * s->n_ctx) * hd;
        float* out = s->attn + head * hd;
        if (len == 1) {
            memcpy(out, vb, hd * sizeof(float));
            continue;
        }
        const float* q = s->q + head * hd;
        float* sc = s->scores + head * s->n_ctx;
        float* pr = s->probs + head * s->n_ctx;
        if (!finite_slice(q, hd) || !finite_slice(kb, len * hd)) { c->err = REF_ERR_NONFINITE; return; }
        for (size_t j = 0; j < len; j++) {
            sc[j] = ref_dot_f32(q, kb + j * hd, hd) * cfg->attn_scale;
            if (!isfinite_f(sc[j])) { c->err = REF_ERR_NONFINITE; return; }
        }
        memcpy(pr, sc, len * sizeof(float));
        int st = softmax(pr, len);
        if (st) { c->err = st; return; }
        if (!finite_slice(vb, len * hd)) { c->err = REF_ERR_NONFINITE; return; }
        for (size_t d = 0; d < hd; d++) out[d] = 0.0f;
        for (size_t j = 0; j < len; j++) {
            float pj = pr[j];
            const float* v = vb + j * hd;
            for (size_t d = 0; d < hd; d++) {
                out[d] += pj * v[d];
                if (!isfinite_f(out[d])) { c->err = REF_ERR_NONFINITE; return; }
            }
        }
    }
}

/* swiglu (:2420-2434) */
static int swiglu(const float* g, const float* u, float* out, size_t n) {
    if (!finite_slice(g, n) || !finite_slice(u, n)) return REF_ERR_NONFINITE;
    for (size_t i = 0; i < n; i++) {
        out[i] = ref_silu(g[i]) * u[i];
        if (!isfinite_f(out[i])) return REF_ERR_NONFINITE;
    }
    return REF_OK;
}

/* ---- state ------------------------------------------------------------------ */
/* RopeTables::llama (:813-846) */
static int build_rope(const ref_config* c, size_t positions, float* cs, float* sn) {
    size_t half = c->rope_dim / 2;
    /* phase = pos * omega with omega <= 1; the restated rem_pio2 covers
     * |phase| < 2^20 * pi/2, so longer tables are rejected here. */
    if (positions > (1u << 20)) return REF_ERR_SHAPE;
    double ln_base = ref_ln_f64((double)c->rope_base);
    for (size_t pos = 0; pos < positions; pos++) {
        for (size_t j = 0; j < half; j++) {
            double exponent = -((double)(2 * j)) / (double)c->rope_dim;
            double omega = ref_exp_f64(exponent * ln_base);
            double phi = (double)pos * omega;
            float cv = (float)ref_cos_f64(phi);
            float sv = (float)ref_sin_f64(phi);
            if (!isfinite_f(cv) || !isfinite_f(sv)) return REF_ERR_NONFINITE;
            cs[pos * half + j] = cv;
            sn[pos * half + j] = sv;
        }
    }
    return REF_OK;
}

/* RopeTables::llama + KvCache::new + ForwardWorkspace (det-model lib.rs:813-846, 849, 963-1031) */
int ref_state_init(ref_state* s, const ref_model* m, size_t n_ctx) {
    memset(s, 0, sizeof *s);
    const ref_config* c = &m->cfg;
    if (n_ctx == 0 || n_ctx > c->ctx) return REF_ERR_SHAPE;
    s->m = m;
    s->n_ctx = n_ctx;
    s->positions = n_ctx;
    size_t half = c->rope_dim / 2, hd = c->head_dim;
    size_t kv = c->block_count * c->n_head_kv * n_ctx * hd;
    s->rope_cos = (float*)malloc(sizeof(float) * n_ctx * half);
    s->rope_sin = (float*)malloc(sizeof(float) * n_ctx * half);
    s->kcache = (float*)calloc(kv, sizeof(float));
    s->vcache = (float*)calloc(kv, sizeof(float));
    s->x = (float*)calloc(c->d, sizeof(float));
    s->h = (float*)calloc(c->d, sizeof(float));
    s->tmp_d = (float*)calloc(c->d, sizeof(float));
    s->q = (float*)calloc(c->n_head * hd, sizeof(float));
    s->attn = (float*)calloc(c->n_head * hd, sizeof(float));
    s->k = (float*)calloc(c->n_head_kv * hd, sizeof(float));
    s->v = (float*)calloc(c->n_head_kv * hd, sizeof(float));
    s->scores = (float*)calloc(c->n_head * n_ctx, sizeof(float));
    s->probs = (float*)calloc(c->n_head * n_ctx, sizeof(float));
    s->gate = (float*)calloc(c->d_ff, sizeof(float));
    s->up = (float*)calloc(c->d_ff, sizeof(float));
    s->ff = (float*)calloc(c->d_ff, sizeof(float));
    size_t maxk = c->d > c->d_ff ? c->d : c->d_ff;
    if (c->n_head * hd > maxk) maxk = c->n_head * hd;
    s->q8a = (ref_q8a_block*)calloc(maxk / 32 + 1, sizeof(ref_q8a_block));
    s->q8k = (ref_q8k_block*)calloc(maxk / 256 + 1, sizeof(ref_q8k_block));
    s->logits = (float*)calloc(m->vocab, sizeof(float));
    if (!s->rope_cos || !s->rope_sin || !s->kcache || !s->vcache || !s->x || !s->h || !s->tmp_d || !s->q ||
        !s->attn || !s->k || !s->v || !s->scores || !s->probs || !s->gate || !s->up || !s->ff || !s->q8a ||
        !s->q8k || !s->logits) {
        ref_state_free(s);
        return REF_ERR_ALLOC;
    }
    int st = build_rope(c, n_ctx, s->rope_cos, s->rope_sin);
    if (st) ref_state_free(s);
    return st;
}

void ref_state_reset_cache(ref_state* s) {
    const ref_config* c = &s->m->cfg;
    size_t kv = c->block_count * c->n_head_kv * s->n_ctx * c->head_dim;
    memset(s->kcache, 0, kv * sizeof(float));
    memset(s->vcache, 0, kv * sizeof(float));
    memset(s->logits, 0, s->m->vocab * sizeof(float));
}

void ref_state_free(ref_state* s) {
    free(s->rope_cos); free(s->rope_sin); free(s->kcache); free(s->vcache);
    free(s->x); free(s->h); free(s->tmp_d); free(s->q); free(s->attn); free(s->k); free(s->v);
    free(s->scores); free(s->probs); free(s->gate); free(s->up); free(s->ff);
    free(s->q8a); free(s->q8k); free(s->logits);
    memset(s, 0, sizeof *s);
}

/* ---- forward_one_with_workspace (:1249-1400) ------------------------------- */
int ref_forward_one(ref_state* s, size_t token, size_t pos) {
    const ref_model* m = s->m;
    const ref_config* c = &m->cfg;
    size_t hd = c->head_dim;
    if (pos >= s->n_ctx || token >= m->tok_embd.rows) return REF_ERR_SHAPE;
    int st = write_row(&m->tok_embd, token, s->x);
    if (st) return st;
    for (size_t l = 0; l < c->block_count; l++) {
        const ref_layer* L = &m->layers[l];
        if ((st = ref_rmsnorm(s->x, L->attn_norm, c->d, c->eps, s->h))) return st;
        const ref_q8a_block* hq = NULL;
        if (needs_q8a(&L->wq) || needs_q8a(&L->wk) || needs_q8a(&L->wv)) {
            if ((st = ref_quantize_q8a(s->h, c->d, s->q8a))) return st;
            hq = s->q8a;
        }
        if ((st = gemv(&L->wq, s->h, hq, s->q8a, s->q8k, s->q))) return st;
        if ((st = add_into(s->q, L->q_bias, c->n_head * hd))) return st;
        if ((st = gemv(&L->wk, s->h, hq, s->q8a, s->q8k, s->k))) return st;
        if ((st = add_into(s->k, L->k_bias, c->n_head_kv * hd))) return st;
        if ((st = gemv(&L->wv, s->h, hq, s->q8a, s->q8k, s->v))) return st;
        if ((st = add_into(s->v, L->v_bias, c->n_head_kv * hd))) return st;
        if ((st = apply_rope(s->q, c->n_head, hd, s, pos))) return st;
        if ((st = apply_rope(s->k, c->n_head_kv, hd, s, pos))) return st;
        /* KvCache::store (:883-913) */
        if (!finite_slice(s->k, c->n_head_kv * hd) || !finite_slice(s->v, c->n_head_kv * hd)) return REF_ERR_NONFINITE;
        for (size_t kh = 0; kh < c->n_head_kv; kh++) {
            size_t off = ((l * c->n_head_kv + kh) * s->n_ctx + pos) * hd;
            memcpy(s->kcache + off, s->k + kh * hd, hd * sizeof(float));
            memcpy(s->vcache + off, s->v + kh * hd, hd * sizeof(float));
        }
        attn_ctx ac = {s, l, pos, 0};
        size_t work = c->n_head * (pos + 1) * hd;
        if (work >= 32768) ref_parallel_for(c->n_head, attn_range, &ac);
        else attn_range(&ac, 0, c->n_head);
        if (ac.err) return ac.err;
        /* wo quantises its own input (gemv_with_quant_scratch) */
        if ((st = gemv(&L->wo, s->attn, NULL, s->q8a, s->q8k, s->tmp_d))) return st;
        if ((st = add_into(s->x, s->tmp_d, c->d))) return st;
        if ((st = ref_rmsnorm(s->x, L->ffn_norm, c->d, c->eps, s->h))) return st;
        hq = NULL;
        if (needs_q8a(&L->w_gate) || needs_q8a(&L->w_up)) {
            if ((st = ref_quantize_q8a(s->h, c->d, s->q8a))) return st;
            hq = s->q8a;
        }
        if ((st = gemv(&L->w_gate, s->h, hq, s->q8a, s->q8k, s->gate))) return st;
        if ((st = gemv(&L->w_up, s->h, hq, s->q8a, s->q8k, s->up))) return st;
        if ((st = swiglu(s->gate, s->up, s->ff, c->d_ff))) return st;
        if ((st = gemv(&L->w_down, s->ff, NULL, s->q8a, s->q8k, s->tmp_d))) return st;
        if ((st = add_into(s->x, s->tmp_d, c->d))) return st;
    }
    if ((st = ref_rmsnorm(s->x, m->output_norm, c->d, c->eps, s->h))) return st;
    return gemv(&m->output, s->h, NULL, s->q8a, s->q8k, s->logits);
}

/* ---- loading --------------------------------------------------------------------- */
/* read_f32_vector and the dense (F32 / F16) matrix readers (det-model lib.rs:1694, 1793-1795) */
static int read_dense(const gg_file* g, const uint8_t* bytes, const char* name, const gg_tensor* t, float** out) {
    const uint8_t* data;
    size_t len;
    int gs = gg_tensor_data(g, bytes, name, &data, &len);
    if (gs) return REF_ERR_GGUF;
    uint64_t n;
    if (gg_element_count(t, &n)) return REF_ERR_SHAPE;
    float* v = (float*)malloc(sizeof(float) * (n ? n : 1));
    if (!v) return REF_ERR_ALLOC;
    if (t->ty == GT_F32) {
        if (len != n * 4) { free(v); return REF_ERR_SHAPE; }
        for (uint64_t i = 0; i < n; i++) {
            uint32_t b = (uint32_t)data[4 * i] | ((uint32_t)data[4 * i + 1] << 8) | ((uint32_t)data[4 * i + 2] << 16) |
                         ((uint32_t)data[4 * i + 3] << 24);
            v[i] = u2f(b);
            if (!isfinite_f(v[i])) { free(v); return REF_ERR_NONFINITE; }
        }
    } else if (t->ty == GT_F16) {
        if (len != n * 2) { free(v); return REF_ERR_SHAPE; }
        for (uint64_t i = 0; i < n; i++) {
            uint16_t b = (uint16_t)(data[2 * i] | (data[2 * i + 1] << 8));
            if ((b & 0x7c00) == 0x7c00) { free(v); return REF_ERR_NONFINITE; }
            v[i] = ref_f16_to_f32(b);
        }
    } else {
        free(v);
        return REF_ERR_UNSUPPORTED_TENSOR_TYPE;
    }
    *out = v;
    return REF_OK;
}

/* read_f32_vector (:1656-1668) / read_optional_f32_vector (:1670-1681) */
static int read_vector(const gg_file* g, const uint8_t* bytes, const char* name, size_t len, float** out,
                       int optional) {
    const gg_tensor* t;
    int gs = gg_find_tensor(g, name, &t);
    if (gs == GG_TENSOR_NOT_FOUND && optional) { *out = NULL; return REF_OK; }
    if (gs) return REF_ERR_GGUF;
    if (t->ndim != 1 || t->dims[0] != len) return REF_ERR_SHAPE;
    return read_dense(g, bytes, name, t, out);
}

static uint16_t le16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* read_weight_matrix (:1778-1810) and the per-type readers (:1812-1953) */
static int read_matrix(const gg_file* g, const uint8_t* bytes, const char* name, size_t rows, size_t cols,
                       ref_matrix* m) {
    memset(m, 0, sizeof *m);
    const gg_tensor* t;
    if (gg_find_tensor(g, name, &t)) return REF_ERR_GGUF;
    if (t->ndim != 2 || t->dims[0] != cols || t->dims[1] != rows) return REF_ERR_SHAPE;
    m->rows = rows;
    m->cols = cols;
    m->src_type = t->ty;
    m->owned = 1;
    if (t->ty == GT_F32 || t->ty == GT_F16) {
        m->type = GT_F32;
        float* v;
        int st = read_dense(g, bytes, name, t, &v);
        if (st) return st;
        if (rows == 0 || cols == 0) { free(v); return REF_ERR_SHAPE; }
        m->data = v;
        return REF_OK;
    }
    size_t bs, ts;
    if (t->ty == GT_Q8_0) { bs = 32; ts = 34; }
    else if (t->ty == GT_Q4_0) { bs = 32; ts = 18; }
    else if (t->ty == GT_Q4_K) { bs = 256; ts = 144; }
    else if (t->ty == GT_Q6_K) { bs = 256; ts = 210; }
    else return REF_ERR_UNSUPPORTED_TENSOR_TYPE;
    if (cols % bs) return REF_ERR_SHAPE;
    m->type = t->ty;
    m->blocks_per_row = cols / bs;
    size_t nb = rows * m->blocks_per_row;
    const uint8_t* data;
    size_t len;
    if (gg_tensor_data(g, bytes, name, &data, &len)) return REF_ERR_GGUF;
    if (len != nb * ts) return REF_ERR_SHAPE;
    if (t->ty == GT_Q8_0) {
        ref_q8a_block* b = (ref_q8a_block*)malloc(sizeof(*b) * (nb ? nb : 1));
        if (!b) return REF_ERR_ALLOC;
        for (size_t i = 0; i < nb; i++) {
            const uint8_t* p = data + i * ts;
            b[i].d = ref_f16_to_f32(le16(p));
            if (!isfinite_f(b[i].d)) { free(b); return REF_ERR_NONFINITE; }
            memcpy(b[i].q, p + 2, 32);
        }
        m->data = b;
    } else if (t->ty == GT_Q4_0) {
        ref_q4_0_block* b = (ref_q4_0_block*)malloc(sizeof(*b) * (nb ? nb : 1));
        if (!b) return REF_ERR_ALLOC;
        for (size_t i = 0; i < nb; i++) {
            const uint8_t* p = data + i * ts;
            b[i].d = ref_f16_to_f32(le16(p));
            if (!isfinite_f(b[i].d)) { free(b); return REF_ERR_NONFINITE; }
            memcpy(b[i].qs, p + 2, 16);
        }
        m->data = b;
    } else if (t->ty == GT_Q4_K) {
        ref_q4k_block* b = (ref_q4k_block*)malloc(sizeof(*b) * (nb ? nb : 1));
        if (!b) return REF_ERR_ALLOC;
        for (size_t i = 0; i < nb; i++) {
            const uint8_t* p = data + i * ts;
            b[i].d = ref_f16_to_f32(le16(p));
            b[i].dmin = ref_f16_to_f32(le16(p + 2));
            if (!isfinite_f(b[i].d) || !isfinite_f(b[i].dmin)) { free(b); return REF_ERR_NONFINITE; }
            memcpy(b[i].scales, p + 4, 12);
            memcpy(b[i].qs, p + 16, 128);
        }
        m->data = b;
    } else {
        ref_q6k_block* b = (ref_q6k_block*)malloc(sizeof(*b) * (nb ? nb : 1));
        if (!b) return REF_ERR_ALLOC;
        for (size_t i = 0; i < nb; i++) {
            const uint8_t* p = data + i * ts;
            memcpy(b[i].ql, p, 128);
            memcpy(b[i].qh, p + 128, 64);
            memcpy(b[i].scales, p + 192, 16);
            b[i].d = ref_f16_to_f32(le16(p + 208));
            if (!isfinite_f(b[i].d)) { free(b); return REF_ERR_NONFINITE; }
        }
        m->data = b;
    }
    if (rows == 0 || cols == 0) return REF_ERR_SHAPE;
    return REF_OK;
}

static int opt_u32(const gg_file* g, const char* key, uint32_t* v, int* present) {
    int gs = gg_u32(g, key, v);
    if (gs == GG_METADATA_NOT_FOUND) { *present = 0; return REF_OK; }
    if (gs) return map_gguf_error(gs);
    *present = 1;
    return REF_OK;
}
static int opt_f32(const gg_file* g, const char* key, float* v, int* present) {
    int gs = gg_f32(g, key, v);
    if (gs == GG_METADATA_NOT_FOUND) { *present = 0; return REF_OK; }
    if (gs) return map_gguf_error(gs);
    *present = 1;
    return REF_OK;
}
/* optional_bool (:1605-1612) */
static int opt_bool(const gg_file* g, const char* key, int* v, int* present) {
    const gg_kv* kv = gg_find(g, key);
    if (!kv) { *present = 0; return REF_OK; }
    if (kv->type != GV_BOOL) return REF_ERR_GGUF;
    *present = 1;
    *v = (int)kv->u;
    return REF_OK;
}
/* reject_nonzero_optional_f32 (:1628-1643) */
static int reject_nonzero_f32(const gg_file* g, const char* key) {
    const gg_kv* kv = gg_find(g, key);
    if (!kv) return REF_OK;
    if (kv->type != GV_F32 && kv->type != GV_F64) return REF_ERR_GGUF;
    double v = kv->f;
    if (!(v - v == 0.0)) return REF_ERR_SHAPE;
    if (v != 0.0) return REF_ERR_UNSUPPORTED_FEATURE;
    return REF_OK;
}

/* LlamaConfig::from_gguf (:1498-1565) + validate (:1572-1596) */
static int config_from_gguf(const gg_file* g, ref_config* c) {
    const gg_kv* arch = gg_find(g, "general.architecture");
    if (!arch) return REF_ERR_MISSING_METADATA;
    if (arch->type != GV_STRING) return REF_ERR_GGUF;
    char prefix[16];
    if (arch->s.len == 5 && memcmp(arch->s.ptr, "llama", 5) == 0) { strcpy(prefix, "llama"); c->pairing = 0; }
    else if (arch->s.len == 5 && memcmp(arch->s.ptr, "qwen2", 5) == 0) { strcpy(prefix, "qwen2"); c->pairing = 1; }
    else return REF_ERR_UNSUPPORTED_ARCH;
    char key[128];
#define KEY(s) (snprintf(key, sizeof key, "%s.%s", prefix, s), key)
    uint32_t v = 0;
    int st, present = 0, gs;
    if ((gs = gg_u32(g, KEY("attention.head_count"), &v))) return map_gguf_error(gs);
    c->n_head = v;
    if ((st = opt_u32(g, KEY("attention.head_count_kv"), &v, &present))) return st;
    c->n_head_kv = present ? v : c->n_head;
    if ((gs = gg_u32(g, KEY("embedding_length"), &v))) return map_gguf_error(gs);
    c->d = v;
    if (c->n_head == 0 || c->d % c->n_head) return REF_ERR_SHAPE;
    if ((st = opt_u32(g, KEY("embedding_length_out"), &v, &present))) return st;
    if (present && v != c->d) return REF_ERR_UNSUPPORTED_FEATURE;
    int b;
    if ((st = opt_bool(g, KEY("attention.causal"), &b, &present))) return st;
    if (present && !b) return REF_ERR_UNSUPPORTED_FEATURE;
    const gg_kv* rs = gg_find(g, KEY("rope.scaling.type"));
    if (rs) {
        if (rs->type != GV_STRING) return REF_ERR_GGUF;
        if (!(rs->s.len == 4 && memcmp(rs->s.ptr, "none", 4) == 0)) return REF_ERR_UNSUPPORTED_ROPE_SCALING;
    }
    if ((st = opt_bool(g, KEY("use_parallel_residual"), &b, &present))) return st;
    if (present && b) return REF_ERR_UNSUPPORTED_FEATURE;
    if ((st = opt_u32(g, KEY("attention.sliding_window"), &v, &present))) return st;
    if (present && v != 0) return REF_ERR_UNSUPPORTED_FEATURE;
    static const char* zero_keys[] = {"attention.max_alibi_bias", "attention.clamp_kqv", "attention.value_scale",
                                      "attn_logit_softcapping", "final_logit_softcapping", "logit_scale",
                                      "embedding_scale", "residual_scale"};
    for (size_t i = 0; i < sizeof zero_keys / sizeof zero_keys[0]; i++)
        if ((st = reject_nonzero_f32(g, KEY(zero_keys[i])))) return st;
    c->head_dim = c->d / c->n_head;
    static const char* len_keys[] = {"attention.key_length", "attention.value_length"};
    for (int i = 0; i < 2; i++) {
        if ((st = opt_u32(g, KEY(len_keys[i]), &v, &present))) return st;
        if (present && v != c->head_dim) return REF_ERR_UNSUPPORTED_HEAD_LEN;
    }
    float f;
    if ((st = opt_f32(g, KEY("attention.scale"), &f, &present))) return st;
    c->attn_scale = present ? f : 1.0f / sqrtf((float)c->head_dim);
    if ((gs = gg_u32(g, KEY("block_count"), &v))) return map_gguf_error(gs);
    c->block_count = v;
    if ((gs = gg_u32(g, KEY("feed_forward_length"), &v))) return map_gguf_error(gs);
    c->d_ff = v;
    if ((gs = gg_f32(g, KEY("attention.layer_norm_rms_epsilon"), &f))) return map_gguf_error(gs);
    c->eps = f;
    if ((st = opt_f32(g, KEY("rope.freq_base"), &f, &present))) return st;
    c->rope_base = present ? f : 10000.0f;
    if ((st = opt_u32(g, KEY("rope.dimension_count"), &v, &present))) return st;
    c->rope_dim = present ? v : c->head_dim;
    if ((gs = gg_u32(g, KEY("context_length"), &v))) return map_gguf_error(gs);
    c->ctx = v;
#undef KEY
    if (c->block_count == 0 || c->d == 0 || c->d_ff == 0 || c->n_head == 0 || c->n_head_kv == 0 || c->ctx == 0 ||
        c->n_head % c->n_head_kv || c->rope_dim == 0 || c->rope_dim % 2 || !isfinite_f(c->eps) || c->eps <= 0.0f ||
        !isfinite_f(c->attn_scale) || c->attn_scale <= 0.0f || !isfinite_f(c->rope_base) || c->rope_base <= 0.0f)
        return REF_ERR_SHAPE;
    if (c->rope_dim > c->head_dim) return REF_ERR_SHAPE;
    return REF_OK;
}

/* vocab_size (:1620-1648) */
static int vocab_size(const gg_file* g, size_t* out) {
    const gg_kv* arch = gg_find(g, "general.architecture");
    if (!arch) return REF_ERR_MISSING_METADATA;
    if (arch->type != GV_STRING) return REF_ERR_GGUF;
    char key[128];
    snprintf(key, sizeof key, "%.*s.vocab_size", (int)arch->s.len, (const char*)arch->s.ptr);
    const char* keys[2] = {key, "llama.vocab_size"};
    for (int i = 0; i < 2; i++) {
        uint32_t v;
        int gs = gg_u32(g, keys[i], &v);
        if (gs == GG_OK) { *out = v; return REF_OK; }
        if (gs != GG_METADATA_NOT_FOUND) return map_gguf_error(gs);
    }
    const gg_kv* toks = gg_find(g, "tokenizer.ggml.tokens");
    if (toks) {
        if (toks->type != GV_ARRAY || toks->elem_type != GV_STRING) return REF_ERR_GGUF;
        *out = (size_t)toks->count;
        return REF_OK;
    }
    const gg_tensor* t;
    if (gg_find_tensor(g, "token_embd.weight", &t)) return REF_ERR_GGUF;
    if (t->ndim == 2) { *out = (size_t)t->dims[1]; return REF_OK; }
    return REF_ERR_MISSING_METADATA;
}

static void matrix_free(ref_matrix* m) {
    if (m->owned) free(m->data);
    m->data = NULL;
}

void ref_model_free(ref_model* m) {
    if (!m) return;
    matrix_free(&m->tok_embd);
    if (m->layers) {
        for (size_t l = 0; l < m->cfg.block_count; l++) {
            ref_layer* L = &m->layers[l];
            free(L->attn_norm); free(L->ffn_norm); free(L->q_bias); free(L->k_bias); free(L->v_bias);
            matrix_free(&L->wq); matrix_free(&L->wk); matrix_free(&L->wv); matrix_free(&L->wo);
            matrix_free(&L->w_gate); matrix_free(&L->w_up); matrix_free(&L->w_down);
        }
        free(m->layers);
    }
    free(m->output_norm);
    if (!m->tied) matrix_free(&m->output);
    free(m);
}

/* F32Llama::from_gguf (:1035-1140) */
int ref_model_load_gguf(const gg_file* g, const uint8_t* bytes, ref_model** out) {
    ref_model* m = (ref_model*)calloc(1, sizeof *m);
    if (!m) return REF_ERR_ALLOC;
    int st = config_from_gguf(g, &m->cfg);
    if (st) { free(m); return st; }
    ref_config* c = &m->cfg;
    size_t V = 0;
    if ((st = vocab_size(g, &V))) { free(m); return st; }
    m->layers = (ref_layer*)calloc(c->block_count, sizeof(ref_layer));
    if (!m->layers) { free(m); return REF_ERR_ALLOC; }
    size_t hd = c->head_dim;
    if ((st = read_matrix(g, bytes, "token_embd.weight", V, c->d, &m->tok_embd))) goto fail;
    for (size_t l = 0; l < c->block_count; l++) {
        ref_layer* L = &m->layers[l];
        char name[96];
#define NM(s) (snprintf(name, sizeof name, "blk.%zu.%s", l, s), name)
        if ((st = read_vector(g, bytes, NM("attn_norm.weight"), c->d, &L->attn_norm, 0))) goto fail;
        if ((st = read_matrix(g, bytes, NM("attn_q.weight"), c->n_head * hd, c->d, &L->wq))) goto fail;
        if ((st = read_vector(g, bytes, NM("attn_q.bias"), c->n_head * hd, &L->q_bias, 1))) goto fail;
        if ((st = read_matrix(g, bytes, NM("attn_k.weight"), c->n_head_kv * hd, c->d, &L->wk))) goto fail;
        if ((st = read_vector(g, bytes, NM("attn_k.bias"), c->n_head_kv * hd, &L->k_bias, 1))) goto fail;
        if ((st = read_matrix(g, bytes, NM("attn_v.weight"), c->n_head_kv * hd, c->d, &L->wv))) goto fail;
        if ((st = read_vector(g, bytes, NM("attn_v.bias"), c->n_head_kv * hd, &L->v_bias, 1))) goto fail;
        if ((st = read_matrix(g, bytes, NM("attn_output.weight"), c->d, c->n_head * hd, &L->wo))) goto fail;
        if ((st = read_vector(g, bytes, NM("ffn_norm.weight"), c->d, &L->ffn_norm, 0))) goto fail;
        if ((st = read_matrix(g, bytes, NM("ffn_gate.weight"), c->d_ff, c->d, &L->w_gate))) goto fail;
        if ((st = read_matrix(g, bytes, NM("ffn_up.weight"), c->d_ff, c->d, &L->w_up))) goto fail;
        if ((st = read_matrix(g, bytes, NM("ffn_down.weight"), c->d, c->d_ff, &L->w_down))) goto fail;
#undef NM
    }
    if ((st = read_vector(g, bytes, "output_norm.weight", c->d, &m->output_norm, 0))) goto fail;
    {
        const gg_tensor* t;
        int gs = gg_find_tensor(g, "output.weight", &t);
        if (gs == GG_OK) {
            if ((st = read_matrix(g, bytes, "output.weight", m->tok_embd.rows, c->d, &m->output))) goto fail;
        } else if (gs == GG_TENSOR_NOT_FOUND) {
            m->output = m->tok_embd;
            m->output.owned = 0;
            m->tied = 1;
        } else {
            st = REF_ERR_GGUF;
            goto fail;
        }
    }
    m->vocab = m->output.rows;
    *out = m;
    return REF_OK;
fail:
    ref_model_free(m);
    return st;
}

/* ---- public entry points ------------------------------------------------------- */
/* F32Llama::from_gguf (det-model lib.rs:1035) */
int ref_model_load(const uint8_t* gguf, size_t len, ref_model** out) {
    gg_file g;
    int gs = gg_parse(gguf, len, &g);
    if (gs) return REF_ERR_GGUF;
    int st = ref_model_load_gguf(&g, gguf, out);
    gg_free(&g);
    return st;
}

int ref_model_get_info(const ref_model* m, ref_model_info* info) {
    memset(info, 0, sizeof *info);
    const ref_config* c = &m->cfg;
    info->block_count = (uint32_t)c->block_count;
    info->embedding_length = (uint32_t)c->d;
    info->feed_forward_length = (uint32_t)c->d_ff;
    info->head_count = (uint32_t)c->n_head;
    info->head_count_kv = (uint32_t)c->n_head_kv;
    info->head_dim = (uint32_t)c->head_dim;
    info->rope_dimension_count = (uint32_t)c->rope_dim;
    info->rope_pairing = (uint32_t)c->pairing;
    info->context_length = (uint32_t)c->ctx;
    info->vocab = (uint32_t)m->vocab;
    info->rms_epsilon = c->eps;
    info->attention_scale = c->attn_scale;
    info->rope_freq_base = c->rope_base;
    const ref_layer* L = &m->layers[0];
    info->weight_types[0] = m->tok_embd.src_type;
    info->weight_types[1] = L->wq.src_type;
    info->weight_types[2] = L->wk.src_type;
    info->weight_types[3] = L->wv.src_type;
    info->weight_types[4] = L->wo.src_type;
    info->weight_types[5] = L->w_gate.src_type;
    info->weight_types[6] = L->w_up.src_type;
    info->weight_types[7] = L->w_down.src_type;
    info->weight_types[8] = m->output.src_type;
    info->has_qkv_bias = L->q_bias != NULL;
    info->tied_output = (uint32_t)m->tied;
    return REF_OK;
}

/* visit_logits_for_tokens_chunked (:1435-1465): positions 0..n-1 in one
 * context; the chunk size never changes the arithmetic. */
int ref_logits(const ref_model* m, const uint32_t* tokens, size_t n, float* out) {
    if (n == 0 || n > m->cfg.ctx) return REF_ERR_SHAPE;
    for (size_t i = 0; i < n; i++)
        if (tokens[i] >= m->tok_embd.rows) return REF_ERR_SHAPE;
    ref_state s;
    int st = ref_state_init(&s, m, n);
    if (st) return st;
    for (size_t i = 0; i < n && !st; i++) {
        st = ref_forward_one(&s, tokens[i], i);
        if (!st) memcpy(out + i * m->vocab, s.logits, m->vocab * sizeof(float));
    }
    ref_state_free(&s);
    return st;
}

/* logits_hash_for_tokens_chunked (:1406-1418) */
int ref_logits_hash(const ref_model* m, const uint32_t* tokens, size_t n, size_t chunk, uint8_t out[32]) {
    if (n == 0 || chunk == 0 || n > m->cfg.ctx) return REF_ERR_SHAPE;
    for (size_t i = 0; i < n; i++)
        if (tokens[i] >= m->tok_embd.rows) return REF_ERR_SHAPE;
    ref_state s;
    int st = ref_state_init(&s, m, n);
    if (st) return st;
    ref_sha256_ctx h;
    ref_sha256_init(&h);
    for (size_t i = 0; i < n && !st; i++) {
        st = ref_forward_one(&s, tokens[i], i);
        if (!st)
            for (size_t v = 0; v < m->vocab; v++) sha_update_f32(&h, s.logits[v]);
    }
    ref_state_free(&s);
    if (!st) ref_sha256_final(&h, out);
    return st;
}

int ref_rope_tables(const ref_model* m, size_t positions, float* cos_out, float* sin_out) {
    if (positions == 0) return REF_ERR_SHAPE;
    return build_rope(&m->cfg, positions, cos_out, sin_out);
}

void ref_free(void* p) { free(p); }
