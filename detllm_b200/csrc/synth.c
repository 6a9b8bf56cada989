/*
 * synth.c -- seeded synthetic GGUF models for the benchmark configurations
 * (libdetsynth.so, host-only harness code; not part of the device path).
 *
 * No checkpoints are available offline, so models are random-init: weights
 * ~ N(0, 0.02) quantised to the GGUF block formats the reference decodes
 * (Q8_0, Q4_0, Q4_K, Q6_K layouts fixed by crates/det-quant/src/lib.rs:
 * 506-568), norm weights 1.0, optional qwen2 QKV biases ~ N(0, 0.02), and a
 * byte-fallback vocabulary (256 "<0xNN>" tokens then filler pieces).
 *
 * Values come from a counter-based generator (splitmix64 of seed, tensor
 * index and element index), so the file is identical for any thread count.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

typedef struct {
    int arch;  /* 0 llama, 1 qwen2 */
    int n_layer, d, d_ff, n_head, n_head_kv, vocab, ctx;
    float rope_base, eps;
    int tied, qkv_bias;
    int t_embd, t_attn, t_gate_up, t_down, t_out;
    uint64_t seed;
    uint8_t escape[32]; /* bitmask of byte tokens marked non-emittable */
} synth_spec;

static uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

static float g_pool[65536];
static uint64_t g_pool_seed = ~0ull;
static pthread_mutex_t g_pool_mu = PTHREAD_MUTEX_INITIALIZER;

static void make_pool(uint64_t seed) {
    pthread_mutex_lock(&g_pool_mu);
    if (g_pool_seed != seed) {
        for (int i = 0; i < 65536; i += 2) {
            uint64_t a = mix64(seed ^ (0x5eedull << 40) ^ (uint64_t)i);
            uint64_t b = mix64(a);
            double u1 = ((double)(a >> 11) + 0.5) * (1.0 / 9007199254740992.0);
            double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
            double r = sqrt(-2.0 * log(u1));
            g_pool[i] = (float)(0.02 * r * cos(6.283185307179586 * u2));
            g_pool[i + 1] = (float)(0.02 * r * sin(6.283185307179586 * u2));
        }
        g_pool_seed = seed;
    }
    pthread_mutex_unlock(&g_pool_mu);
}

static inline float weight(uint64_t seed, uint64_t tensor, uint64_t i) {
    uint64_t r = mix64(seed ^ (tensor << 48) ^ (i >> 2));
    return g_pool[(r >> (16 * (i & 3))) & 0xffff];
}

/* f32 -> f16 bits, round to nearest even */
static uint16_t f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    int32_t e = (int32_t)((x >> 23) & 0xff) - 127 + 15;
    uint32_t m = x & 0x7fffffu;
    if (((x >> 23) & 0xff) == 0xff) return (uint16_t)(sign | 0x7c00u | (m ? 0x200u : 0));
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        m |= 0x800000u;
        int sh = 14 - e;
        uint32_t h = m >> sh, rem = m & ((1u << sh) - 1), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (h & 1))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (m >> 13), rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) h++;
    return (uint16_t)(sign | h);
}

static float f16f(uint16_t h) {
    uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ffu, o;
    if (e == 0) {
        if (!m) o = s;
        else {
            int k = -1;
            do { m <<= 1; k++; } while (!(m & 0x400u));
            o = s | ((uint32_t)(127 - 15 - k) << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31) o = s | 0x7f800000u | (m << 13);
    else o = s | ((e - 15 + 127) << 23) | (m << 13);
    float f;
    memcpy(&f, &o, 4);
    return f;
}

static void put16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* one quantised block of `bk` values into `out` */
static void quant_block(int type, const float* x, uint8_t* out) {
    switch (type) {
        case T_Q8_0: {
            float amax = 0;
            for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[i]));
            uint16_t db = f16(amax / 127.0f);
            float d = f16f(db), id = d > 0 ? 1.0f / d : 0.0f;
            put16(out, db);
            for (int i = 0; i < 32; i++) out[2 + i] = (uint8_t)(int8_t)clampi((int)lrintf(x[i] * id), -127, 127);
            break;
        }
        case T_Q4_0: {
            float amax = 0, mx = 0;
            for (int i = 0; i < 32; i++)
                if (fabsf(x[i]) > amax) { amax = fabsf(x[i]); mx = x[i]; }
            uint16_t db = f16(mx / -8.0f);
            float d = f16f(db), id = d != 0 ? 1.0f / d : 0.0f;
            put16(out, db);
            for (int i = 0; i < 16; i++) {
                int lo = clampi((int)lrintf(x[i] * id) + 8, 0, 15), hi = clampi((int)lrintf(x[i + 16] * id) + 8, 0, 15);
                out[2 + i] = (uint8_t)(lo | (hi << 4));
            }
            break;
        }
        case T_Q4_K: {
            float mn[8], sc_f[8], maxsc = 1e-8f, maxmn = 1e-8f;
            for (int s = 0; s < 8; s++) {
                float lo = 0, hi = -INFINITY;
                for (int i = 0; i < 32; i++) { lo = fminf(lo, x[32 * s + i]); hi = fmaxf(hi, x[32 * s + i]); }
                mn[s] = lo;
                sc_f[s] = (hi - lo) / 15.0f;
                maxsc = fmaxf(maxsc, sc_f[s]);
                maxmn = fmaxf(maxmn, -lo);
            }
            uint16_t db = f16(maxsc / 63.0f), mb = f16(maxmn / 63.0f);
            float d = f16f(db), dmin = f16f(mb);
            int sc[8], m[8];
            for (int s = 0; s < 8; s++) {
                sc[s] = clampi((int)lrintf(sc_f[s] / d), 1, 63);
                m[s] = clampi((int)lrintf(-mn[s] / dmin), 0, 63);
            }
            put16(out, db);
            put16(out + 2, mb);
            uint8_t* scales = out + 4;
            for (int i = 0; i < 4; i++) {
                scales[i] = (uint8_t)((sc[i] & 63) | ((sc[i + 4] >> 4) << 6));
                scales[i + 4] = (uint8_t)((m[i] & 63) | ((m[i + 4] >> 4) << 6));
                scales[i + 8] = (uint8_t)((sc[i + 4] & 15) | ((m[i + 4] & 15) << 4));
            }
            uint8_t* qs = out + 16;
            for (int k = 0; k < 4; k++)
                for (int i = 0; i < 32; i++) {
                    int q[2];
                    for (int h = 0; h < 2; h++) {
                        int s = 2 * k + h;
                        float step = d * (float)sc[s], off = dmin * (float)m[s];
                        q[h] = clampi((int)lrintf((x[32 * s + i] + off) / step), 0, 15);
                    }
                    qs[k * 32 + i] = (uint8_t)(q[0] | (q[1] << 4));
                }
            break;
        }
        case T_Q6_K: {
            float gs[16], maxg = 1e-10f;
            for (int g = 0; g < 16; g++) {
                float a = 0;
                for (int i = 0; i < 16; i++) a = fmaxf(a, fabsf(x[16 * g + i]));
                gs[g] = a / 31.0f;
                maxg = fmaxf(maxg, gs[g]);
            }
            uint16_t db = f16(maxg / 127.0f);
            float d = f16f(db);
            int8_t sc[16];
            for (int g = 0; g < 16; g++) sc[g] = (int8_t)clampi((int)lrintf(gs[g] / d), 1, 127);
            uint8_t* ql = out;
            uint8_t* qh = out + 128;
            memset(ql, 0, 192);
            for (int i = 0; i < 256; i++) {
                int half = i / 128, within = i % 128, part = within / 32, l = within % 32;
                float step = d * (float)sc[i / 16];
                int q = clampi((int)lrintf(x[i] / step) + 32, 0, 63);
                int base = half * 64 + ((part & 1) ? 32 : 0);
                ql[base + l] |= (uint8_t)((part < 2) ? (q & 15) : ((q & 15) << 4));
                qh[half * 32 + l] |= (uint8_t)((q >> 4) << (2 * part));
            }
            memcpy(out + 192, sc, 16);
            put16(out + 208, db);
            break;
        }
    }
}

static void type_geom(int type, int* bk, int* bb) {
    switch (type) {
        case T_F32: *bk = 1; *bb = 4; break;
        case T_F16: *bk = 1; *bb = 2; break;
        case T_Q4_0: *bk = 32; *bb = 18; break;
        case T_Q8_0: *bk = 32; *bb = 34; break;
        case T_Q4_K: *bk = 256; *bb = 144; break;
        default: *bk = 256; *bb = 210; break;
    }
}

typedef struct {
    char name[64];
    int ndim;
    uint64_t dims[2];
    int type;
    int kind; /* 0 random matrix/vector, 1 ones */
    uint64_t offset, bytes;
} tdesc;

typedef struct {
    const tdesc* t;
    uint64_t tindex, seed;
    uint8_t* dst;
    uint64_t b0, b1; /* block range */
} job;

static void* run_job(void* p) {
    job* j = (job*)p;
    int bk, bb;
    type_geom(j->t->type, &bk, &bb);
    float x[256];
    for (uint64_t b = j->b0; b < j->b1; b++) {
        for (int i = 0; i < bk; i++) x[i] = j->t->kind == 1 ? 1.0f : weight(j->seed, j->tindex, b * (uint64_t)bk + i);
        uint8_t* o = j->dst + b * (uint64_t)bb;
        if (j->t->type == T_F32) memcpy(o, x, 4);
        else if (j->t->type == T_F16) put16(o, f16(x[0]));
        else quant_block(j->t->type, x, o);
    }
    return NULL;
}

typedef struct {
    uint8_t* p;
    size_t len, cap;
    int count_only;
} wbuf;

static void wput(wbuf* w, const void* d, size_t n) {
    if (!w->count_only && w->len + n <= w->cap) memcpy(w->p + w->len, d, n);
    w->len += n;
}
static void w32(wbuf* w, uint32_t v) { wput(w, &v, 4); }
static void w64(wbuf* w, uint64_t v) { wput(w, &v, 8); }
static void wstr(wbuf* w, const char* s) { w64(w, strlen(s)); wput(w, s, strlen(s)); }
static void meta_u32(wbuf* w, const char* k, uint32_t v) { wstr(w, k); w32(w, 4); w32(w, v); }
static void meta_f32(wbuf* w, const char* k, float v) { uint32_t b; memcpy(&b, &v, 4); wstr(w, k); w32(w, 6); w32(w, b); }

static int add_tensor(tdesc* ts, int n, const char* name, uint64_t rows, uint64_t cols, int type, int kind, int ndim) {
    tdesc* t = &ts[n];
    snprintf(t->name, sizeof t->name, "%s", name);
    t->ndim = ndim;
    t->dims[0] = cols;
    t->dims[1] = rows;
    t->type = type;
    t->kind = kind;
    int bk, bb;
    type_geom(type, &bk, &bb);
    t->bytes = rows * cols / (uint64_t)bk * (uint64_t)bb;
    return n + 1;
}

/* Writes the GGUF into out (when cap is large enough); returns its size. */
size_t synth_gguf(const synth_spec* s, uint8_t* out, size_t cap, int threads) {
    const char* a = s->arch ? "qwen2" : "llama";
    const uint64_t hd = (uint64_t)(s->d / s->n_head);
    int nt = 0, maxt = 16 + 12 * s->n_layer;
    tdesc* ts = (tdesc*)calloc((size_t)maxt, sizeof(tdesc));
    char nm[64];
    nt = add_tensor(ts, nt, "token_embd.weight", s->vocab, s->d, s->t_embd, 0, 2);
    for (int l = 0; l < s->n_layer; l++) {
#define T(suffix, r, c, ty, kind, nd) \
    (snprintf(nm, sizeof nm, "blk.%d.%s", l, suffix), nt = add_tensor(ts, nt, nm, r, c, ty, kind, nd))
        T("attn_norm.weight", 1, s->d, T_F32, 1, 1);
        T("attn_q.weight", s->n_head * hd, s->d, s->t_attn, 0, 2);
        if (s->qkv_bias) T("attn_q.bias", 1, s->n_head * hd, T_F32, 0, 1);
        T("attn_k.weight", s->n_head_kv * hd, s->d, s->t_attn, 0, 2);
        if (s->qkv_bias) T("attn_k.bias", 1, s->n_head_kv * hd, T_F32, 0, 1);
        T("attn_v.weight", s->n_head_kv * hd, s->d, s->t_attn, 0, 2);
        if (s->qkv_bias) T("attn_v.bias", 1, s->n_head_kv * hd, T_F32, 0, 1);
        T("attn_output.weight", s->d, s->n_head * hd, s->t_attn, 0, 2);
        T("ffn_norm.weight", 1, s->d, T_F32, 1, 1);
        T("ffn_gate.weight", s->d_ff, s->d, s->t_gate_up, 0, 2);
        T("ffn_up.weight", s->d_ff, s->d, s->t_gate_up, 0, 2);
        T("ffn_down.weight", s->d, s->d_ff, s->t_down, 0, 2);
#undef T
    }
    nt = add_tensor(ts, nt, "output_norm.weight", 1, s->d, T_F32, 1, 1);
    if (!s->tied) nt = add_tensor(ts, nt, "output.weight", s->vocab, s->d, s->t_out, 0, 2);
    uint64_t off = 0;
    for (int i = 0; i < nt; i++) {
        off = (off + 31) & ~31ull;
        ts[i].offset = off;
        off += ts[i].bytes;
    }
    const uint64_t data_len = off;
    int any_escape = 0;
    for (int i = 0; i < 32; i++) any_escape |= s->escape[i];
    /* header */
    wbuf w = {out, 0, cap, out == NULL};
    wput(&w, "GGUF", 4);
    w32(&w, 3);
    w64(&w, (uint64_t)nt);
    w64(&w, 11 + (any_escape ? 1 : 0));
    wstr(&w, "general.architecture");
    w32(&w, 8);
    wstr(&w, a);
    char k[96];
#define K(x) (snprintf(k, sizeof k, "%s.%s", a, x), k)
    meta_u32(&w, K("block_count"), (uint32_t)s->n_layer);
    meta_u32(&w, K("embedding_length"), (uint32_t)s->d);
    meta_u32(&w, K("feed_forward_length"), (uint32_t)s->d_ff);
    meta_u32(&w, K("attention.head_count"), (uint32_t)s->n_head);
    meta_u32(&w, K("attention.head_count_kv"), (uint32_t)s->n_head_kv);
    meta_f32(&w, K("attention.layer_norm_rms_epsilon"), s->eps);
    meta_f32(&w, K("rope.freq_base"), s->rope_base);
    meta_u32(&w, K("context_length"), (uint32_t)s->ctx);
    meta_u32(&w, K("vocab_size"), (uint32_t)s->vocab);
#undef K
    wstr(&w, "tokenizer.ggml.tokens");
    w32(&w, 9);
    w32(&w, 8);
    w64(&w, (uint64_t)s->vocab);
    for (int i = 0; i < s->vocab; i++) {
        char piece[32];
        if (i < 256) snprintf(piece, sizeof piece, "<0x%02X>", i);
        else snprintf(piece, sizeof piece, "tok%d", i);
        wstr(&w, piece);
    }
    if (any_escape) {
        wstr(&w, "tokenizer.ggml.token_type");
        w32(&w, 9);
        w32(&w, 5);
        w64(&w, (uint64_t)s->vocab);
        for (int i = 0; i < s->vocab; i++) {
            int32_t ty = (i < 256 && (s->escape[i >> 3] >> (i & 7)) & 1) ? 3 : 1;
            wput(&w, &ty, 4);
        }
    }
    for (int i = 0; i < nt; i++) {
        wstr(&w, ts[i].name);
        w32(&w, (uint32_t)ts[i].ndim);
        for (int d = 0; d < ts[i].ndim; d++) w64(&w, ts[i].dims[d]);
        w32(&w, (uint32_t)ts[i].type);
        w64(&w, ts[i].offset);
    }
    while (w.len % 32) {
        uint8_t z = 0;
        wput(&w, &z, 1);
    }
    const size_t total = w.len + data_len;
    if (!out || cap < total) {
        free(ts);
        return total;
    }
    uint8_t* data = out + w.len;
    memset(data, 0, data_len);
    make_pool(s->seed);
    if (threads < 1) threads = 1;
    pthread_t* th = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
    job* jobs = (job*)calloc((size_t)threads, sizeof(job));
    for (int i = 0; i < nt; i++) {
        int bk, bb;
        type_geom(ts[i].type, &bk, &bb);
        uint64_t nb = ts[i].bytes / (uint64_t)bb;
        int tcount = nb < 4096 ? 1 : threads;
        for (int j = 0; j < tcount; j++) {
            jobs[j] = (job){&ts[i], (uint64_t)i + 1, s->seed, data + ts[i].offset, nb * (uint64_t)j / (uint64_t)tcount,
                            nb * (uint64_t)(j + 1) / (uint64_t)tcount};
            if (tcount == 1) run_job(&jobs[j]);
            else pthread_create(&th[j], NULL, run_job, &jobs[j]);
        }
        if (tcount > 1)
            for (int j = 0; j < tcount; j++) pthread_join(th[j], NULL);
    }
    free(th);
    free(jobs);
    free(ts);
    return total;
}

/* ---- synthetic order-2 Markov byte stream (benchmark input) ----------------
 * n bytes over printable ASCII 0x20..0x7E plus '\n', each byte drawn from a
 * seeded transition table indexed by the two previous bytes.  Row weights are
 * u^12 for u uniform (a few likely successors per context, like text), and
 * the markup bytes '<' and '>' get extra mass in every context.  Sampling is
 * a binary search in the row's cumulative table, driven by splitmix64. */
#define MK_K 96
static uint8_t mk_sym(int i) { return i < 95 ? (uint8_t)(0x20 + i) : (uint8_t)'\n'; }

size_t synth_markov(uint8_t* out, size_t n, uint64_t seed) {
    uint32_t* cdf = (uint32_t*)malloc(sizeof(uint32_t) * MK_K * MK_K * MK_K);
    if (!cdf) return 0;
    const int lt = '<' - 0x20, gt = '>' - 0x20;
    for (int ctx = 0; ctx < MK_K * MK_K; ctx++) {
        double w[MK_K], tot = 0.0;
        for (int c = 0; c < MK_K; c++) {
            const double u = (double)(mix64(seed ^ ((uint64_t)ctx << 8) ^ (uint64_t)c) >> 11) * (1.0 / 9007199254740992.0);
            const double u2 = u * u, u4 = u2 * u2;
            w[c] = u4 * u4 * u4;
            tot += w[c];
        }
        w[lt] += 2.0 * tot / MK_K;
        w[gt] += 2.0 * tot / MK_K;
        tot = 0.0;
        for (int c = 0; c < MK_K; c++) tot += w[c];
        double acc = 0.0;
        for (int c = 0; c < MK_K; c++) {
            acc += w[c];
            double v = acc / tot * 4294967295.0;
            cdf[(size_t)ctx * MK_K + c] = c == MK_K - 1 ? 0xffffffffu : (uint32_t)v;
        }
    }
    int a = 0, b = 1;
    uint64_t st = mix64(seed ^ 0x6d61726b6f76ull);
    for (size_t i = 0; i < n; i++) {
        st = mix64(st);
        const uint32_t u = (uint32_t)(st >> 32);
        const uint32_t* row = cdf + ((size_t)a * MK_K + b) * MK_K;
        int lo = 0, hi = MK_K - 1;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (row[mid] >= u) hi = mid;
            else lo = mid + 1;
        }
        out[i] = mk_sym(lo);
        a = b;
        b = lo;
    }
    free(cdf);
    return n;
}
