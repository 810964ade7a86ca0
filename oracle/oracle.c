/*
 * QORA-TTS decode-path ORACLE (test infrastructure only; see oracle.h).
 *
 * Every function restates one reference function; the citation names the
 * reference file:line it follows.  Floating-point operation order follows the
 * reference exactly (sequential f32 sums, separate multiply and add: this file
 * is compiled with -ffp-contract=off).
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define Q4_GROUP 32

/* ======================================================================== */
/* f16 <-> f32 (the `half` crate 2.7.1 semantics: IEEE binary16, RNE)       */
/* ======================================================================== */

float oq_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1f;
    uint32_t m = h & 0x3ff;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {
            int s = 0;
            while (!(m & 0x400)) { m <<= 1; s++; }
            m &= 0x3ff;
            x = sign | ((uint32_t)(113 - s) << 23) | (m << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

uint16_t oq_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) { /* inf / nan */
        if (ax == 0x7f800000u) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | 0x7e00u | ((ax >> 13) & 0x3ffu));
    }
    uint32_t e = ax >> 23;
    if (e >= 143) return (uint16_t)(sign | 0x7c00u); /* >= 2^16: overflow */
    if (e >= 113) {                                    /* normal f16 range */
        uint32_t mant = ax & 0x7fffffu;
        uint32_t h = ((e - 112) << 10) | (mant >> 13);
        uint32_t rem = mant & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    if (ax < 0x33000000u) return (uint16_t)sign; /* < 2^-25 rounds to zero */
    /* f16 subnormal: m16 = round(v * 2^24) */
    uint32_t M = (ax & 0x7fffffu) | 0x800000u;
    uint32_t s = 126 - e; /* 14..24 */
    uint32_t m16 = M >> s;
    uint32_t rem = M & ((1u << s) - 1u);
    uint32_t half = 1u << (s - 1);
    if (rem > half || (rem == half && (m16 & 1u))) m16++;
    return (uint16_t)(sign | m16);
}

void oq_f32_to_f16_array(const float *src, uint16_t *dst, int64_t n) {
    for (int64_t i = 0; i < n; i++) dst[i] = oq_f32_to_f16(src[i]);
}
void oq_f16_to_f32_array(const uint16_t *src, float *dst, int64_t n) {
    for (int64_t i = 0; i < n; i++) dst[i] = oq_f16_to_f32(src[i]);
}

/* ======================================================================== */
/* Quantiser: gemv.rs:92-130                                                */
/* ======================================================================== */

void oq_quantize_f32_to_q4(const float *data, int64_t k, int64_t n, uint8_t *packed,
                           uint16_t *scales) {
    int64_t gpr = n / Q4_GROUP;
    for (int64_t ki = 0; ki < k; ki++) {
        for (int64_t g = 0; g < gpr; g++) {
            int64_t gi = ki * gpr + g;
            const float *row = data + ki * n + g * Q4_GROUP;
            float absmax = 0.0f;
            for (int j = 0; j < Q4_GROUP; j++) {
                float v = fabsf(row[j]);
                if (v > absmax) absmax = v; /* gemv.rs:111 */
            }
            float scale = absmax / 7.0f;         /* gemv.rs:114 */
            scales[gi] = oq_f32_to_f16(scale);   /* gemv.rs:115 */
            float inv = scale > 0.0f ? 1.0f / scale : 0.0f; /* gemv.rs:116, unrounded scale */
            uint8_t *dst = packed + gi * 16;
            for (int j = 0; j < Q4_GROUP; j += 2) {
                float r0 = roundf(row[j] * inv);     /* half away from zero */
                float r1 = roundf(row[j + 1] * inv);
                r0 = fminf(fmaxf(r0, -8.0f), 7.0f);
                r1 = fminf(fmaxf(r1, -8.0f), 7.0f);
                uint8_t q0 = (uint8_t)(r0 + 8.0f);
                uint8_t q1 = (uint8_t)(r1 + 8.0f);
                dst[j / 2] = (uint8_t)(q0 | (q1 << 4));
            }
        }
    }
}

/* ======================================================================== */
/* Scalar Q4 GEMV: gemv.rs:249-287 (the reference's bit-exact oracle)       */
/* ======================================================================== */

void oq_gemv_q4_scalar(const float *x, const uint8_t *packed, const uint16_t *scales,
                       int64_t n, int64_t k_start, int64_t k_end, float *out) {
    int64_t gpr = n / Q4_GROUP;
    int64_t ppr = gpr * 16;
    memset(out, 0, sizeof(float) * (size_t)n);
    for (int64_t ki = k_start; ki < k_end; ki++) {
        float xv = x[ki];
        if (xv == 0.0f) continue; /* gemv.rs:259 */
        for (int64_t g = 0; g < gpr; g++) {
            float s = oq_f16_to_f32(scales[ki * gpr + g]) * xv; /* gemv.rs:265 */
            if (s == 0.0f) continue;
            float lut[16];
            for (int i = 0; i < 16; i++) lut[i] = s * (float)(i - 8);
            lut[8] = 0.0f; /* gemv.rs:271 literal +0.0 */
            const uint8_t *p = packed + ki * ppr + g * 16;
            float *o = out + g * Q4_GROUP;
            for (int j = 0; j < 16; j++) {
                uint8_t b = p[j];
                o[2 * j] += lut[b & 0x0f];
                o[2 * j + 1] += lut[b >> 4];
            }
        }
    }
}

/* ======================================================================== */
/* Pool: gpool.rs:17-66 (persistent workers on a shared queue)              */
/* ======================================================================== */

typedef struct oq_job {
    void (*fn)(void *arg, int idx);
    void *arg;
    int n_tasks;
    atomic_int next;
    atomic_int done;
} oq_job;

static struct {
    pthread_mutex_t mu;
    pthread_cond_t cv_job, cv_done;
    pthread_mutex_t call_mu;
    pthread_once_t once;
    int workers;
    uint64_t gen;
    oq_job *job;
    int active;
} g_pool = {PTHREAD_MUTEX_INITIALIZER, PTHREAD_COND_INITIALIZER, PTHREAD_COND_INITIALIZER,
            PTHREAD_MUTEX_INITIALIZER, PTHREAD_ONCE_INIT, 0, 0, NULL, 0};

static int g_requested_workers = 0;

static void *pool_worker(void *unused) {
    (void)unused;
    uint64_t seen = 0;
    for (;;) {
        pthread_mutex_lock(&g_pool.mu);
        while (g_pool.gen == seen) pthread_cond_wait(&g_pool.cv_job, &g_pool.mu);
        seen = g_pool.gen;
        oq_job *job = g_pool.job;
        if (job) g_pool.active++;
        pthread_mutex_unlock(&g_pool.mu);
        if (!job) continue;
        for (;;) {
            int i = atomic_fetch_add(&job->next, 1);
            if (i >= job->n_tasks) break;
            job->fn(job->arg, i);
            atomic_fetch_add(&job->done, 1);
        }
        pthread_mutex_lock(&g_pool.mu);
        g_pool.active--;
        pthread_cond_broadcast(&g_pool.cv_done);
        pthread_mutex_unlock(&g_pool.mu);
    }
    return NULL;
}

static void pool_init(void) {
    long avail = sysconf(_SC_NPROCESSORS_ONLN);
    if (avail < 1) avail = 6;
    int workers = g_requested_workers;
    if (workers <= 0) {
        const char *env = getenv("QORA_THREADS"); /* gpool.rs:29-33 */
        int v = env ? atoi(env) : 0;
        workers = v >= 1 ? v : (int)(avail < 16 ? avail : 16);
    }
    if (workers > avail * 2) workers = (int)(avail * 2);
    if (workers < 1) workers = 1;
    g_pool.workers = workers;
    for (int i = 0; i < workers; i++) {
        pthread_t th;
        pthread_create(&th, NULL, pool_worker, NULL);
        pthread_detach(th);
    }
}

int oq_pool_workers(void) {
    pthread_once(&g_pool.once, pool_init);
    return g_pool.workers;
}

void oq_pool_set_workers(int workers) { g_requested_workers = workers; }

static void pool_run(void (*fn)(void *, int), void *arg, int n_tasks) {
    pthread_once(&g_pool.once, pool_init);
    pthread_mutex_lock(&g_pool.call_mu);
    oq_job job;
    job.fn = fn;
    job.arg = arg;
    job.n_tasks = n_tasks;
    atomic_init(&job.next, 0);
    atomic_init(&job.done, 0);
    pthread_mutex_lock(&g_pool.mu);
    g_pool.job = &job;
    g_pool.gen++;
    pthread_cond_broadcast(&g_pool.cv_job);
    /* The caller blocks until every chunk is back (gemv.rs:340-344). */
    while (atomic_load(&job.done) < n_tasks || g_pool.active > 0) {
        if (atomic_load(&job.done) >= n_tasks) g_pool.job = NULL;
        pthread_cond_wait(&g_pool.cv_done, &g_pool.mu);
    }
    g_pool.job = NULL;
    pthread_mutex_unlock(&g_pool.mu);
    pthread_mutex_unlock(&g_pool.call_mu);
}

/* ======================================================================== */
/* GEMV dispatch: gemv.rs:149-154, 230-243, 290-346                          */
/* ======================================================================== */

static int g_simd = -1;

void oq_set_simd(int level) { g_simd = level; }
int oq_get_simd(void) {
    if (g_simd < 0) g_simd = oq_has_avx512() ? 2 : (oq_has_avx2() ? 1 : 0);
    return g_simd;
}

void oq_gemv_q4_inner(const float *x, const oq_q4 *w, int64_t k_start, int64_t k_end,
                      float *out) {
    int simd = oq_get_simd();
    if (simd >= 2 && oq_has_avx512())
        oq_gemv_q4_avx512(x, w->packed, w->scales, w->n, k_start, k_end, out);
    else if (simd >= 1 && oq_has_avx2())
        oq_gemv_q4_avx2(x, w->packed, w->scales, w->n, k_start, k_end, out);
    else
        oq_gemv_q4_scalar(x, w->packed, w->scales, w->n, k_start, k_end, out);
}

typedef struct {
    const float *x;
    const oq_q4 *w;
    int64_t chunk_k;
    float *partials; /* [n_chunks][n] */
} gemv_job_arg;

static void gemv_chunk(void *argp, int t) {
    gemv_job_arg *a = (gemv_job_arg *)argp;
    int64_t k = a->w->k;
    int64_t ks = (int64_t)t * a->chunk_k;
    int64_t ke = ((int64_t)t + 1) * a->chunk_k;
    if (ke > k) ke = k;
    float *out = a->partials + (int64_t)t * a->w->n;
    if (ks >= ke) {
        memset(out, 0, sizeof(float) * (size_t)a->w->n);
        return;
    }
    oq_gemv_q4_inner(a->x, a->w, ks, ke, out);
}

void oq_gemv_workers(const float *x, const oq_q4 *w, float *out, int workers) {
    int64_t k = w->k, n = w->n;
    if (workers <= 0) workers = oq_pool_workers();
    int64_t threads = (k * n) / 500000; /* gemv.rs:303-306 */
    if (threads < 1) threads = 1;
    if (threads > workers) threads = workers;
    if (k * n < 500000) threads = 1;
    if (threads <= 1) {
        oq_gemv_q4_inner(x, w, 0, k, out);
        return;
    }
    int64_t chunks = threads * 4; /* gemv.rs:314-315 */
    if (chunks > k) chunks = k;
    if (chunks < threads) chunks = threads;
    int64_t chunk_k = (k + chunks - 1) / chunks;
    float *partials = (float *)malloc(sizeof(float) * (size_t)(chunks * n));
    gemv_job_arg a = {x, w, chunk_k, partials};
    pool_run(gemv_chunk, &a, (int)chunks);
    memset(out, 0, sizeof(float) * (size_t)n);
    for (int64_t c = 0; c < chunks; c++) { /* chunk order, gemv.rs:340-344 */
        const float *p = partials + c * n;
        for (int64_t j = 0; j < n; j++) out[j] += p[j];
    }
    free(partials);
}

void oq_gemv(const float *x, const oq_q4 *w, float *out) { oq_gemv_workers(x, w, out, 0); }

/* gemm_q4 (gemv.rs:349-412): every token row is one single-pass
 * gemv_q4_inner; threading over tokens does not change any row's bits. */
typedef struct {
    const float *x;
    const oq_q4 *w;
    float *out;
} gemm_job_arg;

static void gemm_row(void *argp, int t) {
    gemm_job_arg *a = (gemm_job_arg *)argp;
    oq_gemv_q4_inner(a->x + (int64_t)t * a->w->k, a->w, 0, a->w->k, a->out + (int64_t)t * a->w->n);
}

void oq_gemm(const float *x, int64_t seq_len, const oq_q4 *w, float *out) {
    gemm_job_arg a = {x, w, out};
    if (w->k * w->n >= 4000000 && seq_len > 1) {
        pool_run(gemm_row, &a, (int)seq_len);
    } else {
        for (int64_t t = 0; t < seq_len; t++) gemm_row(&a, (int)t);
    }
}

/* embed_lookup_q4: gemv.rs:415-437 (also talker.rs:119-150,
 * code_predictor.rs:303-332). */
void oq_embed_lookup(const oq_q4 *w, int64_t token, float *out) {
    int64_t gpr = w->n / Q4_GROUP;
    for (int64_t g = 0; g < gpr; g++) {
        float scale = oq_f16_to_f32(w->scales[token * gpr + g]);
        const uint8_t *p = w->packed + (token * gpr + g) * 16;
        for (int j = 0; j < 16; j++) {
            int q0 = (int)(p[j] & 0x0f) - 8;
            int q1 = (int)((p[j] >> 4) & 0x0f) - 8;
            out[g * Q4_GROUP + 2 * j] = scale * (float)q0;
            out[g * Q4_GROUP + 2 * j + 1] = scale * (float)q1;
        }
    }
}

/* rms_norm_f16: gemv.rs:445-454 */
void oq_rms_norm_f16(const float *x, const uint16_t *gamma, int64_t n, float *out) {
    float sum_sq = 0.0f;
    for (int64_t i = 0; i < n; i++) sum_sq += x[i] * x[i];
    float inv = 1.0f / sqrtf(sum_sq / (float)n + 1e-6f);
    for (int64_t i = 0; i < n; i++) out[i] = x[i] * inv * oq_f16_to_f32(gamma[i]);
}

/* softmax_raw: gemv.rs:471-482 */
void oq_softmax_raw(float *s, int64_t n) {
    float mx = -INFINITY;
    for (int64_t i = 0; i < n; i++) mx = fmaxf(mx, s[i]);
    float sum = 0.0f;
    for (int64_t i = 0; i < n; i++) {
        s[i] = expf(s[i] - mx);
        sum += s[i];
    }
    float inv = 1.0f / sum;
    for (int64_t i = 0; i < n; i++) s[i] *= inv;
}

/* silu: gemv.rs:486-488 */
float oq_silu(float x) { return x / (1.0f + expf(-x)); }

/* ======================================================================== */
/* RoPE: rope.rs:11-41 (tables), rope.rs:51-93 / code_predictor.rs:97-121   */
/* ======================================================================== */

void oq_build_rope_tables(int32_t head_dim, int32_t max_pos, double theta,
                          const int32_t *sections, int32_t n_sections, float *cos_table,
                          float *sin_table) {
    int32_t half = head_dim / 2;
    int32_t dim_offset = 0;
    for (int32_t s = 0; s < n_sections; s++) {
        for (int32_t i = 0; i < sections[s]; i++) {
            int32_t d = dim_offset + i;
            double freq = 1.0 / pow(theta, (double)(2 * d) / (double)head_dim);
            for (int64_t pos = 0; pos < max_pos; pos++) {
                double angle = (double)pos * freq;
                cos_table[pos * half + d] = (float)cos(angle);
                sin_table[pos * half + d] = (float)sin(angle);
            }
        }
        dim_offset += sections[s];
    }
}

/* Split (rotate-half) pairing (i, i+hd/2).  The talker's (pos,pos,pos)
 * multimodal ids select the same table row in every section (rope.rs:63-77),
 * so both the talker and the predictor use this form.  The predictor's guard
 * (code_predictor.rs:107) skips positions past the table. */
void oq_apply_rope_split(float *data, int32_t num_heads, int32_t head_dim, int64_t position,
                         const float *cos_table, const float *sin_table, int64_t table_len) {
    int32_t half = head_dim / 2;
    int64_t off = position * half;
    if (off + half > table_len) return;
    for (int32_t h = 0; h < num_heads; h++) {
        float *b = data + (int64_t)h * head_dim;
        for (int32_t i = 0; i < half; i++) {
            float x1 = b[i], x2 = b[half + i];
            float c = cos_table[off + i], s = sin_table[off + i];
            b[i] = x1 * c - x2 * s;
            b[half + i] = x2 * c + x1 * s;
        }
    }
}

/* apply_qk_norm: talker.rs:89-99, code_predictor.rs:84-93 */
void oq_qk_norm(float *data, int32_t num_heads, int32_t head_dim, const uint16_t *gamma) {
    for (int32_t h = 0; h < num_heads; h++) {
        float *d = data + (int64_t)h * head_dim;
        float sum_sq = 0.0f;
        for (int32_t i = 0; i < head_dim; i++) sum_sq += d[i] * d[i];
        float inv = 1.0f / sqrtf(sum_sq / (float)head_dim + 1e-6f);
        for (int32_t i = 0; i < head_dim; i++) d[i] = d[i] * inv * oq_f16_to_f32(gamma[i]);
    }
}

/* ======================================================================== */
/* KV cache: gemv.rs:75-86 (preallocated instead of grown; same layout)     */
/* ======================================================================== */

struct oq_kv {
    int32_t num_layers, kv_heads, head_dim, max_pos;
    float **k, **v;
    int32_t *len;
};

oq_kv *oq_kv_create(int32_t num_layers, int32_t kv_heads, int32_t head_dim, int32_t max_pos) {
    oq_kv *kv = (oq_kv *)calloc(1, sizeof(oq_kv));
    kv->num_layers = num_layers;
    kv->kv_heads = kv_heads;
    kv->head_dim = head_dim;
    kv->max_pos = max_pos;
    kv->k = (float **)calloc((size_t)num_layers, sizeof(float *));
    kv->v = (float **)calloc((size_t)num_layers, sizeof(float *));
    kv->len = (int32_t *)calloc((size_t)num_layers, sizeof(int32_t));
    size_t sz = (size_t)max_pos * kv_heads * head_dim;
    for (int32_t l = 0; l < num_layers; l++) {
        kv->k[l] = (float *)calloc(sz, sizeof(float));
        kv->v[l] = (float *)calloc(sz, sizeof(float));
    }
    return kv;
}

void oq_kv_destroy(oq_kv *kv) {
    if (!kv) return;
    for (int32_t l = 0; l < kv->num_layers; l++) {
        free(kv->k[l]);
        free(kv->v[l]);
    }
    free(kv->k);
    free(kv->v);
    free(kv->len);
    free(kv);
}

void oq_kv_reset(oq_kv *kv) {
    for (int32_t l = 0; l < kv->num_layers; l++) kv->len[l] = 0;
}
int32_t oq_kv_len(const oq_kv *kv, int32_t layer) { return kv->len[layer]; }
int32_t oq_kv_max_pos(const oq_kv *kv) { return kv->max_pos; }
void oq_kv_set_len(oq_kv *kv, int32_t layer, int32_t len) { kv->len[layer] = len; }
float *oq_kv_k(oq_kv *kv, int32_t layer) { return kv->k[layer]; }
float *oq_kv_v(oq_kv *kv, int32_t layer) { return kv->v[layer]; }

int oq_kv_copy(oq_kv *dst, const oq_kv *src) {
    if (dst->num_layers != src->num_layers || dst->kv_heads != src->kv_heads ||
        dst->head_dim != src->head_dim || dst->max_pos < src->max_pos)
        return -1;
    size_t row = (size_t)src->kv_heads * src->head_dim;
    for (int32_t l = 0; l < src->num_layers; l++) {
        memcpy(dst->k[l], src->k[l], sizeof(float) * row * (size_t)src->len[l]);
        memcpy(dst->v[l], src->v[l], sizeof(float) * row * (size_t)src->len[l]);
        dst->len[l] = src->len[l];
    }
    return 0;
}

/* ======================================================================== */
/* Shared decoder-layer pieces                                              */
/* ======================================================================== */

/* GQA attention for one query vector over kv[0..kv_len) of one layer
 * (talker.rs:304-331; code_predictor.rs:168-192, 474-498). */
static void attend_one(const float *q, const float *kc, const float *vc, int64_t kv_len,
                       int32_t heads, int32_t kv_heads, int32_t hd, float *out, float *scores) {
    float scale = 1.0f / sqrtf((float)hd);
    int32_t groups = heads / kv_heads;
    int64_t stride = (int64_t)kv_heads * hd;
    memset(out, 0, sizeof(float) * (size_t)heads * hd);
    for (int32_t h = 0; h < heads; h++) {
        int32_t kvh = h / groups;
        const float *qv = q + (int64_t)h * hd;
        for (int64_t s = 0; s < kv_len; s++) {
            const float *kr = kc + s * stride + (int64_t)kvh * hd;
            float dot = 0.0f;
            for (int32_t d = 0; d < hd; d++) dot += qv[d] * kr[d];
            scores[s] = dot * scale;
        }
        oq_softmax_raw(scores, kv_len);
        float *o = out + (int64_t)h * hd;
        for (int64_t s = 0; s < kv_len; s++) {
            const float *vr = vc + s * stride + (int64_t)kvh * hd;
            float p = scores[s];
            for (int32_t d = 0; d < hd; d++) o[d] += p * vr[d];
        }
    }
}

/* The attention block of one decode step of one layer, from the raw q / k / v
 * projections (talker.rs:285-331; code_predictor.rs:461-498): qk-norm
 * (talker.rs:89-99), split RoPE at `position` (rope.rs:79-92), append k / v
 * at the layer's cache length, attend over length + 1 positions.  q / k / v
 * are not modified; returns -1 past the cache, -2 past the RoPE table. */
int oq_attend_step(const float *q_raw, const float *k_raw, const float *v_raw, int32_t heads,
                   int32_t kv_heads, int32_t hd, const uint16_t *q_norm, const uint16_t *k_norm,
                   const float *rope_cos, const float *rope_sin, int64_t rope_len,
                   int64_t position, oq_kv *kv, int32_t layer, float *out) {
    int32_t qd = heads * hd, kd = kv_heads * hd;
    int64_t offset = kv->len[layer];
    if (offset + 1 > kv->max_pos) return -1;
    if ((position + 1) * (int64_t)(hd / 2) > rope_len) return -2;
    float *q = (float *)malloc(sizeof(float) * (size_t)qd);
    float *kn = (float *)malloc(sizeof(float) * (size_t)kd);
    float *scores = (float *)malloc(sizeof(float) * (size_t)(offset + 1));
    memcpy(q, q_raw, sizeof(float) * (size_t)qd);
    memcpy(kn, k_raw, sizeof(float) * (size_t)kd);
    oq_qk_norm(q, heads, hd, q_norm);
    oq_qk_norm(kn, kv_heads, hd, k_norm);
    oq_apply_rope_split(q, heads, hd, position, rope_cos, rope_sin, rope_len);
    oq_apply_rope_split(kn, kv_heads, hd, position, rope_cos, rope_sin, rope_len);
    memcpy(kv->k[layer] + offset * kd, kn, sizeof(float) * (size_t)kd);
    memcpy(kv->v[layer] + offset * kd, v_raw, sizeof(float) * (size_t)kd);
    kv->len[layer] = (int32_t)(offset + 1);
    attend_one(q, kv->k[layer], kv->v[layer], offset + 1, heads, kv_heads, hd, out, scores);
    free(q); free(kn); free(scores);
    return 0;
}

typedef struct {
    int32_t hidden, heads, kv_heads, hd, ffn;
    const float *rope_cos, *rope_sin;
    int64_t rope_len; /* entries in each table */
} layer_dims;

/* One decode step of one token through one layer, x updated in place
 * (talker.rs:275-349 with rope at `rope_pos`; code_predictor.rs:450-509 with
 * rope at the cache offset). */
static int decode_layer(const layer_dims *d, const oq_layer *lw, float *x, oq_kv *kv,
                        int32_t layer, int64_t rope_pos, int talker_mode) {
    int32_t qd = d->heads * d->hd, kd = d->kv_heads * d->hd;
    int64_t offset = kv->len[layer];
    if (offset + 1 > kv->max_pos) return -1;
    if (talker_mode && (rope_pos + 1) * (int64_t)(d->hd / 2) > d->rope_len) return -2;
    float *xn = (float *)malloc(sizeof(float) * (size_t)d->hidden);
    float *q = (float *)malloc(sizeof(float) * (size_t)qd);
    float *kn = (float *)malloc(sizeof(float) * (size_t)kd);
    float *vn = (float *)malloc(sizeof(float) * (size_t)kd);
    float *att = (float *)malloc(sizeof(float) * (size_t)qd);
    float *scores = (float *)malloc(sizeof(float) * (size_t)(offset + 1));
    float *tmp = (float *)malloc(sizeof(float) * (size_t)(d->hidden > d->ffn ? d->hidden : d->ffn));
    float *gate = (float *)malloc(sizeof(float) * (size_t)d->ffn);
    float *up = (float *)malloc(sizeof(float) * (size_t)d->ffn);

    oq_rms_norm_f16(x, lw->input_norm, d->hidden, xn);
    oq_gemv(xn, &lw->q_proj, q);
    oq_gemv(xn, &lw->k_proj, kn);
    oq_gemv(xn, &lw->v_proj, vn);
    oq_qk_norm(q, d->heads, d->hd, lw->q_norm);
    oq_qk_norm(kn, d->kv_heads, d->hd, lw->k_norm);
    int64_t pos = talker_mode ? rope_pos : offset;
    oq_apply_rope_split(q, d->heads, d->hd, pos, d->rope_cos, d->rope_sin, d->rope_len);
    oq_apply_rope_split(kn, d->kv_heads, d->hd, pos, d->rope_cos, d->rope_sin, d->rope_len);
    memcpy(kv->k[layer] + offset * kd, kn, sizeof(float) * (size_t)kd);
    memcpy(kv->v[layer] + offset * kd, vn, sizeof(float) * (size_t)kd);
    kv->len[layer] = (int32_t)(offset + 1);
    attend_one(q, kv->k[layer], kv->v[layer], offset + 1, d->heads, d->kv_heads, d->hd, att,
               scores);
    oq_gemv(att, &lw->o_proj, tmp);
    for (int32_t j = 0; j < d->hidden; j++) x[j] += tmp[j];
    oq_rms_norm_f16(x, lw->post_attn_norm, d->hidden, xn);
    oq_gemv(xn, &lw->gate_proj, gate);
    oq_gemv(xn, &lw->up_proj, up);
    for (int32_t j = 0; j < d->ffn; j++) gate[j] = oq_silu(gate[j]) * up[j];
    oq_gemv(gate, &lw->down_proj, tmp);
    for (int32_t j = 0; j < d->hidden; j++) x[j] += tmp[j];

    free(xn); free(q); free(kn); free(vn); free(att); free(scores); free(tmp);
    free(gate); free(up);
    return 0;
}

/* Prefill of seq_len tokens through one layer at absolute positions
 * start_pos.. (talker.rs:389-477 with the mrope batch of rope.rs:98-122;
 * code_predictor.rs:354-432 with per-token rope at t). */
static int prefill_layer(const layer_dims *d, const oq_layer *lw, float *x, int64_t T,
                         oq_kv *kv, int32_t layer, int64_t start_pos) {
    int32_t H = d->hidden, qd = d->heads * d->hd, kd = d->kv_heads * d->hd;
    if (kv->len[layer] != start_pos) return -3;
    if (start_pos + T > kv->max_pos) return -1;
    float *xn = (float *)calloc((size_t)(T * H), sizeof(float));
    float *q = (float *)malloc(sizeof(float) * (size_t)(T * qd));
    float *kn = (float *)malloc(sizeof(float) * (size_t)(T * kd));
    float *vn = (float *)malloc(sizeof(float) * (size_t)(T * kd));
    float *att = (float *)malloc(sizeof(float) * (size_t)(T * qd));
    float *scores = (float *)malloc(sizeof(float) * (size_t)(start_pos + T));
    float *tmp = (float *)malloc(sizeof(float) * (size_t)(T * H));
    float *gate = (float *)malloc(sizeof(float) * (size_t)(T * d->ffn));
    float *up = (float *)malloc(sizeof(float) * (size_t)(T * d->ffn));

    for (int64_t t = 0; t < T; t++) oq_rms_norm_f16(x + t * H, lw->input_norm, H, xn + t * H);
    oq_gemm(xn, T, &lw->q_proj, q);
    oq_gemm(xn, T, &lw->k_proj, kn);
    oq_gemm(xn, T, &lw->v_proj, vn);
    for (int64_t t = 0; t < T; t++) {
        oq_qk_norm(q + t * qd, d->heads, d->hd, lw->q_norm);
        oq_qk_norm(kn + t * kd, d->kv_heads, d->hd, lw->k_norm);
    }
    for (int64_t t = 0; t < T; t++) {
        oq_apply_rope_split(q + t * qd, d->heads, d->hd, start_pos + t, d->rope_cos, d->rope_sin,
                            d->rope_len);
        oq_apply_rope_split(kn + t * kd, d->kv_heads, d->hd, start_pos + t, d->rope_cos,
                            d->rope_sin, d->rope_len);
    }
    memcpy(kv->k[layer] + start_pos * kd, kn, sizeof(float) * (size_t)(T * kd));
    memcpy(kv->v[layer] + start_pos * kd, vn, sizeof(float) * (size_t)(T * kd));
    kv->len[layer] = (int32_t)(start_pos + T);
    /* causal attention, head-outer / token-inner (talker.rs:435-458) */
    float scale = 1.0f / sqrtf((float)d->hd);
    int32_t groups = d->heads / d->kv_heads;
    memset(att, 0, sizeof(float) * (size_t)(T * qd));
    for (int32_t h = 0; h < d->heads; h++) {
        int32_t kvh = h / groups;
        for (int64_t t1 = 0; t1 < T; t1++) {
            int64_t alen = start_pos + t1 + 1;
            const float *qv = q + t1 * qd + (int64_t)h * d->hd;
            for (int64_t s = 0; s < alen; s++) {
                const float *kr = kv->k[layer] + s * kd + (int64_t)kvh * d->hd;
                float dot = 0.0f;
                for (int32_t e = 0; e < d->hd; e++) dot += qv[e] * kr[e];
                scores[s] = dot * scale;
            }
            oq_softmax_raw(scores, alen);
            float *o = att + t1 * qd + (int64_t)h * d->hd;
            for (int64_t s = 0; s < alen; s++) {
                const float *vr = kv->v[layer] + s * kd + (int64_t)kvh * d->hd;
                float p = scores[s];
                for (int32_t e = 0; e < d->hd; e++) o[e] += p * vr[e];
            }
        }
    }
    oq_gemm(att, T, &lw->o_proj, tmp);
    for (int64_t j = 0; j < T * H; j++) x[j] += tmp[j];
    for (int64_t t = 0; t < T; t++) oq_rms_norm_f16(x + t * H, lw->post_attn_norm, H, xn + t * H);
    oq_gemm(xn, T, &lw->gate_proj, gate);
    oq_gemm(xn, T, &lw->up_proj, up);
    for (int64_t j = 0; j < T * d->ffn; j++) gate[j] = oq_silu(gate[j]) * up[j];
    oq_gemm(gate, T, &lw->down_proj, tmp);
    for (int64_t j = 0; j < T * H; j++) x[j] += tmp[j];

    free(xn); free(q); free(kn); free(vn); free(att); free(scores); free(tmp);
    free(gate); free(up);
    return 0;
}

static layer_dims talker_dims(const oq_talker *t) {
    layer_dims d = {t->hidden, t->num_heads, t->num_kv_heads, t->head_dim, t->ffn,
                    t->rope_cos, t->rope_sin, (int64_t)t->rope_max_pos * (t->head_dim / 2)};
    return d;
}

static layer_dims predictor_dims(const oq_predictor *p) {
    layer_dims d = {p->hidden, p->num_heads, p->num_kv_heads, p->head_dim, p->ffn,
                    p->rope_cos, p->rope_sin, (int64_t)p->rope_max_pos * (p->head_dim / 2)};
    return d;
}

/* ======================================================================== */
/* Talker: talker.rs                                                         */
/* ======================================================================== */

int oq_talker_step(const oq_talker *t, const float *embedding, oq_kv *kv, int64_t position,
                   float *out_hidden, float *out_logits) {
    layer_dims d = talker_dims(t);
    float *x = (float *)malloc(sizeof(float) * (size_t)t->hidden);
    memcpy(x, embedding, sizeof(float) * (size_t)t->hidden);
    int rc = 0;
    for (int32_t l = 0; l < t->num_layers && rc == 0; l++)
        rc = decode_layer(&d, &t->layers[l], x, kv, l, position, 1);
    if (rc == 0) {
        oq_rms_norm_f16(x, t->final_norm, t->hidden, out_hidden); /* talker.rs:353 */
        if (out_logits) oq_gemv(out_hidden, &t->codec_head, out_logits); /* :354 */
    }
    free(x);
    return rc;
}

int oq_talker_prefill(const oq_talker *t, const float *x_in, int64_t seq_len, oq_kv *kv,
                      int64_t start_pos, float *out_hidden) {
    layer_dims d = talker_dims(t);
    if (seq_len <= 0) return -4;
    if ((start_pos + seq_len) * (int64_t)(t->head_dim / 2) > d.rope_len) return -2;
    float *x = (float *)malloc(sizeof(float) * (size_t)(seq_len * t->hidden));
    memcpy(x, x_in, sizeof(float) * (size_t)(seq_len * t->hidden));
    int rc = 0;
    for (int32_t l = 0; l < t->num_layers && rc == 0; l++)
        rc = prefill_layer(&d, &t->layers[l], x, seq_len, kv, l, start_pos);
    if (rc == 0)
        oq_rms_norm_f16(x + (seq_len - 1) * t->hidden, t->final_norm, t->hidden, out_hidden);
    free(x);
    return rc;
}

void oq_codec_head(const oq_talker *t, const float *hidden, float *out_logits) {
    oq_gemv(hidden, &t->codec_head, out_logits);
}

void oq_embed_codec_token(const oq_talker *t, uint32_t token, float *out) {
    oq_embed_lookup(&t->codec_embedding, token, out);
}

void oq_embed_text_token(const oq_text_proj *tp, uint32_t token, float *out) {
    const int64_t th = tp->text_embedding.n, mid = tp->fc1.n;
    float *raw = (float *)malloc((size_t)th * sizeof(float));
    float *h = (float *)malloc((size_t)mid * sizeof(float));
    oq_embed_lookup(&tp->text_embedding, token, raw);                  /* :107 */
    oq_gemv(raw, &tp->fc1, h);                                         /* :109 */
    for (int64_t j = 0; j < mid; j++) h[j] += tp->fc1_bias[j];          /* :110 */
    for (int64_t j = 0; j < mid; j++) h[j] = oq_silu(h[j]);            /* :112 */
    oq_gemv(h, &tp->fc2, out);                                         /* :113 */
    for (int64_t j = 0; j < tp->fc2.n; j++) out[j] += tp->fc2_bias[j]; /* :114 */
    free(raw);
    free(h);
}

int oq_talker_decode(const oq_talker *t, const oq_text_proj *tp, uint32_t token, int is_text,
                     oq_kv *kv, int64_t position, float *out_hidden) {
    float *x = (float *)malloc(sizeof(float) * (size_t)t->hidden);
    float *logits = (float *)malloc(sizeof(float) * (size_t)t->vocab);
    if (is_text) oq_embed_text_token(tp, token, x);           /* talker.rs:170-174 */
    else oq_embed_codec_token(t, token, x);
    /* talker.rs:176-257 are forward_with_embedding's layers and final norm */
    const int rc = oq_talker_step(t, x, kv, position, out_hidden, logits);
    free(x);
    free(logits);
    return rc;
}

/* ======================================================================== */
/* Code predictor: code_predictor.rs                                         */
/* ======================================================================== */

void oq_project_input(const oq_predictor *p, const float *in, float *out) {
    if (p->input_proj.packed) { /* code_predictor.rs:51-61 */
        oq_gemv(in, &p->input_proj, out);
        if (p->input_proj_bias)
            for (int32_t j = 0; j < p->hidden; j++) out[j] += p->input_proj_bias[j];
    } else {
        memcpy(out, in, sizeof(float) * (size_t)p->hidden);
    }
}

/* sample_argmax (code_predictor.rs:335-341): Iterator::max_by keeps the LAST
 * maximal element on ties. */
uint32_t oq_argmax(const float *logits, int64_t n) {
    if (n <= 0) return 0;
    int64_t best = 0;
    for (int64_t i = 1; i < n; i++)
        if (!(logits[i] < logits[best])) best = i; /* a >= best => take later */
    return (uint32_t)best;
}

static int predictor_frame_impl(const oq_predictor *p, const float *talker_hidden,
                                const float *semantic_embed, oq_kv *kv,
                                const uint32_t *forced, uint32_t *codes_out,
                                float *logits_out) {
    layer_dims d = predictor_dims(p);
    int32_t H = p->hidden, E = p->codec_embeddings[0].n;
    oq_kv_reset(kv); /* code_predictor.rs:227-231 */
    float *x = (float *)malloc(sizeof(float) * (size_t)(2 * H));
    float *hn = (float *)malloc(sizeof(float) * (size_t)H);
    float *logits = (float *)malloc(sizeof(float) * (size_t)p->vocab);
    float *emb = (float *)malloc(sizeof(float) * (size_t)E);
    int rc = 0;
    oq_project_input(p, talker_hidden, x);       /* :235 */
    oq_project_input(p, semantic_embed, x + H);  /* :236 */
    for (int32_t l = 0; l < p->num_layers && rc == 0; l++)
        rc = prefill_layer(&d, &p->layers[l], x, 2, kv, l, 0);
    if (rc == 0) {
        oq_rms_norm_f16(x + H, p->final_norm, H, hn); /* :435-437 */
        oq_gemv(hn, &p->lm_heads[0], logits);         /* :247 */
        if (logits_out) memcpy(logits_out, logits, sizeof(float) * (size_t)p->vocab);
        codes_out[0] = oq_argmax(logits, p->vocab);
    }
    for (int32_t g = 1; g < p->num_groups && rc == 0; g++) {
        uint32_t prev = forced ? forced[g - 1] : codes_out[g - 1];
        oq_embed_lookup(&p->codec_embeddings[g - 1], prev, emb); /* :255-257 */
        oq_project_input(p, emb, x);                              /* :260 */
        for (int32_t l = 0; l < p->num_layers && rc == 0; l++)
            rc = decode_layer(&d, &p->layers[l], x, kv, l, 0, 0);
        if (rc) break;
        oq_rms_norm_f16(x, p->final_norm, H, hn); /* :512 */
        oq_gemv(hn, &p->lm_heads[g], logits);     /* :266 */
        if (logits_out) memcpy(logits_out + (int64_t)g * p->vocab, logits, sizeof(float) * (size_t)p->vocab);
        codes_out[g] = oq_argmax(logits, p->vocab);
    }
    free(x); free(hn); free(logits); free(emb);
    return rc;
}

int oq_predictor_frame(const oq_predictor *p, const float *talker_hidden,
                       const float *semantic_embed, oq_kv *kv, uint32_t *codes_out,
                       float *logits_out) {
    return predictor_frame_impl(p, talker_hidden, semantic_embed, kv, NULL, codes_out, logits_out);
}

int oq_predictor_frame_forced(const oq_predictor *p, const float *talker_hidden,
                              const float *semantic_embed, oq_kv *kv,
                              const uint32_t *forced_codes, uint32_t *codes_out,
                              float *logits_out) {
    return predictor_frame_impl(p, talker_hidden, semantic_embed, kv, forced_codes, codes_out,
                                logits_out);
}

/* get_acoustic_embeddings_sum: code_predictor.rs:287-300 */
void oq_acoustic_embeddings_sum(const oq_predictor *p, const uint32_t *codes, float *out) {
    int32_t E = p->codec_embeddings[0].n;
    float *e = (float *)malloc(sizeof(float) * (size_t)E);
    memset(out, 0, sizeof(float) * (size_t)E);
    for (int32_t g = 0; g < p->num_groups; g++) {
        oq_embed_lookup(&p->codec_embeddings[g], codes[g], e);
        for (int32_t j = 0; j < E; j++) out[j] += e[j];
    }
    free(e);
}

/* ======================================================================== */
/* Sampler: generate_new.rs:17-22, 771-862                                   */
/* ======================================================================== */

float oq_simple_rand(uint64_t *state) {
    *state ^= *state << 13;
    *state ^= *state >> 7;
    *state ^= *state << 17;
    return (float)(*state) / (float)UINT64_MAX;
}

typedef struct {
    int64_t idx;
    float p;
} idx_p;

/* Stable descending sort by probability (generate_new.rs:806-807). */
static void stable_sort_desc(idx_p *a, int64_t n, idx_p *tmp) {
    for (int64_t w = 1; w < n; w *= 2) {
        for (int64_t lo = 0; lo < n; lo += 2 * w) {
            int64_t mid = lo + w < n ? lo + w : n;
            int64_t hi = lo + 2 * w < n ? lo + 2 * w : n;
            int64_t i = lo, j = mid, o = lo;
            while (i < mid && j < hi) {
                /* take right only if strictly greater: keeps stability */
                if (a[j].p > a[i].p) tmp[o++] = a[j++];
                else tmp[o++] = a[i++];
            }
            while (i < mid) tmp[o++] = a[i++];
            while (j < hi) tmp[o++] = a[j++];
        }
        memcpy(a, tmp, sizeof(idx_p) * (size_t)n);
    }
}

void oq_sample_probs(const float *logits, int64_t n, const oq_sample_params *params,
                     const uint32_t *prev_tokens, int32_t n_prev, float temperature,
                     float *s) {
    memcpy(s, logits, sizeof(float) * (size_t)n);
    if (params->repetition_penalty != 1.0f) { /* :775-785 */
        for (int32_t i = 0; i < n_prev; i++) {
            uint32_t t = prev_tokens[i];
            if ((int64_t)t < n) {
                if (s[t] > 0.0f) s[t] /= params->repetition_penalty;
                else s[t] *= params->repetition_penalty;
            }
        }
    }
    if (temperature != 1.0f && temperature > 0.0f) /* :788-792 */
        for (int64_t i = 0; i < n; i++) s[i] /= temperature;
    float mx = -INFINITY; /* :795-802 */
    for (int64_t i = 0; i < n; i++) mx = fmaxf(mx, s[i]);
    for (int64_t i = 0; i < n; i++) s[i] = expf(s[i] - mx);
    float sum = 0.0f;
    for (int64_t i = 0; i < n; i++) sum += s[i];
    for (int64_t i = 0; i < n; i++) s[i] /= sum;
    idx_p *a = NULL, *tmp = NULL;
    if ((params->top_k > 0 && params->top_k < n) || (params->top_p > 0.0f && params->top_p < 1.0f)) {
        a = (idx_p *)malloc(sizeof(idx_p) * (size_t)n);
        tmp = (idx_p *)malloc(sizeof(idx_p) * (size_t)n);
    }
    if (params->top_k > 0 && params->top_k < n) { /* :805-820 */
        for (int64_t i = 0; i < n; i++) { a[i].idx = i; a[i].p = s[i]; }
        stable_sort_desc(a, n, tmp);
        for (int64_t r = params->top_k; r < n; r++) s[a[r].idx] = 0.0f;
        float sm = 0.0f;
        for (int64_t i = 0; i < n; i++) sm += s[i];
        if (sm > 0.0f)
            for (int64_t i = 0; i < n; i++) s[i] /= sm;
    }
    if (params->top_p > 0.0f && params->top_p < 1.0f) { /* :824-849 */
        for (int64_t i = 0; i < n; i++) { a[i].idx = i; a[i].p = s[i]; }
        stable_sort_desc(a, n, tmp);
        float cum = 0.0f;
        int64_t cutoff = n;
        for (int64_t r = 0; r < n; r++) {
            cum += a[r].p;
            if (cum >= params->top_p) { cutoff = r + 1; break; }
        }
        if (cutoff < 1) cutoff = 1;
        for (int64_t r = cutoff; r < n; r++) s[a[r].idx] = 0.0f;
        float sm = 0.0f;
        for (int64_t i = 0; i < n; i++) sm += s[i];
        if (sm > 0.0f)
            for (int64_t i = 0; i < n; i++) s[i] /= sm;
    }
    free(a);
    free(tmp);
}

uint32_t oq_sample_token(const float *logits, int64_t n, const oq_sample_params *params,
                         const uint32_t *prev_tokens, int32_t n_prev, uint64_t *rng,
                         float temperature) {
    float *s = (float *)malloc(sizeof(float) * (size_t)n);
    oq_sample_probs(logits, n, params, prev_tokens, n_prev, temperature, s);
    float r = oq_simple_rand(rng); /* :852 */
    float cumsum = 0.0f;
    uint32_t out = 0;
    for (int64_t i = 0; i < n; i++) {
        cumsum += s[i];
        if (r < cumsum) { out = (uint32_t)i; break; }
    }
    free(s);
    return out;
}

/* ======================================================================== */
/* One frame of the generation loop: generate_new.rs:606-665                 */
/* ======================================================================== */

int oq_frame(const oq_talker *t, const oq_predictor *p, oq_kv *talker_kv, oq_kv *pred_kv,
             const oq_sample_params *params, const float *text_row, int64_t position,
             float *logits, float *last_hidden, uint32_t *prev_tokens, uint64_t *rng,
             uint32_t *codes_out) {
    int32_t H = t->hidden;
    uint32_t sem = oq_sample_token(logits, t->vocab, params, prev_tokens, 16, rng,
                                   params->temperature);               /* :609 */
    codes_out[0] = sem;
    prev_tokens[0] = sem;                                              /* :617 */
    float *semb = (float *)malloc(sizeof(float) * (size_t)H);
    float *acc = (float *)malloc(sizeof(float) * (size_t)H);
    oq_embed_codec_token(t, sem, semb);                                /* :620 */
    int rc = oq_predictor_frame(p, last_hidden, semb, pred_kv, codes_out + 1, NULL); /* :625 */
    if (rc == 0) {
        for (int32_t i = 0; i < p->num_groups; i++) prev_tokens[i + 1] = codes_out[i + 1];
        oq_acoustic_embeddings_sum(p, codes_out + 1, acc);             /* :640 */
        for (int32_t j = 0; j < H; j++) semb[j] += acc[j];             /* :641-643 */
        for (int32_t j = 0; j < H; j++) semb[j] += text_row[j];        /* :652-654 */
        rc = oq_talker_step(t, semb, talker_kv, position, last_hidden, logits); /* :658 */
    }
    free(semb);
    free(acc);
    return rc;
}

/* ======================================================================== */
/* Synthetic data: counter-based splitmix64 + Box-Muller                     */
/* ======================================================================== */

static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Element pair p of stream `seed`: u1 in (0,1], u2 in [0,1);
 * z0 = r cos(2 pi u2), z1 = r sin(2 pi u2), r = sqrt(-2 ln u1). */
static inline void normal_pair(uint64_t seed, int64_t p, float sigma, float *z0, float *z1) {
    uint64_t base = mix64(seed) ^ 0xD1B54A32D192ED03ull;
    uint64_t a = mix64(base + 2 * (uint64_t)p);
    uint64_t b = mix64(base + 2 * (uint64_t)p + 1);
    double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
    double r = sqrt(-2.0 * log(u1));
    double th = 6.283185307179586 * u2;
    *z0 = (float)((double)sigma * r * cos(th));
    *z1 = (float)((double)sigma * r * sin(th));
}

typedef struct {
    uint64_t seed;
    float sigma;
    int64_t count;
    float *out;
    int64_t per_task;
} synth_arg;

static void synth_task(void *argp, int t) {
    synth_arg *a = (synth_arg *)argp;
    int64_t p0 = (int64_t)t * a->per_task, p1 = p0 + a->per_task;
    int64_t npairs = (a->count + 1) / 2;
    if (p1 > npairs) p1 = npairs;
    for (int64_t p = p0; p < p1; p++) {
        float z0, z1;
        normal_pair(a->seed, p, a->sigma, &z0, &z1);
        a->out[2 * p] = z0;
        if (2 * p + 1 < a->count) a->out[2 * p + 1] = z1;
    }
}

void oq_synth_normal(uint64_t seed, float sigma, int64_t count, float *out) {
    int64_t npairs = (count + 1) / 2;
    int64_t per = 1 << 16;
    int64_t tasks = (npairs + per - 1) / per;
    synth_arg a = {seed, sigma, count, out, per};
    if (tasks <= 1) {
        if (tasks == 1) synth_task(&a, 0);
        return;
    }
    pool_run(synth_task, &a, (int)tasks);
}

typedef struct {
    const float *data;
    int64_t n;
    uint8_t *packed;
    uint16_t *scales;
    int64_t rows_per_task, k;
} quant_arg;

static void quant_task(void *argp, int t) {
    quant_arg *a = (quant_arg *)argp;
    int64_t r0 = (int64_t)t * a->rows_per_task, r1 = r0 + a->rows_per_task;
    if (r1 > a->k) r1 = a->k;
    if (r0 >= r1) return;
    int64_t gpr = a->n / Q4_GROUP;
    oq_quantize_f32_to_q4(a->data + r0 * a->n, r1 - r0, a->n, a->packed + r0 * gpr * 16,
                          a->scales + r0 * gpr);
}

void oq_synth_q4(uint64_t seed, float sigma, int64_t k, int64_t n, uint8_t *packed,
                 uint16_t *scales) {
    float *tmp = (float *)malloc(sizeof(float) * (size_t)(k * n));
    oq_synth_normal(seed, sigma, k * n, tmp);
    int64_t rows = 64;
    int64_t tasks = (k + rows - 1) / rows;
    quant_arg a = {tmp, n, packed, scales, rows, k};
    if (tasks <= 1) quant_task(&a, 0);
    else pool_run(quant_task, &a, (int)tasks);
    free(tmp);
}

/* ======================================================================== */
/* The reference's GEMV-test generators: gemv.rs:693-730                    */
/* ======================================================================== */

uint64_t oq_xrng(uint64_t *state) {
    *state ^= *state << 13;
    *state ^= *state >> 7;
    *state ^= *state << 17;
    return *state;
}

void oq_test_rbytes(uint64_t *state, int64_t n, uint8_t *out) {
    for (int64_t i = 0; i < n; i++) out[i] = (uint8_t)(oq_xrng(state) & 0xff);
}

void oq_test_rscales(uint64_t *state, int64_t n, double zero_frac, uint16_t *out) {
    for (int64_t i = 0; i < n; i++) {
        double r = (double)(oq_xrng(state) % 1000) / 1000.0;
        if (r < zero_frac) {
            out[i] = oq_f32_to_f16(0.0f);
        } else {
            float v = ((float)(oq_xrng(state) % 2000) / 1000.0f - 1.0f) * 0.05f;
            out[i] = oq_f32_to_f16(v);
        }
    }
}

void oq_test_rinput(uint64_t *state, int64_t n, double zero_frac, float *out) {
    for (int64_t i = 0; i < n; i++) {
        double r = (double)(oq_xrng(state) % 1000) / 1000.0;
        if (r < zero_frac) out[i] = 0.0f;
        else out[i] = ((float)(oq_xrng(state) % 2000) / 1000.0f - 1.0f) * 2.0f;
    }
}
