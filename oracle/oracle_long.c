/*
 * Oracle for long sequences (test infrastructure only; see oracle.h).
 *
 * The same arithmetic as oq_gemm and the prefill of oracle.c
 * (prefill_talker_raw_from, talker.rs:379-482; gemm_q4, gemv.rs:349-412),
 * organised so that thousands of positions finish in seconds on the host:
 *   - the Q4 GEMM walks a block of token rows per 32-column group, so each
 *     weight row is read once per block instead of once per token, with
 *     every output element still accumulated in the reference's k order from
 *     the rounded products scale * x * (q - 8) (gemv.rs:249-287);
 *   - the causal attention computes 16 keys' dot products side by side (each
 *     still summed in head-dimension order) and the weighted V sum 16
 *     head-dimension values side by side (each still summed in key order);
 *   - both run on every host core (one pthread per core, tasks taken from a
 *     shared counter).
 * Separate multiplies and adds (compiled with -ffp-contract=off), so every
 * value equals the one oracle.c computes, bit for bit
 * (tests/test_oracle_long.py holds them equal).
 */
#define _GNU_SOURCE
#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "oracle.h"

/* ---- parallel for: fn(arg, i) for i in [0, n), on every host core ---- */
typedef struct {
    void (*fn)(void *, int64_t);
    void *arg;
    int64_t n;
    atomic_llong next;
} par_job;

static void *par_worker(void *p) {
    par_job *j = (par_job *)p;
    for (;;) {
        const int64_t i = atomic_fetch_add(&j->next, 1);
        if (i >= j->n) break;
        j->fn(j->arg, i);
    }
    return NULL;
}

static void par_for(int64_t n, void (*fn)(void *, int64_t), void *arg) {
    long cores = sysconf(_SC_NPROCESSORS_ONLN);
    if (cores < 1) cores = 1;
    if (cores > 256) cores = 256;
    int nt = (int)(n < cores ? n : cores);
    par_job j;
    j.fn = fn;
    j.arg = arg;
    j.n = n;
    atomic_init(&j.next, 0);
    pthread_t th[256];
    int started = 0;
    for (int i = 1; i < nt; i++)
        if (pthread_create(&th[started], NULL, par_worker, &j) == 0) started++;
    par_worker(&j); /* the caller works too; tasks left by failed creations are its */
    for (int i = 0; i < started; i++) pthread_join(th[i], NULL);
}

#define Q4_GROUP 32
#define ROW_BLOCK 12 /* token rows per GEMM task (accumulators stay in registers) */

static const float FACTORS[16] = {-8, -7, -6, -5, -4, -3, -2, -1, 0, 1, 2, 3, 4, 5, 6, 7};

/* One 32-column group g of rows [t0, t0 + nt) over all k: out[t][32g ..] =
 * sum_k x[t][k] * scale[k][g] * (q[k][g][j] - 8), summed in k order from the
 * rounded products, skipping x == 0 and s == 0 as gemv.rs:259, 266 do. */
static void gemm_group_scalar(const float *x, int64_t ldx, const oq_q4 *w, int64_t g, int64_t t0,
                              int nt, float *out, int64_t ldo) {
    const int64_t gpr = w->n / Q4_GROUP, ppr = gpr * 16;
    float acc[ROW_BLOCK][Q4_GROUP];
    memset(acc, 0, sizeof(acc));
    for (int64_t k = 0; k < w->k; k++) {
        const float sc = oq_f16_to_f32(w->scales[k * gpr + g]);
        const uint8_t *p = w->packed + k * ppr + g * 16;
        for (int t = 0; t < nt; t++) {
            const float xv = x[(t0 + t) * ldx + k];
            if (xv == 0.0f) continue;
            const float s = sc * xv;
            if (s == 0.0f) continue;
            for (int j = 0; j < 16; j++) {
                acc[t][2 * j] += s * FACTORS[p[j] & 15];
                acc[t][2 * j + 1] += s * FACTORS[p[j] >> 4];
            }
        }
    }
    for (int t = 0; t < nt; t++) memcpy(out + (t0 + t) * ldo + g * Q4_GROUP, acc[t], sizeof(acc[t]));
}

static const int32_t IL_FIRST[16] = {0, 16, 1, 17, 2, 18, 3, 19, 4, 20, 5, 21, 6, 22, 7, 23};
static const int32_t IL_SECOND[16] = {8, 24, 9, 25, 10, 26, 11, 27, 12, 28, 13, 29, 14, 30, 15, 31};

__attribute__((target("avx512f"))) static void gemm_group_avx512(const float *x, int64_t ldx,
                                                                  const oq_q4 *w, int64_t g,
                                                                  int64_t t0, int nt, float *out,
                                                                  int64_t ldo) {
    const int64_t gpr = w->n / Q4_GROUP, ppr = gpr * 16;
    const __m512 factors = _mm512_loadu_ps(FACTORS);
    const __m512i il_lo = _mm512_loadu_si512((const void *)IL_FIRST);
    const __m512i il_hi = _mm512_loadu_si512((const void *)IL_SECOND);
    const __m512i mask = _mm512_set1_epi32(15);
    __m512 a0[ROW_BLOCK], a1[ROW_BLOCK];
    for (int t = 0; t < ROW_BLOCK; t++) a0[t] = a1[t] = _mm512_setzero_ps();
    for (int64_t k = 0; k < w->k; k++) {
        const float sc = oq_f16_to_f32(w->scales[k * gpr + g]);
        const __m512i b32 = _mm512_cvtepu8_epi32(_mm_loadu_si128((const __m128i *)(w->packed + k * ppr + g * 16)));
        const __m512 lo = _mm512_permutexvar_ps(_mm512_and_epi32(b32, mask), factors);
        const __m512 hi = _mm512_permutexvar_ps(_mm512_srli_epi32(b32, 4), factors);
        /* the (q - 8) factors of columns 0..15 and 16..31 of the group */
        const __m512 f0 = _mm512_permutex2var_ps(lo, il_lo, hi);
        const __m512 f1 = _mm512_permutex2var_ps(lo, il_hi, hi);
        for (int t = 0; t < nt; t++) {
            const float xv = x[(t0 + t) * ldx + k];
            if (xv == 0.0f) continue;
            const float s = sc * xv;
            if (s == 0.0f) continue;
            const __m512 sv = _mm512_set1_ps(s);
            a0[t] = _mm512_add_ps(a0[t], _mm512_mul_ps(f0, sv));
            a1[t] = _mm512_add_ps(a1[t], _mm512_mul_ps(f1, sv));
        }
    }
    for (int t = 0; t < nt; t++) {
        _mm512_storeu_ps(out + (t0 + t) * ldo + g * Q4_GROUP, a0[t]);
        _mm512_storeu_ps(out + (t0 + t) * ldo + g * Q4_GROUP + 16, a1[t]);
    }
}

/* gemm_q4 (gemv.rs:349-412) for seq_len rows: the bits of oq_gemm.  Output
 * columns past the last full group stay zero (gemv.rs:846-861). */
typedef struct {
    const float *x;
    const oq_q4 *w;
    float *out;
    int64_t seq_len, gpr;
    int simd;
} gemm_task;

static void gemm_task_run(void *p, int64_t i) {
    const gemm_task *a = (const gemm_task *)p;
    const int64_t tb = i / a->gpr, g = i % a->gpr;
    const int64_t t0 = tb * ROW_BLOCK;
    const int nt = (int)(a->seq_len - t0 < ROW_BLOCK ? a->seq_len - t0 : ROW_BLOCK);
    if (a->simd) gemm_group_avx512(a->x, a->w->k, a->w, g, t0, nt, a->out, a->w->n);
    else gemm_group_scalar(a->x, a->w->k, a->w, g, t0, nt, a->out, a->w->n);
}

void oq_gemm_long(const float *x, int64_t seq_len, const oq_q4 *w, float *out) {
    gemm_task a = {x, w, out, seq_len, w->n / Q4_GROUP, oq_get_simd() >= 2 && oq_has_avx512()};
    const int64_t blocks = (seq_len + ROW_BLOCK - 1) / ROW_BLOCK;
    if (a.gpr > 0) par_for(blocks * a.gpr, gemm_task_run, &a);
    if (w->n > a.gpr * Q4_GROUP)
        for (int64_t t = 0; t < seq_len; t++)
            memset(out + t * w->n + a.gpr * Q4_GROUP, 0, sizeof(float) * (size_t)(w->n - a.gpr * Q4_GROUP));
}

/* One query vector's attention over keys [0, alen) of one kv head
 * (talker.rs:435-458): scores[s] = (sum_e q[e] k[s][e]) * scale,
 * softmax_raw, o[e] = sum_s p[s] v[s][e].  kt is K transposed,
 * [hd][ldkt] (so 16 keys' sums run side by side), v is [len][stride]. */
static void attend_row_scalar(const float *q, const float *kt, int64_t ldkt, const float *v,
                              int64_t vstride, int64_t alen, int32_t hd, float scale,
                              float *scores, float *o) {
    for (int64_t s = 0; s < alen; s++) {
        float dot = 0.0f;
        for (int32_t e = 0; e < hd; e++) dot += q[e] * kt[(int64_t)e * ldkt + s];
        scores[s] = dot * scale;
    }
    oq_softmax_raw(scores, alen);
    memset(o, 0, sizeof(float) * (size_t)hd);
    for (int64_t s = 0; s < alen; s++) {
        const float p = scores[s];
        const float *vr = v + s * vstride;
        for (int32_t e = 0; e < hd; e++) o[e] += p * vr[e];
    }
}

__attribute__((target("avx512f"))) static void attend_row_avx512(
    const float *q, const float *kt, int64_t ldkt, const float *v, int64_t vstride, int64_t alen,
    int32_t hd, float scale, float *scores, float *o) {
    int64_t s = 0;
    for (; s + 16 <= alen; s += 16) {
        __m512 dot = _mm512_setzero_ps();
        for (int32_t e = 0; e < hd; e++)
            dot = _mm512_add_ps(dot, _mm512_mul_ps(_mm512_set1_ps(q[e]), _mm512_loadu_ps(kt + (int64_t)e * ldkt + s)));
        _mm512_storeu_ps(scores + s, _mm512_mul_ps(dot, _mm512_set1_ps(scale)));
    }
    for (; s < alen; s++) {
        float dot = 0.0f;
        for (int32_t e = 0; e < hd; e++) dot += q[e] * kt[(int64_t)e * ldkt + s];
        scores[s] = dot * scale;
    }
    oq_softmax_raw(scores, alen);
    __m512 acc[8]; /* hd <= 128 */
    const int nv = hd / 16;
    for (int i = 0; i < nv; i++) acc[i] = _mm512_setzero_ps();
    for (s = 0; s < alen; s++) {
        const __m512 p = _mm512_set1_ps(scores[s]);
        const float *vr = v + s * vstride;
        for (int i = 0; i < nv; i++) acc[i] = _mm512_add_ps(acc[i], _mm512_mul_ps(p, _mm512_loadu_ps(vr + 16 * i)));
    }
    for (int i = 0; i < nv; i++) _mm512_storeu_ps(o + 16 * i, acc[i]);
}

/* Per-row pieces of a layer, one task per row. */
typedef struct {
    const oq_talker *t;
    const oq_layer *lw;
    float *x, *xn, *q, *kn;
    int64_t start_pos;
    int stage; /* 0: input norm; 1: qk-norm + RoPE; 2: post-attention norm */
} row_task;

static void row_task_run(void *p, int64_t r) {
    const row_task *a = (const row_task *)p;
    const oq_talker *t = a->t;
    const int32_t H = t->hidden, hd = t->head_dim, qd = t->num_heads * hd, kd = t->num_kv_heads * hd;
    const int64_t rope_len = (int64_t)t->rope_max_pos * (hd / 2);
    if (a->stage == 0) {
        oq_rms_norm_f16(a->x + r * H, a->lw->input_norm, H, a->xn + r * H);
    } else if (a->stage == 1) {
        oq_qk_norm(a->q + r * qd, t->num_heads, hd, a->lw->q_norm);
        oq_qk_norm(a->kn + r * kd, t->num_kv_heads, hd, a->lw->k_norm);
        oq_apply_rope_split(a->q + r * qd, t->num_heads, hd, a->start_pos + r, t->rope_cos, t->rope_sin, rope_len);
        oq_apply_rope_split(a->kn + r * kd, t->num_kv_heads, hd, a->start_pos + r, t->rope_cos, t->rope_sin,
                            rope_len);
    } else {
        oq_rms_norm_f16(a->x + r * H, a->lw->post_attn_norm, H, a->xn + r * H);
    }
}

typedef struct {
    const float *q, *kt, *vc;
    float *att;
    int64_t T, start_pos, ldkt;
    int32_t heads, kvh, hd;
    float scale;
    int simd;
} attn_task;

static void attn_task_run(void *p, int64_t i) {
    const attn_task *a = (const attn_task *)p;
    const int64_t t1 = a->T - 1 - i / a->heads; /* the longest rows first */
    const int32_t h = (int32_t)(i % a->heads);
    const int32_t g = h / (a->heads / a->kvh);
    const int32_t qd = a->heads * a->hd, kd = a->kvh * a->hd;
    const int64_t alen = a->start_pos + t1 + 1;
    float *scores = (float *)malloc(sizeof(float) * (size_t)alen);
    const float *qv = a->q + t1 * qd + (int64_t)h * a->hd;
    const float *ktg = a->kt + (int64_t)g * a->hd * a->ldkt;
    const float *vg = a->vc + (int64_t)g * a->hd;
    float *o = a->att + t1 * qd + (int64_t)h * a->hd;
    if (a->simd) attend_row_avx512(qv, ktg, a->ldkt, vg, kd, alen, a->hd, a->scale, scores, o);
    else attend_row_scalar(qv, ktg, a->ldkt, vg, kd, alen, a->hd, a->scale, scores, o);
    free(scores);
}

typedef struct {
    const float *kc;
    float *kt;
    int64_t L, ldkt;
    int32_t hd, kd;
} transpose_task;

static void transpose_task_run(void *p, int64_t i) { /* i = kv head * hd + e */
    const transpose_task *a = (const transpose_task *)p;
    const int64_t h = i / a->hd, e = i % a->hd;
    float *dst = a->kt + i * a->ldkt;
    for (int64_t s = 0; s < a->L; s++) dst[s] = a->kc[s * a->kd + h * a->hd + e];
}

typedef struct {
    float *gate;
    const float *up;
    int64_t n;
} silu_task;

static void silu_task_run(void *p, int64_t i) { /* chunks of 65536 values */
    const silu_task *a = (const silu_task *)p;
    const int64_t j1 = (i + 1) * 65536 < a->n ? (i + 1) * 65536 : a->n;
    for (int64_t j = i * 65536; j < j1; j++) a->gate[j] = oq_silu(a->gate[j]) * a->up[j];
}

/* prefill_layer of oracle.c (talker.rs:389-477) with the blocked GEMM and the
 * vectorised attention; returns -1 past the cache, -3 on a length mismatch. */
static int prefill_layer_long(const oq_talker *t, const oq_layer *lw, float *x, int64_t T,
                              oq_kv *kv, int32_t layer, int64_t start_pos) {
    const int32_t H = t->hidden, hd = t->head_dim, heads = t->num_heads, kvh = t->num_kv_heads;
    const int32_t qd = heads * hd, kd = kvh * hd, F = t->ffn;
    if (oq_kv_len(kv, layer) != start_pos) return -3;
    if (start_pos + T > oq_kv_max_pos(kv)) return -1;
    float *xn = (float *)malloc(sizeof(float) * (size_t)(T * H));
    float *q = (float *)malloc(sizeof(float) * (size_t)(T * qd));
    float *kn = (float *)malloc(sizeof(float) * (size_t)(T * kd));
    float *vn = (float *)malloc(sizeof(float) * (size_t)(T * kd));
    float *att = (float *)malloc(sizeof(float) * (size_t)(T * qd));
    float *tmp = (float *)malloc(sizeof(float) * (size_t)(T * H));
    float *gate = (float *)malloc(sizeof(float) * (size_t)(T * F));
    float *up = (float *)malloc(sizeof(float) * (size_t)(T * F));

    row_task rt = {t, lw, x, xn, q, kn, start_pos, 0};
    par_for(T, row_task_run, &rt);
    oq_gemm_long(xn, T, &lw->q_proj, q);
    oq_gemm_long(xn, T, &lw->k_proj, kn);
    oq_gemm_long(xn, T, &lw->v_proj, vn);
    rt.stage = 1;
    par_for(T, row_task_run, &rt);
    float *kc = oq_kv_k(kv, layer), *vc = oq_kv_v(kv, layer);
    memcpy(kc + start_pos * kd, kn, sizeof(float) * (size_t)(T * kd));
    memcpy(vc + start_pos * kd, vn, sizeof(float) * (size_t)(T * kd));
    oq_kv_set_len(kv, layer, (int32_t)(start_pos + T));
    /* causal attention (talker.rs:435-458); K of each kv head transposed to [hd][positions] */
    const int64_t L = start_pos + T, ldkt = (L + 15) / 16 * 16;
    float *kt = (float *)malloc(sizeof(float) * (size_t)(kvh * hd * ldkt));
    transpose_task tt = {kc, kt, L, ldkt, hd, kd};
    par_for((int64_t)kvh * hd, transpose_task_run, &tt);
    attn_task at = {q, kt, vc, att, T, start_pos, ldkt, heads, kvh, hd, 1.0f / sqrtf((float)hd),
                    oq_has_avx512() && hd % 16 == 0 && hd <= 128};
    par_for(T * heads, attn_task_run, &at);
    free(kt);
    oq_gemm_long(att, T, &lw->o_proj, tmp);
    for (int64_t j = 0; j < T * H; j++) x[j] += tmp[j];
    rt.stage = 2;
    par_for(T, row_task_run, &rt);
    oq_gemm_long(xn, T, &lw->gate_proj, gate);
    oq_gemm_long(xn, T, &lw->up_proj, up);
    silu_task st = {gate, up, T * F};
    par_for((T * F + 65535) / 65536, silu_task_run, &st);
    oq_gemm_long(gate, T, &lw->down_proj, tmp);
    for (int64_t j = 0; j < T * H; j++) x[j] += tmp[j];
    free(xn); free(q); free(kn); free(vn); free(att); free(tmp); free(gate); free(up);
    return 0;
}

typedef struct {
    const float *x;
    const uint16_t *gamma;
    float *out;
    int32_t H;
} norm_task;

static void norm_task_run(void *p, int64_t r) {
    const norm_task *a = (const norm_task *)p;
    oq_rms_norm_f16(a->x + r * a->H, a->gamma, a->H, a->out + r * a->H);
}

int oq_talker_prefill_rows(const oq_talker *t, const float *x_in, int64_t seq_len, oq_kv *kv,
                           int64_t start_pos, float *out_hidden_rows, float *out_logits_rows) {
    if (seq_len <= 0) return -4;
    if (start_pos + seq_len > t->rope_max_pos) return -2;
    const int32_t H = t->hidden;
    float *x = (float *)malloc(sizeof(float) * (size_t)(seq_len * H));
    memcpy(x, x_in, sizeof(float) * (size_t)(seq_len * H));
    int rc = 0;
    for (int32_t l = 0; l < t->num_layers && rc == 0; l++)
        rc = prefill_layer_long(t, &t->layers[l], x, seq_len, kv, l, start_pos);
    if (rc == 0) {
        norm_task nt = {x, t->final_norm, out_hidden_rows, H};  /* talker.rs:480-481 */
        par_for(seq_len, norm_task_run, &nt);
        if (out_logits_rows) oq_gemm_long(out_hidden_rows, seq_len, &t->codec_head, out_logits_rows);
    }
    free(x);
    return rc;
}
