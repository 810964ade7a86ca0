/*
 * QORA-TTS decode-path ORACLE — CPU restatement of the reference's Rust CPU
 * path (swordreforge/QORA-TTS-12Hz-1.7B, src/gemv.rs, src/simd.rs,
 * src/gpool.rs, src/rope.rs, src/talker.rs, src/code_predictor.rs,
 * src/generate_new.rs).
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library, and
 * only as the checker or as the timed CPU baseline.  The product (the CUDA
 * library) never links or calls it.
 *
 * Parity pin: the reference's Rust toolchain is absent, so the reference
 * cannot be built or run here.  The restatement is pinned by the reference's
 * own known-answer tests, restated (gemv.rs:689-862: SIMD == scalar bit-exact
 * on its xorshift generators, k-chunk assembly, tail-n behaviour;
 * generate_new.rs:918-955: sampler top-p behaviour), plus IEEE binary16
 * conversion checked exhaustively against numpy.  Model-level outputs have no
 * reference golden vectors.
 */
#ifndef QORA_ORACLE_H
#define QORA_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- weights (reference layout, gemv.rs:26-31) ------------------------- */
/* packed: u8[k * (n/32) * 16], byte (ki, g, j) at ki*(n/32)*16 + g*16 + j holds
 * column 32g+2j in the low nibble and 32g+2j+1 in the high nibble.
 * scales: f16 bits [k * (n/32)] at ki*(n/32) + g. */
typedef struct oq_q4 {
    const uint8_t *packed;
    const uint16_t *scales;
    int64_t k, n;
} oq_q4;

typedef struct oq_layer {
    oq_q4 q_proj, k_proj, v_proj, o_proj, gate_proj, up_proj, down_proj;
    const uint16_t *q_norm, *k_norm, *input_norm, *post_attn_norm; /* f16 */
} oq_layer;

/* TalkerWeights (talker.rs:33-56), hot-path fields only. */
typedef struct oq_talker {
    int32_t num_layers, hidden, num_heads, num_kv_heads, head_dim, ffn, vocab;
    int32_t rope_max_pos;
    const oq_layer *layers;
    oq_q4 codec_embedding; /* [vocab][hidden] */
    oq_q4 codec_head;      /* [hidden][vocab] */
    const uint16_t *final_norm;
    const float *rope_cos, *rope_sin; /* [rope_max_pos][head_dim/2] */
} oq_talker;

/* CodePredictorWeights (code_predictor.rs:28-46). */
typedef struct oq_predictor {
    int32_t num_layers, hidden, num_heads, num_kv_heads, head_dim, ffn, vocab;
    int32_t num_groups; /* 15 acoustic groups */
    int32_t rope_max_pos;
    const oq_layer *layers;
    oq_q4 input_proj;             /* [talker_hidden][hidden]; packed==NULL => identity */
    const float *input_proj_bias; /* [hidden] or NULL */
    const oq_q4 *codec_embeddings; /* num_groups x [vocab][embed_dim] */
    const oq_q4 *lm_heads;         /* num_groups x [hidden][vocab] */
    const uint16_t *final_norm;
    const float *rope_cos, *rope_sin;
} oq_predictor;

/* RawKvCache (gemv.rs:75-86): per layer token-major [len][kv_heads][hd] f32. */
typedef struct oq_kv oq_kv;

/* ---- f16 ---------------------------------------------------------------- */
float oq_f16_to_f32(uint16_t h);
uint16_t oq_f32_to_f16(float f); /* IEEE round-to-nearest-even */
void oq_f32_to_f16_array(const float *src, uint16_t *dst, int64_t n);
void oq_f16_to_f32_array(const uint16_t *src, float *dst, int64_t n);

/* ---- gemv.rs ----------------------------------------------------------- */
void oq_quantize_f32_to_q4(const float *data, int64_t k, int64_t n,
                           uint8_t *packed, uint16_t *scales);
void oq_gemv_q4_scalar(const float *x, const uint8_t *packed, const uint16_t *scales,
                       int64_t n, int64_t k_start, int64_t k_end, float *out);
void oq_gemv_q4_avx2(const float *x, const uint8_t *packed, const uint16_t *scales,
                     int64_t n, int64_t k_start, int64_t k_end, float *out);
void oq_gemv_q4_avx512(const float *x, const uint8_t *packed, const uint16_t *scales,
                       int64_t n, int64_t k_start, int64_t k_end, float *out);
int oq_has_avx2(void);
int oq_has_avx512(void);
/* gemv_q4_inner dispatch: avx512 > avx2 > scalar (gemv.rs:230-243);
 * simd = 0 forces scalar. */
void oq_gemv_q4_inner(const float *x, const oq_q4 *w, int64_t k_start, int64_t k_end,
                      float *out);
/* gemv_q4 with the pool chunking of gemv.rs:290-346 for `workers` workers;
 * workers <= 0 uses the pool's own size (min(nproc,16) or QORA_THREADS). */
void oq_gemv(const float *x, const oq_q4 *w, float *out);
void oq_gemv_workers(const float *x, const oq_q4 *w, float *out, int workers);
void oq_gemm(const float *x, int64_t seq_len, const oq_q4 *w, float *out);
void oq_embed_lookup(const oq_q4 *w, int64_t token, float *out);
void oq_rms_norm_f16(const float *x, const uint16_t *gamma, int64_t n, float *out);
void oq_softmax_raw(float *s, int64_t n);
float oq_silu(float x);

/* ---- pool (gpool.rs) ----------------------------------------------------- */
int oq_pool_workers(void);
void oq_pool_set_workers(int workers); /* must precede first use */
/* SIMD selection: 2 = avx512 (if present), 1 = avx2, 0 = scalar. */
void oq_set_simd(int level);
int oq_get_simd(void);

/* ---- rope.rs / loader.rs ------------------------------------------------- */
void oq_build_rope_tables(int32_t head_dim, int32_t max_pos, double theta,
                          const int32_t *sections, int32_t n_sections,
                          float *cos_table, float *sin_table);
void oq_apply_rope_split(float *data, int32_t num_heads, int32_t head_dim, int64_t position,
                         const float *cos_table, const float *sin_table, int64_t table_len);
void oq_qk_norm(float *data, int32_t num_heads, int32_t head_dim, const uint16_t *gamma);

/* ---- KV ------------------------------------------------------------------ */
oq_kv *oq_kv_create(int32_t num_layers, int32_t kv_heads, int32_t head_dim, int32_t max_pos);
void oq_kv_destroy(oq_kv *kv);
void oq_kv_reset(oq_kv *kv);
int32_t oq_kv_len(const oq_kv *kv, int32_t layer);
int32_t oq_kv_max_pos(const oq_kv *kv);
void oq_kv_set_len(oq_kv *kv, int32_t layer, int32_t len);
float *oq_kv_k(oq_kv *kv, int32_t layer);
float *oq_kv_v(oq_kv *kv, int32_t layer);
int oq_kv_copy(oq_kv *dst, const oq_kv *src);

/* Attention block of one decode step of one layer from raw q/k/v projections
 * (talker.rs:285-331): qk-norm, split RoPE at `position`, append, attend. */
int oq_attend_step(const float *q_raw, const float *k_raw, const float *v_raw, int32_t heads,
                   int32_t kv_heads, int32_t hd, const uint16_t *q_norm, const uint16_t *k_norm,
                   const float *rope_cos, const float *rope_sin, int64_t rope_len,
                   int64_t position, oq_kv *kv, int32_t layer, float *out);

/* ---- talker.rs ----------------------------------------------------------- */
/* forward_with_embedding (talker.rs:263-360): out_hidden[hidden], out_logits[vocab]. */
int oq_talker_step(const oq_talker *t, const float *embedding, oq_kv *kv, int64_t position,
                   float *out_hidden, float *out_logits);
/* prefill_talker_raw_from (talker.rs:379-482): returns final-normed last hidden. */
int oq_talker_prefill(const oq_talker *t, const float *x, int64_t seq_len, oq_kv *kv,
                      int64_t start_pos, float *out_hidden);
/* Long sequences (oracle_long.c): the same values as oq_gemm and
 * oq_talker_prefill, blocked and run on every host core.
 * oq_talker_prefill_rows also returns every row's final-normed hidden
 * (out_hidden_rows [seq_len][hidden]) and, when out_logits_rows is not NULL,
 * every row's codec-head logits [seq_len][vocab]. */
void oq_gemm_long(const float *x, int64_t seq_len, const oq_q4 *w, float *out);
int oq_talker_prefill_rows(const oq_talker *t, const float *x, int64_t seq_len, oq_kv *kv,
                           int64_t start_pos, float *out_hidden_rows, float *out_logits_rows);
/* apply_codec_head (talker.rs:647-649). */
void oq_codec_head(const oq_talker *t, const float *hidden, float *out_logits);
void oq_embed_codec_token(const oq_talker *t, uint32_t token, float *out);

/* TalkerWeights text path (talker.rs:33-56, loader.rs:280-284):
 * text_embedding [text_vocab][text_hidden], text_projection.linear_fc1
 * [text_hidden][mid] + bias [mid], linear_fc2 [mid][hidden] + bias [hidden]. */
typedef struct oq_text_proj {
    oq_q4 text_embedding, fc1, fc2;
    const float *fc1_bias, *fc2_bias;
} oq_text_proj;
/* embed_text_token (talker.rs:104-116): out [fc2.n]. */
void oq_embed_text_token(const oq_text_proj *tp, uint32_t token, float *out);
/* forward_talker_decode (talker.rs:161-258): embed the token (text path when
 * is_text, else the codec embedding), one talker step at `position`;
 * out_hidden [hidden] final-normed. */
int oq_talker_decode(const oq_talker *t, const oq_text_proj *tp, uint32_t token, int is_text,
                     oq_kv *kv, int64_t position, float *out_hidden);

/* ---- code_predictor.rs --------------------------------------------------- */
int oq_predictor_frame(const oq_predictor *p, const float *talker_hidden,
                       const float *semantic_embed, oq_kv *kv, uint32_t *codes_out,
                       float *logits_out /* optional [num_groups][vocab] */);
/* Teacher-forced variant: the argmax codes are replaced by forced_codes for
 * the next step's input (logits_out still records every head's logits). */
int oq_predictor_frame_forced(const oq_predictor *p, const float *talker_hidden,
                              const float *semantic_embed, oq_kv *kv,
                              const uint32_t *forced_codes, uint32_t *codes_out,
                              float *logits_out);
void oq_acoustic_embeddings_sum(const oq_predictor *p, const uint32_t *codes, float *out);
uint32_t oq_argmax(const float *logits, int64_t n);
void oq_project_input(const oq_predictor *p, const float *in, float *out);

/* ---- generate_new.rs ----------------------------------------------------- */
typedef struct oq_sample_params {
    float temperature;
    int32_t top_k;
    float top_p;
    float repetition_penalty;
} oq_sample_params;
float oq_simple_rand(uint64_t *state);
uint32_t oq_sample_token(const float *logits, int64_t n, const oq_sample_params *params,
                         const uint32_t *prev_tokens, int32_t n_prev, uint64_t *rng,
                         float temperature);
/* Probabilities after penalty/temperature/softmax/top-k/top-p (the vector the
 * final draw scans), for boundary analysis in tests. */
void oq_sample_probs(const float *logits, int64_t n, const oq_sample_params *params,
                     const uint32_t *prev_tokens, int32_t n_prev, float temperature,
                     float *probs_out);

/* One frame of generate_new.rs:606-665 for one stream (EOS ignored).
 * state: logits[vocab] (in/out), last_hidden[hidden] (in/out), prev_tokens[16]
 * (in/out), rng (in/out); codes_out[16]. */
int oq_frame(const oq_talker *t, const oq_predictor *p, oq_kv *talker_kv, oq_kv *pred_kv,
             const oq_sample_params *params, const float *text_row, int64_t position,
             float *logits, float *last_hidden, uint32_t *prev_tokens, uint64_t *rng,
             uint32_t *codes_out);

/* ---- synthetic data (counter-based, deterministic) ----------------------- */
void oq_synth_normal(uint64_t seed, float sigma, int64_t count, float *out);
void oq_synth_q4(uint64_t seed, float sigma, int64_t k, int64_t n, uint8_t *packed,
                 uint16_t *scales);

/* xorshift generators of the reference's GEMV tests (gemv.rs:693-730). */
uint64_t oq_xrng(uint64_t *state);
void oq_test_rbytes(uint64_t *state, int64_t n, uint8_t *out);
void oq_test_rscales(uint64_t *state, int64_t n, double zero_frac, uint16_t *out);
void oq_test_rinput(uint64_t *state, int64_t n, double zero_frac, float *out);

#ifdef __cplusplus
}
#endif
#endif
