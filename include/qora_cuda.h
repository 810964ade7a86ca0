/*
 * qora_cuda.h — C ABI of the B200 decode engine for QORA-TTS-12Hz-1.7B.
 *
 * Drop-in boundary for the reference's Rust operator surface (paths are
 * within swordreforge/QORA-TTS-12Hz-1.7B).  Each entry point names the
 * reference function it replaces.  Conventions:
 *   - every function returns a status (QORA_OK = 0); no exceptions cross the
 *     ABI; qora_last_error() gives a message for the calling thread;
 *   - tensor pointers are DEVICE pointers unless the name ends in _host;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default);
 *   - handles are owned by the library and freed by their *_destroy; a
 *     context, and everything created from it, is used from one host thread
 *     or stream at a time (calls on one stream are ordered by that stream);
 *   - weights arrive in the reference layout (gemv.rs:26-31, input-major
 *     [k][n], 4-bit nibbles in 32-wide output groups, f16 scale per group)
 *     and are repacked on upload.
 * The reference has no Result on its hot path; its panics (slice bounds,
 * argmax unwrap, debug asserts) become QORA_ERR_* statuses here.
 */
#ifndef QORA_CUDA_H
#define QORA_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QORA_OK 0
#define QORA_ERR_INVALID 1   /* null pointer, bad argument */
#define QORA_ERR_SHAPE 2     /* shape mismatch (e.g. x length != k) */
#define QORA_ERR_CUDA 3      /* a CUDA runtime call failed */
#define QORA_ERR_OOM 4       /* device allocation failed */
#define QORA_ERR_RANGE 5     /* position past RoPE table or KV capacity */
#define QORA_ERR_UNSUPPORTED 6
#define QORA_ERR_TIMEOUT 7   /* bounded device wait expired */

typedef struct qora_ctx qora_ctx;             /* per-device context */
typedef struct qora_w4 qora_w4;               /* device Q4 weight */
typedef struct qora_kv qora_kv;               /* device KV cache, `streams` slabs */
typedef struct qora_talker qora_talker;       /* device TalkerWeights */
typedef struct qora_predictor qora_predictor; /* device CodePredictorWeights */
typedef struct qora_engine qora_engine;       /* per-GPU frame-loop state */
typedef struct qora_model_file qora_model_file; /* a mapped .qora-tts checkpoint */
typedef struct qora_text_proj qora_text_proj;   /* device text projection */

/* Host view of one Q4 weight in the reference layout (gemv.rs:26-31). */
typedef struct qora_q4_host {
    const uint8_t *packed;   /* k * (n/32) * 16 bytes */
    const uint16_t *scales;  /* k * (n/32) f16 bit patterns */
    int64_t k;               /* input dim (rows)  */
    int64_t n;               /* output dim (cols) */
} qora_q4_host;

/* TalkerLayerWeights / PredictorLayerWeights (talker.rs:19-31,
 * code_predictor.rs:14-26). Norm vectors are f16 bit patterns. */
typedef struct qora_layer_host {
    qora_q4_host q_proj, k_proj, v_proj, o_proj, gate_proj, up_proj, down_proj;
    const uint16_t *q_norm, *k_norm, *input_norm, *post_attn_norm;
} qora_layer_host;

/* TalkerWeights hot-path fields (talker.rs:33-56). */
typedef struct qora_talker_host {
    int32_t num_layers, hidden, num_heads, num_kv_heads, head_dim, ffn, vocab;
    int32_t rope_max_pos;            /* max_position_embeddings (config.rs:142) */
    double rope_theta;               /* 1e6 (config.rs:135) */
    const qora_layer_host *layers;
    qora_q4_host codec_embedding;    /* [vocab][hidden] */
    qora_q4_host codec_head;         /* [hidden][vocab] */
    const uint16_t *final_norm;
} qora_talker_host;

/* CodePredictorWeights (code_predictor.rs:28-46). */
typedef struct qora_predictor_host {
    int32_t num_layers, hidden, num_heads, num_kv_heads, head_dim, ffn, vocab;
    int32_t num_groups;              /* 15 acoustic code groups */
    int32_t rope_max_pos;
    double rope_theta;
    const qora_layer_host *layers;
    qora_q4_host input_proj;         /* [talker_hidden][hidden]; packed == NULL => identity */
    const float *input_proj_bias;    /* [hidden] or NULL */
    const qora_q4_host *codec_embeddings; /* num_groups x [vocab][talker_hidden] */
    const qora_q4_host *lm_heads;         /* num_groups x [hidden][vocab] */
    const uint16_t *final_norm;
} qora_predictor_host;

/* TalkerWeights text path (talker.rs:33-56; loader.rs:280-284). */
typedef struct qora_text_proj_host {
    qora_q4_host text_embedding;     /* [text_vocab][text_hidden] */
    qora_q4_host fc1;                /* text_projection.linear_fc1 [text_hidden][mid] */
    qora_q4_host fc2;                /* text_projection.linear_fc2 [mid][hidden] */
    const float *fc1_bias;           /* [mid] */
    const float *fc2_bias;           /* [hidden] */
} qora_text_proj_host;

/* One row of a talker prompt (generate_new.rs:91-466, 756-768): row =
 * text + codec, either part optional.
 *   text  = text_rows[text] (text >= 0; -1: none)
 *   codec = codes_n == 0:  none
 *           codes_n == 1:  codec_embedding[codes[0]]
 *           codes_n == n > 1: codec_embedding[codes[0]] + acoustic_embedding[0][codes[1]]
 *                         + ... + acoustic_embedding[n-2][codes[n-1]], summed in
 *                         that order (a reference frame, generate_new.rs:164-169)
 *           codes_n == -1: the voice embedding (generate_new.rs:214-217, 404-407):
 *                         values past its length are 0, text included. */
typedef struct qora_prompt_row {
    int32_t text;
    int32_t codes_n;
    uint32_t codes[16];
} qora_prompt_row;

/* TTSParams sampling fields (generate_new.rs:38-79). */
typedef struct qora_sample_params {
    float temperature;         /* 0.9 */
    int32_t top_k;             /* 50 */
    float top_p;               /* 1.0 (off) */
    float repetition_penalty;  /* 1.05 */
} qora_sample_params;

/* ---------------------------------------------------------------- context */
int qora_ctx_create(int32_t device, qora_ctx **out);
/* Releases the caller's reference.  Objects created from the context hold
 * references of their own, so the context stays valid until the last of them
 * is destroyed as well. */
void qora_ctx_destroy(qora_ctx *ctx);
const char *qora_status_string(int32_t status);
const char *qora_last_error(void);
/* Device-side error flag raised by kernels (range errors, bounded waits);
 * reading it synchronises `stream`; the flag is cleared. */
int qora_ctx_check_device_error(qora_ctx *ctx, void *stream);

/* ------------------------------------------------------------ gemv.rs */
/* quantize_f32_to_q4 (gemv.rs:92-130), on the host. */
int qora_q4_quantize_host(const float *data_host, int64_t k, int64_t n, uint8_t *packed_host,
                          uint16_t *scales_host);
/* Deterministic synthetic weights (random-init N(0, sigma), then quantised by
 * quantize_f32_to_q4): counter-based splitmix64 + Box-Muller on the host. */
int qora_synth_normal_host(uint64_t seed, float sigma, int64_t count, float *out_host);
int qora_synth_q4_host(uint64_t seed, float sigma, int64_t k, int64_t n, uint8_t *packed_host,
                       uint16_t *scales_host);
/* Q4Weight -> device (repacked to the engine's column-group-major layout). */
int qora_q4_weight_upload(qora_ctx *ctx, const qora_q4_host *w, qora_w4 **out);
void qora_q4_weight_destroy(qora_w4 *w);
/* gemv (gemv.rs:149, 290-346) for `batch` input rows:
 * y[b][0..n) = x[b][0..k) @ W, rows strided by k and n.  batch 1..512. */
int qora_q4_gemv(qora_ctx *ctx, const qora_w4 *w, const float *x, float *y, int32_t batch,
                 void *stream);
/* gemm (gemv.rs:157, 349-412): seq_len token rows. */
int qora_q4_gemm(qora_ctx *ctx, const qora_w4 *w, const float *x, int64_t seq_len, float *y,
                 void *stream);
/* embed_lookup (gemv.rs:165, 415-437): out[i][0..n) = dequantised row tokens[i]
 * (device tokens; one outside the table gives a zero row and QORA_ERR_RANGE at
 * the next qora_ctx_check_device_error). */
int qora_q4_embed_rows(qora_ctx *ctx, const qora_w4 *w, const uint32_t *tokens, int32_t count,
                       float *out, void *stream);
/* rms_norm_f16 (gemv.rs:445-454) over `rows` rows of length n. */
int qora_rms_norm_f16(qora_ctx *ctx, const float *x, const uint16_t *gamma, int64_t n,
                      int32_t rows, float *out, void *stream);

/* ------------------------------------------------------------ rope.rs */
/* build_mrope_tables (rope.rs:11-41; predictor: loader.rs:859-874), host. */
int qora_rope_tables_host(int32_t head_dim, int32_t max_pos, double theta,
                          const int32_t *sections, int32_t n_sections, float *cos_host,
                          float *sin_host);

/* ------------------------------------------------------------ KV cache */
/* RawKvCache / empty_kv_cache (gemv.rs:75-86) for `streams` independent
 * streams, preallocated to max_pos positions.  Device layout per layer:
 * [stream][kv_head][max_pos][head_dim] f32, plus a length per stream. */
int qora_kv_create(qora_ctx *ctx, int32_t num_layers, int32_t kv_heads, int32_t head_dim,
                   int32_t max_pos, int32_t streams, qora_kv **out);
/* RawKvCache / empty_kv_cache (gemv.rs:75-86) with paged storage: where the
 * reference grows one Vec per layer as positions append, a paged cache draws
 * fixed pages from a pool preallocated here: pool_pages pages of
 * page_positions positions (a power of two >= 32) each, a page holding those
 * positions for every layer and kv head.  A stream's pages are mapped from
 * the pool as the entry points append to it (QORA_ERR_OOM, before any
 * launch, when the pool is exhausted) and go back by qora_kv_reset;
 * qora_kv_copy_stream between paged caches with the same page size shares
 * the source's full pages instead of copying them (prefix snapshot,
 * generate_new.rs:317-355).  max_pos bounds each stream's length.  Every
 * entry point that takes a qora_kv accepts a paged one except
 * qora_kv_layer_ptrs (no slab to point at). */
int qora_kv_create_paged(qora_ctx *ctx, int32_t num_layers, int32_t kv_heads, int32_t head_dim,
                         int32_t max_pos, int32_t streams, int32_t page_positions,
                         int32_t pool_pages, qora_kv **out);
/* Pages of a paged cache referenced by at least one stream, and free pages. */
int qora_kv_pages_host(const qora_kv *kv, int32_t *mapped, int32_t *free_pages);
void qora_kv_destroy(qora_kv *kv);
/* Clear streams (code_predictor.rs:227-231).  ids_host NULL => all streams. */
int qora_kv_reset(qora_kv *kv, const int32_t *ids_host, int32_t count, void *stream);
int qora_kv_lengths_host(qora_kv *kv, int32_t *len_host, void *stream);
/* Copy one stream's cache (prefix snapshot / restore, generate_new.rs:317-355). */
int qora_kv_copy_stream(qora_kv *dst, int32_t dst_stream, const qora_kv *src,
                        int32_t src_stream, void *stream);
/* Device pointers of one layer's K and V slabs and the length array. */
int qora_kv_layer_ptrs(qora_kv *kv, int32_t layer, float **k, float **v, int32_t **len);
/* Copy one layer's K and V slabs (all streams, [stream][kv_head][max_pos][head_dim])
 * into caller device buffers (KV snapshot of the reference's RawKvCache). */
int qora_kv_export_layer(qora_kv *kv, int32_t layer, float *k_out, float *v_out, void *stream);
/* KV-cache append + attend of one decoder layer for streams 0..B-1, T = 1
 * (the attention block of the decode step, talker.rs:285-331 and
 * code_predictor.rs:461-498; apply_qk_norm talker.rs:89-99; split RoPE
 * rope.rs:79-92).  qkv [B][(num_heads + 2*kv_heads)*head_dim]: the raw q | k | v
 * projections of this layer (read only).  q and k get the per-head RMS norm
 * (q_norm / k_norm: f16 [head_dim]) and RoPE at positions[b] (int32 [B]) from
 * rope_cos / rope_sin ([rope_max_pos][head_dim/2] f32); k and v are written at
 * the stream's cache length; out [B][num_heads*head_dim] = softmax(q.k /
 * sqrt(head_dim)) . v over length+1 positions.  advance != 0 adds one to each
 * stream's length afterwards (the cache has one length per stream for all
 * layers: advance once per step, on the last layer).  num_heads / kv_heads is
 * 1, 2 or 4.  The first call on a cache allocates its split-merge scratch. */
int qora_kv_attend(qora_kv *kv, int32_t layer, const float *qkv, int32_t num_heads,
                   const uint16_t *q_norm, const uint16_t *k_norm, const float *rope_cos,
                   const float *rope_sin, int32_t rope_max_pos, const int32_t *positions,
                   int32_t B, int32_t advance, float *out, void *stream);
/* No counterpart in the reference (its CPU path allocates freely).  Same
 * arguments and results as qora_kv_attend, but allocates no device memory:
 * for callers that cannot let a library call cudaMalloc, such as a real-time
 * audio loop that must not stall on an allocation, or an application whose
 * own memory manager already holds the GPU's memory.  The split-merge scratch
 * is a fixed ~1.1 MB array in the library's static device memory, present on
 * every GPU that loads the library until the process exits.  Limit:
 * B * num_heads * head_dim <= 16384 (the talker's 16 x 128 heads: B <= 8) and
 * B * kv_heads <= 512; larger calls return QORA_ERR_UNSUPPORTED.  The first
 * call on each device looks up the array's device address (make that first
 * call before any stream capture).  All calls share the array: calls that
 * overlap on the GPU race, so issue them on one stream. */
int qora_kv_attend_noalloc(qora_kv *kv, int32_t layer, const float *qkv, int32_t num_heads,
                           const uint16_t *q_norm, const uint16_t *k_norm, const float *rope_cos,
                           const float *rope_sin, int32_t rope_max_pos, const int32_t *positions,
                           int32_t B, int32_t advance, float *out, void *stream);

/* ------------------------------------------------------------ save.rs */
/* load_model (save.rs:262-409; records gemv.rs:595-687): maps a .qora-tts
 * checkpoint (Q4 format) read-only and parses its talker and code-predictor
 * sections (the speech decoder after them is read by qora_model_file_decoder,
 * with the decoder's entry points below).  Every length is
 * checked against the file; a malformed file, a version other than 1 or an
 * f16 (format 0) checkpoint is an error.  The RoPE base is recovered from the
 * stored tables and must reproduce them exactly. */
int qora_model_file_open(const char *path, qora_model_file **out);
/* Host views of the file's TalkerWeights / CodePredictorWeights for
 * qora_talker_create / qora_predictor_create; their pointers stay valid until
 * qora_model_file_close (nibbles point into the mapping, the small f16 / f32
 * arrays into aligned copies). */
int qora_model_file_talker(const qora_model_file *f, qora_talker_host *out);
int qora_model_file_predictor(const qora_model_file *f, qora_predictor_host *out);
/* The talker's text embedding and text projection (save.rs:78-82). */
int qora_model_file_text_proj(const qora_model_file *f, qora_text_proj_host *out);
void qora_model_file_close(qora_model_file *f);

/* ------------------------------------------------------------ talker.rs */
int qora_talker_create(qora_ctx *ctx, const qora_talker_host *host, int32_t max_batch,
                       qora_talker **out);
void qora_talker_destroy(qora_talker *t);
/* forward_with_embedding (talker.rs:263-360) for B streams of `kv`:
 * emb [B][hidden] (not modified); positions [B] RoPE positions (int32);
 * hidden [B][hidden] final-normed; logits [B][vocab] (may be NULL).
 * Appends one position to each stream's cache. */
int qora_talker_step(qora_talker *t, qora_kv *kv, const float *emb, const int32_t *positions,
                     int32_t B, float *hidden, float *logits, void *stream);
/* prefill_talker_raw_from (talker.rs:379-482) for one stream:
 * x [T][hidden], start_pos must equal the stream's cache length. */
int qora_talker_prefill(qora_talker *t, qora_kv *kv, int32_t kv_stream, const float *x,
                        int32_t T, int32_t start_pos, float *hidden, void *stream);
/* forward_talker_decode (talker.rs:161-258) for B streams: embeds
 * tokens_host[b] (a HOST array) through the text projection `tp` when is_text,
 * else through the codec embedding, runs the talker step at positions[b]
 * (device int32) and writes the final-normed hidden [B][hidden]; no codec
 * head.  `tp` may be NULL when is_text == 0.  Out-of-vocabulary tokens are
 * QORA_ERR_RANGE before any launch. */
int qora_talker_decode(qora_talker *t, qora_kv *kv, qora_text_proj *tp, const uint32_t *tokens_host,
                       int32_t is_text, const int32_t *positions, int32_t B, float *hidden,
                       void *stream);
/* apply_codec_head (talker.rs:647-649). */
int qora_talker_codec_head(qora_talker *t, const float *hidden, int32_t B, float *logits,
                           void *stream);
/* embed_codec_token (talker.rs:152-154) for B device tokens (range as
 * qora_q4_embed_rows). */
int qora_talker_embed_codec(qora_talker *t, const uint32_t *tokens, int32_t B, float *out,
                            void *stream);

/* embed_text_token (talker.rs:104-116): text-embedding row -> fc1 + bias ->
 * SiLU -> fc2 + bias, for a run of prompt tokens.  `tokens` is a HOST array
 * of `count` text token ids (the tokenizer's output); `out` is device
 * [count][hidden].  A token >= text_vocab is QORA_ERR_RANGE before any
 * launch.  One object serves one stream at a time (its scratch is shared). */
int qora_text_proj_create(qora_ctx *ctx, const qora_text_proj_host *host, qora_text_proj **out);
void qora_text_proj_destroy(qora_text_proj *tp);
int qora_text_proj_embed(qora_text_proj *tp, const uint32_t *tokens, int32_t count, float *out,
                         void *stream);

/* Prompt assembly (generate_new.rs:91-466): `count` rows described by the
 * HOST array `rows` into device out [count][hidden]; text_rows is device
 * [n_text][hidden] (e.g. from qora_text_proj_embed), voice a device vector of
 * voice_len floats (NULL when no row is a voice row); `p` may be NULL when no
 * row has more than one code.  Every index is checked before any launch
 * (QORA_ERR_RANGE). */
int qora_prompt_assemble(qora_talker *t, qora_predictor *p, const float *text_rows,
                         int32_t n_text, const float *voice, int32_t voice_len,
                         const qora_prompt_row *rows, int32_t count, float *out, void *stream);

/* ------------------------------------------------------------ code_predictor.rs */
int qora_predictor_create(qora_ctx *ctx, const qora_predictor_host *host, int32_t max_batch,
                          qora_predictor **out);
void qora_predictor_destroy(qora_predictor *p);
/* generate_acoustic_codes (code_predictor.rs:218-273) for B streams:
 * hidden [B][talker_hidden], semantic [B][talker_hidden] -> codes [B][num_groups].
 * logits [B][num_groups][vocab] optional (NULL).  forced [B][num_groups]
 * optional: teacher forcing, the forced code (not the argmax) feeds the next
 * step.  kv must have num_groups+1 positions per stream; it is reset. */
int qora_predictor_frame(qora_predictor *p, qora_kv *kv, const float *hidden,
                         const float *semantic, int32_t B, uint32_t *codes, float *logits,
                         const uint32_t *forced, void *stream);
/* get_acoustic_embeddings_sum (code_predictor.rs:287-300): codes [B][num_groups]. */
int qora_predictor_embed_sum(qora_predictor *p, const uint32_t *codes, int32_t B, float *out,
                             void *stream);

/* ------------------------------------------------------------ generate_new.rs */
/* sample_token (generate_new.rs:771-862) for B rows of V logits.
 * prev [B][n_prev] (repetition penalty), rng [B] xorshift64 states (in/out),
 * out [B].  top_p in (0,1) needs 0 < top_k <= 1024. */
int qora_sample(qora_ctx *ctx, const float *logits, int32_t B, int32_t V, const uint32_t *prev,
                int32_t n_prev, uint64_t *rng, const qora_sample_params *params, uint32_t *out,
                void *stream);

/* The frame loop (generate_new.rs:606-665) for B streams on one GPU: sample
 * code0 -> semantic embedding -> predictor (15 codes) -> embedding sum +
 * text row -> talker step.  EOS is not acted on (streams run every frame). */
int qora_engine_create(qora_talker *t, qora_predictor *p, int32_t B, int32_t max_pos,
                       const qora_sample_params *params, qora_engine **out);
void qora_engine_destroy(qora_engine *e);
/* Prefill every stream with x_host [B][T][hidden] (one talker prefill per
 * stream), set RNG seeds (seeds_host [B]) and clear the previous-code window. */
int qora_engine_prefill(qora_engine *e, const float *x_host, int32_t T, const uint64_t *seeds_host,
                        void *stream);
/* The prefix-cache path of generate_speech (generate_new.rs:509-530): every
 * stream's cache becomes a copy of stream `prefix_stream` of `prefix` (a
 * talker cache holding exactly prefix_len positions, e.g. the role prefix,
 * codec header and ICL reference part prefilled once per run), then
 * x_host [B][T][hidden] (the text-dependent suffix) is prefilled on top at
 * positions prefix_len.., as prefill_talker_raw_from does.  A prefix of
 * another length is QORA_ERR_SHAPE (the reference then prefills in full). */
int qora_engine_prefill_from(qora_engine *e, const qora_kv *prefix, int32_t prefix_stream,
                             int32_t prefix_len, const float *x_host, int32_t T,
                             const uint64_t *seeds_host, void *stream);
/* Run one frame (device buffers): text [B][hidden] -> codes [B][16].
 * On the persistent frame kernel (the default at B = 1) each launch carries
 * its own synchronisation tags, so the call must not be captured into a CUDA
 * graph by the caller: under stream capture it returns QORA_ERR_UNSUPPORTED.
 * The per-op path (qora_engine_use_persistent(e, 0), or B > 1) may be
 * captured, and qora_engine_use_graph captures it internally. */
int qora_engine_frame(qora_engine *e, const float *text, uint32_t *codes, void *stream);
/* Run one frame from HOST buffers: text_host [B][hidden] in, codes_host [B][16]
 * out; both copies are issued on `stream` and the call returns after the
 * codes have landed. */
int qora_engine_frame_host(qora_engine *e, const float *text_host, uint32_t *codes_host,
                           void *stream);
/* Capture one frame of the per-op path into a CUDA graph (enable=1) and
 * replay it per frame (no effect while the persistent frame kernel runs the
 * frames: that path is one launch per frame already). */
int qora_engine_use_graph(qora_engine *e, int32_t enable);
/* Run each frame as ONE launch of the persistent frame kernel (enable = 1, the
 * default where supported) or as the sequence of per-op kernels (enable = 0).
 * The persistent kernel needs B = 1, an input projection, head_dim 64 or 128,
 * heads / kv_heads of 1, 2 or 4, widths <= 6144 and vocab <= 4096;
 * QORA_ERR_UNSUPPORTED otherwise (the per-op path then stays in use). */
int qora_engine_use_persistent(qora_engine *e, int32_t enable);
/* frame_temperature (generate_new.rs:82-88, used at :608): sets the
 * temperature of the following frames' first sample_token.  The onset
 * schedule (onset_frames frames at onset_temperature, then temperature) is a
 * call at the start and one at frame onset_frames; a captured frame graph is
 * captured again on the next frame.  NaN is QORA_ERR_INVALID. */
int qora_engine_set_temperature(qora_engine *e, float temperature);
/* Per-op timing of the persistent frame kernel (a profiling aid, no
 * reference counterpart).  enable != 0 makes later frames record, for each
 * op, globaltimer ns over the SMs that have items in it: the earliest input
 * ready (stored bit-complemented), the latest input ready, the latest
 * completion and the latest start; then, on the SM that runs the op's first
 * item, the cycles its GEMV items waited for weight slots, computed and
 * reduced, and the slots consumed.  With ops_host / stamps_host non-NULL it
 * first copies the last recorded frame: op types (0 GEMV, 1 attention,
 * 2 sampler) into ops_host[capacity] and the records into
 * stamps_host[capacity][8].  *n_ops receives the op count. */
int qora_engine_trace(qora_engine *e, int32_t enable, int32_t capacity, int32_t *n_ops,
                      int32_t *ops_host, uint64_t *stamps_host);
/* Number of kernels one frame launches (for launch accounting). */
int qora_engine_kernels_per_frame(qora_engine *e, int32_t *count);
/* Device pointers of the engine state: logits [B][vocab], hidden [B][hidden],
 * prev [B][16], rng [B], positions [B]. */
int qora_engine_state(qora_engine *e, float **logits, float **hidden, uint32_t **prev,
                      uint64_t **rng, int32_t **positions);

/* ------------------------------------------------------------ decoder.rs */
/* The speech decoder (SpeechDecoderWeights + decode_to_audio, decoder.rs:24-66,
 * 395-582): 16 codes per 12.5 Hz frame -> 24 kHz f32 samples, all in f32. */
typedef struct qora_decoder qora_decoder;

/* Its configuration (decoder.rs:1-14, loader.rs:503-716; the 12 Hz
 * tokenizer's values in the comments).  Fixed by the reference and not
 * configurable: pre-conv taps 3, upsample ConvTranspose kernel 2 / stride 2,
 * ConvNeXt depthwise taps 7, Vocos conv taps 7, residual dilations 1, 3, 9,
 * output conv taps 7, norm eps 1e-5. */
typedef struct qora_decoder_dims {
    int32_t codebook_dim;      /* 256 */
    int32_t codebook_size;     /* 2048 */
    int32_t num_quantizers;    /* 16: rvq_first + 15 rvq_rest */
    int32_t vq_dim;            /* 512: width of the codebook output projections */
    int32_t latent;            /* 1024: pre-conv and upsample channels */
    int32_t hidden;            /* 512 */
    int32_t num_heads;         /* 16 */
    int32_t head_dim;          /* 64 (the only value supported) */
    int32_t intermediate;      /* 1024 (a multiple of 64) */
    int32_t num_layers;        /* 8 */
    int32_t sliding_window;    /* 72 (at most 128) */
    int32_t upsample_stages;   /* 2 */
    int32_t upsample_inner;    /* 4096: ConvNeXt pwconv1 width */
    int32_t vocos_blocks;      /* 4 (at most 7) */
    int32_t vocos_channels[8]; /* 1536, 768, 384, 192, 96: blocks + 1 entries used */
    int32_t vocos_kernels[8];  /* 16, 10, 8, 6: each the stride or twice it */
    int32_t vocos_strides[8];  /* 8, 5, 4, 3 */
    int32_t rope_max_pos;      /* 8000 (loader.rs:671): later positions are not rotated */
    double rope_theta;         /* 10000 */
} qora_decoder_dims;

/* load_speech_decoder (loader.rs:503-716) in three steps: create, one
 * qora_decoder_set_tensor per checkpoint tensor (its safetensors name and its
 * values in the checkpoint's own layout, read as f32: Linear [out][in], Conv1d
 * [out][in][k], ConvTranspose1d [in][out][k], codebooks as embedding_sum and
 * cluster_usage, normalised here as ema_codebook does, loader.rs:488-501),
 * then finalize (uploads; QORA_ERR_INVALID naming the first tensor not set).
 * An unknown name or a wrong value count is an error. */
int qora_decoder_create(qora_ctx *ctx, const qora_decoder_dims *dims, qora_decoder **out);
int qora_decoder_set_tensor(qora_decoder *dec, const char *name, const float *data_host,
                            int64_t count);
int qora_decoder_finalize(qora_decoder *dec);
void qora_decoder_destroy(qora_decoder *dec);
/* load_model's speech decoder (load_decoder_weights, save.rs:446-552): the
 * decoder section of a .qora-tts file opened by qora_model_file_open, uploaded
 * as a finalized decoder (its dims taken from the section; the file's
 * processed tensors are handed over under their checkpoint names, so the
 * decoder equals one loaded tensor by tensor from the speech tokenizer).
 * QORA_ERR_INVALID when the file has no well-formed decoder section,
 * QORA_ERR_UNSUPPORTED for a decoder structure this engine does not run. */
int qora_model_file_decoder(const qora_model_file *f, qora_ctx *ctx, qora_decoder **out);
/* The dims the decoder was created with. */
int qora_decoder_get_dims(const qora_decoder *dec, qora_decoder_dims *dims);
/* Which convolutions run on the tensor cores (3 x TF32 products, f32
 * accumulation): mode 0 none (all on the CUDA cores), 1 (the default) those
 * whose tiles fill the GPU, 2 every one that has a tensor-core form (the
 * Vocos convolutions and transposed convolutions, the upsample transposed
 * convolutions and ConvNeXt pointwise convolutions). */
int qora_decoder_use_tensor_cores(qora_decoder *dec, int32_t mode);
/* Samples decoded from `frames` frames: frames * 1920 at the 12 Hz dims. */
int qora_decoder_samples(const qora_decoder *dec, int64_t frames, int64_t *samples);
/* decode_to_audio (decoder.rs:395-582) from host codes [num_quantizers][frames]
 * (quantizer-major, as the reference's codes[q][t]); warmup_host
 * [num_quantizers][warmup_frames] is prepended and its share of the samples
 * trimmed (warmup_trim_len, decoder.rs:649-656) when it is non-NULL and
 * warmup_frames > 0.  Writes *n_samples = frames * hop samples, clamped to
 * [-1, 1], into samples_host (capacity values; QORA_ERR_SHAPE when too
 * small).  frames == 0 gives no samples (decoder.rs:401-404).  A code outside
 * the codebook reads row 0 and gives QORA_ERR_RANGE at the next
 * qora_ctx_check_device_error (the reference panics on the slice). */
int qora_decode_to_audio(qora_decoder *dec, const uint32_t *codes_host, int64_t frames,
                         const uint32_t *warmup_host, int64_t warmup_frames, float *samples_host,
                         int64_t capacity, int64_t *n_samples, void *stream);
/* The same on the device: codes [num_quantizers][warmup_frames + frames]
 * (each row its warm-up codes, then its codes), samples receives
 * frames * hop values; *launches (optional) the kernels launched.
 * Asynchronous on `stream`. */
int qora_decode_to_audio_device(qora_decoder *dec, const uint32_t *codes, int64_t frames,
                                int64_t warmup_frames, float *samples, int32_t *launches,
                                void *stream);

#ifdef __cplusplus
}
#endif
#endif /* QORA_CUDA_H */
