// Talker, code predictor, KV cache and the per-frame engine (host orchestration).
//
// Kernel sequence of one talker step for B streams (talker.rs:263-360):
//   per layer (5 launches):
//     [qkv GEMV, RMSNorm prologue] -> [attention: qk-norm, RoPE, KV append,
//     split-position GQA] -> [o GEMV + residual] -> [gate|up GEMV, RMSNorm
//     prologue, SwiGLU epilogue] -> [down GEMV + residual]
//   then [codec head GEMV, final-norm prologue, hidden side output, length advance].
// Residual-producing epilogues also write per-32-column sum-of-squares
// partials, which the next RMSNorm prologue sums in fixed order.
//
// The predictor frame (code_predictor.rs:218-273) runs the same layer
// sequence: one 2-token pass (projected talker hidden + projected semantic
// embedding) and 14 one-token passes; each pass ends in a head GEMV whose
// final CTA takes the argmax (last index on ties) and advances the cache.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "attention.cuh"
#include "gemv.cuh"
#include "kv.cuh"
#include "frame.cuh"
#include "model.cuh"
#include "sampler.cuh"

namespace qora {

int host_rope_tables(int32_t head_dim, int32_t max_pos, double theta, const int32_t *sections,
                     int32_t n_sections, float *cos_t, float *sin_t);

namespace {

__global__ void k_advance(int *len, int *pos, int count, int by) {
    griddep_launch_dependents();
    griddep_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) {
        len[i] += by;
        if (pos) pos[i] += by;
    }
}

__global__ void k_fill_i32(int *p, int count, int v) {
    griddep_launch_dependents();
    griddep_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) p[i] = v;
}

// Prefix snapshot / restore (generate_new.rs:317-355): rows [row0, len) of
// one source stream, every (layer, kv head), into `ndst` destination streams
// dst0.., and their lengths.  Only the source's live rows move; the source
// length is read on the device, so the copy needs no host round trip.  Both
// caches are addressed through their layer views (slab or paged; layer l's
// rows sit `step` elements after layer 0's).  grid (layers * kvh, ndst, row
// chunks); K and V rows are head_dim floats.
__global__ void k_kv_copy_rows(KVLayer src, int64_t src_step, KVLayer dst, int64_t dst_step, int dst0,
                               int kvh, int hd, int row0, const int *src_len, int *dst_len) {
    griddep_launch_dependents();
    griddep_wait();
    const int l = blockIdx.x / kvh, h = blockIdx.x % kvh;
    const int ds = dst0 + blockIdx.y;
    const int len = min(__ldcg(src_len), min(src.max_pos, dst.max_pos));
    const int d4n = hd / 4;  // head_dim is a multiple of 4
    const int n4 = (len - row0) * d4n;
    for (int i = blockIdx.z * blockDim.x + threadIdx.x; i < n4; i += gridDim.z * blockDim.x) {
        const int p = row0 + i / d4n, d4 = i % d4n;
        const int64_t so = l * src_step + src.row(0, h, p) + 4 * d4;
        const int64_t dof = l * dst_step + dst.row(ds, h, p) + 4 * d4;
        *reinterpret_cast<float4 *>(dst.k + dof) = __ldcg(reinterpret_cast<const float4 *>(src.k + so));
        *reinterpret_cast<float4 *>(dst.v + dof) = __ldcg(reinterpret_cast<const float4 *>(src.v + so));
    }
    if (blockIdx.x == 0 && blockIdx.z == 0 && threadIdx.x == 0) dst_len[ds] = __ldcg(src_len);
}

// One layer of a cache gathered into [stream][kv_head][max_pos][head_dim]
// (the slab layout), rows [0, max_pos) of every stream.
__global__ void k_kv_gather_layer(KVLayer L, int kvh, int hd, int max_pos, float *k_out, float *v_out) {
    const int b = blockIdx.y, h = blockIdx.x % kvh;
    const int64_t n4 = (int64_t)max_pos * hd / 4;
    float4 *ko = reinterpret_cast<float4 *>(k_out + ((int64_t)b * kvh + h) * max_pos * hd);
    float4 *vo = reinterpret_cast<float4 *>(v_out + ((int64_t)b * kvh + h) * max_pos * hd);
    for (int64_t i = (int64_t)(blockIdx.x / kvh) * blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)(gridDim.x / kvh) * blockDim.x) {
        const int p = (int)(i / (hd / 4)), d4 = (int)(i % (hd / 4));
        const int64_t off = L.row(b, h, p) + 4 * d4;
        ko[i] = __ldcg(reinterpret_cast<const float4 *>(L.k + off));
        vo[i] = __ldcg(reinterpret_cast<const float4 *>(L.v + off));
    }
}

int upload_f16(const uint16_t *h, int64_t n, DevBuf &buf) {
    if (!h) return set_error(QORA_ERR_INVALID, "null norm vector");
    QORA_TRY(buf.alloc((size_t)n * 2));
    QORA_CUDA(cudaMemcpy(buf.p, h, (size_t)n * 2, cudaMemcpyHostToDevice));
    return QORA_OK;
}

}  // namespace

// --------------------------------------------------------------------- layers
int LayerDev::upload(const qora_layer_host &h, int64_t hidden, int heads, int kvh, int hd,
                     int64_t ffn) {
    const int64_t qd = (int64_t)heads * hd, kd = (int64_t)kvh * hd;
    if (h.q_proj.k != hidden || h.q_proj.n != qd || h.k_proj.n != kd || h.v_proj.n != kd ||
        h.o_proj.k != qd || h.o_proj.n != hidden || h.gate_proj.n != ffn ||
        h.up_proj.n != ffn || h.down_proj.k != ffn || h.down_proj.n != hidden)
        return set_error(QORA_ERR_SHAPE, "layer weight shapes do not match the config");
    {   // fused [q | k | v]
        const qora_q4_host parts[3] = {h.q_proj, h.k_proj, h.v_proj};
        const int64_t offs[3] = {0, qd / kGroup, (qd + kd) / kGroup};
        const int64_t strides[3] = {1, 1, 1};
        QORA_TRY(upload_q4_parts(parts, offs, strides, 3, hidden, (qd + 2 * kd) / kGroup,
                                 qkv_nib, qkv_scl, qkv, nullptr));
    }
    {
        const int64_t off = 0, st = 1;
        QORA_TRY(upload_q4_parts(&h.o_proj, &off, &st, 1, qd, hidden / kGroup, o_nib, o_scl, o,
                                 nullptr));
        QORA_TRY(upload_q4_parts(&h.down_proj, &off, &st, 1, ffn, hidden / kGroup, dn_nib,
                                 dn_scl, dn, nullptr));
    }
    {   // gate/up interleaved by 32-column group: g0 u0 g1 u1 ...
        const qora_q4_host parts[2] = {h.gate_proj, h.up_proj};
        const int64_t offs[2] = {0, 1};
        const int64_t strides[2] = {2, 2};
        QORA_TRY(upload_q4_parts(parts, offs, strides, 2, hidden, 2 * ffn / kGroup, gu_nib,
                                 gu_scl, gu, nullptr));
    }
    QORA_TRY(upload_f16(h.q_norm, hd, q_norm));
    QORA_TRY(upload_f16(h.k_norm, hd, k_norm));
    QORA_TRY(upload_f16(h.input_norm, hidden, in_norm));
    QORA_TRY(upload_f16(h.post_attn_norm, hidden, post_norm));
    return QORA_OK;
}

// Activation and scratch buffers sized for `rows` rows.

}  // namespace qora

using namespace qora;

// --------------------------------------------------------------------- talker

namespace qora {

struct Launcher {
    qora_ctx *ctx;
    Work *w;
    cudaStream_t st;
    int count = 0;      // kernels launched
    bool fixed = false; // prefill: a row's rounding must not depend on the rows of its launch

    int gemv(GemvArgs a, int xm, int em) {
        GemvPlan p;
        if (!a.err) a.err = ctx->err.as<int>();
        if (fixed && gemm_mma_supported(a, xm, em)) {
            // prefill: the tensor-core GEMM (k_gemv_mma's bits without a K split)
            return launch_gemm_mma(a, xm, em, w->gemm_scratch(), st, &count);
        }
        if (fixed && gemv_mma_supported(a, xm, em)) {
            // the tensor-core kernel with the K split planned for a full
            // kMaxRows chunk, whatever this launch's row count: the same split
            // (hence the same bits) for a row in any chunk, as the reference's
            // prefix cache needs (generate_new.rs:320-322)
            p = plan_gemv_mma(a.w.k, a.w.C, kMaxRows, em, ctx->num_sms);
            p.Z = (a.rows + p.rows_per_z - 1) / p.rows_per_z;
            p.grid.z = (unsigned)p.Z;
        } else {
            p = plan_gemv_for(a, xm, em, ctx->num_sms);
        }
        if (!a.err) a.err = ctx->err.as<int>();
        count++;
        return launch_gemv(a, xm, em, p, w->gticket.as<unsigned>(), st);
    }
};

// One decoder layer over `rows` rows (T tokens per stream).
// `next` is the weight the GEMV after this layer streams (L2 prefetch target).
static int run_layer(Launcher &ln, const LayerDev &ld, int H, int heads, int kvh, int hd,
                     int64_t ffn, int rows, int T, const KVLayer &kv, const int *len,
                     const int *pos, const float *rope_cos, const float *rope_sin, int rope_max,
                     const Q4Dev &next) {
    Work &w = *ln.w;
    const int64_t qd = (int64_t)heads * hd, qkvn = qd + 2 * (int64_t)kvh * hd;
    {
        GemvArgs a;
        a.w = ld.qkv;
        a.rows = rows;
        a.x = w.x.as<float>();
        a.ldx = H;
        a.gamma = ld.in_norm.as<__half>();
        a.ss = w.ss.as<float>();
        a.ldss = H / kGroup;
        a.ss_tiles = H / kGroup;
        a.y = w.qkv.as<float>();
        a.ldy = qkvn;
        prefetch_next(a, ld.o);
        QORA_TRY(ln.gemv(a, X_RMSNORM, E_STORE));
    }
    AttnArgs at;
    at.qkv = w.qkv.as<float>();
    at.ldqkv = qkvn;
    at.heads = heads;
    at.kv_heads = kvh;
    at.T = T;
    at.streams = rows / T;
    at.q_gamma = ld.q_norm.as<__half>();
    at.k_gamma = ld.k_norm.as<__half>();
    at.rope_cos = rope_cos;
    at.rope_sin = rope_sin;
    at.rope_max_pos = rope_max;
    at.pos = pos;
    at.len = len;
    at.kv = kv;
    at.out = w.attn.as<float>();
    at.ldout = qd;
    at.part_o = w.apo.as<float>();
    at.part_ml = w.apml.as<float>();
    at.tickets = w.atk.as<unsigned>();
    at.err = ln.ctx->err.as<int>();
    if (T > 1 || ln.fixed) {  // prefill (any length): append first, then the causal kernel
        QORA_TRY(launch_qkv_post(at, ln.st));
        ln.count++;
        at.preappended = true;
    }
    QORA_TRY(launch_attention(at, ln.st));
    ln.count++;
    {
        GemvArgs a;
        a.w = ld.o;
        a.rows = rows;
        a.x = w.attn.as<float>();
        a.ldx = qd;
        a.y = w.x.as<float>();
        a.ldy = H;
        a.ss_out = w.ss.as<float>();
        a.ldss_out = H / kGroup;
        prefetch_next(a, ld.gu);
        QORA_TRY(ln.gemv(a, X_PLAIN, E_RESID));
    }
    {
        GemvArgs a;
        a.w = ld.gu;
        a.rows = rows;
        a.x = w.x.as<float>();
        a.ldx = H;
        a.gamma = ld.post_norm.as<__half>();
        a.ss = w.ss.as<float>();
        a.ldss = H / kGroup;
        a.ss_tiles = H / kGroup;
        a.y = w.h.as<float>();
        a.ldy = ffn;
        prefetch_next(a, ld.dn);
        QORA_TRY(ln.gemv(a, X_RMSNORM, E_SWIGLU));
    }
    {
        GemvArgs a;
        a.w = ld.dn;
        a.rows = rows;
        a.x = w.h.as<float>();
        a.ldx = ffn;
        a.y = w.x.as<float>();
        a.ldy = H;
        a.ss_out = w.ss.as<float>();
        a.ldss_out = H / kGroup;
        prefetch_next(a, next);
        QORA_TRY(ln.gemv(a, X_PLAIN, E_RESID));
    }
    return QORA_OK;
}

// Talker forward for B streams (T = 1) starting from w.x / w.ss.
// hidden: final-normed rows (ldh); logits may be null (then a plain norm).
static int talker_forward_step(qora_talker *t, qora_kv *kv, Launcher &ln, int B, const int *pos,
                               float *hidden, int64_t ldh, float *logits, int64_t ldl,
                               int *adv_pos) {
    for (int l = 0; l < t->L; l++)
        QORA_TRY(run_layer(ln, t->layers[l], t->H, t->heads, t->kvh, t->hd, t->ffn, B, 1,
                           kv->layer(l), kv->lens(), pos, t->rope_cos.as<float>(),
                           t->rope_sin.as<float>(), t->rope_max,
                           l + 1 < t->L ? t->layers[l + 1].qkv : t->head));
    GemvArgs a;
    a.w = t->head;
    a.rows = B;
    a.x = ln.w->x.as<float>();
    a.ldx = t->H;
    a.gamma = t->final_norm.as<__half>();
    a.ss = ln.w->ss.as<float>();
    a.ldss = t->H / kGroup;
    a.ss_tiles = t->H / kGroup;
    a.side = hidden;
    a.ldside = ldh;
    a.y = logits ? logits : ln.w->logits.as<float>();
    a.ldy = logits ? ldl : t->vocab;
    a.adv_len = kv->lens();
    a.adv_pos = adv_pos;
    a.adv_T = 1;
    a.adv_streams = B;
    return ln.gemv(a, X_RMSNORM, E_STORE);
}

}  // namespace qora

// ------------------------------------------------------------------ predictor

namespace qora {

// Projects rows of width Ht into w.x (+ ss).  Source: plain rows, or the
// embedding row of a code (X_EMBED).
static int predictor_project(qora_predictor *p, Launcher &ln, int rows, const float *x,
                             int64_t ldx, const EmbDev *emb, const uint32_t *tok, int64_t ldtok) {
    Work &w = *ln.w;
    if (!p->has_proj) {
        const float *src = x;
        int64_t lds = ldx;
        if (emb) {
            QORA_TRY(launch_embed_rows(*emb, tok, ldtok, rows, p->xe.as<float>(), p->Ht, p->ctx->err.as<int>(), ln.st));
            ln.count++;
            src = p->xe.as<float>();
            lds = p->Ht;
        }
        QORA_TRY(launch_copy_rowstats(src, lds, w.x.as<float>(), p->H, rows, p->H,
                                      w.ss.as<float>(), p->H / kGroup, ln.st));
        ln.count++;
        return QORA_OK;
    }
    GemvArgs a;
    a.w = p->proj;
    a.rows = rows;
    a.x = x;
    a.ldx = ldx;
    if (emb) {
        a.emb = *emb;
        a.tok = tok;
        a.ldtok = ldtok;
    }
    a.bias = p->proj_bias.as<float>();
    a.y = w.x.as<float>();
    a.ldy = p->H;
    a.ss_out = w.ss.as<float>();
    a.ldss_out = p->H / kGroup;
    return ln.gemv(a, emb ? X_EMBED : X_PLAIN, E_BIAS);
}

static int predictor_head(qora_predictor *p, Launcher &ln, int B, int g, int T, qora_kv *kv,
                          uint32_t *codes, int64_t ldcodes, float *logits, int64_t ldl) {
    Work &w = *ln.w;
    GemvArgs a;
    a.w = p->heads_w[g];
    a.rows = B;
    // last token of each stream: row b*T + T-1
    a.x = w.x.as<float>() + (int64_t)(T - 1) * p->H;
    a.ldx = (int64_t)T * p->H;
    a.gamma = p->final_norm.as<__half>();
    a.ss = w.ss.as<float>() + (int64_t)(T - 1) * (p->H / kGroup);
    a.ldss = (int64_t)T * (p->H / kGroup);
    a.ss_tiles = p->H / kGroup;
    a.y = logits ? logits + (int64_t)g * p->vocab : w.logits.as<float>();
    a.ldy = logits ? ldl : p->vocab;
    a.tbest_v = w.tbest_v.as<float>();
    a.tbest_i = w.tbest_i.as<int>();
    a.amax = codes + g;
    a.ldamax = ldcodes;
    a.adv_len = kv->lens();
    a.adv_T = T;
    a.adv_streams = B;
    return ln.gemv(a, X_RMSNORM, E_STORE);
}

// generate_acoustic_codes for B streams; hidden rows are x2[b][0], semantic x2[b][1]
// (x2 row stride 2*Ht).  codes [B][groups] (ldcodes), optional logits, forced.
static int predictor_frame_impl(qora_predictor *p, qora_kv *kv, Launcher &ln, int B,
                                const float *x2, uint32_t *codes, int64_t ldcodes, float *logits,
                                int64_t ldl, const uint32_t *forced, int64_t ldforced) {
    // reset the per-frame cache (code_predictor.rs:227-231)
    QORA_TRY(launch_ex(k_fill_i32, dim3((B + 255) / 256), dim3(256), 0, ln.st, 1u, kv->lens(), B, 0));
    ln.count++;
    // 2-token prefill: [proj(hidden), proj(semantic)]
    QORA_TRY(predictor_project(p, ln, 2 * B, x2, p->Ht, nullptr, nullptr, 0));
    for (int l = 0; l < p->L; l++)
        QORA_TRY(run_layer(ln, p->layers[l], p->H, p->heads, p->kvh, p->hd, p->ffn, 2 * B, 2,
                           kv->layer(l), kv->lens(), nullptr, p->rope_cos.as<float>(),
                           p->rope_sin.as<float>(), p->rope_max,
                           l + 1 < p->L ? p->layers[l + 1].qkv : p->heads_w[0]));
    QORA_TRY(predictor_head(p, ln, B, 0, 2, kv, codes, ldcodes, logits, ldl));
    for (int g = 1; g < p->groups; g++) {
        const uint32_t *tok = forced ? forced + (g - 1) : codes + (g - 1);
        const int64_t ldtok = forced ? ldforced : ldcodes;
        QORA_TRY(predictor_project(p, ln, B, nullptr, 0, &p->embs[g - 1], tok, ldtok));
        for (int l = 0; l < p->L; l++)
            QORA_TRY(run_layer(ln, p->layers[l], p->H, p->heads, p->kvh, p->hd, p->ffn, B, 1,
                               kv->layer(l), kv->lens(), nullptr, p->rope_cos.as<float>(),
                               p->rope_sin.as<float>(), p->rope_max,
                               l + 1 < p->L ? p->layers[l + 1].qkv : p->heads_w[g]));
        QORA_TRY(predictor_head(p, ln, B, g, 1, kv, codes, ldcodes, logits, ldl));
    }
    return QORA_OK;
}

}  // namespace qora

// --------------------------------------------------------------------- engine

namespace qora {

// Page-table helpers of paged caches (host side; no-ops for a slab).
void kv_release_stream(qora_kv *kv, int sid) {
    if (!kv->paged()) return;
    for (int j = 0; j < kv->pages_per_stream; j++) {
        int &e = kv->host_table[(size_t)sid * kv->pages_per_stream + j];
        if (e != kv->guard_page() && --kv->refs[(size_t)e] == 0) kv->free_pages.push_back(e);
        e = kv->guard_page();
    }
}

int kv_prepare(qora_kv *kv, int s0, int n, int add, cudaStream_t st) {
    if (!kv->paged() || add <= 0) return QORA_OK;
    // all or nothing: count the pages first, so a failed call maps none
    size_t want = 0;
    for (int sid = s0; sid < s0 + n; sid++) {
        const int need = std::min(kv->max_pos, kv->host_len[(size_t)sid] + add);
        const int pages = (need + kv->page_pos - 1) / kv->page_pos;
        for (int j = 0; j < pages; j++)
            want += kv->host_table[(size_t)sid * kv->pages_per_stream + j] == kv->guard_page();
    }
    if (want > kv->free_pages.size())
        return set_error(QORA_ERR_OOM, "paged KV cache: %zu more pages needed, %zu of %d free", want,
                         kv->free_pages.size(), kv->pool_pages);
    bool changed = false;
    for (int sid = s0; sid < s0 + n; sid++) {
        const int need = std::min(kv->max_pos, kv->host_len[(size_t)sid] + add);
        const int pages = (need + kv->page_pos - 1) / kv->page_pos;
        for (int j = 0; j < pages; j++) {
            int &e = kv->host_table[(size_t)sid * kv->pages_per_stream + j];
            if (e != kv->guard_page()) continue;
            e = kv->free_pages.back();
            kv->free_pages.pop_back();
            kv->refs[(size_t)e] = 1;
            changed = true;
        }
    }
    if (changed)
        QORA_CUDA(cudaMemcpyAsync(kv->table.as<int>() + (size_t)s0 * kv->pages_per_stream,
                                  kv->host_table.data() + (size_t)s0 * kv->pages_per_stream,
                                  (size_t)n * kv->pages_per_stream * 4, cudaMemcpyHostToDevice, st));
    return QORA_OK;
}

void kv_note_growth(qora_kv *kv, int s0, int n, int add) {
    for (int sid = s0; sid < s0 + n; sid++)
        kv->host_len[(size_t)sid] = std::min(kv->max_pos, kv->host_len[(size_t)sid] + add);
}

// Copies stream `ss` of `src` into streams [ds, ds + n) of `dst` (live rows only).
int kv_copy_streams(qora_kv *dst, int32_t ds, int32_t n, const qora_kv *src, int32_t ss,
                    cudaStream_t st) {
    if (!dst || !src || dst->layers != src->layers || dst->kvh != src->kvh || dst->hd != src->hd ||
        dst->max_pos < src->max_pos || ds < 0 || n <= 0 || ds + n > dst->streams || ss < 0 ||
        ss >= src->streams)
        return set_error(QORA_ERR_INVALID, "qora_kv_copy_stream: incompatible caches");
    int len = src->host_len[(size_t)ss];
    if (src->paged() || dst->paged()) {
        // page mapping needs the exact length: read it (a prefix copy is rare)
        QORA_CUDA(cudaMemcpyAsync(&len, src->lens() + ss, 4, cudaMemcpyDeviceToHost, st));
        QORA_CUDA(cudaStreamSynchronize(st));
    }
    int row0 = 0;
    if (dst->paged()) {
        const bool share = src->paged() && src != dst && src->page_pos == dst->page_pos;
        const bool share_self = src == dst;
        const int full = (share || share_self) ? len / src->page_pos : 0;
        for (int d = ds; d < ds + n; d++) {
            if (share_self && d == ss) continue;
            kv_release_stream(dst, d);
            dst->host_len[(size_t)d] = 0;
            if (share || share_self) {  // full pages are shared, not copied
                for (int j = 0; j < full; j++) {
                    const int pg = src->host_table[(size_t)ss * src->pages_per_stream + j];
                    dst->host_table[(size_t)d * dst->pages_per_stream + j] = pg;
                    dst->refs[(size_t)pg]++;
                }
                dst->host_len[(size_t)d] = full * src->page_pos;
            }
        }
        row0 = full * src->page_pos;
        for (int d = ds; d < ds + n; d++) {
            if (share_self && d == ss) continue;
            QORA_TRY(kv_prepare(dst, d, 1, len - dst->host_len[(size_t)d], st));
            dst->host_len[(size_t)d] = len;
        }
        QORA_CUDA(cudaMemcpyAsync(dst->table.as<int>() + (size_t)ds * dst->pages_per_stream,
                                  dst->host_table.data() + (size_t)ds * dst->pages_per_stream,
                                  (size_t)n * dst->pages_per_stream * 4, cudaMemcpyHostToDevice, st));
    } else {
        for (int d = ds; d < ds + n; d++) dst->host_len[(size_t)d] = len;
    }
    const KVLayer sl = src->layer(0, ss), dl = dst->layer(0, 0);
    const int64_t s_step = src->paged() ? (int64_t)src->kvh * src->page_pos * src->hd : (int64_t)src->layer_elems();
    const int64_t d_step = dst->paged() ? (int64_t)dst->kvh * dst->page_pos * dst->hd : (int64_t)dst->layer_elems();
    // row chunks: enough CTAs to keep HBM busy for a long prefix
    const int chunks = std::max(1, std::min(64, src->max_pos * src->hd / 4 / 256 / 4));
    return launch_ex(k_kv_copy_rows, dim3(src->layers * src->kvh, n, chunks), dim3(256), 0, st, 1u, sl,
                     s_step, dl, d_step, ds, src->kvh, src->hd, row0, src->lens() + ss, dst->lens());
}
}  // namespace qora

// =========================================================================
// extern "C" entry points
// =========================================================================
extern "C" {

int qora_kv_create_paged(qora_ctx *ctx, int32_t num_layers, int32_t kv_heads, int32_t head_dim,
                         int32_t max_pos, int32_t streams, int32_t page_positions, int32_t pool_pages,
                         qora_kv **out) {
    if (!ctx || !out || num_layers <= 0 || kv_heads <= 0 || max_pos <= 0 || streams <= 0 ||
        pool_pages <= 0)
        return set_error(QORA_ERR_INVALID, "qora_kv_create_paged: bad arguments");
    if (head_dim != 64 && head_dim != 128)
        return set_error(QORA_ERR_UNSUPPORTED, "head_dim %d (supported: 64, 128)", head_dim);
    // every tile the kernels read (16 or 32 positions, aligned) must lie in one page
    if (page_positions < kPageMinPositions || (page_positions & (page_positions - 1)))
        return set_error(QORA_ERR_INVALID, "page_positions %d: a power of two >= %d", page_positions,
                         kPageMinPositions);
    QORA_CUDA(cudaSetDevice(ctx->device));
    qora_kv *kv = new qora_kv();
    kv->ctx = ctx;
    kv->layers = num_layers;
    kv->kvh = kv_heads;
    kv->hd = head_dim;
    kv->max_pos = max_pos;
    kv->streams = streams;
    kv->page_pos = page_positions;
    while ((1 << kv->page_shift) < page_positions) kv->page_shift++;
    kv->pages_per_stream = (max_pos + page_positions - 1) / page_positions;
    kv->pool_pages = pool_pages;
    const size_t bytes = (size_t)(pool_pages + 1) * kv->page_elems() * 4;  // + the guard page
    int rc = kv->k.alloc(bytes);
    if (rc == QORA_OK) rc = kv->v.alloc(bytes);
    if (rc == QORA_OK) rc = kv->len.alloc((size_t)streams * 4);
    if (rc == QORA_OK) rc = kv->len.zero();
    if (rc == QORA_OK) rc = kv->table.alloc((size_t)streams * kv->pages_per_stream * 4);
    if (rc == QORA_OK) {
        kv->host_table.assign((size_t)streams * kv->pages_per_stream, kv->guard_page());
        kv->refs.assign((size_t)pool_pages, 0);
        kv->free_pages.reserve((size_t)pool_pages);
        for (int pg = pool_pages - 1; pg >= 0; pg--) kv->free_pages.push_back(pg);
        kv->host_len.assign((size_t)streams, 0);
        if (cudaMemcpy(kv->table.p, kv->host_table.data(), kv->table.bytes, cudaMemcpyHostToDevice) !=
            cudaSuccess)
            rc = set_error(QORA_ERR_CUDA, "qora_kv_create_paged: table upload failed");
    }
    if (rc == QORA_OK && cudaDeviceSynchronize() != cudaSuccess)
        rc = set_error(QORA_ERR_CUDA, "qora_kv_create_paged: sync failed");
    if (rc != QORA_OK) {
        delete kv;
        return rc;
    }
    *out = kv;
    return QORA_OK;
}

int qora_kv_pages_host(const qora_kv *kv, int32_t *mapped, int32_t *free_pages) {
    if (!kv) return set_error(QORA_ERR_INVALID, "null kv");
    if (!kv->paged()) return set_error(QORA_ERR_UNSUPPORTED, "qora_kv_pages_host: not a paged cache");
    int used = 0;
    for (int r : kv->refs) used += r > 0;
    if (mapped) *mapped = used;
    if (free_pages) *free_pages = (int32_t)kv->free_pages.size();
    return QORA_OK;
}

int qora_kv_create(qora_ctx *ctx, int32_t num_layers, int32_t kv_heads, int32_t head_dim,
                   int32_t max_pos, int32_t streams, qora_kv **out) {
    if (!ctx || !out || num_layers <= 0 || kv_heads <= 0 || max_pos <= 0 || streams <= 0)
        return set_error(QORA_ERR_INVALID, "qora_kv_create: bad arguments");
    if (head_dim != 64 && head_dim != 128)
        return set_error(QORA_ERR_UNSUPPORTED, "head_dim %d (supported: 64, 128)", head_dim);
    QORA_CUDA(cudaSetDevice(ctx->device));
    qora_kv *kv = new qora_kv();
    kv->ctx = ctx;
    kv->layers = num_layers;
    kv->kvh = kv_heads;
    kv->hd = head_dim;
    kv->max_pos = max_pos;
    kv->streams = streams;
    const size_t bytes = kv->layer_elems() * num_layers * 4;
    int rc = kv->k.alloc(bytes);
    if (rc == QORA_OK) rc = kv->v.alloc(bytes);
    if (rc == QORA_OK) rc = kv->len.alloc((size_t)streams * 4);
    if (rc == QORA_OK) rc = kv->len.zero();
    kv->host_len.assign((size_t)streams, 0);
    if (rc == QORA_OK && cudaDeviceSynchronize() != cudaSuccess)
        rc = set_error(QORA_ERR_CUDA, "qora_kv_create: sync failed");
    if (rc != QORA_OK) {
        delete kv;
        return rc;
    }
    *out = kv;
    return QORA_OK;
}

void qora_kv_destroy(qora_kv *kv) { delete kv; }

int qora_kv_reset(qora_kv *kv, const int32_t *ids_host, int32_t count, void *stream) {
    if (!kv) return set_error(QORA_ERR_INVALID, "null kv");
    cudaStream_t st = as_stream(stream);
    if (ids_host)
        for (int i = 0; i < count; i++)
            if (ids_host[i] < 0 || ids_host[i] >= kv->streams)
                return set_error(QORA_ERR_INVALID, "stream id %d out of range", ids_host[i]);
    const int n = ids_host ? count : kv->streams;
    for (int i = 0; i < n; i++) {
        const int sid = ids_host ? ids_host[i] : i;
        kv_release_stream(kv, sid);
        kv->host_len[(size_t)sid] = 0;
    }
    if (!ids_host) {
        QORA_CUDA(cudaMemsetAsync(kv->len.p, 0, kv->len.bytes, st));
    } else {
        for (int i = 0; i < count; i++) QORA_CUDA(cudaMemsetAsync(kv->lens() + ids_host[i], 0, 4, st));
    }
    if (kv->paged())  // released entries point at the guard page again
        QORA_CUDA(cudaMemcpyAsync(kv->table.p, kv->host_table.data(), kv->table.bytes,
                                  cudaMemcpyHostToDevice, st));
    return QORA_OK;
}

int qora_kv_lengths_host(qora_kv *kv, int32_t *len_host, void *stream) {
    if (!kv || !len_host) return set_error(QORA_ERR_INVALID, "null argument");
    QORA_CUDA(cudaMemcpyAsync(len_host, kv->len.p, kv->len.bytes, cudaMemcpyDeviceToHost,
                              as_stream(stream)));
    QORA_CUDA(cudaStreamSynchronize(as_stream(stream)));
    return QORA_OK;
}

int qora_kv_copy_stream(qora_kv *dst, int32_t ds, const qora_kv *src, int32_t ss, void *stream) {
    return kv_copy_streams(dst, ds, 1, src, ss, as_stream(stream));
}

int qora_kv_layer_ptrs(qora_kv *kv, int32_t layer, float **k, float **v, int32_t **len) {
    if (!kv || layer < 0 || layer >= kv->layers) return set_error(QORA_ERR_INVALID, "bad layer");
    if (kv->paged()) return set_error(QORA_ERR_UNSUPPORTED, "qora_kv_layer_ptrs: a paged cache has no slab");
    KVLayer L = kv->layer(layer);
    if (k) *k = L.k;
    if (v) *v = L.v;
    if (len) *len = kv->lens();
    return QORA_OK;
}

int qora_kv_export_layer(qora_kv *kv, int32_t layer, float *k_out, float *v_out, void *stream) {
    if (!kv || layer < 0 || layer >= kv->layers || !k_out || !v_out)
        return set_error(QORA_ERR_INVALID, "qora_kv_export_layer: bad arguments");
    KVLayer L = kv->layer(layer);
    if (kv->paged())  // gathered into the slab layout
        return launch_ex(k_kv_gather_layer, dim3(kv->kvh * 8, kv->streams), dim3(256), 0, as_stream(stream), 1u,
                         L, kv->kvh, kv->hd, kv->max_pos, k_out, v_out);
    const size_t bytes = kv->layer_elems() * 4;
    QORA_CUDA(cudaMemcpyAsync(k_out, L.k, bytes, cudaMemcpyDeviceToDevice, as_stream(stream)));
    QORA_CUDA(cudaMemcpyAsync(v_out, L.v, bytes, cudaMemcpyDeviceToDevice, as_stream(stream)));
    return QORA_OK;
}

// ------------------------------------------------------------------ talker
int qora_talker_create(qora_ctx *ctx, const qora_talker_host *h, int32_t max_batch,
                       qora_talker **out) {
    if (!ctx || !h || !out || !h->layers || max_batch <= 0 || max_batch > kMaxRows)
        return set_error(QORA_ERR_INVALID, "qora_talker_create: bad arguments");
    if (h->hidden % kGroup || h->ffn % kGroup || h->vocab % kGroup || h->num_heads % h->num_kv_heads)
        return set_error(QORA_ERR_SHAPE, "talker dims must be multiples of 32");
    QORA_CUDA(cudaSetDevice(ctx->device));
    auto *t = new qora_talker();
    t->ctx = ctx;
    t->L = h->num_layers;
    t->H = h->hidden;
    t->heads = h->num_heads;
    t->kvh = h->num_kv_heads;
    t->hd = h->head_dim;
    t->ffn = h->ffn;
    t->vocab = h->vocab;
    t->rope_max = h->rope_max_pos;
    t->max_batch = max_batch;
    t->layers.resize(t->L);
    int rc = QORA_OK;
    for (int l = 0; l < t->L && rc == QORA_OK; l++)
        rc = t->layers[l].upload(h->layers[l], t->H, t->heads, t->kvh, t->hd, t->ffn);
    if (rc == QORA_OK) rc = upload_emb(h->codec_embedding, t->ce_packed, t->ce_scl, t->codec_emb);
    if (rc == QORA_OK && (h->codec_head.k != t->H || h->codec_head.n != t->vocab))
        rc = set_error(QORA_ERR_SHAPE, "codec_head shape");
    if (rc == QORA_OK) {
        const int64_t off = 0, st = 1;
        rc = upload_q4_parts(&h->codec_head, &off, &st, 1, t->H, t->vocab / kGroup, t->head_nib,
                             t->head_scl, t->head, nullptr);
    }
    if (rc == QORA_OK) rc = upload_f16(h->final_norm, t->H, t->final_norm);
    if (rc == QORA_OK) {
        const int half = t->hd / 2;
        std::vector<float> c((size_t)t->rope_max * half), s((size_t)t->rope_max * half);
        int32_t secs[3] = {24, 20, 20};
        const bool mrope = (half == 64);
        rc = host_rope_tables(t->hd, t->rope_max, h->rope_theta, mrope ? secs : &half,
                              mrope ? 3 : 1, c.data(), s.data());
        if (rc == QORA_OK) rc = t->rope_cos.alloc(c.size() * 4);
        if (rc == QORA_OK) rc = t->rope_sin.alloc(s.size() * 4);
        if (rc == QORA_OK && (cudaMemcpy(t->rope_cos.p, c.data(), c.size() * 4, cudaMemcpyHostToDevice) ||
                              cudaMemcpy(t->rope_sin.p, s.data(), s.size() * 4, cudaMemcpyHostToDevice)))
            rc = set_error(QORA_ERR_CUDA, "rope upload");
    }
    if (rc == QORA_OK)  // prefill chunks use up to kMaxRows rows
        rc = t->w.alloc(kMaxRows, t->H, t->qkvn(), t->qd(), t->ffn, t->vocab, t->kvh, t->heads,
                        t->hd);
    if (rc == QORA_OK) rc = t->emb_in.alloc((size_t)max_batch * t->H * 4);
    if (rc == QORA_OK) rc = t->tok_in.alloc((size_t)max_batch * 4);
    if (rc != QORA_OK) {
        delete t;
        return rc;
    }
    *out = t;
    return QORA_OK;
}

void qora_talker_destroy(qora_talker *t) { delete t; }

int qora_talker_step(qora_talker *t, qora_kv *kv, const float *emb, const int32_t *positions,
                     int32_t B, float *hidden, float *logits, void *stream) {
    if (!t || !kv || !emb || !positions || !hidden || B <= 0 || B > t->max_batch || B > kv->streams)
        return set_error(QORA_ERR_INVALID, "qora_talker_step: bad arguments");
    if (kv->layers != t->L || kv->kvh != t->kvh || kv->hd != t->hd)
        return set_error(QORA_ERR_SHAPE, "KV cache does not match the talker");
    Launcher ln{t->ctx, &t->w, as_stream(stream)};
    QORA_TRY(kv_prepare(kv, 0, B, 1, ln.st));
    QORA_TRY(launch_copy_rowstats(emb, t->H, t->w.x.as<float>(), t->H, B, t->H,
                                  t->w.ss.as<float>(), t->H / kGroup, ln.st));
    QORA_TRY(talker_forward_step(t, kv, ln, B, positions, hidden, t->H, logits, t->vocab, nullptr));
    kv_note_growth(kv, 0, B, 1);
    return QORA_OK;
}

int qora_talker_decode(qora_talker *t, qora_kv *kv, qora_text_proj *tp, const uint32_t *tokens_host,
                       int32_t is_text, const int32_t *positions, int32_t B, float *hidden,
                       void *stream) {
    if (!t || !kv || !tokens_host || !positions || !hidden || B <= 0 || B > t->max_batch ||
        (is_text && !tp))
        return set_error(QORA_ERR_INVALID, "qora_talker_decode: bad arguments");
    cudaStream_t st = as_stream(stream);
    float *emb = t->emb_in.as<float>();
    if (is_text) {  // embed_text_token (talker.rs:171)
        if (text_proj_hidden(tp) != t->H)
            return set_error(QORA_ERR_SHAPE, "text projection is %lld wide, talker %d",
                             (long long)text_proj_hidden(tp), t->H);
        QORA_TRY(qora_text_proj_embed(tp, tokens_host, B, emb, stream));
    } else {  // embed_codec_token (talker.rs:173)
        for (int32_t b = 0; b < B; b++)
            if ((int64_t)tokens_host[b] >= t->codec_emb.rows)
                return set_error(QORA_ERR_RANGE, "codec token %u outside the codec vocabulary (%lld)",
                                 tokens_host[b], (long long)t->codec_emb.rows);
        QORA_CUDA(cudaMemcpyAsync(t->tok_in.p, tokens_host, (size_t)B * 4, cudaMemcpyHostToDevice, st));
        QORA_TRY(launch_embed_rows(t->codec_emb, t->tok_in.as<uint32_t>(), 1, B, emb, t->H,
                                   t->ctx->err.as<int>(), st));
    }
    return qora_talker_step(t, kv, emb, positions, B, hidden, nullptr, stream);
}

namespace {
// Prefill `T` tokens for streams [s0, s0+ns) (ns*T <= kMaxRows); x rows are
// stream-major [ns][T][H] with row stride H.  Appends T positions per stream.
int talker_prefill_rows(qora_talker *t, qora_kv *kv, int s0, int ns, int T, const float *x,
                        cudaStream_t st) {
    Launcher ln{t->ctx, &t->w, st};
    ln.fixed = true;
    const int rows = ns * T;
    QORA_TRY(kv_prepare(kv, s0, ns, T, st));
    QORA_TRY(launch_copy_rowstats(x, t->H, t->w.x.as<float>(), t->H, rows, t->H,
                                  t->w.ss.as<float>(), t->H / kGroup, st));
    for (int l = 0; l < t->L; l++)
        QORA_TRY(run_layer(ln, t->layers[l], t->H, t->heads, t->kvh, t->hd, t->ffn, rows, T,
                           kv->layer(l, s0), kv->lens() + s0, nullptr, t->rope_cos.as<float>(),
                           t->rope_sin.as<float>(), t->rope_max,
                           l + 1 < t->L ? t->layers[l + 1].qkv : t->head));
    QORA_TRY(launch_ex(k_advance, dim3((ns + 255) / 256), dim3(256), 0, st, 1u, kv->lens() + s0,
                       (int *)nullptr, ns, T));
    kv_note_growth(kv, s0, ns, T);
    return QORA_OK;
}
}  // namespace

int qora_talker_prefill(qora_talker *t, qora_kv *kv, int32_t kv_stream, const float *x, int32_t T,
                        int32_t start_pos, float *hidden, void *stream) {
    if (!t || !kv || !x || !hidden || T <= 0 || kv_stream < 0 || kv_stream >= kv->streams)
        return set_error(QORA_ERR_INVALID, "qora_talker_prefill: bad arguments");
    cudaStream_t st = as_stream(stream);
    int32_t cur = 0;
    QORA_CUDA(cudaMemcpyAsync(&cur, kv->lens() + kv_stream, 4, cudaMemcpyDeviceToHost, st));
    QORA_CUDA(cudaStreamSynchronize(st));
    if (cur != start_pos)  // talker.rs:422-423
        return set_error(QORA_ERR_INVALID, "prefix cache length %d != start_pos %d", cur, start_pos);
    if (start_pos + T > kv->max_pos || start_pos + T > t->rope_max)
        return set_error(QORA_ERR_RANGE, "prefill past capacity");
    kv->host_len[(size_t)kv_stream] = cur;
    for (int t0 = 0; t0 < T; t0 += kMaxRows) {
        const int tc = std::min(kMaxRows, T - t0);
        QORA_TRY(talker_prefill_rows(t, kv, kv_stream, 1, tc, x + (int64_t)t0 * t->H, st));
    }
    // final norm of the last token (talker.rs:480-481)
    const int last = (T - 1) % kMaxRows;
    QORA_TRY(launch_rmsnorm_rows(t->w.x.as<float>() + (int64_t)last * t->H,
                                 t->final_norm.as<__half>(), t->H, 1, hidden, st));
    return QORA_OK;
}

int qora_talker_codec_head(qora_talker *t, const float *hidden, int32_t B, float *logits,
                           void *stream) {
    if (!t || !hidden || !logits || B <= 0 || B > kMaxRows)
        return set_error(QORA_ERR_INVALID, "qora_talker_codec_head: bad arguments");
    Launcher ln{t->ctx, &t->w, as_stream(stream)};
    GemvArgs a;
    a.w = t->head;
    a.rows = B;
    a.x = hidden;
    a.ldx = t->H;
    a.y = logits;
    a.ldy = t->vocab;
    return ln.gemv(a, X_PLAIN, E_STORE);
}

int qora_talker_embed_codec(qora_talker *t, const uint32_t *tokens, int32_t B, float *out,
                            void *stream) {
    if (!t || !tokens || !out || B <= 0) return set_error(QORA_ERR_INVALID, "bad arguments");
    return launch_embed_rows(t->codec_emb, tokens, 1, B, out, t->H, t->ctx->err.as<int>(), as_stream(stream));
}

// --------------------------------------------------------------- predictor
int qora_predictor_create(qora_ctx *ctx, const qora_predictor_host *h, int32_t max_batch,
                          qora_predictor **out) {
    if (!ctx || !h || !out || !h->layers || !h->codec_embeddings || !h->lm_heads ||
        max_batch <= 0 || 2 * max_batch > kMaxRows || h->num_groups > kMaxEmbedGroups)
        return set_error(QORA_ERR_INVALID, "qora_predictor_create: bad arguments");
    QORA_CUDA(cudaSetDevice(ctx->device));
    auto *p = new qora_predictor();
    p->ctx = ctx;
    p->L = h->num_layers;
    p->H = h->hidden;
    p->heads = h->num_heads;
    p->kvh = h->num_kv_heads;
    p->hd = h->head_dim;
    p->ffn = h->ffn;
    p->vocab = h->vocab;
    p->groups = h->num_groups;
    p->rope_max = h->rope_max_pos;
    p->Ht = h->codec_embeddings[0].n;
    p->max_batch = max_batch;
    p->layers.resize(p->L);
    int rc = QORA_OK;
    for (int l = 0; l < p->L && rc == QORA_OK; l++)
        rc = p->layers[l].upload(h->layers[l], p->H, p->heads, p->kvh, p->hd, p->ffn);
    p->has_proj = h->input_proj.packed != nullptr;
    if (rc == QORA_OK && p->has_proj) {
        if (h->input_proj.k != p->Ht || h->input_proj.n != p->H)
            rc = set_error(QORA_ERR_SHAPE, "input_proj shape");
        const int64_t off = 0, st = 1;
        if (rc == QORA_OK)
            rc = upload_q4_parts(&h->input_proj, &off, &st, 1, p->Ht, p->H / kGroup, p->proj_nib,
                                 p->proj_scl, p->proj, nullptr);
        if (rc == QORA_OK) {
            rc = p->proj_bias.alloc((size_t)p->H * 4);
            std::vector<float> zero(p->H, 0.0f);
            const float *b = h->input_proj_bias ? h->input_proj_bias : zero.data();
            if (rc == QORA_OK && cudaMemcpy(p->proj_bias.p, b, (size_t)p->H * 4, cudaMemcpyHostToDevice))
                rc = set_error(QORA_ERR_CUDA, "bias upload");
        }
    } else if (rc == QORA_OK && p->Ht != p->H) {
        rc = set_error(QORA_ERR_SHAPE, "identity projection needs talker hidden == predictor hidden");
    }
    p->emb_packed.resize(p->groups);
    p->emb_scl.resize(p->groups);
    p->head_nib.resize(p->groups);
    p->head_scl.resize(p->groups);
    p->embs.resize(p->groups);
    p->heads_w.resize(p->groups);
    for (int g = 0; g < p->groups && rc == QORA_OK; g++) {
        rc = upload_emb(h->codec_embeddings[g], p->emb_packed[g], p->emb_scl[g], p->embs[g]);
        if (rc == QORA_OK && (h->lm_heads[g].k != p->H || h->lm_heads[g].n != p->vocab))
            rc = set_error(QORA_ERR_SHAPE, "lm_head shape");
        const int64_t off = 0, st = 1;
        if (rc == QORA_OK)
            rc = upload_q4_parts(&h->lm_heads[g], &off, &st, 1, p->H, p->vocab / kGroup,
                                 p->head_nib[g], p->head_scl[g], p->heads_w[g], nullptr);
    }
    if (rc == QORA_OK) rc = upload_f16(h->final_norm, p->H, p->final_norm);
    if (rc == QORA_OK) {
        const int half = p->hd / 2;
        std::vector<float> c((size_t)p->rope_max * half), s((size_t)p->rope_max * half);
        rc = host_rope_tables(p->hd, p->rope_max, h->rope_theta, &half, 1, c.data(), s.data());
        if (rc == QORA_OK) rc = p->rope_cos.alloc(c.size() * 4);
        if (rc == QORA_OK) rc = p->rope_sin.alloc(s.size() * 4);
        if (rc == QORA_OK && (cudaMemcpy(p->rope_cos.p, c.data(), c.size() * 4, cudaMemcpyHostToDevice) ||
                              cudaMemcpy(p->rope_sin.p, s.data(), s.size() * 4, cudaMemcpyHostToDevice)))
            rc = set_error(QORA_ERR_CUDA, "rope upload");
    }
    if (rc == QORA_OK) {
        const int rows = 2 * max_batch;
        const int64_t qkvn = (int64_t)(p->heads + 2 * p->kvh) * p->hd;
        rc = p->w.alloc(rows, p->H, qkvn, (int64_t)p->heads * p->hd, p->ffn, p->vocab, p->kvh,
                        p->heads, p->hd);
        if (rc == QORA_OK) rc = p->x2.alloc((size_t)rows * p->Ht * 4);
        if (rc == QORA_OK) rc = p->codes.alloc((size_t)max_batch * p->groups * 4);
        if (rc == QORA_OK) rc = p->xe.alloc((size_t)rows * p->Ht * 4);
    }
    if (rc != QORA_OK) {
        delete p;
        return rc;
    }
    *out = p;
    return QORA_OK;
}

void qora_predictor_destroy(qora_predictor *p) { delete p; }

int qora_predictor_frame(qora_predictor *p, qora_kv *kv, const float *hidden, const float *semantic,
                         int32_t B, uint32_t *codes, float *logits, const uint32_t *forced,
                         void *stream) {
    if (!p || !kv || !hidden || !semantic || !codes || B <= 0 || B > p->max_batch || B > kv->streams)
        return set_error(QORA_ERR_INVALID, "qora_predictor_frame: bad arguments");
    if (kv->layers != p->L || kv->kvh != p->kvh || kv->hd != p->hd || kv->max_pos < p->groups + 1)
        return set_error(QORA_ERR_SHAPE, "KV cache does not match the predictor");
    cudaStream_t st = as_stream(stream);
    // interleave [hidden | semantic] rows into x2
    const size_t row = (size_t)p->Ht * 4;
    QORA_CUDA(cudaMemcpy2DAsync(p->x2.p, 2 * row, hidden, row, row, B, cudaMemcpyDeviceToDevice, st));
    QORA_CUDA(cudaMemcpy2DAsync(p->x2.as<char>() + row, 2 * row, semantic, row, row, B,
                                cudaMemcpyDeviceToDevice, st));
    Launcher ln{p->ctx, &p->w, st};
    // the frame resets the streams' caches and fills groups + 1 positions
    for (int b = 0; b < B; b++) kv->host_len[(size_t)b] = 0;
    QORA_TRY(kv_prepare(kv, 0, B, p->groups + 1, st));
    QORA_TRY(predictor_frame_impl(p, kv, ln, B, p->x2.as<float>(), codes, p->groups, logits,
                                  (int64_t)p->groups * p->vocab, forced, p->groups));
    kv_note_growth(kv, 0, B, p->groups + 1);
    return QORA_OK;
}

int qora_predictor_embed_sum(qora_predictor *p, const uint32_t *codes, int32_t B, float *out,
                             void *stream) {
    if (!p || !codes || !out || B <= 0) return set_error(QORA_ERR_INVALID, "bad arguments");
    FrameEmbedArgs a;
    a.n = p->Ht;
    for (int g = 0; g < p->groups; g++) a.tables[g] = p->embs[g];
    a.ngroups = p->groups;
    a.codes = codes;
    a.ldcodes = p->groups;
    a.out = out;
    a.ldout = p->Ht;
    return launch_frame_embed(a, B, as_stream(stream));
}

// ------------------------------------------------------------------ engine
int qora_engine_create(qora_talker *t, qora_predictor *p, int32_t B, int32_t max_pos,
                       const qora_sample_params *params, qora_engine **out) {
    if (!t || !p || !params || !out || B <= 0 || B > t->max_batch || B > p->max_batch ||
        max_pos <= 0 || max_pos > t->rope_max || p->Ht != t->H || p->groups + 1 > 16)
        return set_error(QORA_ERR_INVALID, "qora_engine_create: bad arguments");
    auto *e = new qora_engine();
    e->t = t;
    e->p = p;
    e->B = B;
    e->max_pos = max_pos;
    e->params = *params;
    int rc = qora_kv_create(t->ctx, t->L, t->kvh, t->hd, max_pos, B, &e->tkv);
    if (rc == QORA_OK) rc = qora_kv_create(t->ctx, p->L, p->kvh, p->hd, p->groups + 1, B, &e->pkv);
    if (rc == QORA_OK) rc = e->logits.alloc((size_t)B * t->vocab * 4);
    if (rc == QORA_OK) rc = e->codes.alloc((size_t)B * 16 * 4);
    if (rc == QORA_OK) rc = e->prev.alloc((size_t)B * 16 * 4);
    if (rc == QORA_OK) rc = e->rng.alloc((size_t)B * 8);
    if (rc == QORA_OK) rc = e->pos.alloc((size_t)B * 4);
    if (rc == QORA_OK) rc = e->text.alloc((size_t)B * t->H * 4);
    if (rc == QORA_OK) rc = e->prev.zero();
    if (rc == QORA_OK) rc = e->pos.zero();
    if (rc == QORA_OK) rc = e->codes.zero();
    if (rc != QORA_OK) {
        qora_engine_destroy(e);
        return rc;
    }
    *out = e;
    return QORA_OK;
}

void qora_engine_destroy(qora_engine *e) {
    if (!e) return;
    frame_program_destroy(e->frame);
    if (e->exec) cudaGraphExecDestroy(e->exec);
    if (e->graph) cudaGraphDestroy(e->graph);
    qora_kv_destroy(e->tkv);
    qora_kv_destroy(e->pkv);
    delete e;
}

namespace {
// Prefills T rows per stream on top of each stream's cache (which holds
// `start` positions), then sets up the first frame: logits, positions, rng.
int engine_prefill_rows(qora_engine *e, const float *x_host, int32_t T, const uint64_t *seeds_host,
                        int32_t start, void *stream) {
    qora_talker *t = e->t;
    qora_predictor *p = e->p;
    cudaStream_t st = as_stream(stream);
    DevBuf xd;
    QORA_TRY(xd.alloc((size_t)e->B * T * t->H * 4));
    QORA_CUDA(cudaMemcpyAsync(xd.p, x_host, xd.bytes, cudaMemcpyHostToDevice, st));
    const int per = std::max(1, kMaxRows / T);
    for (int s0 = 0; s0 < e->B; s0 += per) {
        const int ns = std::min(per, e->B - s0);
        if (T <= kMaxRows) {
            QORA_TRY(talker_prefill_rows(t, e->tkv, s0, ns, T, xd.as<float>() + (int64_t)s0 * T * t->H, st));
            // last-token hidden of each stream -> predictor input row 0
            for (int i = 0; i < ns; i++)
                QORA_TRY(launch_rmsnorm_rows(t->w.x.as<float>() + ((int64_t)i * T + T - 1) * t->H,
                                             t->final_norm.as<__half>(), t->H, 1,
                                             p->x2.as<float>() + (int64_t)(s0 + i) * 2 * p->Ht, st));
        } else {
            for (int i = 0; i < ns; i++)
                QORA_TRY(qora_talker_prefill(t, e->tkv, s0 + i, xd.as<float>() + (int64_t)(s0 + i) * T * t->H,
                                             T, start, p->x2.as<float>() + (int64_t)(s0 + i) * 2 * p->Ht, stream));
        }
    }
    // first logits (generate_new.rs:473)
    {
        Launcher ln{t->ctx, &t->w, st};
        GemvArgs a;
        a.w = t->head;
        a.rows = e->B;
        a.x = p->x2.as<float>();
        a.ldx = 2 * p->Ht;
        a.y = e->logits.as<float>();
        a.ldy = t->vocab;
        QORA_TRY(ln.gemv(a, X_PLAIN, E_STORE));
    }
    QORA_TRY(launch_ex(k_fill_i32, dim3((e->B + 255) / 256), dim3(256), 0, st, 1u, e->pos.as<int>(),
                       e->B, start + T));
    QORA_CUDA(cudaMemcpyAsync(e->rng.p, seeds_host, (size_t)e->B * 8, cudaMemcpyHostToDevice, st));
    QORA_CUDA(cudaMemsetAsync(e->prev.p, 0, e->prev.bytes, st));
    QORA_CUDA(cudaStreamSynchronize(st));
    return QORA_OK;
}

}  // namespace

int qora_engine_prefill(qora_engine *e, const float *x_host, int32_t T, const uint64_t *seeds_host,
                        void *stream) {
    if (!e || !x_host || !seeds_host || T <= 0 || T >= e->max_pos)
        return set_error(QORA_ERR_INVALID, "qora_engine_prefill: bad arguments");
    QORA_TRY(qora_kv_reset(e->tkv, nullptr, 0, stream));
    return engine_prefill_rows(e, x_host, T, seeds_host, 0, stream);
}

int qora_engine_prefill_from(qora_engine *e, const qora_kv *prefix, int32_t prefix_stream,
                             int32_t prefix_len, const float *x_host, int32_t T,
                             const uint64_t *seeds_host, void *stream) {
    if (!e || !prefix || !x_host || !seeds_host || T <= 0 || prefix_len < 0 ||
        prefix_len + T >= e->max_pos || prefix_stream < 0 || prefix_stream >= prefix->streams)
        return set_error(QORA_ERR_INVALID, "qora_engine_prefill_from: bad arguments");
    if (prefix->layers != e->t->L || prefix->kvh != e->t->kvh || prefix->hd != e->t->hd ||
        prefix->max_pos > e->max_pos)
        return set_error(QORA_ERR_SHAPE, "qora_engine_prefill_from: the prefix cache does not fit the engine");
    cudaStream_t st = as_stream(stream);
    int32_t have = -1;
    QORA_CUDA(cudaMemcpyAsync(&have, prefix->lens() + prefix_stream, 4, cudaMemcpyDeviceToHost, st));
    QORA_CUDA(cudaStreamSynchronize(st));
    if (have != prefix_len)  // the reference falls back to a full prefill here (generate_new.rs:307-316)
        return set_error(QORA_ERR_SHAPE, "qora_engine_prefill_from: prefix holds %d positions, not %d",
                         have, prefix_len);
    QORA_TRY(kv_copy_streams(e->tkv, 0, e->B, prefix, prefix_stream, st));
    return engine_prefill_rows(e, x_host, T, seeds_host, prefix_len, stream);
}

namespace {
int engine_frame_kernels(qora_engine *e, const float *text, uint32_t *codes_out, cudaStream_t st,
                         int *count) {
    qora_talker *t = e->t;
    qora_predictor *p = e->p;
    const int B = e->B;
    int n = 0;
    // 1. code0 = sample_token(logits); prev[0] = code0; semantic row -> x2[b][1]
    SampleArgs sa;
    sa.logits = e->logits.as<float>();
    sa.ldlogits = t->vocab;
    sa.V = t->vocab;
    sa.prev = e->prev.as<uint32_t>();
    sa.ldprev = 16;
    sa.n_prev = 16;
    sa.rng = e->rng.as<uint64_t>();
    sa.params = e->params;
    sa.out = e->codes.as<uint32_t>();
    sa.ldout = 16;
    sa.prev_update = e->prev.as<uint32_t>();
    sa.ldprev_update = 16;
    sa.emb = t->codec_emb;
    sa.emb_out = p->x2.as<float>() + p->Ht;
    sa.ldemb_out = 2 * p->Ht;
    sa.err = t->ctx->err.as<int>();
    QORA_TRY(launch_sample(sa, B, st));
    n++;
    // 2. acoustic codes 1..15
    {
        Launcher ln{p->ctx, &p->w, st};
        QORA_TRY(predictor_frame_impl(p, e->pkv, ln, B, p->x2.as<float>(),
                                      e->codes.as<uint32_t>() + 1, 16, nullptr, 0, nullptr, 0));
        n += ln.count;
    }
    // 3. talker input: (semantic + acoustic sum) + text; prev[1..15] = codes
    {
        FrameEmbedArgs fa;
        fa.n = t->H;
        for (int g = 0; g < p->groups; g++) fa.tables[g] = p->embs[g];
        fa.ngroups = p->groups;
        fa.codes = e->codes.as<uint32_t>();
        fa.ldcodes = 16;
        fa.code_off = 1;
        fa.sem = p->x2.as<float>() + p->Ht;
        fa.ldsem = 2 * p->Ht;
        fa.text = text;
        fa.ldtext = t->H;
        fa.out = t->w.x.as<float>();
        fa.ldout = t->H;
        fa.ss = t->w.ss.as<float>();
        fa.ldss = t->H / kGroup;
        fa.prev = e->prev.as<uint32_t>();
        fa.ldprev = 16;
        QORA_TRY(launch_frame_embed(fa, B, st));
        n++;
    }
    // 4. talker step: hidden -> x2[b][0], logits -> engine logits, advance len and pos
    {
        Launcher ln{t->ctx, &t->w, st};
        QORA_TRY(talker_forward_step(t, e->tkv, ln, B, e->pos.as<int>(), p->x2.as<float>(),
                                     2 * p->Ht, e->logits.as<float>(), t->vocab, e->pos.as<int>()));
        n += ln.count;
    }
    if (codes_out && codes_out != e->codes.as<uint32_t>())
        QORA_CUDA(cudaMemcpyAsync(codes_out, e->codes.p, (size_t)B * 16 * 4, cudaMemcpyDeviceToDevice, st));
    if (count) *count = n;
    return QORA_OK;
}
}  // namespace

int qora_engine_frame(qora_engine *e, const float *text, uint32_t *codes, void *stream) {
    if (!e || !text) return set_error(QORA_ERR_INVALID, "qora_engine_frame: bad arguments");
    cudaStream_t st = as_stream(stream);
    if (e->persistent && frame_supported(e)) {
        // one launch for the whole frame (frame.cu)
        if (!e->frame) QORA_TRY(frame_build(e, &e->frame));
        QORA_TRY(frame_launch(e->frame, text, st));
        if (codes && codes != e->codes.as<uint32_t>())
            QORA_CUDA(cudaMemcpyAsync(codes, e->codes.p, (size_t)e->B * 16 * 4, cudaMemcpyDeviceToDevice, st));
        e->kernels = 1;
        return QORA_OK;
    }
    if (!e->use_graph) {
        int n = 0;
        QORA_TRY(engine_frame_kernels(e, text, codes, st, &n));
        e->kernels = n;
        return QORA_OK;
    }
    if (!e->exec || e->graph_text != text || e->graph_codes != codes || e->cap_stream != st) {
        if (e->exec) cudaGraphExecDestroy(e->exec);
        if (e->graph) cudaGraphDestroy(e->graph);
        e->exec = nullptr;
        e->graph = nullptr;
        cudaStream_t cs = st;
        bool own = false;
        if (cs == nullptr) {  // the legacy stream cannot be captured
            QORA_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
            own = true;
        }
        QORA_CUDA(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
        int n = 0;
        const int rc = engine_frame_kernels(e, text, codes, cs, &n);
        cudaGraph_t g = nullptr;
        const cudaError_t ce = cudaStreamEndCapture(cs, &g);
        if (own) cudaStreamDestroy(cs);
        if (rc != QORA_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (ce != cudaSuccess) return set_error(QORA_ERR_CUDA, "graph capture: %s", cudaGetErrorString(ce));
        e->graph = g;
        QORA_CUDA(cudaGraphInstantiate(&e->exec, g, 0));
        e->graph_text = text;
        e->graph_codes = codes;
        e->cap_stream = st;
        e->kernels = n;
    }
    QORA_CUDA(cudaGraphLaunch(e->exec, st));
    return QORA_OK;
}

int qora_engine_frame_host(qora_engine *e, const float *text_host, uint32_t *codes_host, void *stream) {
    if (!e || !text_host || !codes_host) return set_error(QORA_ERR_INVALID, "bad arguments");
    cudaStream_t st = as_stream(stream);
    QORA_CUDA(cudaMemcpyAsync(e->text.p, text_host, (size_t)e->B * e->t->H * 4,
                              cudaMemcpyHostToDevice, st));
    QORA_TRY(qora_engine_frame(e, e->text.as<float>(), e->codes.as<uint32_t>(), stream));
    QORA_CUDA(cudaMemcpyAsync(codes_host, e->codes.p, (size_t)e->B * 16 * 4, cudaMemcpyDeviceToHost, st));
    QORA_CUDA(cudaStreamSynchronize(st));
    return QORA_OK;
}

int qora_engine_use_graph(qora_engine *e, int32_t enable) {
    if (!e) return set_error(QORA_ERR_INVALID, "null engine");
    e->use_graph = enable != 0;
    return QORA_OK;
}

int qora_engine_set_temperature(qora_engine *e, float temperature) {
    if (!e || temperature != temperature) return set_error(QORA_ERR_INVALID, "qora_engine_set_temperature: bad arguments");
    if (e->params.temperature == temperature) return QORA_OK;
    e->params.temperature = temperature;
    if (e->frame) frame_program_set_temperature(e->frame, temperature);
    // the per-op graph holds the old value in its sampler node: capture again
    if (e->exec) cudaGraphExecDestroy(e->exec);  // (freed after an in-flight launch completes)
    if (e->graph) cudaGraphDestroy(e->graph);
    e->exec = nullptr;
    e->graph = nullptr;
    return QORA_OK;
}

int qora_engine_use_persistent(qora_engine *e, int32_t enable) {
    if (!e) return set_error(QORA_ERR_INVALID, "null engine");
    if (enable && !frame_supported(e))
        return set_error(QORA_ERR_UNSUPPORTED,
                         "persistent frame kernel: needs batch 1, an input projection, head_dim 64/128, "
                         "heads/kv_heads 1/2/4, widths <= 6144 and vocab <= 4096");
    e->persistent = enable != 0;
    return QORA_OK;
}

int qora_engine_trace(qora_engine *e, int32_t enable, int32_t capacity, int32_t *n_ops,
                      int32_t *ops_host, uint64_t *stamps_host) {
    if (!e) return set_error(QORA_ERR_INVALID, "null engine");
    if (!e->persistent || !frame_supported(e))
        return set_error(QORA_ERR_UNSUPPORTED, "tracing needs the persistent frame kernel");
    if (!e->frame) QORA_TRY(frame_build(e, &e->frame));
    FrameProgram *fp = e->frame;
    const int n = (int)fp->ops.size();
    if (n_ops) *n_ops = n;
    if (ops_host || stamps_host) {
        if (capacity < n) return set_error(QORA_ERR_SHAPE, "trace capacity %d < %d ops", capacity, n);
        if (ops_host)
            for (int i = 0; i < n; i++) ops_host[i] = fp->ops[i].type;
        if (stamps_host) {
            QORA_CUDA(cudaDeviceSynchronize());
            QORA_CUDA(cudaMemcpy(stamps_host, fp->d_trace.p, (size_t)n * fk::kTraceFields * 8,
                                 cudaMemcpyDeviceToHost));
        }
    }
    fp->trace = enable != 0;
    return QORA_OK;
}

int qora_engine_kernels_per_frame(qora_engine *e, int32_t *count) {
    if (!e || !count) return set_error(QORA_ERR_INVALID, "bad arguments");
    *count = e->kernels;
    return QORA_OK;
}

int qora_engine_state(qora_engine *e, float **logits, float **hidden, uint32_t **prev,
                      uint64_t **rng, int32_t **positions) {
    if (!e) return set_error(QORA_ERR_INVALID, "null engine");
    if (logits) *logits = e->logits.as<float>();
    if (hidden) *hidden = e->p->x2.as<float>();
    if (prev) *prev = e->prev.as<uint32_t>();
    if (rng) *rng = e->rng.as<uint64_t>();
    if (positions) *positions = e->pos.as<int>();
    return QORA_OK;
}

}  // extern "C"
