// The talker's text projection on the device: embed_text_token
// (talker.rs:104-116) for a run of prompt tokens.
//
//   [fc1 GEMV: X_EMBED prologue (dequantised text-embedding row of each
//    token, gemv.rs:425-433), bias epilogue]
//   -> [SiLU in place (gemv.rs:486-488)]
//   -> [fc2 GEMV, bias epilogue] -> out[count][hidden]
//
// Up to kMaxRows tokens share one launch sequence, so the fc1 / fc2 weights
// are streamed once per chunk rather than once per token, on the tensor-core
// GEMV; each token's row is the same bits whatever else is in the chunk.
// Token ids arrive from the host (the tokenizer's output) and are
// range-checked there, before any launch.
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "gemv.cuh"

struct qora_text_proj {
    qora::CtxRef ctx;
    int64_t vocab = 0, th = 0, mid = 0, H = 0;
    qora::DevBuf emb_packed, emb_scl, fc1_nib, fc1_scl, fc2_nib, fc2_scl, b1, b2, tok, h;
    qora::EmbDev emb;
    qora::Q4Dev fc1, fc2;
};

namespace qora {
namespace {

// silu (gemv.rs:486-488): x / (1 + exp(-x)), in place over n values.
__global__ void k_silu(float *h, int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        h[i] = silu_ref(h[i]);
}

int upload_f32(const float *src, int64_t n, DevBuf &buf) {
    if (!src) return set_error(QORA_ERR_INVALID, "null bias vector");
    QORA_TRY(buf.alloc((size_t)n * 4));
    QORA_CUDA(cudaMemcpy(buf.p, src, (size_t)n * 4, cudaMemcpyHostToDevice));
    return QORA_OK;
}

// A token's row must not depend on which other tokens share the call: the
// reference projects one token at a time, and its prefix cache relies on a
// prompt row coming out the same in the prefix build and in the full build.
// So every chunk runs the tensor-core GEMV with the K split planned for a
// single row tile, whatever the chunk's size (its clusters are independent,
// so any number of row tiles is valid).  Where the tensor-core path does not
// apply, each token gets its own launch.
int bias_gemv(qora_text_proj *tp, const Q4Dev &w, int xmode, const float *x, const uint32_t *tok,
              const float *bias, float *y, int rows, cudaStream_t st) {
    GemvArgs a;
    a.w = w;
    a.rows = rows;
    if (xmode == X_EMBED) {
        a.emb = tp->emb;
        a.tok = tok;
        a.ldtok = 1;
    } else {
        a.x = x;
        a.ldx = w.k;
    }
    a.bias = bias;
    a.y = y;
    a.ldy = w.n;
    a.err = tp->ctx->err.as<int>();
    if (gemv_mma_supported(a, xmode, E_BIAS)) {
        GemvPlan p = plan_gemv_mma(w.k, w.C, 1, E_BIAS, tp->ctx->num_sms);
        p.Z = (rows + p.rows_per_z - 1) / p.rows_per_z;
        p.grid.z = (unsigned)p.Z;
        return launch_gemv(a, xmode, E_BIAS, p, nullptr, st);
    }
    for (int r = 0; r < rows; r++) {
        GemvArgs b = a;
        b.rows = 1;
        if (xmode == X_EMBED) b.tok = tok + r;
        else b.x = x + (int64_t)r * w.k;
        b.y = y + (int64_t)r * w.n;
        const GemvPlan p = plan_gemv(w.k, w.C, 1, E_BIAS, tp->ctx->num_sms);
        QORA_TRY(launch_gemv(b, xmode, E_BIAS, p, nullptr, st));
    }
    return QORA_OK;
}

}  // namespace

int64_t text_proj_hidden(const qora_text_proj *tp) { return tp->H; }

}  // namespace qora

using namespace qora;

extern "C" {

int qora_text_proj_create(qora_ctx *ctx, const qora_text_proj_host *h, qora_text_proj **out) {
    if (!ctx || !h || !out) return set_error(QORA_ERR_INVALID, "qora_text_proj_create: bad arguments");
    *out = nullptr;
    const qora_q4_host &e = h->text_embedding, &f1 = h->fc1, &f2 = h->fc2;
    if (e.k <= 0 || e.n <= 0 || e.n % kGroup || f1.k != e.n || f1.n % kGroup || f2.k != f1.n ||
        f2.n <= 0 || f2.n % kGroup)
        return set_error(QORA_ERR_SHAPE,
                         "text projection shapes: embedding [%lld][%lld], fc1 [%lld][%lld], fc2 [%lld][%lld]",
                         (long long)e.k, (long long)e.n, (long long)f1.k, (long long)f1.n,
                         (long long)f2.k, (long long)f2.n);
    QORA_CUDA(cudaSetDevice(ctx->device));
    auto *tp = new qora_text_proj();
    tp->ctx = ctx;
    tp->vocab = e.k;
    tp->th = e.n;
    tp->mid = f1.n;
    tp->H = f2.n;
    const int64_t off = 0, st = 1;
    int rc = upload_emb(e, tp->emb_packed, tp->emb_scl, tp->emb);
    if (rc == QORA_OK)
        rc = upload_q4_parts(&f1, &off, &st, 1, tp->th, tp->mid / kGroup, tp->fc1_nib, tp->fc1_scl,
                             tp->fc1, nullptr);
    if (rc == QORA_OK)
        rc = upload_q4_parts(&f2, &off, &st, 1, tp->mid, tp->H / kGroup, tp->fc2_nib, tp->fc2_scl,
                             tp->fc2, nullptr);
    if (rc == QORA_OK) rc = upload_f32(h->fc1_bias, tp->mid, tp->b1);
    if (rc == QORA_OK) rc = upload_f32(h->fc2_bias, tp->H, tp->b2);
    if (rc == QORA_OK) rc = tp->tok.alloc((size_t)kMaxRows * 4);
    if (rc == QORA_OK) rc = tp->h.alloc((size_t)kMaxRows * tp->mid * 4);
    if (rc == QORA_OK && cudaDeviceSynchronize() != cudaSuccess)
        rc = set_error(QORA_ERR_CUDA, "qora_text_proj_create: upload failed");
    if (rc != QORA_OK) {
        delete tp;
        return rc;
    }
    *out = tp;
    return QORA_OK;
}

void qora_text_proj_destroy(qora_text_proj *tp) { delete tp; }

int qora_text_proj_embed(qora_text_proj *tp, const uint32_t *tokens, int32_t count, float *out,
                         void *stream) {
    if (!tp || (count > 0 && (!tokens || !out)) || count < 0)
        return set_error(QORA_ERR_INVALID, "qora_text_proj_embed: bad arguments");
    for (int32_t i = 0; i < count; i++)
        if ((int64_t)tokens[i] >= tp->vocab)  // embed_lookup indexes the table (talker.rs:107)
            return set_error(QORA_ERR_RANGE, "text token %u at %d outside the text vocabulary (%lld)",
                             tokens[i], i, (long long)tp->vocab);
    cudaStream_t st = as_stream(stream);
    for (int32_t c0 = 0; c0 < count; c0 += kMaxRows) {
        const int rows = std::min<int32_t>(kMaxRows, count - c0);
        QORA_CUDA(cudaMemcpyAsync(tp->tok.p, tokens + c0, (size_t)rows * 4, cudaMemcpyHostToDevice, st));
        float *h = tp->h.as<float>();
        QORA_TRY(bias_gemv(tp, tp->fc1, X_EMBED, nullptr, tp->tok.as<uint32_t>(), tp->b1.as<float>(),
                           h, rows, st));
        const int64_t n = (int64_t)rows * tp->mid;
        const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)tp->ctx->num_sms * 8);
        k_silu<<<blocks, 256, 0, st>>>(h, n);
        QORA_CUDA(cudaGetLastError());
        QORA_TRY(bias_gemv(tp, tp->fc2, X_PLAIN, h, nullptr, tp->b2.as<float>(),
                           out + (int64_t)c0 * tp->H, rows, st));
    }
    return QORA_OK;
}

}  // extern "C"
