// Standalone KV-cache append + attend for one decoder layer (the attention
// block of the decode step: talker.rs:285-331, code_predictor.rs:461-498).
// The model code fuses this into its layer sequence; this entry point exposes
// the same kernel (k_attention) to callers that drive the layers themselves.
#include "kv.cuh"

namespace qora {

namespace {
__global__ void k_len_advance(int *len, int count) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) len[i] += 1;
}
}  // namespace

int kv_attend_args(qora_kv *kv, int32_t layer, const float *qkv, int32_t num_heads,
                   const uint16_t *q_norm, const uint16_t *k_norm, const float *rope_cos,
                   const float *rope_sin, int32_t rope_max_pos, const int32_t *positions,
                   int32_t B, float *out, AttnArgs &at) {
    if (!kv || !qkv || !q_norm || !k_norm || !rope_cos || !rope_sin || !positions || !out)
        return set_error(QORA_ERR_INVALID, "qora_kv_attend: null argument");
    if (layer < 0 || layer >= kv->layers || B <= 0 || B > kv->streams || rope_max_pos <= 0)
        return set_error(QORA_ERR_INVALID, "qora_kv_attend: layer %d / B %d out of range", layer, B);
    if (num_heads <= 0 || num_heads % kv->kvh != 0)
        return set_error(QORA_ERR_SHAPE, "qora_kv_attend: %d heads over %d kv heads", num_heads,
                         kv->kvh);
    const int G = num_heads / kv->kvh;
    if (G != 1 && G != 2 && G != 4)
        return set_error(QORA_ERR_UNSUPPORTED, "qora_kv_attend: heads / kv_heads = %d (1, 2, 4)", G);
    at = AttnArgs();
    at.qkv = const_cast<float *>(qkv);  // read only: q/k are normed and roped in shared memory
    at.ldqkv = (int64_t)(num_heads + 2 * kv->kvh) * kv->hd;
    at.heads = num_heads;
    at.kv_heads = kv->kvh;
    at.T = 1;
    at.streams = B;
    at.q_gamma = reinterpret_cast<const __half *>(q_norm);
    at.k_gamma = reinterpret_cast<const __half *>(k_norm);
    at.rope_cos = rope_cos;
    at.rope_sin = rope_sin;
    at.rope_max_pos = rope_max_pos;
    at.pos = positions;
    at.len = kv->lens();
    at.kv = kv->layer(layer);
    at.out = out;
    at.ldout = (int64_t)num_heads * kv->hd;
    at.err = kv->ctx->err.as<int>();
    return QORA_OK;
}

int kv_advance(qora_kv *kv, int32_t B, cudaStream_t st) {
    k_len_advance<<<(B + 255) / 256, 256, 0, st>>>(kv->lens(), B);
    QORA_LAUNCH_CHECK();
    return QORA_OK;
}

}  // namespace qora

using namespace qora;

extern "C" int qora_kv_attend(qora_kv *kv, int32_t layer, const float *qkv, int32_t num_heads,
                              const uint16_t *q_norm, const uint16_t *k_norm, const float *rope_cos,
                              const float *rope_sin, int32_t rope_max_pos,
                              const int32_t *positions, int32_t B, int32_t advance, float *out,
                              void *stream) {
    AttnArgs at;
    QORA_TRY(kv_attend_args(kv, layer, qkv, num_heads, q_norm, k_norm, rope_cos, rope_sin,
                            rope_max_pos, positions, B, out, at));
    DeviceGuard dg;  // the cache's device, whatever the calling thread has current
    QORA_TRY(dg.set(kv->ctx->device));
    if (!kv->attn_po.p || kv->attn_heads != num_heads) {  // first call on this cache: size scratch
        QORA_TRY(kv->attn_po.alloc(attn_part_o_floats(kv->streams, kv->kvh, num_heads, kv->hd) * 4));
        QORA_TRY(kv->attn_pml.alloc(attn_part_ml_floats(kv->streams, kv->kvh, num_heads) * 4));
        QORA_TRY(kv->attn_tk.alloc((size_t)kv->streams * kv->kvh * 4));
        QORA_TRY(kv->attn_tk.zero());
        QORA_CUDA(cudaDeviceSynchronize());
        kv->attn_heads = num_heads;
    }
    at.part_o = kv->attn_po.as<float>();
    at.part_ml = kv->attn_pml.as<float>();
    at.tickets = kv->attn_tk.as<unsigned>();
    cudaStream_t st = as_stream(stream);
    QORA_TRY(kv_prepare(kv, 0, B, 1, st));  // the append at each stream's length
    QORA_TRY(launch_attention(at, st));
    if (advance) {
        QORA_TRY(kv_advance(kv, B, st));
        kv_note_growth(kv, 0, B, 1);
    }
    return QORA_OK;
}
