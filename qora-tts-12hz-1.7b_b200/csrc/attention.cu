// GQA decode attention with fused qk-norm, RoPE and KV append (sm_100a).
//
// Replaces the per-layer attention block of the talker and the predictor
// (talker.rs:285-331, code_predictor.rs:461-498, prefill variants
// talker.rs:402-458 and code_predictor.rs:369-414):
//   * apply_qk_norm (talker.rs:89-99): per-head RMS norm, eps 1e-6, f16 gamma;
//   * split / rotate-half RoPE (rope.rs:79-92, code_predictor.rs:97-121);
//   * KV append at the stream's cache length (extend_from_slice);
//   * scores (q.k) * 1/sqrt(hd), softmax, weighted V sum.
// One CTA handles one (kv head, position split, query row) and all G query
// heads sharing that kv head, so every K/V byte is read once per row.  Splits
// are merged flash-decoding style by the last-arriving CTA in split order.
#include "attention_impl.cuh"

namespace qora {

namespace {

using attn::kTile;
using attn::norm_rope_head;
using attn::rope_rows;

constexpr int kThreads = 128;

template <int HD>
__global__ void __launch_bounds__(kThreads) k_qkv_post(const AttnArgs a) {
    constexpr int J = HD / 32;
    griddep_launch_dependents();
    griddep_wait();
    const int r = blockIdx.x;
    const int b = r / a.T, t = r % a.T;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int L0 = __ldcg(a.len + b);
    if (L0 + a.T > a.kv.max_pos) {
        if (threadIdx.x == 0) raise_error(a.err, kDevRange);
        return;
    }
    const float *cr, *sr;
    if (!rope_rows<HD>(a, b, t, L0, cr, sr)) {
        if (threadIdx.x == 0) raise_error(a.err, kDevRange);
        return;
    }
    float *row = a.qkv + (int64_t)r * a.ldqkv;
    const int nitems = a.heads + 2 * a.kv_heads;
    for (int it = warp; it < nitems; it += kThreads / 32) {
        float v[J];
        const float *src = row + (int64_t)it * HD;  // q heads, then k heads, then v heads
#pragma unroll
        for (int j = 0; j < J; j++) v[j] = src[lane + 32 * j];
        if (it < a.heads) {
            norm_rope_head<HD>(v, a.q_gamma, cr, sr, true, lane);
#pragma unroll
            for (int j = 0; j < J; j++) row[(int64_t)it * HD + lane + 32 * j] = v[j];
        } else if (it < a.heads + a.kv_heads) {
            const int h = it - a.heads;
            norm_rope_head<HD>(v, a.k_gamma, cr, sr, true, lane);
            float *dst = a.kv.k + (((int64_t)b * a.kv_heads + h) * a.kv.max_pos + L0 + t) * HD;
#pragma unroll
            for (int j = 0; j < J; j++) dst[lane + 32 * j] = v[j];
        } else {
            const int h = it - a.heads - a.kv_heads;
            float *dst = a.kv.v + (((int64_t)b * a.kv_heads + h) * a.kv.max_pos + L0 + t) * HD;
#pragma unroll
            for (int j = 0; j < J; j++) dst[lane + 32 * j] = v[j];
        }
    }
}

template <int HD, int G>
__global__ void __launch_bounds__(kThreads) k_attention(const AttnArgs a) {
    __shared__ attn::AttnSmem<HD, G, kThreads> sm;
    griddep_launch_dependents();
    griddep_wait();
    attn::attn_item<HD, G, kThreads, 0>(a, blockIdx.x, blockIdx.y, blockIdx.z, threadIdx.x, sm);
}

template <int HD>
int launch_attn_hd(const AttnArgs &a, cudaStream_t st) {
    const int G = a.heads / a.kv_heads;
    const int rows = a.streams * a.T;
    // position splits: the kernel uses min(16, ceil(positions / 32)) of them
    // and positions never exceed the cache capacity, so that bounds the grid
    // (a short cache such as the predictor's launches one split per row)
    const int ysplit = std::max(1, std::min(kAttnMaxSplit, (a.kv.max_pos + attn::kTile - 1) / attn::kTile));
    dim3 grid(a.kv_heads, ysplit, rows);
    switch (G) {
        case 1: return launch_ex(k_attention<HD, 1>, grid, dim3(kThreads), 0, st, 1u, a);
        case 2: return launch_ex(k_attention<HD, 2>, grid, dim3(kThreads), 0, st, 1u, a);
        case 4: return launch_ex(k_attention<HD, 4>, grid, dim3(kThreads), 0, st, 1u, a);
    }
    return set_error(QORA_ERR_UNSUPPORTED, "heads/kv_heads = %d", G);
}

}  // namespace

int launch_qkv_post(const AttnArgs &a, cudaStream_t st) {
    const int rows = a.streams * a.T;
    if (rows <= 0) return QORA_OK;
    switch (a.kv.head_dim) {
        case 64: return launch_ex(k_qkv_post<64>, dim3(rows), dim3(kThreads), 0, st, 1u, a);
        case 128: return launch_ex(k_qkv_post<128>, dim3(rows), dim3(kThreads), 0, st, 1u, a);
    }
    return set_error(QORA_ERR_UNSUPPORTED, "head_dim %d", a.kv.head_dim);
}

int launch_attention(const AttnArgs &a, cudaStream_t st) {
    if (!a.preappended && a.T != 1)
        return set_error(QORA_ERR_INVALID, "fused append needs T == 1");
    if (a.streams * a.T <= 0) return QORA_OK;
    switch (a.kv.head_dim) {
        case 64: return launch_attn_hd<64>(a, st);
        case 128: return launch_attn_hd<128>(a, st);
    }
    return set_error(QORA_ERR_UNSUPPORTED, "head_dim %d", a.kv.head_dim);
}

}  // namespace qora
