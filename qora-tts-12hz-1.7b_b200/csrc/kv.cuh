// Device KV cache handle (RawKvCache / empty_kv_cache, gemv.rs:75-86) shared
// by the model code and the standalone append/attend entry points.
#pragma once

#include "attention.cuh"

struct qora_kv {
    qora::CtxRef ctx;
    int layers = 0, kvh = 0, hd = 0, max_pos = 0, streams = 0;
    qora::DevBuf k, v, len;
    // split-merge scratch of qora_kv_attend, sized on its first call
    qora::DevBuf attn_po, attn_pml, attn_tk;
    int attn_heads = 0;
    size_t layer_elems() const { return (size_t)streams * kvh * max_pos * hd; }
    qora::KVLayer layer(int l, int stream0 = 0) const {
        qora::KVLayer L;
        const size_t off = (size_t)l * layer_elems() + (size_t)stream0 * kvh * max_pos * hd;
        L.k = k.as<float>() + off;
        L.v = v.as<float>() + off;
        L.kv_heads = kvh;
        L.head_dim = hd;
        L.max_pos = max_pos;
        return L;
    }
    int *lens() const { return len.as<int>(); }
};

namespace qora {
// Fills the attention arguments of one standalone decode append/attend call
// (T = 1, B streams starting at stream 0); scratch pointers are left null.
int kv_attend_args(qora_kv *kv, int32_t layer, const float *qkv, int32_t num_heads,
                   const uint16_t *q_norm, const uint16_t *k_norm, const float *rope_cos,
                   const float *rope_sin, int32_t rope_max_pos, const int32_t *positions,
                   int32_t B, float *out, AttnArgs &at);
// Adds one position to streams [0, B) of `kv` (after the last layer's attend).
int kv_advance(qora_kv *kv, int32_t B, cudaStream_t st);
}  // namespace qora
