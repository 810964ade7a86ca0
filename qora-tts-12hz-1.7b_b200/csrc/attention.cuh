// Decode / prefill attention over the device KV cache.
#pragma once

#include "common.cuh"

namespace qora {

// Layer view of the KV cache (f32 rows of head_dim values).
//   slab (table == nullptr): [stream][kv_head][max_pos][head_dim] from k / v;
//   paged: a physical page holds 2^page_shift consecutive positions of every
//   layer and kv head ([layer][kv_head][page_pos][head_dim], page_elems
//   floats; k / v point at this layer's part of page 0), and logical page j
//   of stream b lives in physical page table[b * table_stride + j].
// Within one page (or a slab) a kv head's rows are contiguous, so any run of
// positions that does not cross a multiple of the page size is one block.
struct KVLayer {
    float *k = nullptr;
    float *v = nullptr;
    int kv_heads = 0, head_dim = 0, max_pos = 0;
    const int *table = nullptr;
    int table_stride = 0, page_shift = 0;
    int64_t page_elems = 0;

    // Element offset (from k / v) of position p of (stream b, kv head h).
    __host__ __device__ __forceinline__ int64_t row(int b, int h, int p) const {
        if (!table) return (((int64_t)b * kv_heads + h) * max_pos + p) * head_dim;
        const int pg = table[(int64_t)b * table_stride + (p >> page_shift)];
        return (int64_t)pg * page_elems +
               ((int64_t)(h << page_shift) + (p & ((1 << page_shift) - 1))) * head_dim;
    }
};

struct alignas(16) AttnArgs {
    // raw projections, row r = stream * T + t: [q (heads*hd) | k (kvh*hd) | v (kvh*hd)]
    float *qkv = nullptr;
    int64_t ldqkv = 0;
    int heads = 0, kv_heads = 0;
    int T = 1;                      // query tokens per stream in this call
    int streams = 0;
    const __half *q_gamma = nullptr, *k_gamma = nullptr;  // qk-norm (talker.rs:89-99)
    const float *rope_cos = nullptr, *rope_sin = nullptr; // [rope_max_pos][hd/2]
    int rope_max_pos = 0;
    const int *pos = nullptr;       // RoPE position of token 0 per stream; NULL => cache length
    const int *len = nullptr;       // cache length per stream before this call
    int pos_static = -1;            // >= 0: RoPE position of token 0 for every stream (overrides pos)
    int len_static = -1;            // >= 0: cache length for every stream (overrides len)
    int stable_len = -1;            // cache rows [0, stable_len) were written before this launch
                                    // (may be read before the item's inputs arrive); < 0: all of
                                    // them (a kernel of its own, after griddepcontrol.wait)
    int stable_writer = -1;         // frame kernel: op index of the attention op that wrote row
                                    // len - 1 in this launch (-1: none); an SM that has waited on
                                    // the input of a later op may read rows [0, len) early
    KVLayer kv;
    bool preappended = false;       // q/k already normed+roped and K/V appended
    float *out = nullptr;           // [rows][heads*hd]
    int64_t ldout = 0;
    // split merge scratch
    float *part_o = nullptr;        // [rows][kvh][kAttnMaxSplit][G][hd]
    float *part_ml = nullptr;       // [rows][kvh][kAttnMaxSplit][G][2]
    unsigned *tickets = nullptr;    // [rows][kvh]
    int *err = nullptr;
    // tagged input / output (persistent frame kernel): when qkv_t is set the
    // q | k | v rows are read from tagged words carrying qkv_tag, and when
    // out_t is set the output is written as tagged words carrying out_tag
    const uint64_t *qkv_t = nullptr;
    uint32_t qkv_tag = 0, out_tag = 0;
    uint64_t *out_t = nullptr;
    uint32_t tag_base = 0;          // added to qkv_tag and out_tag
    int *abort_flag = nullptr;
};

// qk-norm + RoPE + append for T tokens per stream (used when T > 1).
int launch_qkv_post(const AttnArgs &a, cudaStream_t stream);
// Attention for every row; fused qk-norm/RoPE/append when !a.preappended (T == 1).
int launch_attention(const AttnArgs &a, cudaStream_t stream);

inline size_t attn_part_o_floats(int rows, int kvh, int heads, int hd) {
    return (size_t)rows * kvh * kAttnMaxSplit * (heads / kvh) * hd;
}
inline size_t attn_part_ml_floats(int rows, int kvh, int heads) {
    return (size_t)rows * kvh * kAttnMaxSplit * (heads / kvh) * 2;
}

}  // namespace qora
