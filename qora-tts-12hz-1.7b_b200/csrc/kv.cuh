// Device KV cache handle (RawKvCache / empty_kv_cache, gemv.rs:75-86) shared
// by the model code and the standalone append/attend entry points.
#pragma once

#include "attention.cuh"

#include <vector>

struct qora_kv {
    qora::CtxRef ctx;
    int layers = 0, kvh = 0, hd = 0, max_pos = 0, streams = 0;
    qora::DevBuf k, v, len;
    // split-merge scratch of qora_kv_attend, sized on its first call
    qora::DevBuf attn_po, attn_pml, attn_tk;
    int attn_heads = 0;
    // ---- paged layout (page_pos > 0): a pool of pool_pages pages (+ one
    // guard page that unmapped table entries point at), a page table per
    // stream, pages mapped from the pool as a stream grows and returned when
    // it is reset.  Pages are reference counted: a prefix copy shares the
    // source's full pages.  host_len mirrors the device lengths as the host
    // entry points set them.
    int page_pos = 0, page_shift = 0, pages_per_stream = 0, pool_pages = 0;
    qora::DevBuf table;
    std::vector<int> host_table, refs, free_pages, host_len;
    bool paged() const { return page_pos > 0; }
    int guard_page() const { return pool_pages; }
    int64_t page_elems() const { return (int64_t)layers * kvh * page_pos * hd; }

    size_t layer_elems() const { return (size_t)streams * kvh * max_pos * hd; }
    qora::KVLayer layer(int l, int stream0 = 0) const {
        qora::KVLayer L;
        L.kv_heads = kvh;
        L.head_dim = hd;
        L.max_pos = max_pos;
        if (paged()) {
            const size_t off = (size_t)l * kvh * page_pos * hd;
            L.k = k.as<float>() + off;
            L.v = v.as<float>() + off;
            L.table = table.as<int>() + (size_t)stream0 * pages_per_stream;
            L.table_stride = pages_per_stream;
            L.page_shift = page_shift;
            L.page_elems = page_elems();
            return L;
        }
        const size_t off = (size_t)l * layer_elems() + (size_t)stream0 * kvh * max_pos * hd;
        L.k = k.as<float>() + off;
        L.v = v.as<float>() + off;
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
// Smallest page of a paged cache: every tile the attention kernels read
// (16 or 32 positions starting at a multiple of its size) lies in one page.
constexpr int kPageMinPositions = 32;
// Paged caches: returns a stream's pages (its table entries point at the
// guard page again; a page shared with another stream stays mapped there).
void kv_release_stream(qora_kv *kv, int sid);
// Paged caches: maps pages so that streams [s0, s0 + n) hold their current
// length plus `add` positions (QORA_ERR_OOM when the pool runs out, before
// any launch), uploading changed table entries on `st`.  No-op for a slab.
int kv_prepare(qora_kv *kv, int s0, int n, int add, cudaStream_t st);
// Records on the host that streams [s0, s0 + n) grew by `add` positions.
void kv_note_growth(qora_kv *kv, int s0, int n, int add);
// Copies stream `ss` of `src` into streams [ds, ds + n) of `dst` (live rows
// only; a paged destination shares the source's full pages when both are
// paged alike).
int kv_copy_streams(qora_kv *dst, int32_t ds, int32_t n, const qora_kv *src, int32_t ss,
                    cudaStream_t st);
}  // namespace qora
