// Device-side pieces of the GQA decode attention (sm_100a), shared by the
// standalone kernels (attention.cu) and the persistent frame kernel.
//
// Restates the attention block of the decode step (talker.rs:285-331,
// code_predictor.rs:461-498): apply_qk_norm (talker.rs:89-99), split /
// rotate-half RoPE (rope.rs:79-92), KV append at the stream's cache length,
// scores (q.k) * 1/sqrt(hd), softmax, weighted V sum.  One work item handles
// one (kv head, position split, query row) and all G query heads sharing that
// kv head, so every K/V byte is read once per row; splits are merged
// flash-decoding style by the last-arriving item in split order.
#pragma once

#include "attention.cuh"

namespace qora {
namespace attn {

constexpr int kTile = 32;

// Block-wide barrier over the NT threads that run an item: BAR 0 is
// __syncthreads (the whole CTA), BAR > 0 a named barrier of NT threads.
template <int NT, int BAR>
__device__ __forceinline__ void block_sync() {
    if constexpr (BAR == 0) {
        __syncthreads();
    } else {
        asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
    }
}

// qk-norm + RoPE of one head vector held by one warp: element i = lane + 32 j.
template <int HD>
__device__ __forceinline__ void norm_rope_head(float (&v)[HD / 32], const __half *gamma,
                                               const float *cos_row, const float *sin_row,
                                               bool do_rope, int lane) {
    constexpr int J = HD / 32;
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < J; j++) ss += __fmul_rn(v[j], v[j]);
    ss = warp_sum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), 1e-6f)));
#pragma unroll
    for (int j = 0; j < J; j++) v[j] = __fmul_rn(__fmul_rn(v[j], inv), __half2float(gamma[lane + 32 * j]));
    if (do_rope) {
        // pairs (i, i + HD/2): x1' = x1 c - x2 s ; x2' = x2 c + x1 s
#pragma unroll
        for (int j = 0; j < J / 2; j++) {
            const int i = lane + 32 * j;
            const float c = cos_row[i], s = sin_row[i];
            const float x1 = v[j], x2 = v[j + J / 2];
            v[j] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
            v[j + J / 2] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
        }
    }
}

// The same with gamma and the RoPE row already in registers (g[j] = gamma
// element lane + 32 j, c / sn[j] = cos / sin element lane + 32 j, j < HD/64).
template <int HD>
__device__ __forceinline__ void norm_rope_head_pre(float (&v)[HD / 32], const float (&g)[HD / 32],
                                                   const float (&c)[HD / 64], const float (&sn)[HD / 64]) {
    constexpr int J = HD / 32;
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < J; j++) ss += __fmul_rn(v[j], v[j]);
    ss = warp_sum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), 1e-6f)));
#pragma unroll
    for (int j = 0; j < J; j++) v[j] = __fmul_rn(__fmul_rn(v[j], inv), g[j]);
#pragma unroll
    for (int j = 0; j < J / 2; j++) {
        const float x1 = v[j], x2 = v[j + J / 2];
        v[j] = __fsub_rn(__fmul_rn(x1, c[j]), __fmul_rn(x2, sn[j]));
        v[j + J / 2] = __fadd_rn(__fmul_rn(x2, c[j]), __fmul_rn(x1, sn[j]));
    }
}

// Asynchronous global -> shared copies of 16 bytes (L2 only) and 4 bytes.
__device__ __forceinline__ void attn_cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void attn_cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}

template <int HD>
__device__ __forceinline__ bool rope_rows(const AttnArgs &a, int b, int t, int L0,
                                          const float *&cr, const float *&sr) {
    const int rp = (a.pos_static >= 0 ? a.pos_static : (a.pos ? __ldcg(a.pos + b) : L0)) + t;
    if (rp < 0 || rp >= a.rope_max_pos) return false;
    cr = a.rope_cos + (int64_t)rp * (HD / 2);
    sr = a.rope_sin + (int64_t)rp * (HD / 2);
    return true;
}

template <int HD, int G, int NT>
struct AttnSmem {
    float q_s[G][HD];
    float kt_s[HD][kTile + 1];
    __align__(16) float v_s[kTile][HD];
    float sc_s[G][(NT / 32) / G][kTile];
    float p_s[G][kTile];
    float m_s[G], l_s[G], corr_s[G];
    int last_flag;
};

// `stable_all`: every cache row before this call's new ones is final (the
// caller knows it), whatever a.stable_len says.
template <int HD, int G, int NT, int BAR>
__device__ __forceinline__ void attn_item(const AttnArgs &a, int kvh, int split, int r, int tid,
                                          AttnSmem<HD, G, NT> &sm, bool stable_all = false) {
    constexpr int J = HD / 32;
    constexpr int PARTS = (NT / 32) / G;   // warps per head in the score phase
    constexpr int DPART = HD / PARTS;
    constexpr int NO = (G * HD + NT - 1) / NT;
    auto &q_s = sm.q_s;
    auto &kt_s = sm.kt_s;
    auto &v_s = sm.v_s;
    auto &sc_s = sm.sc_s;
    auto &p_s = sm.p_s;
    auto &m_s = sm.m_s;
    auto &l_s = sm.l_s;
    auto &corr_s = sm.corr_s;
    auto &last_flag = sm.last_flag;
    const int b = r / a.T, t = r % a.T;
    const int lane = tid & 31, warp = tid >> 5;
    const int L0 = a.len_static >= 0 ? a.len_static : __ldcg(a.len + b);
    if (L0 + a.T > a.kv.max_pos) {
        if (tid == 0 && split == 0 && kvh == 0) raise_error(a.err, kDevRange);
        return;
    }
    const int Lq = L0 + t + 1;
    const int nsplit = min(kAttnMaxSplit, (Lq + kTile - 1) / kTile);
    if (split >= nsplit) return;
    const int chunk = (Lq + nsplit - 1) / nsplit;
    const int p0 = split * chunk;
    const int p1 = min(Lq, p0 + chunk);

    // row p of this (stream, kv head) in the cache (slab or paged)
    auto krow = [&](int p) { return a.kv.k + a.kv.row(b, kvh, p); };
    auto vrow = [&](int p) { return a.kv.v + a.kv.row(b, kvh, p); };
    const float *row = a.qkv + (int64_t)r * a.ldqkv;

    // ---- prologue: query heads (normed + roped unless pre-appended), append
    bool staged0 = false;  // the split's first K / V tile is complete in shared memory
    if (a.preappended) {
        for (int i = tid; i < G * HD; i += NT)
            q_s[i / HD][i % HD] = __ldcg(row + (int64_t)(kvh * G) * HD + i);
    } else {
        const float *cr = nullptr, *sr = nullptr;
        if (!rope_rows<HD>(a, b, t, L0, cr, sr)) {
            if (tid == 0 && split == 0 && kvh == 0) raise_error(a.err, kDevRange);
            return;
        }
        const bool appender = (p1 == Lq);
        // What does not depend on this op's inputs is requested before waiting
        // for them: the qk-norm gamma and RoPE row of the warp's head, and the
        // cached K / V rows of the split's first tile (positions < L0) that were
        // written before this launch (V as 16-byte pieces, K elements straight
        // into the transposed tile).  Rows written earlier in this launch are
        // read only after the inputs: the first tile is then loaded whole after
        // the barrier below.
        const int old0 = max(0, min(min(kTile, p1 - p0), L0 - p0));
        const int stable = (stable_all || a.stable_len < 0) ? L0 : min(L0, a.stable_len);
        const int pre0 = max(0, min(old0, stable - p0));
        staged0 = (pre0 == old0);
        for (int i = tid; i < pre0 * (HD / 4); i += NT) {
            const int pp = i / (HD / 4), d4 = i % (HD / 4);
            attn_cp_async16(&v_s[pp][4 * d4], vrow(p0 + pp) + 4 * d4);
        }
        for (int i = tid; i < pre0 * HD; i += NT) {
            const int pp = i / HD, d = i % HD;
            attn_cp_async4(&kt_s[d][pp], krow(p0 + pp) + d);
        }
        for (int it = warp; it < G + 2; it += NT / 32) {
            if (it >= G && !appender) continue;
            float gv[J], cv[J / 2], sv[J / 2];
            if (it <= G) {
                const __half *gm = it < G ? a.q_gamma : a.k_gamma;
#pragma unroll
                for (int j = 0; j < J; j++) gv[j] = __half2float(gm[lane + 32 * j]);
#pragma unroll
                for (int j = 0; j < J / 2; j++) {
                    cv[j] = cr[lane + 32 * j];
                    sv[j] = sr[lane + 32 * j];
                }
            }
            float v[J];
            const int64_t off = it < G ? (int64_t)(kvh * G + it) * HD
                                       : (it == G ? (int64_t)(a.heads + kvh) * HD
                                                  : (int64_t)(a.heads + a.kv_heads + kvh) * HD);
            if (a.qkv_t) {
                bool all[J];
#pragma unroll
                for (int j = 0; j < J; j++) all[j] = true;
                // acquire: the K/V rows read below were appended by earlier ops
                poll_tagged<J, true>(a.qkv_t + (int64_t)r * a.ldqkv + off + lane, 32, a.tag_base + a.qkv_tag,
                                     v, all, a.err, a.abort_flag);
            } else {
                const float *src = row + off;
#pragma unroll
                for (int j = 0; j < J; j++) v[j] = __ldcg(src + lane + 32 * j);
            }
            // the new row sits in the split's first tile when L0 - p0 < kTile
            const int nt = L0 + t - p0;
            const bool in_tile0 = appender && nt < kTile;
            if (it < G) {
                norm_rope_head_pre<HD>(v, gv, cv, sv);
#pragma unroll
                for (int j = 0; j < J; j++) q_s[it][lane + 32 * j] = v[j];
            } else if (it == G) {
                norm_rope_head_pre<HD>(v, gv, cv, sv);
                float *dst = krow(L0 + t);
#pragma unroll
                for (int j = 0; j < J; j++) dst[lane + 32 * j] = v[j];
                if (in_tile0) {
#pragma unroll
                    for (int j = 0; j < J; j++) kt_s[lane + 32 * j][nt] = v[j];
                }
            } else {
                float *dst = vrow(L0 + t);
#pragma unroll
                for (int j = 0; j < J; j++) dst[lane + 32 * j] = v[j];
                if (in_tile0) {
#pragma unroll
                    for (int j = 0; j < J; j++) v_s[nt][lane + 32 * j] = v[j];
                }
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    }
    if (tid < G) {
        m_s[tid] = -INFINITY;
        l_s[tid] = 0.0f;
    }
    block_sync<NT, BAR>();

    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));  // talker.rs:305
    float o_acc[NO];
#pragma unroll
    for (int i = 0; i < NO; i++) o_acc[i] = 0.0f;

    for (int base = p0; base < p1; base += kTile) {
        const int cnt = min(kTile, p1 - base);
        // K tile (transposed) and V tile into shared memory; every load of the
        // tile is in flight at once (a staged first tile is already in place)
        const bool staged = staged0 && base == p0;
        for (int i = staged ? kTile * (HD / 4) : tid; i < kTile * (HD / 4); i += NT) {
            const int pp = i / (HD / 4), d4 = i % (HD / 4);
            float4 k4 = make_float4(0.f, 0.f, 0.f, 0.f), v4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (pp < cnt) {
                k4 = __ldcg(reinterpret_cast<const float4 *>(krow(base + pp)) + d4);
                v4 = __ldcg(reinterpret_cast<const float4 *>(vrow(base + pp)) + d4);
            }
            kt_s[4 * d4 + 0][pp] = k4.x;
            kt_s[4 * d4 + 1][pp] = k4.y;
            kt_s[4 * d4 + 2][pp] = k4.z;
            kt_s[4 * d4 + 3][pp] = k4.w;
            reinterpret_cast<float4 *>(&v_s[pp][0])[d4] = v4;
        }
        block_sync<NT, BAR>();
        {
            const int hh = warp % G, part = warp / G;
            float dot = 0.0f;
#pragma unroll 8
            for (int d = part * DPART; d < (part + 1) * DPART; d++)
                dot = __fmaf_rn(q_s[hh][d], kt_s[d][lane], dot);
            sc_s[hh][part][lane] = dot;
        }
        block_sync<NT, BAR>();
        if (warp < G) {
            const int hh = warp;
            float dot = 0.0f;
#pragma unroll
            for (int pt = 0; pt < PARTS; pt++) dot += sc_s[hh][pt][lane];
            const float sc = lane < cnt ? __fmul_rn(dot, scale) : -INFINITY;
            const float m_old = m_s[hh];
            const float m_new = fmaxf(m_old, warp_max(sc));
            const float p = lane < cnt ? expf(sc - m_new) : 0.0f;
            const float psum = warp_sum(p);
            p_s[hh][lane] = p;
            if (lane == 0) {
                const float corr = expf(m_old - m_new);  // exp(-inf) = 0 on the first tile
                corr_s[hh] = corr;
                l_s[hh] = __fmaf_rn(l_s[hh], corr, psum);
                m_s[hh] = m_new;
            }
        }
        block_sync<NT, BAR>();
#pragma unroll
        for (int i = 0; i < NO; i++) {
            const int o = tid + i * NT;
            if (o < G * HD) {
                const int hh = o / HD, d = o % HD;
                float acc = __fmul_rn(o_acc[i], corr_s[hh]);
#pragma unroll 8
                for (int pp = 0; pp < cnt; pp++) acc = __fmaf_rn(p_s[hh][pp], v_s[pp][d], acc);
                o_acc[i] = acc;
            }
        }
        block_sync<NT, BAR>();
    }

    const int64_t out_base = (int64_t)r * a.ldout + (int64_t)kvh * G * HD;
    if (nsplit == 1) {
        if (a.out_t) fence_acq_rel_gpu();  // the K/V append is published before the output
#pragma unroll
        for (int i = 0; i < NO; i++) {
            const int o = tid + i * NT;
            if (o < G * HD) {
                const float y = __fdiv_rn(o_acc[i], l_s[o / HD]);
                if (a.out_t) st_relaxed_u64(a.out_t + out_base + o, tag_pack(y, a.tag_base + a.out_tag));
                else a.out[out_base + o] = y;
            }
        }
        return;
    }
    // ---- split partials, last arriver merges in split order
    const int64_t slot = ((int64_t)r * a.kv_heads + kvh) * kAttnMaxSplit;
#pragma unroll
    for (int i = 0; i < NO; i++) {
        const int o = tid + i * NT;
        if (o < G * HD) __stcg(a.part_o + (slot + split) * (G * HD) + o, o_acc[i]);
    }
    if (tid < G) {
        __stcg(a.part_ml + ((slot + split) * G + tid) * 2 + 0, m_s[tid]);
        __stcg(a.part_ml + ((slot + split) * G + tid) * 2 + 1, l_s[tid]);
    }
    __threadfence();
    block_sync<NT, BAR>();
    if (tid == 0) {
        const unsigned tk = atomicAdd(&a.tickets[(int64_t)r * a.kv_heads + kvh], 1u);
        last_flag = (tk == (unsigned)(nsplit - 1));
    }
    block_sync<NT, BAR>();
    if (!last_flag) return;
    __threadfence();
    for (int o = tid; o < G * HD; o += NT) {
        const int hh = o / HD;
        float M = -INFINITY;
        for (int sp = 0; sp < nsplit; sp++)
            M = fmaxf(M, __ldcg(a.part_ml + ((slot + sp) * G + hh) * 2));
        float L = 0.0f, O = 0.0f;
        for (int sp = 0; sp < nsplit; sp++) {
            const float w = expf(__ldcg(a.part_ml + ((slot + sp) * G + hh) * 2) - M);
            L = __fmaf_rn(__ldcg(a.part_ml + ((slot + sp) * G + hh) * 2 + 1), w, L);
            O = __fmaf_rn(__ldcg(a.part_o + (slot + sp) * (G * HD) + o), w, O);
        }
        const float y = __fdiv_rn(O, L);
        if (a.out_t) st_relaxed_u64(a.out_t + out_base + o, tag_pack(y, a.tag_base + a.out_tag));
        else a.out[out_base + o] = y;
    }
    if (tid == 0) a.tickets[(int64_t)r * a.kv_heads + kvh] = 0u;
}

}  // namespace attn
}  // namespace qora
