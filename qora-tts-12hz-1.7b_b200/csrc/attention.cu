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
#include "attention.cuh"

namespace qora {

namespace {

constexpr int kThreads = 128;
constexpr int kTile = 32;

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

template <int HD>
__device__ __forceinline__ bool rope_rows(const AttnArgs &a, int b, int t, int L0,
                                          const float *&cr, const float *&sr) {
    const int rp = (a.pos ? __ldcg(a.pos + b) : L0) + t;
    if (rp < 0 || rp >= a.rope_max_pos) return false;
    cr = a.rope_cos + (int64_t)rp * (HD / 2);
    sr = a.rope_sin + (int64_t)rp * (HD / 2);
    return true;
}

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
    constexpr int J = HD / 32;
    constexpr int PARTS = 4 / G;           // warps per head in the score phase
    constexpr int DPART = HD / PARTS;
    constexpr int NO = (G * HD + kThreads - 1) / kThreads;
    __shared__ float q_s[G][HD];
    __shared__ float kt_s[HD][kTile + 1];
    __shared__ __align__(16) float v_s[kTile][HD];
    __shared__ float sc_s[G][PARTS][kTile];
    __shared__ float p_s[G][kTile];
    __shared__ float m_s[G], l_s[G], corr_s[G];
    __shared__ int last_flag;

    griddep_launch_dependents();
    griddep_wait();
    const int kvh = blockIdx.x, split = blockIdx.y, r = blockIdx.z;
    const int b = r / a.T, t = r % a.T;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int L0 = __ldcg(a.len + b);
    if (L0 + a.T > a.kv.max_pos) {
        if (threadIdx.x == 0 && split == 0 && kvh == 0) raise_error(a.err, kDevRange);
        return;
    }
    const int Lq = L0 + t + 1;
    const int nsplit = min(kAttnMaxSplit, (Lq + kTile - 1) / kTile);
    if (split >= nsplit) return;
    const int chunk = (Lq + nsplit - 1) / nsplit;
    const int p0 = split * chunk;
    const int p1 = min(Lq, p0 + chunk);

    const float *krow_base = a.kv.k + ((int64_t)b * a.kv_heads + kvh) * a.kv.max_pos * HD;
    const float *vrow_base = a.kv.v + ((int64_t)b * a.kv_heads + kvh) * a.kv.max_pos * HD;
    const float *row = a.qkv + (int64_t)r * a.ldqkv;

    // ---- prologue: query heads (normed + roped unless pre-appended), append
    if (a.preappended) {
        for (int i = threadIdx.x; i < G * HD; i += kThreads)
            q_s[i / HD][i % HD] = row[(int64_t)(kvh * G) * HD + i];
    } else {
        const float *cr = nullptr, *sr = nullptr;
        if (!rope_rows<HD>(a, b, t, L0, cr, sr)) {
            if (threadIdx.x == 0 && split == 0 && kvh == 0) raise_error(a.err, kDevRange);
            return;
        }
        const bool appender = (p1 == Lq);
        for (int it = warp; it < G + 2; it += kThreads / 32) {
            if (it >= G && !appender) continue;
            float v[J];
            const float *src = it < G ? row + (int64_t)(kvh * G + it) * HD
                                      : (it == G ? row + (int64_t)(a.heads + kvh) * HD
                                                 : row + (int64_t)(a.heads + a.kv_heads + kvh) * HD);
#pragma unroll
            for (int j = 0; j < J; j++) v[j] = src[lane + 32 * j];
            if (it < G) {
                norm_rope_head<HD>(v, a.q_gamma, cr, sr, true, lane);
#pragma unroll
                for (int j = 0; j < J; j++) q_s[it][lane + 32 * j] = v[j];
            } else if (it == G) {
                norm_rope_head<HD>(v, a.k_gamma, cr, sr, true, lane);
                float *dst = const_cast<float *>(krow_base) + (int64_t)(L0 + t) * HD;
#pragma unroll
                for (int j = 0; j < J; j++) dst[lane + 32 * j] = v[j];
            } else {
                float *dst = const_cast<float *>(vrow_base) + (int64_t)(L0 + t) * HD;
#pragma unroll
                for (int j = 0; j < J; j++) dst[lane + 32 * j] = v[j];
            }
        }
    }
    if (threadIdx.x < G) {
        m_s[threadIdx.x] = -INFINITY;
        l_s[threadIdx.x] = 0.0f;
    }
    __syncthreads();

    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));  // talker.rs:305
    float o_acc[NO];
#pragma unroll
    for (int i = 0; i < NO; i++) o_acc[i] = 0.0f;

    for (int base = p0; base < p1; base += kTile) {
        const int cnt = min(kTile, p1 - base);
        // K tile (transposed) and V tile into shared memory; every load of the
        // tile is in flight at once
        for (int i = threadIdx.x; i < kTile * (HD / 4); i += kThreads) {
            const int pp = i / (HD / 4), d4 = i % (HD / 4);
            float4 k4 = make_float4(0.f, 0.f, 0.f, 0.f), v4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (pp < cnt) {
                k4 = __ldcg(reinterpret_cast<const float4 *>(krow_base + (int64_t)(base + pp) * HD) + d4);
                v4 = __ldcg(reinterpret_cast<const float4 *>(vrow_base + (int64_t)(base + pp) * HD) + d4);
            }
            kt_s[4 * d4 + 0][pp] = k4.x;
            kt_s[4 * d4 + 1][pp] = k4.y;
            kt_s[4 * d4 + 2][pp] = k4.z;
            kt_s[4 * d4 + 3][pp] = k4.w;
            reinterpret_cast<float4 *>(&v_s[pp][0])[d4] = v4;
        }
        __syncthreads();
        {
            const int hh = warp % G, part = warp / G;
            float dot = 0.0f;
#pragma unroll 8
            for (int d = part * DPART; d < (part + 1) * DPART; d++)
                dot = __fmaf_rn(q_s[hh][d], kt_s[d][lane], dot);
            sc_s[hh][part][lane] = dot;
        }
        __syncthreads();
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
        __syncthreads();
#pragma unroll
        for (int i = 0; i < NO; i++) {
            const int o = threadIdx.x + i * kThreads;
            if (o < G * HD) {
                const int hh = o / HD, d = o % HD;
                float acc = __fmul_rn(o_acc[i], corr_s[hh]);
#pragma unroll 8
                for (int pp = 0; pp < cnt; pp++) acc = __fmaf_rn(p_s[hh][pp], v_s[pp][d], acc);
                o_acc[i] = acc;
            }
        }
        __syncthreads();
    }

    const int64_t out_base = (int64_t)r * a.ldout + (int64_t)kvh * G * HD;
    if (nsplit == 1) {
#pragma unroll
        for (int i = 0; i < NO; i++) {
            const int o = threadIdx.x + i * kThreads;
            if (o < G * HD) a.out[out_base + o] = __fdiv_rn(o_acc[i], l_s[o / HD]);
        }
        return;
    }
    // ---- split partials, last arriver merges in split order
    const int64_t slot = ((int64_t)r * a.kv_heads + kvh) * kAttnMaxSplit;
#pragma unroll
    for (int i = 0; i < NO; i++) {
        const int o = threadIdx.x + i * kThreads;
        if (o < G * HD) __stcg(a.part_o + (slot + split) * (G * HD) + o, o_acc[i]);
    }
    if (threadIdx.x < G) {
        __stcg(a.part_ml + ((slot + split) * G + threadIdx.x) * 2 + 0, m_s[threadIdx.x]);
        __stcg(a.part_ml + ((slot + split) * G + threadIdx.x) * 2 + 1, l_s[threadIdx.x]);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned tk = atomicAdd(&a.tickets[(int64_t)r * a.kv_heads + kvh], 1u);
        last_flag = (tk == (unsigned)(nsplit - 1));
    }
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    for (int o = threadIdx.x; o < G * HD; o += kThreads) {
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
        a.out[out_base + o] = __fdiv_rn(O, L);
    }
    if (threadIdx.x == 0) a.tickets[(int64_t)r * a.kv_heads + kvh] = 0u;
}

template <int HD>
int launch_attn_hd(const AttnArgs &a, cudaStream_t st) {
    const int G = a.heads / a.kv_heads;
    const int rows = a.streams * a.T;
    dim3 grid(a.kv_heads, kAttnMaxSplit, rows);
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
