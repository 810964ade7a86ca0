// Device-side sampler (sm_100a), shared by the standalone k_sample and the
// persistent frame kernel.
//
// sample_row restates sample_token (generate_new.rs:771-862) for one row:
// repetition penalty over the previous codes (divide if > 0, else multiply;
// repeated ids apply repeatedly), temperature, softmax, top-k (the first k of
// a stable descending sort, i.e. ties keep index order), renormalisation,
// optional top-p, then the xorshift64 draw of simple_rand
// (generate_new.rs:17-22) and a cumulative scan in index order.  The top-k
// threshold is found by a 4-pass radix select on the probability bits
// instead of a sort; survivor sums and the final scan run sequentially in
// index order, as in the reference.
#pragma once

#include "attention_impl.cuh"
#include "sampler.cuh"

namespace qora {
namespace samp {

constexpr int kSampleMaxV = 4096;


template <int NT, int BAR>
__device__ __forceinline__ float block_reduce_max(float v, float *red, int tid) {
    v = warp_max(v);
    const int lane = tid & 31, warp = tid >> 5;
    attn::block_sync<NT, BAR>();
    if (lane == 0) red[warp] = v;
    attn::block_sync<NT, BAR>();
    if (warp == 0) {
        float x = lane < (NT / 32) ? red[lane] : -INFINITY;
        x = warp_max(x);
        if (lane == 0) red[0] = x;
    }
    attn::block_sync<NT, BAR>();
    return red[0];
}

template <int NT, int BAR>
__device__ __forceinline__ float block_reduce_sum(float v, float *red, int tid) {
    v = warp_sum(v);
    const int lane = tid & 31, warp = tid >> 5;
    attn::block_sync<NT, BAR>();
    if (lane == 0) red[warp] = v;
    attn::block_sync<NT, BAR>();
    if (warp == 0) {
        float x = lane < (NT / 32) ? red[lane] : 0.0f;
        x = warp_sum(x);
        if (lane == 0) red[0] = x;
    }
    attn::block_sync<NT, BAR>();
    return red[0];
}

// Exclusive prefix sum of one int per thread over the block (index order).
template <int NT, int BAR>
__device__ __forceinline__ int block_exclusive_scan(int v, int *wsum, int &total, int tid) {
    const int lane = tid & 31, warp = tid >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    attn::block_sync<NT, BAR>();
    if (lane == 31) wsum[warp] = x;
    attn::block_sync<NT, BAR>();
    if (warp == 0) {
        int w = lane < (NT / 32) ? wsum[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        wsum[lane] = w;  // inclusive warp totals
    }
    attn::block_sync<NT, BAR>();
    total = wsum[(NT / 32) - 1];
    const int before = warp > 0 ? wsum[warp - 1] : 0;
    return before + x - v;
}


template <int NT, int BAR>
struct SampleSmem {
    float red[32];
    int wsum[32];
    unsigned hist[256];
    unsigned sel_prefix, sel_mask;
    int sel_need;
    int surv_idx[kMaxSurvivors];
    float surv_p[kMaxSurvivors];
    int sorted_pos[kMaxSurvivors];
    int n_surv;
    int out_code;
    float all_p[kSampleMaxV];
};

// sample_token (generate_new.rs:771-862) for one row, run by NT threads
// (tid 0..NT-1) that synchronise with block_sync<NT, BAR>.
template <int NT, int BAR>
__device__ __forceinline__ void sample_row(const SampleArgs &a, int row, int tid,
                                           SampleSmem<NT, BAR> &sm) {
    constexpr int PER = (kSampleMaxV + NT - 1) / NT;
    auto &red = sm.red;
    auto &wsum = sm.wsum;
    auto &hist = sm.hist;
    auto &sel_prefix = sm.sel_prefix;
    auto &sel_mask = sm.sel_mask;
    auto &sel_need = sm.sel_need;
    auto &surv_idx = sm.surv_idx;
    auto &surv_p = sm.surv_p;
    auto &sorted_pos = sm.sorted_pos;
    auto &n_surv = sm.n_surv;
    auto &out_code = sm.out_code;
    const int V = a.V;
    const int E = (V + NT - 1) / NT;
    const int i0 = tid * E;
    float s[PER];
#pragma unroll
    for (int e = 0; e < PER; e++) {
        const int i = i0 + e;
        s[e] = (e < E && i < V) ? __ldcg(a.logits + (int64_t)row * a.ldlogits + i) : -INFINITY;
    }
    // repetition penalty (generate_new.rs:775-785)
    if (a.params.repetition_penalty != 1.0f && a.prev) {
        for (int j = 0; j < a.n_prev; j++) {
            const uint32_t pt = __ldcg(a.prev + (int64_t)row * a.ldprev + j);
            if ((int)pt >= i0 && (int)pt < i0 + E && (int)pt < V) {
                const int e = (int)pt - i0;
#pragma unroll
                for (int q = 0; q < PER; q++)
                    if (q == e) s[q] = s[q] > 0.0f ? __fdiv_rn(s[q], a.params.repetition_penalty)
                                                   : __fmul_rn(s[q], a.params.repetition_penalty);
            }
        }
    }
    // temperature (generate_new.rs:788-792)
    const float temp = a.params.temperature;
    if (temp != 1.0f && temp > 0.0f) {
#pragma unroll
        for (int e = 0; e < PER; e++)
            if (e < E && i0 + e < V) s[e] = __fdiv_rn(s[e], temp);
    }
    // softmax (generate_new.rs:795-802)
    float mx = -INFINITY;
#pragma unroll
    for (int e = 0; e < PER; e++) mx = fmaxf(mx, s[e]);
    mx = block_reduce_max<NT, BAR>(mx, red, tid);
    float loc = 0.0f;
#pragma unroll
    for (int e = 0; e < PER; e++) {
        s[e] = (e < E && i0 + e < V) ? expf(s[e] - mx) : 0.0f;
        loc += s[e];
    }
    const float sum = block_reduce_sum<NT, BAR>(loc, red, tid);
#pragma unroll
    for (int e = 0; e < PER; e++) s[e] = __fdiv_rn(s[e], sum);
    if (!(sum > 0.0f) || sum != sum) {
        if (tid == 0) raise_error(a.err, kDevNaN);
    }

    const int top_k = a.params.top_k;
    const bool use_topk = top_k > 0 && top_k < V;
    if (use_topk) {
        // radix select of the top_k-th largest probability (bits are monotone for p >= 0)
        if (tid == 0) {
            sel_prefix = 0u;
            sel_mask = 0u;
            sel_need = top_k;
        }
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int i = tid; i < 256; i += NT) hist[i] = 0u;
            attn::block_sync<NT, BAR>();
            const unsigned pre = sel_prefix, msk = sel_mask;
#pragma unroll
            for (int e = 0; e < PER; e++) {
                if (e < E && i0 + e < V) {
                    const unsigned bits = __float_as_uint(s[e]);
                    if ((bits & msk) == pre) atomicAdd(&hist[(bits >> shift) & 255u], 1u);
                }
            }
            attn::block_sync<NT, BAR>();
            if (tid < 32) {
                // lane l owns bins [248 - 8l .. 255 - 8l] (descending digit order)
                const int lane = tid;
                unsigned cnt[8];
                unsigned tot = 0;
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    cnt[q] = hist[255 - (lane * 8 + q)];
                    tot += cnt[q];
                }
                unsigned incl = tot;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += y;
                }
                unsigned before = incl - tot;
                const unsigned need = (unsigned)sel_need;
                __syncwarp();
                if (before < need && need <= incl) {
                    for (int q = 0; q < 8; q++) {
                        if (before + cnt[q] >= need) {
                            const unsigned digit = 255u - (unsigned)(lane * 8 + q);
                            sel_prefix = pre | (digit << shift);
                            sel_mask = msk | (255u << shift);
                            sel_need = (int)(need - before);
                            break;
                        }
                        before += cnt[q];
                    }
                }
            }
            attn::block_sync<NT, BAR>();
        }
        const unsigned tau = sel_prefix;
        const int need_eq = sel_need;
        int eq_cnt = 0;
#pragma unroll
        for (int e = 0; e < PER; e++)
            if (e < E && i0 + e < V && __float_as_uint(s[e]) == tau) eq_cnt++;
        int eq_total;
        int eq_rank = block_exclusive_scan<NT, BAR>(eq_cnt, wsum, eq_total, tid);
        int keep = 0;
#pragma unroll
        for (int e = 0; e < PER; e++) {
            if (e < E && i0 + e < V) {
                const unsigned bits = __float_as_uint(s[e]);
                bool k = bits > tau;
                if (bits == tau) {
                    k = eq_rank < need_eq;
                    eq_rank++;
                }
                if (!k) s[e] = 0.0f;
                else if (s[e] != 0.0f) keep++;  // zero survivors add nothing
            }
        }
        int total;
        int pos = block_exclusive_scan<NT, BAR>(keep, wsum, total, tid);
#pragma unroll
        for (int e = 0; e < PER; e++) {
            if (e < E && i0 + e < V && s[e] != 0.0f && pos < kMaxSurvivors) {
                surv_idx[pos] = i0 + e;
                surv_p[pos] = s[e];
                pos++;
            }
        }
        if (tid == 0) n_surv = min(total, kMaxSurvivors);
        attn::block_sync<NT, BAR>();
        // renormalise in index order (generate_new.rs:814-819)
        if (tid == 0) {
            float sm = 0.0f;
            for (int i = 0; i < n_surv; i++) sm += surv_p[i];
            red[0] = sm;
        }
        attn::block_sync<NT, BAR>();
        const float sm = red[0];
        if (sm > 0.0f)
            for (int i = tid; i < n_surv; i += NT) surv_p[i] = __fdiv_rn(surv_p[i], sm);
        attn::block_sync<NT, BAR>();
        // top-p over the survivors (generate_new.rs:824-849)
        const float top_p = a.params.top_p;
        if (top_p > 0.0f && top_p < 1.0f) {
            for (int i = tid; i < n_surv; i += NT) {
                const float pi = surv_p[i];
                int rank = 0;
                for (int j = 0; j < n_surv; j++) {
                    const float pj = surv_p[j];
                    rank += (pj > pi) || (pj == pi && j < i);
                }
                sorted_pos[rank] = i;
            }
            attn::block_sync<NT, BAR>();
            if (tid == 0) {
                float cum = 0.0f;
                int cutoff = n_surv;
                for (int rk = 0; rk < n_surv; rk++) {
                    cum += surv_p[sorted_pos[rk]];
                    if (cum >= top_p) {
                        cutoff = rk + 1;
                        break;
                    }
                }
                if (cutoff < 1) cutoff = 1;
                for (int rk = cutoff; rk < n_surv; rk++) surv_p[sorted_pos[rk]] = 0.0f;
                float s2 = 0.0f;
                for (int i = 0; i < n_surv; i++) s2 += surv_p[i];
                if (s2 > 0.0f)
                    for (int i = 0; i < n_surv; i++) surv_p[i] = __fdiv_rn(surv_p[i], s2);
            }
            attn::block_sync<NT, BAR>();
        }
        // draw (generate_new.rs:852-861)
        if (tid == 0) {
            uint64_t st = __ldcg(a.rng + row);
            st ^= st << 13;
            st ^= st >> 7;
            st ^= st << 17;
            a.rng[row] = st;
            const float rr = __fdiv_rn(__ull2float_rn(st), 18446744073709551616.0f);
            float cum = 0.0f;
            int code = 0;
            for (int i = 0; i < n_surv; i++) {
                cum += surv_p[i];
                if (rr < cum) {
                    code = surv_idx[i];
                    break;
                }
            }
            out_code = code;
        }
    } else {
        // no top-k: scan every probability in index order (top-p unsupported here)
        float *all_p = sm.all_p;
#pragma unroll
        for (int e = 0; e < PER; e++)
            if (e < E && i0 + e < V) all_p[i0 + e] = s[e];
        attn::block_sync<NT, BAR>();
        if (tid == 0) {
            uint64_t st = __ldcg(a.rng + row);
            st ^= st << 13;
            st ^= st >> 7;
            st ^= st << 17;
            a.rng[row] = st;
            const float rr = __fdiv_rn(__ull2float_rn(st), 18446744073709551616.0f);
            float cum = 0.0f;
            int code = 0;
            for (int i = 0; i < V; i++) {
                cum += all_p[i];
                if (rr < cum) {
                    code = i;
                    break;
                }
            }
            out_code = code;
        }
    }
    attn::block_sync<NT, BAR>();
    const int code = out_code;
    if (tid == 0) {
        a.out[(int64_t)row * a.ldout] = (uint32_t)code;
        if (a.prev_update) a.prev_update[(int64_t)row * a.ldprev_update] = (uint32_t)code;
    }
    if (a.emb_out) {
        // semantic embedding of the drawn code (talker.rs:152-154)
        const uint8_t *p = a.emb.packed + (int64_t)code * (a.emb.n >> 1);
        const __half *sc = a.emb.scl + (int64_t)code * (a.emb.n >> 5);
        for (int64_t j = tid; j < a.emb.n; j += NT) {
            const uint8_t byte = p[j >> 1];
            const int q = (j & 1) ? (byte >> 4) : (byte & 15);
            a.emb_out[(int64_t)row * a.ldemb_out + j] = __fmul_rn(__half2float(sc[j >> 5]), (float)(q - 8));
        }
    }
}

}  // namespace samp
}  // namespace qora
