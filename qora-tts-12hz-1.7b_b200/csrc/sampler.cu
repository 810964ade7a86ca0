// Device sampler and frame-input assembly (sm_100a).
//
// k_sample restates sample_token (generate_new.rs:771-862) for one row per
// CTA: repetition penalty over the previous codes (divide if > 0, else
// multiply; repeated ids apply repeatedly), temperature, softmax, top-k
// (the first k of a stable descending sort, i.e. ties keep index order),
// renormalisation, optional top-p, then the xorshift64 draw of simple_rand
// (generate_new.rs:17-22) and a cumulative scan in index order.
// The top-k threshold is found by a 4-pass radix select on the probability
// bits instead of a sort; survivor sums and the final scan run sequentially
// in index order, as in the reference.
//
// k_frame_embed restates the frame-input assembly (generate_new.rs:639-654,
// code_predictor.rs:287-300): emb = (E_talker[c0] + sum_g E_g[c_g]) + text.
#include "sampler.cuh"

namespace qora {

namespace {

constexpr int kSampleThreads = 1024;
constexpr int kMaxPerThread = 4;   // V <= 4096

__device__ __forceinline__ float block_reduce_max(float v, float *red) {
    v = warp_max(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float x = lane < (int)(blockDim.x >> 5) ? red[lane] : -INFINITY;
        x = warp_max(x);
        if (lane == 0) red[0] = x;
    }
    __syncthreads();
    return red[0];
}

__device__ __forceinline__ float block_reduce_sum(float v, float *red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float x = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
        x = warp_sum(x);
        if (lane == 0) red[0] = x;
    }
    __syncthreads();
    return red[0];
}

// Exclusive prefix sum of one int per thread over the block (index order).
__device__ __forceinline__ int block_exclusive_scan(int v, int *wsum, int &total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < (int)(blockDim.x >> 5) ? wsum[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        wsum[lane] = w;  // inclusive warp totals
    }
    __syncthreads();
    total = wsum[(blockDim.x >> 5) - 1];
    const int before = warp > 0 ? wsum[warp - 1] : 0;
    return before + x - v;
}

__global__ void __launch_bounds__(kSampleThreads) k_sample(SampleArgs a) {
    __shared__ float red[32];
    __shared__ int wsum[32];
    __shared__ unsigned hist[256];
    __shared__ unsigned sel_prefix, sel_mask;
    __shared__ int sel_need;
    __shared__ int surv_idx[kMaxSurvivors];
    __shared__ float surv_p[kMaxSurvivors];
    __shared__ int sorted_pos[kMaxSurvivors];
    __shared__ int n_surv;
    __shared__ int out_code;

    griddep_launch_dependents();
    griddep_wait();
    const int row = blockIdx.x;
    const int V = a.V;
    const int E = (V + kSampleThreads - 1) / kSampleThreads;
    const int i0 = threadIdx.x * E;
    float s[kMaxPerThread];
#pragma unroll
    for (int e = 0; e < kMaxPerThread; e++) {
        const int i = i0 + e;
        s[e] = (e < E && i < V) ? a.logits[(int64_t)row * a.ldlogits + i] : -INFINITY;
    }
    // repetition penalty (generate_new.rs:775-785)
    if (a.params.repetition_penalty != 1.0f && a.prev) {
        for (int j = 0; j < a.n_prev; j++) {
            const uint32_t pt = a.prev[(int64_t)row * a.ldprev + j];
            if ((int)pt >= i0 && (int)pt < i0 + E && (int)pt < V) {
                const int e = (int)pt - i0;
#pragma unroll
                for (int q = 0; q < kMaxPerThread; q++)
                    if (q == e) s[q] = s[q] > 0.0f ? __fdiv_rn(s[q], a.params.repetition_penalty)
                                                   : __fmul_rn(s[q], a.params.repetition_penalty);
            }
        }
    }
    // temperature (generate_new.rs:788-792)
    const float temp = a.params.temperature;
    if (temp != 1.0f && temp > 0.0f) {
#pragma unroll
        for (int e = 0; e < kMaxPerThread; e++)
            if (e < E && i0 + e < V) s[e] = __fdiv_rn(s[e], temp);
    }
    // softmax (generate_new.rs:795-802)
    float mx = -INFINITY;
#pragma unroll
    for (int e = 0; e < kMaxPerThread; e++) mx = fmaxf(mx, s[e]);
    mx = block_reduce_max(mx, red);
    float loc = 0.0f;
#pragma unroll
    for (int e = 0; e < kMaxPerThread; e++) {
        s[e] = (e < E && i0 + e < V) ? expf(s[e] - mx) : 0.0f;
        loc += s[e];
    }
    const float sum = block_reduce_sum(loc, red);
#pragma unroll
    for (int e = 0; e < kMaxPerThread; e++) s[e] = __fdiv_rn(s[e], sum);
    if (!(sum > 0.0f) || sum != sum) {
        if (threadIdx.x == 0) raise_error(a.err, kDevNaN);
    }

    const int top_k = a.params.top_k;
    const bool use_topk = top_k > 0 && top_k < V;
    if (use_topk) {
        // radix select of the top_k-th largest probability (bits are monotone for p >= 0)
        if (threadIdx.x == 0) {
            sel_prefix = 0u;
            sel_mask = 0u;
            sel_need = top_k;
        }
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0u;
            __syncthreads();
            const unsigned pre = sel_prefix, msk = sel_mask;
#pragma unroll
            for (int e = 0; e < kMaxPerThread; e++) {
                if (e < E && i0 + e < V) {
                    const unsigned bits = __float_as_uint(s[e]);
                    if ((bits & msk) == pre) atomicAdd(&hist[(bits >> shift) & 255u], 1u);
                }
            }
            __syncthreads();
            if (threadIdx.x < 32) {
                // lane l owns bins [248 - 8l .. 255 - 8l] (descending digit order)
                const int lane = threadIdx.x;
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
            __syncthreads();
        }
        const unsigned tau = sel_prefix;
        const int need_eq = sel_need;
        int eq_cnt = 0;
#pragma unroll
        for (int e = 0; e < kMaxPerThread; e++)
            if (e < E && i0 + e < V && __float_as_uint(s[e]) == tau) eq_cnt++;
        int eq_total;
        int eq_rank = block_exclusive_scan(eq_cnt, wsum, eq_total);
        int keep = 0;
#pragma unroll
        for (int e = 0; e < kMaxPerThread; e++) {
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
        int pos = block_exclusive_scan(keep, wsum, total);
#pragma unroll
        for (int e = 0; e < kMaxPerThread; e++) {
            if (e < E && i0 + e < V && s[e] != 0.0f && pos < kMaxSurvivors) {
                surv_idx[pos] = i0 + e;
                surv_p[pos] = s[e];
                pos++;
            }
        }
        if (threadIdx.x == 0) n_surv = min(total, kMaxSurvivors);
        __syncthreads();
        // renormalise in index order (generate_new.rs:814-819)
        if (threadIdx.x == 0) {
            float sm = 0.0f;
            for (int i = 0; i < n_surv; i++) sm += surv_p[i];
            red[0] = sm;
        }
        __syncthreads();
        const float sm = red[0];
        if (sm > 0.0f)
            for (int i = threadIdx.x; i < n_surv; i += blockDim.x) surv_p[i] = __fdiv_rn(surv_p[i], sm);
        __syncthreads();
        // top-p over the survivors (generate_new.rs:824-849)
        const float top_p = a.params.top_p;
        if (top_p > 0.0f && top_p < 1.0f) {
            for (int i = threadIdx.x; i < n_surv; i += blockDim.x) {
                const float pi = surv_p[i];
                int rank = 0;
                for (int j = 0; j < n_surv; j++) {
                    const float pj = surv_p[j];
                    rank += (pj > pi) || (pj == pi && j < i);
                }
                sorted_pos[rank] = i;
            }
            __syncthreads();
            if (threadIdx.x == 0) {
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
            __syncthreads();
        }
        // draw (generate_new.rs:852-861)
        if (threadIdx.x == 0) {
            uint64_t st = a.rng[row];
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
        __shared__ float all_p[kMaxPerThread * kSampleThreads];
#pragma unroll
        for (int e = 0; e < kMaxPerThread; e++)
            if (e < E && i0 + e < V) all_p[i0 + e] = s[e];
        __syncthreads();
        if (threadIdx.x == 0) {
            uint64_t st = a.rng[row];
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
    __syncthreads();
    const int code = out_code;
    if (threadIdx.x == 0) {
        a.out[(int64_t)row * a.ldout] = (uint32_t)code;
        if (a.prev_update) a.prev_update[(int64_t)row * a.ldprev_update] = (uint32_t)code;
    }
    if (a.emb_out) {
        // semantic embedding of the drawn code (talker.rs:152-154)
        const uint8_t *p = a.emb.packed + (int64_t)code * (a.emb.n >> 1);
        const __half *sc = a.emb.scl + (int64_t)code * (a.emb.n >> 5);
        for (int64_t j = threadIdx.x; j < a.emb.n; j += blockDim.x) {
            const uint8_t byte = p[j >> 1];
            const int q = (j & 1) ? (byte >> 4) : (byte & 15);
            a.emb_out[(int64_t)row * a.ldemb_out + j] = __fmul_rn(__half2float(sc[j >> 5]), (float)(q - 8));
        }
    }
}

__global__ void k_frame_embed(FrameEmbedArgs a) {
    griddep_launch_dependents();
    griddep_wait();
    const int r = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int64_t n = a.n;
    for (int64_t g = warp; g * 32 < n; g += nw) {
        const int64_t j = g * 32 + lane;
        float acc = 0.0f;
        if (j < n) {
            for (int q = 0; q < a.ngroups; q++) {
                const uint32_t code = a.codes[(int64_t)r * a.ldcodes + a.code_off + q];
                const EmbDev &e = a.tables[q];
                const uint8_t byte = e.packed[(int64_t)code * (n >> 1) + (j >> 1)];
                const int qq = (j & 1) ? (byte >> 4) : (byte & 15);
                acc = __fadd_rn(acc, __fmul_rn(__half2float(e.scl[(int64_t)code * (n >> 5) + (j >> 5)]),
                                               (float)(qq - 8)));
            }
            if (a.sem) acc = __fadd_rn(a.sem[(int64_t)r * a.ldsem + j], acc);
            if (a.text) acc = __fadd_rn(acc, a.text[(int64_t)r * a.ldtext + j]);
            a.out[(int64_t)r * a.ldout + j] = acc;
        }
        if (a.ss) {
            const float sq = warp_sum(j < n ? __fmul_rn(acc, acc) : 0.0f);
            if (lane == 0) a.ss[(int64_t)r * a.ldss + g] = sq;
        }
    }
    if (a.prev && threadIdx.x < a.ngroups)
        a.prev[(int64_t)r * a.ldprev + 1 + threadIdx.x] =
            a.codes[(int64_t)r * a.ldcodes + a.code_off + threadIdx.x];
}

}  // namespace

int launch_sample(const SampleArgs &a, int rows, cudaStream_t st) {
    if (rows <= 0) return QORA_OK;
    if (a.V <= 0 || a.V > kMaxPerThread * kSampleThreads)
        return set_error(QORA_ERR_UNSUPPORTED, "sampler vocab %d (max %d)", a.V,
                         kMaxPerThread * kSampleThreads);
    const bool topk = a.params.top_k > 0 && a.params.top_k < a.V;
    if (topk && a.params.top_k > kMaxSurvivors)
        return set_error(QORA_ERR_UNSUPPORTED, "top_k %d > %d", a.params.top_k, kMaxSurvivors);
    if (!topk && a.params.top_p > 0.0f && a.params.top_p < 1.0f)
        return set_error(QORA_ERR_UNSUPPORTED, "top_p needs 0 < top_k <= %d", kMaxSurvivors);
    return launch_ex(k_sample, dim3(rows), dim3(kSampleThreads), 0, st, 1u, a);
}

int launch_frame_embed(const FrameEmbedArgs &a, int rows, cudaStream_t st) {
    if (rows <= 0) return QORA_OK;
    if (a.ngroups > kMaxEmbedGroups) return set_error(QORA_ERR_INVALID, "too many groups");
    return launch_ex(k_frame_embed, dim3(rows), dim3(256), 0, st, 1u, a);
}

}  // namespace qora
