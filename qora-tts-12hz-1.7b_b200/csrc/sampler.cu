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
#include "sampler_impl.cuh"

namespace qora {

namespace {

constexpr int kSampleThreads = 1024;
constexpr int kMaxPerThread = samp::kSampleMaxV / kSampleThreads;

__global__ void __launch_bounds__(kSampleThreads) k_sample(SampleArgs a) {
    __shared__ samp::SampleSmem<kSampleThreads, 0> sm;
    griddep_launch_dependents();
    griddep_wait();
    samp::sample_row<kSampleThreads, 0>(a, blockIdx.x, threadIdx.x, sm);
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
