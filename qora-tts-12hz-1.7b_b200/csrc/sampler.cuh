// Device sampler and frame-input assembly.
#pragma once

#include "common.cuh"

namespace qora {

constexpr int kMaxSurvivors = 1024;  // top_k limit of the device sampler
constexpr int kMaxEmbedGroups = 16;

struct SampleArgs {
    const float *logits = nullptr;
    int64_t ldlogits = 0;
    int V = 0;
    const uint32_t *prev = nullptr;  // [rows][ldprev], first n_prev used
    int64_t ldprev = 0;
    int n_prev = 0;
    uint64_t *rng = nullptr;         // [rows] xorshift64 state, in/out
    qora_sample_params params{};
    uint32_t *out = nullptr;
    int64_t ldout = 1;
    uint32_t *prev_update = nullptr; // optional: also store the code here
    int64_t ldprev_update = 0;
    EmbDev emb;                      // optional: write emb row of the code
    float *emb_out = nullptr;
    int64_t ldemb_out = 0;
    int *err = nullptr;
};

struct FrameEmbedArgs {
    int64_t n = 0;                  // embedding width
    EmbDev tables[kMaxEmbedGroups]; // acoustic tables, group order
    int ngroups = 0;
    const uint32_t *codes = nullptr;
    int64_t ldcodes = 0;
    int code_off = 0;               // codes[r][code_off + g] is group g's code
    const float *sem = nullptr;     // optional semantic row (added first)
    int64_t ldsem = 0;
    const float *text = nullptr;    // optional text row (added last)
    int64_t ldtext = 0;
    float *out = nullptr;
    int64_t ldout = 0;
    float *ss = nullptr;            // optional per-32-column sum of squares
    int64_t ldss = 0;
    uint32_t *prev = nullptr;       // optional: prev[r][1 + g] = group g's code
    int64_t ldprev = 0;
};

int launch_sample(const SampleArgs &a, int rows, cudaStream_t st);
int launch_frame_embed(const FrameEmbedArgs &a, int rows, cudaStream_t st);

}  // namespace qora
