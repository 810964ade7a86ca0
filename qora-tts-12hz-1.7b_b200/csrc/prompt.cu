// Prompt assembly on the device: the talker's prefill rows of
// generate_new.rs:91-466 (role prefix, codec header with the TTS pad / BOS
// overlay or the voice row, ICL block and prefix, first-text row) and the
// trailing text rows of the frame loop, built from rows of the text
// projection and the codec / acoustic embedding tables already on the device.
//
// Every row is text + codec with either part optional (the reference's
// add_embed and the `combined[j] = a[j] + b[j]` loops; f32 addition commutes,
// so the operand order of those loops does not change a bit).  The codec part
// of a reference-frame row sums its 16 embeddings in the reference's order,
// codec(c0) + acoustic_0(c1) + ... + acoustic_14(c15) (generate_new.rs:164-169).
// One CTA builds one row; recipes travel in the launch parameters.
#include <algorithm>

#include "common.cuh"
#include "model.cuh"

namespace qora {
namespace {

constexpr int kPromptRowsPerLaunch = 40;  // recipes per launch (parameter space < 4 KB)

struct PromptArgs {
    EmbDev tables[16];  // [0] talker codec embedding, [1 + g] predictor acoustic group g
    const float *text = nullptr;
    int64_t ldtext = 0;
    const float *voice = nullptr;
    int voice_len = 0;
    int n = 0;          // row width (talker hidden)
    float *out = nullptr;
    int count = 0;
    qora_prompt_row rows[kPromptRowsPerLaunch];
};
static_assert(sizeof(PromptArgs) <= 4000, "kernel parameters must stay under 4 KB");

// embed_lookup_q4 (gemv.rs:425-433): scale * (q - 8), one element
__device__ __forceinline__ float emb_at(const EmbDev &e, uint32_t row, int j) {
    const uint8_t b = e.packed[(int64_t)row * (e.n >> 1) + (j >> 1)];
    const int q = (j & 1) ? (b >> 4) : (b & 15);
    return __fmul_rn(__half2float(e.scl[(int64_t)row * (e.n >> 5) + (j >> 5)]), (float)(q - 8));
}

__global__ void k_prompt_rows(const __grid_constant__ PromptArgs a) {
    const qora_prompt_row &r = a.rows[blockIdx.x];
    const float *text = r.text >= 0 ? a.text + (int64_t)r.text * a.ldtext : nullptr;
    float *out = a.out + (int64_t)blockIdx.x * a.n;
    for (int j = threadIdx.x; j < a.n; j += blockDim.x) {
        float v;
        if (r.codes_n < 0) {  // voice row: voice + text over the voice's length, zeros after
            v = j < a.voice_len ? (text ? __fadd_rn(a.voice[j], text[j]) : a.voice[j]) : 0.0f;
        } else if (r.codes_n == 0) {
            v = text ? text[j] : 0.0f;
        } else {
            float c = emb_at(a.tables[0], r.codes[0], j);
            for (int g = 1; g < r.codes_n; g++) c = __fadd_rn(c, emb_at(a.tables[g], r.codes[g], j));
            v = text ? __fadd_rn(text[j], c) : c;
        }
        out[j] = v;
    }
}

}  // namespace
}  // namespace qora

using namespace qora;

extern "C" int qora_prompt_assemble(qora_talker *t, qora_predictor *p, const float *text_rows,
                                    int32_t n_text, const float *voice, int32_t voice_len,
                                    const qora_prompt_row *rows, int32_t count, float *out,
                                    void *stream) {
    if (!t || count < 0 || (count > 0 && (!rows || !out)) || n_text < 0 || voice_len < 0)
        return set_error(QORA_ERR_INVALID, "qora_prompt_assemble: bad arguments");
    const int max_codes = p ? 1 + p->groups : 1;
    if (p && p->Ht != t->H)
        return set_error(QORA_ERR_SHAPE, "qora_prompt_assemble: predictor embeddings are %lld wide, talker %d",
                         (long long)p->Ht, t->H);
    for (int32_t i = 0; i < count; i++) {
        const qora_prompt_row &r = rows[i];
        if (r.text >= n_text || r.text < -1 || (r.text >= 0 && !text_rows))
            return set_error(QORA_ERR_RANGE, "prompt row %d: text row %d of %d", i, r.text, n_text);
        if (r.codes_n < -1 || r.codes_n > max_codes)
            return set_error(QORA_ERR_INVALID, "prompt row %d: %d codes (at most %d%s)", i, r.codes_n,
                             max_codes, p ? "" : " without a predictor");
        if (r.codes_n < 0 && !voice)
            return set_error(QORA_ERR_INVALID, "prompt row %d: voice row without a voice embedding", i);
        if (r.codes_n >= 1 && (int64_t)r.codes[0] >= t->codec_emb.rows)
            return set_error(QORA_ERR_RANGE, "prompt row %d: codec token %u of %lld", i, r.codes[0],
                             (long long)t->codec_emb.rows);
        for (int g = 1; g < r.codes_n; g++)
            if ((int64_t)r.codes[g] >= p->embs[(size_t)g - 1].rows)
                return set_error(QORA_ERR_RANGE, "prompt row %d: group %d code %u of %lld", i, g, r.codes[g],
                                 (long long)p->embs[(size_t)g - 1].rows);
    }
    PromptArgs a;
    a.tables[0] = t->codec_emb;
    if (p)
        for (int g = 0; g < p->groups; g++) a.tables[1 + g] = p->embs[(size_t)g];
    a.text = text_rows;
    a.ldtext = t->H;
    a.voice = voice;
    a.voice_len = std::min<int32_t>(voice_len, t->H);  // generate_new.rs:215, :405
    a.n = t->H;
    cudaStream_t st = as_stream(stream);
    for (int32_t c0 = 0; c0 < count; c0 += kPromptRowsPerLaunch) {
        a.count = std::min<int32_t>(kPromptRowsPerLaunch, count - c0);
        std::copy(rows + c0, rows + c0 + a.count, a.rows);
        a.out = out + (int64_t)c0 * t->H;
        k_prompt_rows<<<a.count, 256, 0, st>>>(a);
        QORA_CUDA(cudaGetLastError());
    }
    return QORA_OK;
}
