// Device-side model objects (talker, code predictor, frame engine) shared by
// the per-op host orchestration (model.cu) and the persistent frame kernel
// (frame.cu).
#pragma once

#include <vector>

#include "attention.cuh"
#include "gemv.cuh"
#include "kv.cuh"
#include "sampler.cuh"

namespace qora {

// One decoder layer's device weights: fused [q|k|v], o, interleaved gate/up
// (g0 u0 g1 u1 ...), down, and the f16 norm vectors.
struct LayerDev {
    DevBuf qkv_nib, qkv_scl, o_nib, o_scl, gu_nib, gu_scl, dn_nib, dn_scl;
    Q4Dev qkv, o, gu, dn;
    DevBuf q_norm, k_norm, in_norm, post_norm;

    int upload(const qora_layer_host &h, int64_t hidden, int heads, int kvh, int hd, int64_t ffn);
};

// Activation and scratch buffers sized for `rows` rows.
struct Work {
    DevBuf x, ss, qkv, attn, h, logits, gticket, tbest_v, tbest_i, apo, apml, atk, rexp, rinv, bop;
    int rows = 0;

    GemmScratch gemm_scratch() {
        GemmScratch s;
        s.rexp = rexp.as<int>();
        s.rinv = rinv.as<float>();
        s.bop = bop.as<uint8_t>();
        s.rows = rows;
        s.bop_bytes = bop.bytes;
        return s;
    }

    int alloc(int rows_, int64_t hidden, int64_t qkvn, int64_t qd, int64_t ffn, int64_t vocab,
              int kvh, int heads, int hd) {
        rows = rows_;
        QORA_TRY(x.alloc((size_t)rows * hidden * 4));
        QORA_TRY(ss.alloc((size_t)rows * (hidden / kGroup) * 4));
        QORA_TRY(qkv.alloc((size_t)rows * qkvn * 4));
        QORA_TRY(attn.alloc((size_t)rows * qd * 4));
        QORA_TRY(h.alloc((size_t)rows * ffn * 4));
        QORA_TRY(logits.alloc((size_t)rows * vocab * 4));
        QORA_TRY(gticket.alloc(64));
        QORA_TRY(gticket.zero());
        QORA_TRY(tbest_v.alloc((size_t)rows * (vocab / kGroup + 1) * 4));
        QORA_TRY(tbest_i.alloc((size_t)rows * (vocab / kGroup + 1) * 4));
        QORA_TRY(apo.alloc(attn_part_o_floats(rows, kvh, heads, hd) * 4));
        QORA_TRY(apml.alloc(attn_part_ml_floats(rows, kvh, heads) * 4));
        QORA_TRY(atk.alloc((size_t)rows * kvh * 4));
        QORA_TRY(atk.zero());
        QORA_TRY(rexp.alloc((size_t)rows * 4));
        QORA_TRY(rinv.alloc((size_t)rows * 4));
        // prefill GEMM B tiles: rows rounded up to 128, the widest K (hidden, qd or ffn)
        const int64_t kmax = std::max<int64_t>(hidden, std::max<int64_t>(qd, ffn));
        QORA_TRY(bop.alloc((size_t)((rows + 127) / 128) * 128 * kmax * 4));
        QORA_CUDA(cudaDeviceSynchronize());
        return QORA_OK;
    }
};

struct FrameProgram;  // persistent frame kernel state (frame.cu)
void frame_program_destroy(FrameProgram *p);
void frame_program_set_temperature(FrameProgram *p, float temperature);
int64_t text_proj_hidden(const qora_text_proj *tp);  // output width (text_proj.cu)

}  // namespace qora

struct qora_talker {
    qora::CtxRef ctx;
    int L = 0, H = 0, heads = 0, kvh = 0, hd = 0, ffn = 0, vocab = 0, rope_max = 0;
    std::vector<qora::LayerDev> layers;
    qora::DevBuf ce_packed, ce_scl, head_nib, head_scl, final_norm, rope_cos, rope_sin;
    qora::EmbDev codec_emb;
    qora::Q4Dev head;
    int max_batch = 0;
    qora::Work w;
    qora::DevBuf emb_in, tok_in;  // qora_talker_decode: [max_batch][H] input rows, their tokens

    int64_t qd() const { return (int64_t)heads * hd; }
    int64_t kd() const { return (int64_t)kvh * hd; }
    int64_t qkvn() const { return qd() + 2 * kd(); }
};

struct qora_predictor {
    qora::CtxRef ctx;
    int L = 0, H = 0, heads = 0, kvh = 0, hd = 0, ffn = 0, vocab = 0, groups = 0, rope_max = 0;
    int64_t Ht = 0;  // talker hidden (input / embedding width)
    std::vector<qora::LayerDev> layers;
    bool has_proj = false;
    qora::DevBuf proj_nib, proj_scl, proj_bias, final_norm, rope_cos, rope_sin;
    qora::Q4Dev proj;
    std::vector<qora::DevBuf> emb_packed, emb_scl, head_nib, head_scl;
    std::vector<qora::EmbDev> embs;
    std::vector<qora::Q4Dev> heads_w;
    int max_batch = 0;
    qora::Work w;
    qora::DevBuf x2;     // [rows][2][Ht]: talker hidden | semantic embedding
    qora::DevBuf codes;  // [rows][groups] internal code buffer
    qora::DevBuf xe;     // identity-projection staging [rows][Ht]
};

struct qora_engine {
    qora_talker *t = nullptr;
    qora_predictor *p = nullptr;
    int B = 0, max_pos = 0;
    qora_sample_params params{};
    qora_kv *tkv = nullptr, *pkv = nullptr;
    qora::DevBuf logits, codes, prev, rng, pos, text;
    bool use_graph = false;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    const float *graph_text = nullptr;
    uint32_t *graph_codes = nullptr;
    int kernels = qora::kEngineKernelsUnknown;
    cudaStream_t cap_stream = nullptr;
    bool persistent = true;              // run frames on the persistent frame kernel when supported
    qora::FrameProgram *frame = nullptr; // built on the first persistent frame
};
