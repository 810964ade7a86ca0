// Reader of the reference's single-file checkpoint (.qora-tts, save.rs:262-409,
// record helpers gemv.rs:595-687), for callers that load weights without the
// reference's Rust loader.
//
// Layout (little endian): "QTTS", u32 version (1), u8 format (1 = Q4, 0 = f16),
// then the talker section (save.rs:300-351, with the text embedding and text
// projection the prompt is built from), the code-predictor section
// (save.rs:353-438) and the speech decoder (save.rs:171-262), read on demand
// by qora_model_file_decoder.  Arrays are u64 element counts followed by the
// elements; a weight is u64 k, u64 n, then (Q4) the packed bytes and the f16
// scales.
//
// The file is mapped read-only: packed nibbles (the bulk of the file) are
// used in place; f16 / f32 arrays, which can sit at odd offsets, are copied
// into aligned buffers.  The RoPE base is not stored, only its f32 tables: it
// is recovered from the slowest-turning column, rounded to an integer and
// accepted only if the tables rebuilt from it equal the file's bit for bit.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>
#include <deque>
#include <string>
#include <utility>
#include <vector>

#include "common.cuh"
#include "sampler.cuh"

namespace qora {
int host_rope_tables(int32_t head_dim, int32_t max_pos, double theta, const int32_t *sections,
                     int32_t n_sections, float *cos_host, float *sin_host);
}

struct qora_model_file {
    void *map = nullptr;
    size_t size = 0;
    std::deque<std::vector<uint16_t>> u16;  // aligned copies (stable addresses)
    std::deque<std::vector<float>> f32;
    std::vector<qora_layer_host> t_layers, p_layers;
    std::vector<qora_q4_host> p_embs, p_heads;
    qora_talker_host talker{};
    qora_predictor_host predictor{};
    qora_text_proj_host text{};
    size_t dec_off = 0;   // where the speech-decoder section starts
};

namespace {

using namespace qora;

struct Cursor {
    const uint8_t *p, *end;
    const char *what = "";
    bool ok = true;

    bool need(uint64_t n) {
        if (!ok || n > (uint64_t)(end - p)) ok = false;
        return ok;
    }
    uint64_t u(int bytes) {
        uint64_t v = 0;
        if (!need((uint64_t)bytes)) return 0;
        for (int i = 0; i < bytes; i++) v |= (uint64_t)p[i] << (8 * i);
        p += bytes;
        return v;
    }
    const uint8_t *bytes(uint64_t n) {
        if (!need(n)) return nullptr;
        const uint8_t *r = p;
        p += n;
        return r;
    }
};

// u64 count + f16 elements, copied into an aligned buffer; expect < 0: any count
const uint16_t *read_f16(Cursor &c, qora_model_file *f, int64_t expect, int64_t *count = nullptr) {
    const uint64_t n = c.u(8);
    if (n > (1ull << 40) || (expect >= 0 && n != (uint64_t)expect)) c.ok = false;
    const uint8_t *b = c.bytes(n * 2);
    if (!c.ok) return nullptr;
    f->u16.emplace_back(n);
    if (n) std::memcpy(f->u16.back().data(), b, n * 2);
    if (count) *count = (int64_t)n;
    return f->u16.back().data();
}

const float *read_f32(Cursor &c, qora_model_file *f, int64_t expect, int64_t *count = nullptr) {
    const uint64_t n = c.u(8);
    if (n > (1ull << 40) || (expect >= 0 && n != (uint64_t)expect)) c.ok = false;
    const uint8_t *b = c.bytes(n * 4);
    if (!c.ok) return nullptr;
    f->f32.emplace_back(n);
    if (n) std::memcpy(f->f32.back().data(), b, n * 4);
    if (count) *count = (int64_t)n;
    return f->f32.back().data();
}

// write_weight_io / read_weight_io (gemv.rs:595-610, 672-687), Q4 format
qora_q4_host read_q4(Cursor &c, qora_model_file *f) {
    qora_q4_host w{};
    const uint64_t k = c.u(8), n = c.u(8);
    if (!c.ok || k == 0 || n == 0 || n % kGroup != 0 || k > (1u << 24) || n > (1u << 24)) {
        c.ok = false;
        return w;
    }
    const uint64_t nb = c.u(8);
    if (nb != k * n / 2) c.ok = false;
    w.packed = c.bytes(nb);
    w.scales = read_f16(c, f, (int64_t)(k * (n / kGroup)));
    w.k = (int64_t)k;
    w.n = (int64_t)n;
    return w;
}

qora_layer_host read_layer(Cursor &c, qora_model_file *f, int hidden, int hd) {
    qora_layer_host l{};
    l.q_proj = read_q4(c, f);
    l.k_proj = read_q4(c, f);
    l.v_proj = read_q4(c, f);
    l.o_proj = read_q4(c, f);
    l.q_norm = read_f16(c, f, hd);
    l.k_norm = read_f16(c, f, hd);
    l.gate_proj = read_q4(c, f);
    l.up_proj = read_q4(c, f);
    l.down_proj = read_q4(c, f);
    l.input_norm = read_f16(c, f, hidden);
    l.post_attn_norm = read_f16(c, f, hidden);
    return l;
}

// The RoPE base behind f32 tables cos/sin[max_pos][hd/2] (rope.rs:11-41): from
// column hd/2 - 1 at position 1 (angle = theta^(-(hd-2)/hd), far from any
// wrap), rounded to an integer, and kept only if the rebuilt tables match.
int recover_theta(const float *cs, const float *sn, int hd, int max_pos, double *theta_out) {
    const int half = hd / 2;
    if (max_pos < 2 || half < 2) return set_error(QORA_ERR_INVALID, "model file: RoPE tables too small");
    const double ang = std::atan2((double)sn[half + half - 1], (double)cs[half + half - 1]);
    if (!(ang > 0.0)) return set_error(QORA_ERR_INVALID, "model file: RoPE tables do not rotate");
    const double theta = std::round(std::pow(ang, -(double)hd / (double)(hd - 2)));
    std::vector<float> c2((size_t)max_pos * half), s2((size_t)max_pos * half);
    // (the sectioning of build_mrope_tables does not change the tables: a
    // dimension's frequency depends on its index only)
    const int32_t one = half;
    QORA_TRY(host_rope_tables(hd, max_pos, theta, &one, 1, c2.data(), s2.data()));
    if (std::memcmp(c2.data(), cs, c2.size() * 4) != 0 || std::memcmp(s2.data(), sn, s2.size() * 4) != 0)
        return set_error(QORA_ERR_UNSUPPORTED,
                         "model file: RoPE tables are not those of an integer base (best fit %.1f)", theta);
    *theta_out = theta;
    return QORA_OK;
}

int parse(qora_model_file *f) {
    Cursor c{static_cast<const uint8_t *>(f->map), static_cast<const uint8_t *>(f->map) + f->size};
    const uint8_t *magic = c.bytes(4);
    if (!magic || std::memcmp(magic, "QTTS", 4) != 0)
        return set_error(QORA_ERR_INVALID, "model file: not a .qora-tts file (magic)");
    const uint64_t version = c.u(4);
    if (version != 1) return set_error(QORA_ERR_UNSUPPORTED, "model file: version %llu (expected 1)",
                                       (unsigned long long)version);
    const uint64_t fmt = c.u(1);
    if (fmt != 1)
        return set_error(QORA_ERR_UNSUPPORTED,
                         "model file: format %llu (only Q4 checkpoints, format 1, run on this engine)",
                         (unsigned long long)fmt);

    // ---- talker (save.rs:300-351)
    qora_talker_host &t = f->talker;
    t.num_layers = (int32_t)c.u(4);
    t.hidden = (int32_t)c.u(4);
    const uint64_t text_hidden = c.u(4);
    t.num_heads = (int32_t)c.u(4);
    t.num_kv_heads = (int32_t)c.u(4);
    t.head_dim = (int32_t)c.u(4);
    c.u(4);  // num_kv_groups
    const uint64_t nsec = c.u(4);
    if (!c.ok || nsec > 8 || t.num_layers <= 0 || t.num_layers > 1024 || t.hidden <= 0 ||
        t.head_dim <= 0 || t.head_dim % 2 || t.num_heads <= 0 || t.num_kv_heads <= 0)
        return set_error(QORA_ERR_INVALID, "model file: bad talker header");
    for (uint64_t i = 0; i < nsec; i++) c.u(4);  // mrope_section (position ids are (p, p, p))
    f->t_layers.resize((size_t)t.num_layers);
    for (int i = 0; i < t.num_layers && c.ok; i++) f->t_layers[(size_t)i] = read_layer(c, f, t.hidden, t.head_dim);
    t.codec_embedding = read_q4(c, f);
    qora_text_proj_host &x = f->text;
    x.text_embedding = read_q4(c, f);
    x.fc1 = read_q4(c, f);
    x.fc1_bias = read_f32(c, f, x.fc1.n);
    x.fc2 = read_q4(c, f);
    x.fc2_bias = read_f32(c, f, x.fc2.n);
    if (c.ok && ((uint64_t)x.text_embedding.n != text_hidden || x.fc1.k != x.text_embedding.n ||
                 x.fc2.k != x.fc1.n || x.fc2.n != t.hidden))
        return set_error(QORA_ERR_INVALID, "model file: text projection shapes do not chain");
    t.codec_head = read_q4(c, f);
    t.final_norm = read_f16(c, f, t.hidden);
    int64_t tc = 0, ts = 0;
    const float *t_cos = read_f32(c, f, -1, &tc);
    const float *t_sin = read_f32(c, f, -1, &ts);
    if (!c.ok) return set_error(QORA_ERR_INVALID, "model file: truncated or malformed talker section");
    t.layers = f->t_layers.data();
    t.ffn = (int32_t)f->t_layers[0].gate_proj.n;
    t.vocab = (int32_t)t.codec_head.n;
    if (tc != ts || tc % (t.head_dim / 2) != 0)
        return set_error(QORA_ERR_INVALID, "model file: talker RoPE tables");
    t.rope_max_pos = (int32_t)(tc / (t.head_dim / 2));
    QORA_TRY(recover_theta(t_cos, t_sin, t.head_dim, t.rope_max_pos, &t.rope_theta));

    // ---- code predictor (save.rs:353-438)
    qora_predictor_host &p = f->predictor;
    p.num_layers = (int32_t)c.u(4);
    p.hidden = (int32_t)c.u(4);
    p.num_heads = (int32_t)c.u(4);
    p.num_kv_heads = (int32_t)c.u(4);
    p.head_dim = (int32_t)c.u(4);
    c.u(4);  // num_kv_groups
    if (!c.ok || p.num_layers <= 0 || p.num_layers > 1024 || p.hidden <= 0 || p.head_dim <= 0 ||
        p.head_dim % 2 || p.num_heads <= 0 || p.num_kv_heads <= 0)
        return set_error(QORA_ERR_INVALID, "model file: bad code-predictor header");
    const uint64_t has_proj = c.u(1);
    if (has_proj == 1) {
        p.input_proj = read_q4(c, f);
        p.input_proj_bias = read_f32(c, f, p.input_proj.n);
    } else if (has_proj != 0) {
        return set_error(QORA_ERR_INVALID, "model file: input projection flag %llu",
                         (unsigned long long)has_proj);
    }
    const uint64_t n_emb = c.u(4);
    if (!c.ok || n_emb == 0 || n_emb > kMaxEmbedGroups)
        return set_error(QORA_ERR_INVALID, "model file: %llu code-predictor embeddings",
                         (unsigned long long)n_emb);
    f->p_embs.resize((size_t)n_emb);
    for (uint64_t i = 0; i < n_emb && c.ok; i++) f->p_embs[(size_t)i] = read_q4(c, f);
    f->p_layers.resize((size_t)p.num_layers);
    for (int i = 0; i < p.num_layers && c.ok; i++) f->p_layers[(size_t)i] = read_layer(c, f, p.hidden, p.head_dim);
    const uint64_t n_heads = c.u(4);
    if (!c.ok || n_heads != n_emb)
        return set_error(QORA_ERR_INVALID, "model file: %llu heads for %llu embeddings",
                         (unsigned long long)n_heads, (unsigned long long)n_emb);
    f->p_heads.resize((size_t)n_heads);
    for (uint64_t i = 0; i < n_heads && c.ok; i++) f->p_heads[(size_t)i] = read_q4(c, f);
    p.final_norm = read_f16(c, f, p.hidden);
    int64_t pc = 0, ps = 0;
    const float *p_cos = read_f32(c, f, -1, &pc);
    const float *p_sin = read_f32(c, f, -1, &ps);
    if (!c.ok) return set_error(QORA_ERR_INVALID, "model file: truncated or malformed code-predictor section");
    p.layers = f->p_layers.data();
    p.codec_embeddings = f->p_embs.data();
    p.lm_heads = f->p_heads.data();
    p.num_groups = (int32_t)n_heads;
    p.ffn = (int32_t)f->p_layers[0].gate_proj.n;
    p.vocab = (int32_t)f->p_heads[0].n;
    if (pc != ps || pc % (p.head_dim / 2) != 0)
        return set_error(QORA_ERR_INVALID, "model file: code-predictor RoPE tables");
    p.rope_max_pos = (int32_t)(pc / (p.head_dim / 2));
    f->dec_off = (size_t)(c.p - static_cast<const uint8_t *>(f->map));
    return recover_theta(p_cos, p_sin, p.head_dim, p.rope_max_pos, &p.rope_theta);
}

// ---- speech decoder (save_decoder, save.rs:171-262; load_decoder_weights,
// save.rs:446-552).  The section holds load_speech_decoder's processed
// tensors (loader.rs:503-716): codebooks already divided by their usage,
// linear and ConvNeXt pointwise weights transposed to input-major.  They are
// handed to the decoder under their checkpoint names in the checkpoint's
// layouts (transposes undone exactly; each codebook with a usage of 1, so
// the decoder's division leaves it unchanged).
using DecTensors = std::vector<std::pair<std::string, std::vector<float>>>;

bool dec_vec(Cursor &c, std::vector<float> &out, int64_t expect = -1) {
    const uint64_t n = c.u(8);
    if (n > (1ull << 36) || (expect >= 0 && n != (uint64_t)expect)) c.ok = false;
    const uint8_t *b = c.bytes(n * 4);
    if (!c.ok) return false;
    out.resize((size_t)n);
    if (n) std::memcpy(out.data(), b, (size_t)n * 4);
    return true;
}

// [rows][cols] -> [cols][rows] (transpose_2d, loader.rs:466-474, undone)
std::vector<float> dec_t(const std::vector<float> &a, int64_t rows, int64_t cols) {
    std::vector<float> o(a.size());
    for (int64_t r = 0; r < rows; r++)
        for (int64_t q = 0; q < cols; q++) o[(size_t)(q * rows + r)] = a[(size_t)(r * cols + q)];
    return o;
}

struct DecConv {
    uint32_t in = 0, out = 0, k = 0, stride = 0, pad = 0, dil = 1;
};

// save_conv1d / save_conv_t1d / save_dw_conv (save.rs:139-169): header,
// weight, bias, stored under `name`weight / `name`bias.  kind 0: Conv1d (in,
// out, k, stride, pad, dil); 1: ConvTranspose1d (in, out, k, stride, pad);
// 2: depthwise (channels, k, pad).
bool dec_conv(Cursor &c, DecTensors &T, const std::string &name, int kind, DecConv &h) {
    if (kind == 2) {
        h.in = h.out = (uint32_t)c.u(4);
        h.k = (uint32_t)c.u(4);
        h.pad = (uint32_t)c.u(4);
        h.stride = h.dil = 1;
    } else {
        h.in = (uint32_t)c.u(4);
        h.out = (uint32_t)c.u(4);
        h.k = (uint32_t)c.u(4);
        h.stride = (uint32_t)c.u(4);
        h.pad = (uint32_t)c.u(4);
        h.dil = kind == 0 ? (uint32_t)c.u(4) : 1u;
    }
    if (!c.ok || h.in == 0 || h.out == 0 || h.k == 0 || h.in > 65536 || h.out > 65536 || h.k > 64) return c.ok = false;
    std::vector<float> w, b;
    const int64_t wn = kind == 2 ? (int64_t)h.out * h.k : (int64_t)h.in * h.out * h.k;
    if (!dec_vec(c, w, wn) || !dec_vec(c, b, h.out)) return false;
    T.emplace_back(name + "weight", std::move(w));
    T.emplace_back(name + "bias", std::move(b));
    return true;
}

int decoder_section(const qora_model_file *f, qora_decoder_dims &d, DecTensors &T) {
    const uint8_t *base = static_cast<const uint8_t *>(f->map);
    Cursor c{base + f->dec_off, base + f->size};
    d = qora_decoder_dims{};
    d.hidden = (int32_t)c.u(4);
    d.num_heads = (int32_t)c.u(4);
    d.head_dim = (int32_t)c.u(4);
    d.intermediate = (int32_t)c.u(4);
    d.sliding_window = (int32_t)c.u(4);
    d.codebook_dim = (int32_t)c.u(4);
    if (!c.ok || d.hidden <= 0 || d.hidden > 65536 || d.num_heads <= 0 || d.num_heads > 1024 || d.head_dim <= 0 ||
        d.head_dim > 1024 || d.intermediate <= 0 || d.intermediate > (1 << 20) || d.sliding_window <= 0 ||
        d.codebook_dim <= 0 || d.codebook_dim > 65536)
        return set_error(QORA_ERR_INVALID, "model file: no speech-decoder section, or a bad decoder header");
    const int64_t HD = (int64_t)d.num_heads * d.head_dim;
    const std::string q = "decoder.quantizer.";
    auto ones = [](int64_t n) { return std::vector<float>((size_t)n, 1.0f); };
    std::vector<float> v, w;
    // codebooks (save.rs:180-186)
    if (!dec_vec(c, v) || v.empty() || v.size() % (size_t)d.codebook_dim)
        return set_error(QORA_ERR_INVALID, "model file: decoder codebook 0");
    d.codebook_size = (int32_t)(v.size() / (size_t)d.codebook_dim);
    T.emplace_back(q + "rvq_first.vq.layers.0._codebook.embedding_sum", std::move(v));
    T.emplace_back(q + "rvq_first.vq.layers.0._codebook.cluster_usage", ones(d.codebook_size));
    if (!dec_vec(c, w) || w.empty() || w.size() % (size_t)d.codebook_dim)
        return set_error(QORA_ERR_INVALID, "model file: decoder codebook projection");
    d.vq_dim = (int32_t)(w.size() / (size_t)d.codebook_dim);
    T.emplace_back(q + "rvq_first.output_proj.weight", dec_t(w, d.codebook_dim, d.vq_dim));
    const uint64_t n_rest = c.u(4);
    if (!c.ok || n_rest == 0 || n_rest > 64) return set_error(QORA_ERR_INVALID, "model file: decoder codebooks");
    d.num_quantizers = (int32_t)n_rest + 1;
    for (uint64_t g = 0; g < n_rest; g++) {
        if (!dec_vec(c, v, (int64_t)d.codebook_size * d.codebook_dim))
            return set_error(QORA_ERR_INVALID, "model file: decoder codebook %llu", (unsigned long long)g + 1);
        const std::string cb = q + "rvq_rest.vq.layers." + std::to_string(g) + "._codebook.";
        T.emplace_back(cb + "embedding_sum", std::move(v));
        T.emplace_back(cb + "cluster_usage", ones(d.codebook_size));
    }
    if (!dec_vec(c, w, (int64_t)d.codebook_dim * d.vq_dim))
        return set_error(QORA_ERR_INVALID, "model file: decoder codebook projection");
    T.emplace_back(q + "rvq_rest.output_proj.weight", dec_t(w, d.codebook_dim, d.vq_dim));
    // pre-conv (save.rs:189)
    DecConv h;
    if (!dec_conv(c, T, "decoder.pre_conv.conv.", 0, h) || h.in != (uint32_t)d.vq_dim || h.k != 3 || h.stride != 1 ||
        h.dil != 1)
        return set_error(QORA_ERR_INVALID, "model file: decoder pre-conv");
    d.latent = (int32_t)h.out;
    // transformer (save.rs:192-211): linear weights stored [in][out]
    const std::string t = "decoder.pre_transformer.";
    auto lin = [&](const std::string &name, int64_t in, int64_t out) {
        if (!dec_vec(c, w, in * out)) return false;
        T.emplace_back(name, dec_t(w, in, out));
        return true;
    };
    auto raw = [&](const std::string &name, int64_t n) {
        if (!dec_vec(c, v, n)) return false;
        T.emplace_back(name, std::move(v));
        return true;
    };
    if (!lin(t + "input_proj.weight", d.latent, d.hidden) || !raw(t + "input_proj.bias", d.hidden))
        return set_error(QORA_ERR_INVALID, "model file: decoder input projection");
    const uint64_t n_tf = c.u(4);
    if (!c.ok || n_tf > 256) return set_error(QORA_ERR_INVALID, "model file: decoder layers");
    d.num_layers = (int32_t)n_tf;
    for (uint64_t i = 0; i < n_tf; i++) {
        const std::string l = t + "layers." + std::to_string(i) + ".";
        const bool ok = lin(l + "self_attn.q_proj.weight", d.hidden, HD) &&
                        lin(l + "self_attn.k_proj.weight", d.hidden, HD) &&
                        lin(l + "self_attn.v_proj.weight", d.hidden, HD) &&
                        lin(l + "self_attn.o_proj.weight", HD, d.hidden) &&
                        lin(l + "mlp.gate_proj.weight", d.hidden, d.intermediate) &&
                        lin(l + "mlp.up_proj.weight", d.hidden, d.intermediate) &&
                        lin(l + "mlp.down_proj.weight", d.intermediate, d.hidden) &&
                        raw(l + "input_layernorm.weight", d.hidden) &&
                        raw(l + "post_attention_layernorm.weight", d.hidden) &&
                        raw(l + "self_attn_layer_scale.scale", d.hidden) && raw(l + "mlp_layer_scale.scale", d.hidden);
        if (!ok) return set_error(QORA_ERR_INVALID, "model file: decoder layer %llu", (unsigned long long)i);
    }
    if (!raw(t + "norm.weight", d.hidden) || !lin(t + "output_proj.weight", d.hidden, d.latent) ||
        !raw(t + "output_proj.bias", d.latent))
        return set_error(QORA_ERR_INVALID, "model file: decoder output projection");
    // upsample (save.rs:214-227)
    const uint64_t n_up = c.u(4);
    if (!c.ok || n_up > 8) return set_error(QORA_ERR_INVALID, "model file: decoder upsample stages");
    d.upsample_stages = (int32_t)n_up;
    for (uint64_t i = 0; i < n_up; i++) {
        const std::string ct = "decoder.upsample." + std::to_string(i) + ".0.conv.";
        const std::string cn = "decoder.upsample." + std::to_string(i) + ".1.";
        const uint64_t ch = c.u(4);
        DecConv hc, hd;
        if (!c.ok || ch != (uint64_t)d.latent || !dec_conv(c, T, ct, 1, hc) || hc.in != ch || hc.out != ch ||
            hc.k != 2 || hc.stride != 2 || hc.pad != 0 || !dec_conv(c, T, cn + "dwconv.conv.", 2, hd) ||
            hd.out != ch || hd.k != 7)
            return set_error(QORA_ERR_INVALID, "model file: decoder upsample stage %llu", (unsigned long long)i);
        if (!raw(cn + "norm.weight", d.latent) || !raw(cn + "norm.bias", d.latent) || !dec_vec(c, w) || w.empty() ||
            w.size() % (size_t)d.latent)
            return set_error(QORA_ERR_INVALID, "model file: decoder upsample stage %llu", (unsigned long long)i);
        const int64_t inner = (int64_t)(w.size() / (size_t)d.latent);
        if (i == 0) d.upsample_inner = (int32_t)inner;
        if (inner != d.upsample_inner) return set_error(QORA_ERR_INVALID, "model file: decoder upsample widths");
        T.emplace_back(cn + "pwconv1.weight", dec_t(w, d.latent, inner));
        if (!raw(cn + "pwconv1.bias", inner) || !dec_vec(c, w, inner * d.latent))
            return set_error(QORA_ERR_INVALID, "model file: decoder upsample stage %llu", (unsigned long long)i);
        T.emplace_back(cn + "pwconv2.weight", dec_t(w, inner, d.latent));
        if (!raw(cn + "pwconv2.bias", d.latent) || !raw(cn + "gamma", d.latent))
            return set_error(QORA_ERR_INVALID, "model file: decoder upsample stage %llu", (unsigned long long)i);
    }
    if (n_up == 0) d.upsample_inner = 4 * d.latent;
    // Vocos (save.rs:230-246)
    if (!dec_conv(c, T, "decoder.decoder.0.conv.", 0, h) || h.in != (uint32_t)d.latent || h.k != 7 ||
        h.stride != 1 || h.dil != 1)
        return set_error(QORA_ERR_INVALID, "model file: decoder Vocos input conv");
    d.vocos_channels[0] = (int32_t)h.out;
    const uint64_t n_vb = c.u(4);
    if (!c.ok || n_vb == 0 || n_vb > 7) return set_error(QORA_ERR_INVALID, "model file: decoder Vocos blocks");
    d.vocos_blocks = (int32_t)n_vb;
    static const uint32_t kDil[3] = {1, 3, 9};
    for (uint64_t b = 0; b < n_vb; b++) {
        const std::string p = "decoder.decoder." + std::to_string(b + 1) + ".block.";
        const int64_t ci = d.vocos_channels[b];
        DecConv hc;
        if (!raw(p + "0.alpha", ci) || !raw(p + "0.beta", ci) || !dec_conv(c, T, p + "1.conv.", 1, hc) ||
            hc.in != (uint32_t)ci || hc.pad != 0)
            return set_error(QORA_ERR_INVALID, "model file: decoder Vocos block %llu", (unsigned long long)b);
        d.vocos_channels[b + 1] = (int32_t)hc.out;
        d.vocos_kernels[b] = (int32_t)hc.k;
        d.vocos_strides[b] = (int32_t)hc.stride;
        const uint64_t n_res = c.u(4);
        if (!c.ok || n_res != 3)
            return set_error(QORA_ERR_UNSUPPORTED, "model file: decoder Vocos block with %llu residual units",
                             (unsigned long long)n_res);
        for (int r = 0; r < 3; r++) {
            const std::string u = p + std::to_string(r + 2) + ".";
            DecConv h1, h2;
            const int64_t co = hc.out;
            if (!raw(u + "act1.alpha", co) || !raw(u + "act1.beta", co) || !dec_conv(c, T, u + "conv1.conv.", 0, h1) ||
                !raw(u + "act2.alpha", co) || !raw(u + "act2.beta", co) || !dec_conv(c, T, u + "conv2.conv.", 0, h2))
                return set_error(QORA_ERR_INVALID, "model file: decoder residual unit %llu.%d", (unsigned long long)b, r);
            if (h1.in != (uint32_t)co || h1.out != (uint32_t)co || h1.k != 7 || h1.stride != 1 || h1.dil != kDil[r] ||
                h2.in != (uint32_t)co || h2.out != (uint32_t)co || h2.k != 1 || h2.stride != 1)
                return set_error(QORA_ERR_UNSUPPORTED, "model file: decoder residual unit %llu.%d shape",
                                 (unsigned long long)b, r);
        }
    }
    // output (save.rs:249-252)
    const int64_t cl = d.vocos_channels[n_vb];
    const std::string fo = "decoder.decoder." + std::to_string(n_vb + 1) + ".";
    const std::string oo = "decoder.decoder." + std::to_string(n_vb + 2) + ".conv.";
    if (!raw(fo + "alpha", cl) || !raw(fo + "beta", cl) || !dec_conv(c, T, oo, 0, h) || h.in != (uint32_t)cl ||
        h.out != 1 || h.k != 7 || h.stride != 1 || h.dil != 1)
        return set_error(QORA_ERR_INVALID, "model file: decoder output conv");
    // RoPE tables (save.rs:255-256): the base is recovered as for the talker
    std::vector<float> rc, rs;
    if (!dec_vec(c, rc) || !dec_vec(c, rs) || rc.size() != rs.size() || d.head_dim % 2 || rc.empty() ||
        rc.size() % (size_t)(d.head_dim / 2))
        return set_error(QORA_ERR_INVALID, "model file: decoder RoPE tables");
    d.rope_max_pos = (int32_t)(rc.size() / (size_t)(d.head_dim / 2));
    return recover_theta(rc.data(), rs.data(), d.head_dim, d.rope_max_pos, &d.rope_theta);
}

}  // namespace

extern "C" {

int qora_model_file_open(const char *path, qora_model_file **out) {
    if (!path || !out) return set_error(QORA_ERR_INVALID, "qora_model_file_open: bad arguments");
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return set_error(QORA_ERR_INVALID, "model file: cannot open %s", path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
        close(fd);
        return set_error(QORA_ERR_INVALID, "model file: cannot stat %s", path);
    }
    void *map = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return set_error(QORA_ERR_OOM, "model file: cannot map %s", path);
    auto *f = new qora_model_file();
    f->map = map;
    f->size = (size_t)st.st_size;
    const int rc = parse(f);
    if (rc != QORA_OK) {
        qora_model_file_close(f);
        return rc;
    }
    *out = f;
    return QORA_OK;
}

int qora_model_file_talker(const qora_model_file *f, qora_talker_host *out) {
    if (!f || !out) return set_error(QORA_ERR_INVALID, "qora_model_file_talker: bad arguments");
    *out = f->talker;
    return QORA_OK;
}

int qora_model_file_predictor(const qora_model_file *f, qora_predictor_host *out) {
    if (!f || !out) return set_error(QORA_ERR_INVALID, "qora_model_file_predictor: bad arguments");
    *out = f->predictor;
    return QORA_OK;
}

int qora_model_file_text_proj(const qora_model_file *f, qora_text_proj_host *out) {
    if (!f || !out) return set_error(QORA_ERR_INVALID, "qora_model_file_text_proj: bad arguments");
    *out = f->text;
    return QORA_OK;
}

int qora_model_file_decoder(const qora_model_file *f, qora_ctx *ctx, qora_decoder **out) {
    if (!f || !ctx || !out) return set_error(QORA_ERR_INVALID, "qora_model_file_decoder: bad arguments");
    *out = nullptr;
    qora_decoder_dims d;
    DecTensors T;
    QORA_TRY(decoder_section(f, d, T));
    qora_decoder *dec = nullptr;
    QORA_TRY(qora_decoder_create(ctx, &d, &dec));
    int rc = QORA_OK;
    for (auto &kv : T) {
        rc = qora_decoder_set_tensor(dec, kv.first.c_str(), kv.second.data(), (int64_t)kv.second.size());
        if (rc != QORA_OK) break;
        std::vector<float>().swap(kv.second);   // the decoder keeps its own copy
    }
    if (rc == QORA_OK) rc = qora_decoder_finalize(dec);
    if (rc != QORA_OK) {
        qora_decoder_destroy(dec);
        return rc;
    }
    *out = dec;
    return QORA_OK;
}

void qora_model_file_close(qora_model_file *f) {
    if (!f) return;
    if (f->map) munmap(f->map, f->size);
    delete f;
}

}  // extern "C"
