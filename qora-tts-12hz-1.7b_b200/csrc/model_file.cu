// Reader of the reference's single-file checkpoint (.qora-tts, save.rs:262-409,
// record helpers gemv.rs:595-687), for callers that load weights without the
// reference's Rust loader.
//
// Layout (little endian): "QTTS", u32 version (1), u8 format (1 = Q4, 0 = f16),
// then the talker section (save.rs:300-351, with the text embedding and text
// projection the prompt is built from), the code-predictor section
// (save.rs:353-438) and the speech decoder, which this engine does not use and
// which is not read.  Arrays are u64 element counts followed by the elements;
// a weight is u64 k, u64 n, then (Q4) the packed bytes and the f16 scales.
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
    return recover_theta(p_cos, p_sin, p.head_dim, p.rope_max_pos, &p.rope_theta);
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

void qora_model_file_close(qora_model_file *f) {
    if (!f) return;
    if (f->map) munmap(f->map, f->size);
    delete f;
}

}  // extern "C"
