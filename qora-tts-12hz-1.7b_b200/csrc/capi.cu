// extern "C" entry points: context, weights, generic GEMV/GEMM, RoPE tables,
// sampler.  Model-level entry points (KV, talker, predictor, engine) live in
// model.cu.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "gemv.cuh"
#include "sampler.cuh"

namespace qora {

static thread_local char g_err[512] = "";

int set_error(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

// ---------------------------------------------------------------- host f16
static uint16_t f32_to_f16_rne(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | (ax == 0x7f800000u ? 0x7c00u : 0x7e00u));
    const uint32_t e = ax >> 23;
    if (e >= 143) return (uint16_t)(sign | 0x7c00u);
    if (e >= 113) {
        const uint32_t mant = ax & 0x7fffffu;
        uint32_t h = ((e - 112) << 10) | (mant >> 13);
        const uint32_t rem = mant & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    if (ax < 0x33000000u) return (uint16_t)sign;
    const uint32_t M = (ax & 0x7fffffu) | 0x800000u, s = 126 - e;
    uint32_t m16 = M >> s;
    const uint32_t rem = M & ((1u << s) - 1u), half = 1u << (s - 1);
    if (rem > half || (rem == half && (m16 & 1u))) m16++;
    return (uint16_t)(sign | m16);
}

// quantize_f32_to_q4 (gemv.rs:92-130) for rows [r0, r1).
static void quantize_rows(const float *data, int64_t r0, int64_t r1, int64_t n, uint8_t *packed,
                          uint16_t *scales) {
    const int64_t gpr = n / kGroup;
    for (int64_t ki = r0; ki < r1; ki++) {
        for (int64_t g = 0; g < gpr; g++) {
            const float *v = data + ki * n + g * kGroup;
            float absmax = 0.0f;
            for (int j = 0; j < kGroup; j++) {
                const float a = std::fabs(v[j]);
                if (a > absmax) absmax = a;
            }
            const float scale = absmax / 7.0f;
            scales[ki * gpr + g] = f32_to_f16_rne(scale);
            const float inv = scale > 0.0f ? 1.0f / scale : 0.0f;  // unrounded scale
            uint8_t *dst = packed + (ki * gpr + g) * 16;
            for (int j = 0; j < kGroup; j += 2) {
                const float q0 = std::fmin(std::fmax(std::round(v[j] * inv), -8.0f), 7.0f) + 8.0f;
                const float q1 = std::fmin(std::fmax(std::round(v[j + 1] * inv), -8.0f), 7.0f) + 8.0f;
                dst[j / 2] = (uint8_t)((uint8_t)q0 | ((uint8_t)q1 << 4));
            }
        }
    }
}

template <class F>
static void parallel_for(int64_t n, int64_t grain, F fn) {
    const int64_t tasks = (n + grain - 1) / grain;
    unsigned hw = std::thread::hardware_concurrency();
    const int64_t nth = std::max<int64_t>(1, std::min<int64_t>(tasks, hw ? hw : 4));
    if (nth <= 1) {
        for (int64_t t = 0; t < tasks; t++) fn(t * grain, std::min(n, (t + 1) * grain));
        return;
    }
    std::vector<std::thread> th;
    std::atomic<int64_t> next{0};
    for (int64_t i = 0; i < nth; i++)
        th.emplace_back([&] {
            for (;;) {
                const int64_t t = next.fetch_add(1);
                if (t >= tasks) break;
                fn(t * grain, std::min(n, (t + 1) * grain));
            }
        });
    for (auto &x : th) x.join();
}

static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Counter-based N(0, sigma): pair p of stream `seed` from two splitmix64
// outputs, Box-Muller in double precision.
static void synth_normal_range(uint64_t seed, float sigma, int64_t count, float *out, int64_t p0,
                               int64_t p1) {
    const uint64_t base = mix64(seed) ^ 0xD1B54A32D192ED03ull;
    for (int64_t p = p0; p < p1; p++) {
        const uint64_t a = mix64(base + 2 * (uint64_t)p), b = mix64(base + 2 * (uint64_t)p + 1);
        const double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740992.0);
        const double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
        const double r = std::sqrt(-2.0 * std::log(u1));
        const double th = 6.283185307179586 * u2;
        out[2 * p] = (float)((double)sigma * r * std::cos(th));
        if (2 * p + 1 < count) out[2 * p + 1] = (float)((double)sigma * r * std::sin(th));
    }
}

int host_rope_tables(int32_t head_dim, int32_t max_pos, double theta, const int32_t *sections,
                     int32_t n_sections, float *cos_t, float *sin_t) {
    const int32_t half = head_dim / 2;
    int32_t sum = 0;
    for (int i = 0; i < n_sections; i++) sum += sections[i];
    if (sum != half) return set_error(QORA_ERR_SHAPE, "rope sections sum %d != head_dim/2 %d", sum, half);
    int32_t off = 0;
    for (int s = 0; s < n_sections; s++) {  // rope.rs:26-38
        for (int32_t i = 0; i < sections[s]; i++) {
            const int32_t d = off + i;
            const double freq = 1.0 / std::pow(theta, (double)(2 * d) / (double)head_dim);
            for (int64_t pos = 0; pos < max_pos; pos++) {
                const double ang = (double)pos * freq;
                cos_t[pos * half + d] = (float)std::cos(ang);
                sin_t[pos * half + d] = (float)std::sin(ang);
            }
        }
        off += sections[s];
    }
    return QORA_OK;
}

}  // namespace qora

using namespace qora;

bool qora::pdl_enabled() {
    static const bool on = [] {
        const char *e = getenv("QORA_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

extern "C" {

const char *qora_status_string(int32_t s) {
    switch (s) {
        case QORA_OK: return "ok";
        case QORA_ERR_INVALID: return "invalid argument";
        case QORA_ERR_SHAPE: return "shape mismatch";
        case QORA_ERR_CUDA: return "CUDA error";
        case QORA_ERR_OOM: return "out of device memory";
        case QORA_ERR_RANGE: return "position out of range";
        case QORA_ERR_UNSUPPORTED: return "unsupported configuration";
        case QORA_ERR_TIMEOUT: return "device wait timed out";
    }
    return "unknown status";
}

const char *qora_last_error(void) { return g_err; }

int qora_ctx_create(int32_t device, qora_ctx **out) {
    if (!out) return set_error(QORA_ERR_INVALID, "null out");
    int n = 0;
    QORA_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return set_error(QORA_ERR_INVALID, "device %d of %d", device, n);
    QORA_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    QORA_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10)
        return set_error(QORA_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a",
                         device, prop.major, prop.minor);
    auto *c = new qora_ctx();
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    int rc = c->err.alloc(64);
    if (rc == QORA_OK) rc = c->err.zero();
    if (rc == QORA_OK) rc = gemv_init();
    if (rc == QORA_OK && cudaDeviceSynchronize() != cudaSuccess)
        rc = set_error(QORA_ERR_CUDA, "qora_ctx_create: sync failed");
    if (rc != QORA_OK) {
        delete c;
        return rc;
    }
    *out = c;
    return QORA_OK;
}

void qora_ctx_destroy(qora_ctx *ctx) { qora::CtxRef::drop(ctx); }

int qora_ctx_check_device_error(qora_ctx *ctx, void *stream) {
    if (!ctx) return set_error(QORA_ERR_INVALID, "null ctx");
    int v = 0;
    cudaStream_t st = as_stream(stream);
    QORA_CUDA(cudaMemcpyAsync(&v, ctx->err.p, 4, cudaMemcpyDeviceToHost, st));
    QORA_CUDA(cudaStreamSynchronize(st));
    if (v == kDevOk) return QORA_OK;
    QORA_CUDA(cudaMemsetAsync(ctx->err.p, 0, 4, st));
    QORA_CUDA(cudaStreamSynchronize(st));
    switch (v) {
        case kDevRange: return set_error(QORA_ERR_RANGE, "device: position past RoPE table or KV capacity");
        case kDevNaN: return set_error(QORA_ERR_INVALID, "device: NaN reached argmax/sampler");
        case kDevTimeout: return set_error(QORA_ERR_TIMEOUT, "device: bounded wait expired");
        case kDevF16Range:
            return set_error(QORA_ERR_RANGE, "device: infinite GEMV input value on the tensor-core path");
    }
    return set_error(QORA_ERR_CUDA, "device error code %d", v);
}

int qora_q4_quantize_host(const float *data, int64_t k, int64_t n, uint8_t *packed, uint16_t *scales) {
    if (!data || !packed || !scales || k <= 0 || n <= 0 || n % kGroup)
        return set_error(QORA_ERR_INVALID, "qora_q4_quantize_host: bad arguments (n %% 32 == 0 required)");
    parallel_for(k, 64, [&](int64_t a, int64_t b) { quantize_rows(data, a, b, n, packed, scales); });
    return QORA_OK;
}

int qora_synth_normal_host(uint64_t seed, float sigma, int64_t count, float *out) {
    if (!out || count < 0) return set_error(QORA_ERR_INVALID, "bad arguments");
    const int64_t npairs = (count + 1) / 2;
    parallel_for(npairs, 1 << 16, [&](int64_t a, int64_t b) { synth_normal_range(seed, sigma, count, out, a, b); });
    return QORA_OK;
}

int qora_synth_q4_host(uint64_t seed, float sigma, int64_t k, int64_t n, uint8_t *packed, uint16_t *scales) {
    if (!packed || !scales || k <= 0 || n <= 0 || n % kGroup) return set_error(QORA_ERR_INVALID, "bad arguments");
    std::vector<float> tmp((size_t)(k * n));
    QORA_TRY(qora_synth_normal_host(seed, sigma, k * n, tmp.data()));
    return qora_q4_quantize_host(tmp.data(), k, n, packed, scales);
}

int qora_q4_weight_upload(qora_ctx *ctx, const qora_q4_host *w, qora_w4 **out) {
    if (!ctx || !w || !out || !w->packed || !w->scales || w->k <= 0 || w->n < kGroup)
        return set_error(QORA_ERR_INVALID, "qora_q4_weight_upload: bad arguments");
    QORA_CUDA(cudaSetDevice(ctx->device));
    auto *d = new qora_w4();
    d->ctx = ctx;
    const int64_t C = w->n / kGroup;
    qora_q4_host full = *w;  // the tail (n % 32) has no stored groups (gemv.rs:846-861)
    full.n = C * kGroup;
    const int64_t off = 0, st = 1;
    int rc = upload_q4_parts(&full, &off, &st, 1, w->k, C, d->nib, d->scl, d->dev, nullptr);
    d->dev.n = w->n;
    if (rc == QORA_OK) rc = upload_emb(full, d->rowmajor_packed, d->rowmajor_scl, d->emb);
    if (rc != QORA_OK) {
        delete d;
        return rc;
    }
    *out = d;
    return QORA_OK;
}

void qora_q4_weight_destroy(qora_w4 *w) { delete w; }

static int generic_gemv(qora_ctx *ctx, const qora_w4 *w, const float *x, float *y, int rows,
                        cudaStream_t st) {
    GemvArgs a;
    a.w = w->dev;
    a.rows = rows;
    a.x = x;
    a.ldx = w->dev.k;
    a.y = y;
    a.ldy = w->dev.n;
    a.err = ctx->err.as<int>();
    const GemvPlan p = plan_gemv_for(a, X_PLAIN, E_STORE, ctx->num_sms);
    return launch_gemv(a, X_PLAIN, E_STORE, p, nullptr, st);
}

int qora_q4_gemv(qora_ctx *ctx, const qora_w4 *w, const float *x, float *y, int32_t batch, void *stream) {
    if (!ctx || !w || !x || !y || batch <= 0 || batch > kMaxRows)
        return set_error(QORA_ERR_INVALID, "qora_q4_gemv: bad arguments (batch 1..%d)", kMaxRows);
    return generic_gemv(ctx, w, x, y, batch, as_stream(stream));
}

int qora_q4_gemm(qora_ctx *ctx, const qora_w4 *w, const float *x, int64_t seq_len, float *y, void *stream) {
    if (!ctx || !w || !x || !y || seq_len <= 0) return set_error(QORA_ERR_INVALID, "qora_q4_gemm: bad arguments");
    for (int64_t t0 = 0; t0 < seq_len; t0 += kMaxRows) {
        const int rows = (int)std::min<int64_t>(kMaxRows, seq_len - t0);
        QORA_TRY(generic_gemv(ctx, w, x + t0 * w->dev.k, y + t0 * w->dev.n, rows, as_stream(stream)));
    }
    return QORA_OK;
}

int qora_q4_embed_rows(qora_ctx *ctx, const qora_w4 *w, const uint32_t *tokens, int32_t count,
                       float *out, void *stream) {
    if (!ctx || !w || !tokens || !out || count < 0) return set_error(QORA_ERR_INVALID, "bad arguments");
    return launch_embed_rows(w->emb, tokens, 1, count, out, w->emb.n, ctx->err.as<int>(), as_stream(stream));
}

int qora_rms_norm_f16(qora_ctx *ctx, const float *x, const uint16_t *gamma, int64_t n, int32_t rows,
                      float *out, void *stream) {
    if (!ctx || !x || !gamma || !out || n <= 0 || rows <= 0) return set_error(QORA_ERR_INVALID, "bad arguments");
    return launch_rmsnorm_rows(x, reinterpret_cast<const __half *>(gamma), n, rows, out, as_stream(stream));
}

int qora_rope_tables_host(int32_t head_dim, int32_t max_pos, double theta, const int32_t *sections,
                          int32_t n_sections, float *cos_host, float *sin_host) {
    if (!cos_host || !sin_host || head_dim <= 0 || head_dim % 2 || max_pos <= 0)
        return set_error(QORA_ERR_INVALID, "bad arguments");
    const int32_t half = head_dim / 2;
    if (!sections || n_sections <= 0) return host_rope_tables(head_dim, max_pos, theta, &half, 1, cos_host, sin_host);
    return host_rope_tables(head_dim, max_pos, theta, sections, n_sections, cos_host, sin_host);
}

int qora_sample(qora_ctx *ctx, const float *logits, int32_t B, int32_t V, const uint32_t *prev,
                int32_t n_prev, uint64_t *rng, const qora_sample_params *params, uint32_t *out,
                void *stream) {
    if (!ctx || !logits || !rng || !params || !out || B <= 0 || V <= 0 || (n_prev > 0 && !prev))
        return set_error(QORA_ERR_INVALID, "qora_sample: bad arguments");
    SampleArgs a;
    a.logits = logits;
    a.ldlogits = V;
    a.V = V;
    a.prev = prev;
    a.ldprev = n_prev;
    a.n_prev = n_prev;
    a.rng = rng;
    a.params = *params;
    a.out = out;
    a.ldout = 1;
    a.err = ctx->err.as<int>();
    return launch_sample(a, B, as_stream(stream));
}

}  // extern "C"
