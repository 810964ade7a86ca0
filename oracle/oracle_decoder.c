/*
 * Speech-decoder ORACLE (test infrastructure only: tests/, the checker in
 * __graft_entry__.smoke() and bench.py's CPU legs use it; the product never
 * does).  A CPU restatement of the reference's f32 speech decoder primitives
 * (src/conv.rs, src/decoder.rs); oracle/pydecoder.py strings them together
 * as decode_to_audio (decoder.rs:395-582).
 *
 * Per output element the floating-point operations are the reference's, in
 * its order: sums start where the reference starts them (the bias, or 0),
 * add terms in the reference's order, and round every multiply and add
 * separately (this file is compiled with -ffp-contract=off).  The loops run
 * independent output elements side by side so the compiler can vectorise
 * them; no element's own sum is reordered, so the results are the
 * reference's bits (the golden vectors of conv.rs's own tests pin the
 * convolutions; tests/test_oracle_decoder.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OD_TILE 512

static inline int64_t od_min(int64_t a, int64_t b) { return a < b ? a : b; }
static inline int64_t od_max(int64_t a, int64_t b) { return a > b ? a : b; }

/* causal_conv1d (conv.rs:114-150) through causal_conv1d_range_scalar
 * (conv.rs:191-230): in [ic][len], w [oc][ic][ks], out [oc][len];
 * out[oc][o] = bias[oc] + sum over ic ascending, then k ascending, of
 * in[ic][o + k*dil - pad] * w[oc][ic][k], pad = (ks - 1) * dil, positions
 * outside [0, len) skipped (no term added). */
void od_causal_conv1d(const float *in, const float *w, const float *bias, int32_t ic_n, int32_t oc_n,
                      int32_t ks, int32_t dil, int64_t len, float *out) {
    const int64_t pad = (int64_t)(ks - 1) * dil;
    float acc[OD_TILE];
    for (int32_t oc = 0; oc < oc_n; oc++) {
        for (int64_t t0 = 0; t0 < len; t0 += OD_TILE) {
            const int64_t n = od_min(OD_TILE, len - t0);
            for (int64_t i = 0; i < n; i++) acc[i] = bias[oc];
            for (int32_t ic = 0; ic < ic_n; ic++) {
                const float *src = in + (int64_t)ic * len;
                const float *wr = w + ((int64_t)oc * ic_n + ic) * ks;
                for (int32_t k = 0; k < ks; k++) {
                    const int64_t sh = (int64_t)k * dil - pad;  /* input index = o + sh */
                    const int64_t lo = od_max(t0, -sh), hi = od_min(t0 + n, len - sh);
                    const float wv = wr[k];
                    for (int64_t o = lo; o < hi; o++) acc[o - t0] += src[o + sh] * wv;
                }
            }
            memcpy(out + (int64_t)oc * len + t0, acc, (size_t)n * sizeof(float));
        }
    }
}

/* Output length of conv_transpose1d (conv.rs:249). */
int64_t od_conv_transpose1d_len(int64_t len, int32_t ks, int32_t stride, int32_t pad) {
    return (len - 1) * stride - 2 * (int64_t)pad + ks;
}

/* conv_transpose1d (conv.rs:247-289) through the scalar range
 * (conv.rs:291-349): in [ic][len], w [ic][oc][ks], out [oc][out_len]; every
 * output starts at its bias, then for ic ascending, input position i
 * ascending (a zero input value skipped), tap k ascending:
 * out[oc][i*stride + k - pad] += in[ic][i] * w[ic][oc][k] when in range. */
void od_conv_transpose1d(const float *in, const float *w, const float *bias, int32_t ic_n, int32_t oc_n,
                         int32_t ks, int32_t stride, int32_t pad, int64_t len, float *out) {
    const int64_t out_len = od_conv_transpose1d_len(len, ks, stride, pad);
    for (int32_t oc = 0; oc < oc_n; oc++) {
        float *row = out + (int64_t)oc * out_len;
        for (int64_t o = 0; o < out_len; o++) row[o] = bias[oc];
        for (int32_t ic = 0; ic < ic_n; ic++) {
            const float *src = in + (int64_t)ic * len;
            const float *wb = w + ((int64_t)ic * oc_n + oc) * ks;
            for (int64_t i = 0; i < len; i++) {
                const float val = src[i];
                if (val == 0.0f) continue;
                const int64_t base = i * stride - pad;
                const int32_t k0 = (int32_t)od_max(0, -base);
                const int32_t k1 = (int32_t)od_min(ks, out_len - base);
                for (int32_t k = k0; k < k1; k++) row[base + k] += val * wb[k];
            }
        }
    }
}

/* depthwise_conv1d (conv.rs:361-432): causal, pad = ks - 1 (the weight's
 * padding field is not used); out[c][o] = bias[c] + sum over k ascending of
 * in[c][o + k - pad] * w[c][k], positions outside [0, len) skipped. */
void od_depthwise_conv1d(const float *in, const float *w, const float *bias, int32_t ch, int32_t ks,
                         int64_t len, float *out) {
    const int64_t pad = ks - 1;
    for (int32_t c = 0; c < ch; c++) {
        const float *src = in + (int64_t)c * len;
        float *dst = out + (int64_t)c * len;
        for (int64_t o = 0; o < len; o++) dst[o] = bias[c];
        for (int32_t k = 0; k < ks; k++) {
            const int64_t sh = k - pad;
            const int64_t lo = od_max(0, -sh), hi = od_min(len, len - sh);
            const float wv = w[(int64_t)c * ks + k];
            for (int64_t o = lo; o < hi; o++) dst[o] += src[o + sh] * wv;
        }
    }
}

/* layer_norm_channel_first (decoder.rs:657-684): per position t, over the
 * channels in order: mean = (sum x) / C; var = sum (x - mean)^2;
 * inv_std = 1 / sqrt(var / C + eps); out = (x - mean) * inv_std * gamma + beta. */
void od_layer_norm_cf(const float *in, const float *gamma, const float *beta, int32_t ch, int64_t len,
                      float eps, float *out) {
    float mean[OD_TILE], var[OD_TILE], inv[OD_TILE];
    for (int64_t t0 = 0; t0 < len; t0 += OD_TILE) {
        const int64_t n = od_min(OD_TILE, len - t0);
        for (int64_t i = 0; i < n; i++) mean[i] = 0.0f, var[i] = 0.0f;
        for (int32_t c = 0; c < ch; c++) {
            const float *src = in + (int64_t)c * len + t0;
            for (int64_t i = 0; i < n; i++) mean[i] += src[i];
        }
        for (int64_t i = 0; i < n; i++) mean[i] /= (float)ch;
        for (int32_t c = 0; c < ch; c++) {
            const float *src = in + (int64_t)c * len + t0;
            for (int64_t i = 0; i < n; i++) {
                const float d = src[i] - mean[i];
                var[i] += d * d;
            }
        }
        for (int64_t i = 0; i < n; i++) inv[i] = 1.0f / sqrtf(var[i] / (float)ch + eps);
        for (int32_t c = 0; c < ch; c++) {
            const float *src = in + (int64_t)c * len + t0;
            float *dst = out + (int64_t)c * len + t0;
            for (int64_t i = 0; i < n; i++) dst[i] = (src[i] - mean[i]) * inv[i] * gamma[c] + beta[c];
        }
    }
}

/* snake_beta (conv.rs:545-641): a = exp(alpha[c]), inv_b = exp(-beta[c]);
 * out = x + inv_b * sin(a x)^2, evaluated as x + ((inv_b * s) * s). */
void od_snake_beta(const float *in, const float *alpha, const float *beta, int32_t ch, int64_t len,
                   float *out) {
    for (int32_t c = 0; c < ch; c++) {
        const float a = expf(alpha[c]);
        const float inv_b = expf(-beta[c]);
        const float *src = in + (int64_t)c * len;
        float *dst = out + (int64_t)c * len;
        for (int64_t t = 0; t < len; t++) {
            const float x = src[t];
            const float s = sinf(a * x);
            dst[t] = x + inv_b * s * s;
        }
    }
}

/* gelu (conv.rs:692-694), in place: x * 0.5 * (1 + tanh(x * 0.70710677)). */
void od_gelu(float *x, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        const float v = x[i];
        x[i] = v * 0.5f * (1.0f + tanhf(v * 0.7071067811865476f));
    }
}

/* f32_gemm_bias (conv.rs:434-526) via f32_gemm_block_scalar: a [m][k],
 * b [k][n], c [m][n] = bias[m] + sum over kk ascending of a[m][kk] * b[kk][j],
 * a zero a[m][kk] skipped. */
void od_f32_gemm_bias(const float *a, const float *b, const float *bias, int64_t m, int64_t n, int64_t k,
                      float *c) {
    for (int64_t mi = 0; mi < m; mi++) {
        float *row = c + mi * n;
        for (int64_t j = 0; j < n; j++) row[j] = bias[mi];
        for (int64_t kk = 0; kk < k; kk++) {
            const float av = a[mi * k + kk];
            if (av == 0.0f) continue;
            const float *br = b + kk * n;
            for (int64_t j = 0; j < n; j++) row[j] += av * br[j];
        }
    }
}

/* f32_gemv / f32_gemv_bias (decoder.rs:596-622) for `rows` input rows:
 * x [rows][k], w [k][n] (input-major, the reference's transposed layout),
 * out[r][j] = (bias ? bias[j] : 0) + sum over ki ascending of x[r][ki] * w[ki][j],
 * a zero x[r][ki] skipped. */
void od_f32_gemv_rows(const float *x, const float *w, const float *bias, int64_t rows, int64_t k, int64_t n,
                      float *out) {
    for (int64_t r = 0; r < rows; r++) {
        float *o = out + r * n;
        for (int64_t j = 0; j < n; j++) o[j] = bias ? bias[j] : 0.0f;
        for (int64_t ki = 0; ki < k; ki++) {
            const float iv = x[r * k + ki];
            if (iv == 0.0f) continue;
            const float *wr = w + ki * n;
            for (int64_t j = 0; j < n; j++) o[j] += iv * wr[j];
        }
    }
}

/* rms_norm_f32 (decoder.rs:585-594) per row: ss = sum x^2 (in order);
 * inv = 1 / sqrt(ss / n + eps); out = x * inv * gamma. */
void od_rms_norm_rows(const float *x, const float *gamma, int64_t rows, int64_t n, float eps, float *out) {
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * n;
        float ss = 0.0f;
        for (int64_t i = 0; i < n; i++) ss += xr[i] * xr[i];
        const float inv = 1.0f / sqrtf(ss / (float)n + eps);
        for (int64_t i = 0; i < n; i++) out[r * n + i] = xr[i] * inv * gamma[i];
    }
}

/* Decoder RoPE tables (loader.rs:668-682): standard (not multimodal),
 * freq_i = 1 / theta^(2i / head_dim) in f64, cos / sin of pos * freq_i in f64,
 * rounded to f32; [max_pos][head_dim / 2]. */
void od_rope_tables(int32_t head_dim, int32_t max_pos, double theta, float *cos_t, float *sin_t) {
    const int32_t half = head_dim / 2;
    for (int32_t i = 0; i < half; i++) {
        const double freq = 1.0 / pow(theta, (double)(2 * i) / (double)head_dim);
        for (int32_t pos = 0; pos < max_pos; pos++) {
            const double angle = (double)pos * freq;
            cos_t[(int64_t)pos * half + i] = (float)cos(angle);
            sin_t[(int64_t)pos * half + i] = (float)sin(angle);
        }
    }
}

/* apply_rope_split_half (decoder.rs:624-647) to every row of x
 * [rows][heads * head_dim], row r at position r: pairs (x[i], x[i + half]);
 * a position whose table row is past the table (max_pos rows) is left as is. */
void od_rope_split_half_rows(float *x, int64_t rows, int32_t heads, int32_t head_dim, const float *cos_t,
                             const float *sin_t, int32_t max_pos) {
    const int32_t half = head_dim / 2;
    for (int64_t pos = 0; pos < rows; pos++) {
        const int64_t off = pos * half;
        if (off + half > (int64_t)max_pos * half) continue;
        float *row = x + pos * (int64_t)heads * head_dim;
        for (int32_t h = 0; h < heads; h++) {
            float *b = row + (int64_t)h * head_dim;
            for (int32_t i = 0; i < half; i++) {
                const float x0 = b[i], x1 = b[half + i];
                const float c = cos_t[off + i], s = sin_t[off + i];
                b[i] = x0 * c - x1 * s;
                b[half + i] = x1 * c + x0 * s;
            }
        }
    }
}

/* The decoder transformer's causal sliding-window attention
 * (decoder.rs:251-284) for all positions: q, k, v [T][heads * head_dim];
 * position t attends to positions max(0, t + 1 - window) .. t;
 * score = (sum over d of q k, in order) * scale; softmax_raw (gemv.rs:471-482):
 * max, exp(s - max) summed in order, multiplied by 1 / sum; out accumulates
 * p * v over the keys in order, from 0. */
void od_window_attention(const float *q, const float *k, const float *v, int64_t T, int32_t heads,
                         int32_t head_dim, int32_t window, float scale, float *out) {
    const int64_t dim = (int64_t)heads * head_dim;
    float *scores = (float *)malloc(sizeof(float) * (size_t)(window > 0 ? window : 1));
    for (int64_t t = 0; t < T; t++) {
        const int64_t start = t + 1 > window ? t + 1 - window : 0;
        const int64_t n = t + 1 - start;
        float *o = out + t * dim;
        for (int64_t i = 0; i < dim; i++) o[i] = 0.0f;
        for (int32_t h = 0; h < heads; h++) {
            const float *qh = q + t * dim + (int64_t)h * head_dim;
            for (int64_t s = 0; s < n; s++) {
                const float *kh = k + (start + s) * dim + (int64_t)h * head_dim;
                float dot = 0.0f;
                for (int32_t d = 0; d < head_dim; d++) dot += qh[d] * kh[d];
                scores[s] = dot * scale;
            }
            float mx = -INFINITY;
            for (int64_t s = 0; s < n; s++) mx = fmaxf(mx, scores[s]);
            float sum = 0.0f;
            for (int64_t s = 0; s < n; s++) {
                scores[s] = expf(scores[s] - mx);
                sum += scores[s];
            }
            const float inv = 1.0f / sum;
            for (int64_t s = 0; s < n; s++) scores[s] *= inv;
            float *oh = o + (int64_t)h * head_dim;
            for (int64_t s = 0; s < n; s++) {
                const float *vh = v + (start + s) * dim + (int64_t)h * head_dim;
                const float p = scores[s];
                for (int32_t d = 0; d < head_dim; d++) oh[d] += p * vh[d];
            }
        }
    }
    free(scores);
}

/* The decoder MLP's activation (decoder.rs:286-296):
 * out = (g / (1 + exp(-g))) * up. */
void od_silu_mul(const float *gate, const float *up, int64_t n, float *out) {
    for (int64_t i = 0; i < n; i++) {
        const float g = gate[i];
        out[i] = (g / (1.0f + expf(-g))) * up[i];
    }
}

/* warmup_trim_len (decoder.rs:649-656): Tv / (Tv + T) of the samples, in
 * integer arithmetic, at most out_len. */
int64_t od_warmup_trim_len(int64_t tv_frames, int64_t total_frames, int64_t out_len) {
    if (total_frames == 0) return 0;
    return od_min(tv_frames * out_len / total_frames, out_len);
}

/* rvec of conv.rs's tests (conv.rs:700-711), the generator of their golden
 * vectors: xorshift64 (x ^= x << 13; x ^= x >> 7; x ^= x << 17), each value
 * ((x % 2000) / 1000 - 1) * mag in f32. */
void od_xrng_vec(uint64_t *state, int64_t n, float mag, float *out) {
    uint64_t s = *state;
    for (int64_t i = 0; i < n; i++) {
        s ^= s << 13;
        s ^= s >> 7;
        s ^= s << 17;
        out[i] = ((float)(s % 2000) / 1000.0f - 1.0f) * mag;
    }
    *state = s;
}
