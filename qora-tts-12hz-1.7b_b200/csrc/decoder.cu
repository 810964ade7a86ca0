// The speech decoder on the device: decode_to_audio (decoder.rs:395-582),
// 16 codes per 12.5 Hz frame -> 24 kHz f32 samples.
//
//   codebook lookup + output projections (decoder.rs:142-193)   [vq_dim][T]
//   pre-conv, causal k=3 (decoder.rs:433)                        [latent][T]
//   8-layer sliding-window transformer (decoder.rs:196-333)      [latent][T]
//   2 x (ConvTranspose k=2 s=2 + ConvNeXt) (decoder.rs:337-382)  [latent][4T]
//   Vocos: causal conv k=7, 4 blocks of SnakeBeta + ConvTranspose + 3
//   residual units (SnakeBeta, dilated conv k=7, SnakeBeta, conv k=1),
//   SnakeBeta + conv to one channel, clamp (decoder.rs:478-545)  [1][1920 T]
//
// Every tensor is channel-first ([channels][positions], as in the reference),
// so every convolution, linear layer and transposed convolution is one
// implicit GEMM on the CUDA cores (k_dec_conv): out[oc][t] = bias[oc] +
// sum over ic, tap of W[oc][ic][tap] * X[ic][t + tap * dil - pad], with the
// element-wise op before it (SnakeBeta, RMSNorm or LayerNorm of the input)
// applied while its input tile is staged, and the element-wise op after it
// (residual add, layer scale, GELU, SwiGLU) in its epilogue.  A transposed
// convolution with kernel k = m * stride and no padding becomes `stride`
// phase convolutions of m taps, each writing every stride-th output.  Each
// output element sums its terms in the reference's order (input channel
// ascending, then tap ascending, from the bias), with fused multiply-adds;
// the reference rounds the product and the sum separately, so results agree
// to f32 rounding, not bit for bit.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "tc.cuh"

namespace qora {
namespace {

constexpr int kCvBM = 128;      // output channels per CTA tile
constexpr int kCvBN = 128;      // positions per CTA tile
constexpr int kCvThreads = 256;
constexpr int kCvMaxHalo = 64;  // (taps - 1) * dilation
// input channels per pipeline stage: 16 for pointwise convolutions (8 K rows
// per stage would leave the stage's loads and barrier uncovered), 8 otherwise
template <int KS> constexpr int cv_bk() { return KS == 1 ? 16 : 8; }
template <int KS> constexpr int cv_halo() { return KS == 1 ? 0 : kCvMaxHalo; }
template <int KS> constexpr int cv_xper() {
    return (cv_bk<KS>() * (kCvBN + cv_halo<KS>()) + kCvThreads - 1) / kCvThreads;
}
template <int KS> constexpr int cv_smem_floats(int halo) {
    return 2 * cv_bk<KS>() * KS * kCvBM + 2 * cv_bk<KS>() * (kCvBN + halo);
}
constexpr int kCvRecvFloats = kCvBM * kCvBN;   // a K-split cluster's partial tiles (split-wide)
constexpr int kCvMaxSplit = 8;

enum DecPro { P_NONE = 0, P_SNAKE = 1, P_RMS = 2, P_LN = 3 };
enum DecEpi { E_BIAS = 0, E_RESID = 1, E_SCALE_RESID = 2, E_GELU = 3, E_SWIGLU = 4 };

struct ConvArgs {
    const float *in = nullptr;     // [ic][len]
    int64_t len = 0;               // input positions (= output positions per phase)
    const float *w = nullptr;      // [phases][ic][taps][oc_pad]
    const float *bias = nullptr;   // [oc] or null (no bias)
    float *out = nullptr;          // [oc_out][len * phases]; element (oc, j, phase p) at j * phases + p
    int ic = 0, oc = 0, oc_pad = 0, dil = 1, phases = 1;
    int ksplit = 1;                // CTAs of a cluster (blockIdx.z) splitting the input channels
    const float *pa = nullptr, *pb = nullptr;  // per input channel: SnakeBeta exp(alpha), exp(-beta);
                                               // RMSNorm gamma; LayerNorm gamma, beta
    const float *ra = nullptr, *rb = nullptr;  // per position: RMSNorm 1/rms; LayerNorm mean, 1/std
    const float *resid = nullptr;  // [oc][len * phases] (E_RESID, E_SCALE_RESID; may alias out)
    const float *escale = nullptr; // [oc] (E_SCALE_RESID)
    const uint8_t *wtc = nullptr;  // tensor-core weight image (tc_image) or null
    int *err = nullptr;            // device error flag
};

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// sin(x)^2.  sin^2 has period pi, so x is first reduced to r = x - k pi,
// k the integer nearest x / pi, by Cody and Waite's two-constant reduction
// (pi = PI_HI + PI_LO, each product taken with a fused multiply-add), which
// leaves |r| <= pi / 2 with an error far below f32 rounding for |x| < 1e5;
// there the hardware sine __sinf is within 2^-21.4 of sin(r).  Infinite or
// NaN x gives NaN, as sin does.
__device__ __forceinline__ float sin_sq(float x) {
    const float k = rintf(x * 0.318309886183790672f);
    float r = fmaf(-k, 3.14159274101257324f, x);
    r = fmaf(-k, -8.74227766e-08f, r);
    const float s = __sinf(r);
    return s * s;
}

// snake_beta (conv.rs:620-641) with a = exp(alpha), ib = exp(-beta) precomputed
// on the host: x + ib * sin(a x)^2.
__device__ __forceinline__ float snake(float x, float a, float ib) {
    return x + ib * sin_sq(a * x);
}

// gelu (conv.rs:692-694): x * 0.5 * (1 + tanh(x * 0.70710677)).
__device__ __forceinline__ float gelu_ref(float x) {
    return x * 0.5f * (1.0f + tanhf(x * 0.7071067811865476f));
}

template <int PRO>
__device__ __forceinline__ float prologue(float v, int ic, int64_t pos, const ConvArgs &a) {
    if constexpr (PRO == P_SNAKE) {
        return snake(v, __ldg(a.pa + ic), __ldg(a.pb + ic));
    } else if constexpr (PRO == P_RMS) {
        // rms_norm_f32 (decoder.rs:585-594): x * inv * gamma
        return v * __ldg(a.ra + pos) * __ldg(a.pa + ic);
    } else if constexpr (PRO == P_LN) {
        // layer_norm_channel_first (decoder.rs:678-681): (x - mean) * inv * gamma + beta
        return (v - __ldg(a.ra + pos)) * __ldg(a.rb + pos) * __ldg(a.pa + ic) + __ldg(a.pb + ic);
    } else {
        return v;
    }
}

// Implicit-GEMM convolution: one CTA per (128 positions, 128 output channels,
// phase); the phases of a position tile are adjacent CTAs (blockIdx.x =
// tile * phases + phase), so their interleaved outputs are written to the
// same L2 sectors at about the same time and their common input tile is
// read from DRAM once.  Thread (tx, ty) of the 16 x 16 grid owns output channels
// ty*4 .. +3 and 64 + ty*4 .. +3 of the tile and positions tx + 16 i
// (i = 0..7), so a warp's input reads are 16 consecutive words (broadcast to
// the two ty rows) and its weight reads two float4 broadcasts.  Weights reach
// shared memory by cp.async (one row of 128 output channels per (ic, tap)),
// input rows through registers (the prologue is applied on the way), both
// double-buffered over stages of cv_bk input channels.
template <int KS, int PRO, int EPI>
__global__ void __launch_bounds__(kCvThreads, 2) k_dec_conv(const ConvArgs a) {
    extern __shared__ float4 dsm4[];
    float *dsm = reinterpret_cast<float *>(dsm4);
    constexpr int kCvBK = cv_bk<KS>();
    constexpr int kCvXPer = cv_xper<KS>();
    constexpr int WK = kCvBK * KS;
    const int halo = (KS - 1) * a.dil;
    const int XW = kCvBN + halo;
    float *Ws = dsm;                        // [2][WK][kCvBM]
    float *Xs = dsm + 2 * WK * kCvBM;       // [2][kCvBK][XW]
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int oc0 = blockIdx.y * kCvBM;
    const int p = (int)(blockIdx.x % (unsigned)a.phases);
    const int64_t j0 = (int64_t)(blockIdx.x / (unsigned)a.phases) * kCvBN;
    const float *wp = a.w + (int64_t)p * a.ic * KS * a.oc_pad;
    // K split: cluster rank q (= blockIdx.z) takes stages [st0, st1)
    const int S = a.ksplit, q = blockIdx.z;
    const int nall = (a.ic + kCvBK - 1) / kCvBK;
    const int st0 = q * nall / S, st1 = (q + 1) * nall / S;

    auto orow = [&](int r) { return r < 4 ? ty * 4 + r : 64 + ty * 4 + (r - 4); };
    float acc[8][8];
#pragma unroll
    for (int r = 0; r < 8; r++) {
        const int oc = oc0 + orow(r);
        const float b = (EPI != E_SWIGLU && a.bias && oc < a.oc && q == 0) ? __ldg(a.bias + oc) : 0.0f;
#pragma unroll
        for (int i = 0; i < 8; i++) acc[r][i] = b;
    }

    auto load_w = [&](int st, int buf) {
        const int ic0 = st * kCvBK;
        for (int e = tid; e < WK * (kCvBM / 4); e += kCvThreads) {
            const int kk = e / (kCvBM / 4), c4 = e % (kCvBM / 4);
            const int ic = ic0 + kk / KS, k = kk % KS;
            const int oc = oc0 + c4 * 4;
            float *dst = Ws + ((int64_t)buf * WK + kk) * kCvBM + c4 * 4;
            if (ic < a.ic && oc < a.oc_pad) cp_async16(dst, wp + ((int64_t)ic * KS + k) * a.oc_pad + oc);
            else *reinterpret_cast<float4 *>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        cp_async_commit();
    };
    float xr[kCvXPer];
    auto fetch_x = [&](int st) {
        const int ic0 = st * kCvBK;
#pragma unroll
        for (int u = 0; u < kCvXPer; u++) {
            const int e = tid + u * kCvThreads;
            float v = 0.0f;
            if (e < kCvBK * XW) {
                const int icl = e / XW, col = e - icl * XW;
                const int ic = ic0 + icl;
                const int64_t pos = j0 - halo + col;
                if (ic < a.ic && pos >= 0 && pos < a.len) v = __ldg(a.in + (int64_t)ic * a.len + pos);
            }
            xr[u] = v;
        }
    };
    auto store_x = [&](int st, int buf) {
        const int ic0 = st * kCvBK;
#pragma unroll
        for (int u = 0; u < kCvXPer; u++) {
            const int e = tid + u * kCvThreads;
            if (e < kCvBK * XW) {
                const int icl = e / XW, col = e - icl * XW;
                const int ic = ic0 + icl;
                const int64_t pos = j0 - halo + col;
                float v = xr[u];
                // positions outside the input are the convolution's zero
                // padding (of the prologue's output)
                if (PRO != P_NONE && ic < a.ic && pos >= 0 && pos < a.len) v = prologue<PRO>(v, ic, pos, a);
                Xs[(int64_t)buf * kCvBK * XW + e] = v;
            }
        }
    };

    load_w(st0, 0);
    fetch_x(st0);
    store_x(st0, 0);
    cp_async_wait_all();
    __syncthreads();
    for (int st = st0; st < st1; st++) {
        const int buf = (st - st0) & 1;
        const bool more = st + 1 < st1;
        if (more) {
            load_w(st + 1, buf ^ 1);
            fetch_x(st + 1);
        }
        const float *W = Ws + (int64_t)buf * WK * kCvBM;
        const float *X = Xs + (int64_t)buf * kCvBK * XW;
#pragma unroll 2
        for (int icl = 0; icl < kCvBK; icl++) {
#pragma unroll
            for (int k = 0; k < KS; k++) {
                const float4 wa = *reinterpret_cast<const float4 *>(W + (icl * KS + k) * kCvBM + ty * 4);
                const float4 wb = *reinterpret_cast<const float4 *>(W + (icl * KS + k) * kCvBM + 64 + ty * 4);
                const float *xp = X + icl * XW + tx + k * a.dil;
                float xv[8];
#pragma unroll
                for (int i = 0; i < 8; i++) xv[i] = xp[16 * i];
                const float wr[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
                for (int r = 0; r < 8; r++)
#pragma unroll
                    for (int i = 0; i < 8; i++) acc[r][i] = fmaf(wr[r], xv[i], acc[r][i]);
            }
        }
        if (more) {
            store_x(st + 1, buf ^ 1);
            cp_async_wait_all();
        }
        __syncthreads();
    }

    const int64_t out_len = a.len * a.phases;
    // K split: rank q finishes positions tx + 16 i for i in [q * 8 / S, (q + 1) * 8 / S)
    // of the tile; every rank sends it those partial sums (distributed shared
    // memory, receive buffer [S][128 rows][128 / S positions]), which it adds
    // in rank order, rank 0's (bias-first) partial first.
    int i_lo = 0, i_hi = 8;
    if (S > 1) {
        const int per = 8 / S, cw = kCvBN / S;
        float *recv = dsm;                 // the stages' buffers are free after the loop
        asm volatile("barrier.cluster.arrive.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
#pragma unroll
        for (int r = 0; r < 8; r++)
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int owner = i / per, cl = tx + 16 * (i - owner * per);
                float *dst = recv + ((int64_t)q * kCvBM + orow(r)) * cw + cl;
                uint32_t ra;
                asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                             : "=r"(ra)
                             : "r"((uint32_t)__cvta_generic_to_shared(dst)), "r"(owner));
                asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(acc[r][i]) : "memory");
            }
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
        i_lo = q * per;
        i_hi = i_lo + per;
#pragma unroll
        for (int r = 0; r < 8; r++)
#pragma unroll
            for (int i = 0; i < 8; i++) {
                if (i < i_lo || i >= i_hi) continue;
                const int cl = tx + 16 * (i - i_lo);
                float v = 0.0f;
                for (int s2 = 0; s2 < S; s2++) v += recv[((int64_t)s2 * kCvBM + orow(r)) * cw + cl];
                acc[r][i] = v;
            }
    }
    if constexpr (EPI == E_SWIGLU) {
        // rows ty*4 + r are gate channels and 64 + ty*4 + r the matching up
        // channels of output channels blockIdx.y * 64 + ty*4 + r
        // (decoder.rs:290-295: (g / (1 + exp(-g))) * up)
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int ch = blockIdx.y * 64 + ty * 4 + r;
            if (oc0 + orow(r) >= a.oc) continue;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int64_t j = j0 + tx + 16 * i;
                if (j >= a.len || i < i_lo || i >= i_hi) continue;
                const float g = acc[r][i], u = acc[r + 4][i];
                a.out[(int64_t)ch * out_len + j] = (g / (1.0f + expf(-g))) * u;
            }
        }
    } else {
#pragma unroll
        for (int r = 0; r < 8; r++) {
            const int oc = oc0 + orow(r);
            if (oc >= a.oc) continue;
            const float sc = (EPI == E_SCALE_RESID) ? __ldg(a.escale + oc) : 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int64_t j = j0 + tx + 16 * i;
                if (j >= a.len || i < i_lo || i >= i_hi) continue;
                const int64_t o = (int64_t)oc * out_len + j * a.phases + p;
                float v = acc[r][i];
                if constexpr (EPI == E_RESID) v = v + a.resid[o];           // signal[j] += residual[j]
                if constexpr (EPI == E_SCALE_RESID) v = a.resid[o] + v * sc; // x += o * scale
                if constexpr (EPI == E_GELU) v = gelu_ref(v);
                a.out[o] = v;
            }
        }
    }
}

// Per-position statistics over the channels of x [C][L] (columns):
//   RMS: ra = 1 / sqrt(sum x^2 / C + eps)                 (rms_norm_f32, decoder.rs:585-594)
//   LN:  ra = mean, rb = 1 / sqrt(sum (x - mean)^2 / C + eps)  (decoder.rs:657-677)
// A CTA takes 32 positions; its 8 warps split the channels.
template <bool LN>
__global__ void __launch_bounds__(256) k_dec_colstats(const float *x, int C, int64_t L, float eps, float *ra,
                                                      float *rb) {
    __shared__ float part[8][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int64_t t = (int64_t)blockIdx.x * 32 + tx;
    const bool ok = t < L;
    float s = 0.0f;
    for (int c = ty; c < C; c += 8) {
        const float v = ok ? __ldg(x + (int64_t)c * L + t) : 0.0f;
        s += LN ? v : v * v;
    }
    part[ty][tx] = s;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; w++) tot += part[w][tx];
    if (!LN) {
        if (ty == 0 && ok) ra[t] = 1.0f / sqrtf(tot / (float)C + eps);
        return;
    }
    const float mean = tot / (float)C;
    __syncthreads();
    float v2 = 0.0f;
    for (int c = ty; c < C; c += 8) {
        const float d = (ok ? __ldg(x + (int64_t)c * L + t) : 0.0f) - mean;
        v2 += d * d;
    }
    part[ty][tx] = v2;
    __syncthreads();
    float var = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; w++) var += part[w][tx];
    if (ty == 0 && ok) {
        ra[t] = mean;
        rb[t] = 1.0f / sqrtf(var / (float)C + eps);
    }
}

// Codebook lookup (decoder.rs:142-193): e0[d][t] = codebook 0 row codes[0][t];
// er[d][t] = sum over g = 1..nq-1 in order of codebook g row codes[g][t]
// (from 0).  A code outside the codebook raises kDevRange and reads row 0.
__global__ void k_dec_vq(const uint32_t *codes, int64_t T, int nq, const float *cb, int size, int dim,
                         float *e0, float *er, int *err) {
    const int64_t n = (int64_t)dim * T;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int d = (int)(i / T);
        const int64_t t = i - (int64_t)d * T;
        float s = 0.0f, f = 0.0f;
        for (int g = 0; g < nq; g++) {
            uint32_t c = __ldg(codes + (int64_t)g * T + t);
            if (c >= (uint32_t)size) {
                raise_error(err, kDevRange);
                c = 0;
            }
            const float v = __ldg(cb + ((int64_t)g * size + c) * dim + d);
            if (g == 0) f = v;
            else s += v;
        }
        e0[i] = f;
        er[i] = s;
    }
}

// depthwise_conv1d (conv.rs:398-432): causal, pad = taps - 1;
// out[c][t] = bias[c] + sum over k ascending of in[c][t + k - pad] * w[c][k].
__global__ void k_dec_dwconv(const float *in, const float *w, const float *bias, int C, int ks, int64_t L,
                             float *out) {
    const int64_t n = (int64_t)C * L;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i / L);
        const int64_t t = i - (int64_t)c * L;
        float s = __ldg(bias + c);
        for (int k = 0; k < ks; k++) {
            const int64_t pos = t + k - (ks - 1);
            if (pos >= 0) s = fmaf(__ldg(in + (int64_t)c * L + pos), __ldg(w + (int64_t)c * ks + k), s);
        }
        out[i] = s;
    }
}

// The transformer's causal sliding-window attention (decoder.rs:230-284) with
// split-half RoPE (decoder.rs:624-647) applied to q and k as they are staged.
// qkv [3 * heads * 64][T] (q, k, v channel blocks); out [heads * 64][T].
// One CTA per (64 queries, head); four threads per query (keys split four
// ways for the scores, dims four ways for the output).
constexpr int kAttQ = 64;
constexpr int kAttMaxWindow = 128;
constexpr int kAttD = 64;
constexpr int kAttRow = kAttD + 1;

__global__ void __launch_bounds__(256) k_dec_attn(const float *qkv, int64_t T, int heads, int window,
                                                  float scale, const float *cos_t, const float *sin_t,
                                                  int rope_max, float *out) {
    extern __shared__ float4 asm4[];
    float *sm = reinterpret_cast<float *>(asm4);
    const int nk = kAttQ + window - 1;
    float *Qs = sm;                          // [kAttQ][kAttRow]
    float *Ks = Qs + kAttQ * kAttRow;        // [nk][kAttRow]
    float *Vs = Ks + nk * kAttRow;           // [nk][kAttRow]
    float *Ps = Vs + nk * kAttRow;           // [kAttQ][window]
    const int h = blockIdx.y;
    const int64_t t0 = (int64_t)blockIdx.x * kAttQ;
    const int64_t k0 = t0 - (window - 1);    // position of key row 0
    const int64_t HD = (int64_t)heads * kAttD;
    const float *q = qkv + (int64_t)h * kAttD * T;
    const float *k = qkv + (HD + (int64_t)h * kAttD) * T;
    const float *v = qkv + (2 * HD + (int64_t)h * kAttD) * T;
    constexpr int half = kAttD / 2;
    // stage q (rows t0 ..) and k, v (rows k0 ..), rotating the (d, d + 32) pairs
    for (int e = threadIdx.x; e < half * (kAttQ + nk); e += blockDim.x) {
        const int d = e % half, r = e / half;
        const bool isq = r < kAttQ;
        const int row = isq ? r : r - kAttQ;
        const int64_t pos = isq ? t0 + row : k0 + row;
        float x0 = 0.f, x1 = 0.f, v0 = 0.f, v1 = 0.f;
        if (pos >= 0 && pos < T) {
            const float *src = isq ? q : k;
            x0 = __ldg(src + (int64_t)d * T + pos);
            x1 = __ldg(src + (int64_t)(d + half) * T + pos);
            if (pos < rope_max) {
                const float c = __ldg(cos_t + pos * half + d), s = __ldg(sin_t + pos * half + d);
                const float y0 = x0 * c - x1 * s, y1 = x1 * c + x0 * s;
                x0 = y0;
                x1 = y1;
            }
            if (!isq) {
                v0 = __ldg(v + (int64_t)d * T + pos);
                v1 = __ldg(v + (int64_t)(d + half) * T + pos);
            }
        }
        if (isq) {
            Qs[row * kAttRow + d] = x0;
            Qs[row * kAttRow + d + half] = x1;
        } else {
            Ks[row * kAttRow + d] = x0;
            Ks[row * kAttRow + d + half] = x1;
            Vs[row * kAttRow + d] = v0;
            Vs[row * kAttRow + d + half] = v1;
        }
    }
    __syncthreads();
    const int ql = threadIdx.x >> 2, part = threadIdx.x & 3;
    const int64_t t = t0 + ql;
    // keys of query t: positions max(0, t + 1 - window) .. t, i.e. key rows
    // ql + (window - 1) - (n - 1) .. ql + window - 1
    const int64_t start = t + 1 > window ? t + 1 - window : 0;
    const int n = (int)(t + 1 - start);
    const int r0 = (int)(start - k0);
    float mx = -INFINITY;
    for (int s = part; s < n; s += 4) {
        const float *kr = Ks + (r0 + s) * kAttRow;
        const float *qr = Qs + ql * kAttRow;
        float dot = 0.0f;
#pragma unroll 16
        for (int d = 0; d < kAttD; d++) dot = fmaf(qr[d], kr[d], dot);
        const float sc = dot * scale;
        Ps[ql * window + s] = sc;
        mx = fmaxf(mx, sc);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    float sum = 0.0f;
    for (int s = part; s < n; s += 4) {
        const float e = expf(Ps[ql * window + s] - mx);
        Ps[ql * window + s] = e;
        sum += e;
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    const float inv = 1.0f / sum;
    __syncwarp();
    float o[16];
#pragma unroll
    for (int i = 0; i < 16; i++) o[i] = 0.0f;
    for (int s = 0; s < n; s++) {
        const float pw = Ps[ql * window + s] * inv;
        const float *vr = Vs + (r0 + s) * kAttRow + part * 16;
#pragma unroll
        for (int i = 0; i < 16; i++) o[i] = fmaf(pw, vr[i], o[i]);
    }
    if (t < T) {
#pragma unroll
        for (int i = 0; i < 16; i++) out[((int64_t)h * kAttD + part * 16 + i) * T + t] = o[i];
    }
}

// The output stage (decoder.rs:541-555): SnakeBeta, causal conv C -> 1
// (taps ks), clamp to [-1, 1]; samples before `skip` are dropped (the warm-up
// trim, decoder.rs:548-552).  A CTA takes 256 positions; the SnakeBeta of
// 32 channels at a time is staged in shared memory once.
constexpr int kFinT = 256;
constexpr int kFinC = 32;
constexpr int kFinMaxTaps = 16;

__global__ void __launch_bounds__(kFinT) k_dec_final(const float *in, int C, int64_t L, const float *sa,
                                                     const float *sib, const float *w, const float *bias,
                                                     int ks, int64_t skip, float *out) {
    __shared__ float S[kFinC][kFinT + kFinMaxTaps];
    const int64_t t0 = (int64_t)blockIdx.x * kFinT;
    const int64_t t = t0 + threadIdx.x;
    const int W = kFinT + ks - 1;
    float acc = __ldg(bias);
    for (int c0 = 0; c0 < C; c0 += kFinC) {
        const int cn = min(kFinC, C - c0);
        __syncthreads();
        for (int e = threadIdx.x; e < cn * W; e += blockDim.x) {
            const int cl = e / W, col = e - cl * W;
            const int64_t pos = t0 - (ks - 1) + col;
            float v = 0.0f;
            if (pos >= 0 && pos < L)
                v = snake(__ldg(in + (int64_t)(c0 + cl) * L + pos), __ldg(sa + c0 + cl), __ldg(sib + c0 + cl));
            S[cl][col] = v;
        }
        __syncthreads();
        for (int cl = 0; cl < cn; cl++)
            for (int k = 0; k < ks; k++) acc = fmaf(S[cl][threadIdx.x + k], __ldg(w + (int64_t)(c0 + cl) * ks + k), acc);
    }
    // f32::clamp(-1, 1): a NaN stays NaN
    if (t < L && t >= skip) out[t - skip] = acc < -1.0f ? -1.0f : (acc > 1.0f ? 1.0f : acc);
}

// ----------------------------------------------------------------------
// The same implicit-GEMM convolution on the tcgen05 tensor cores, f32-exact
// to within f32 rounding: both operands are split into TF32 hi + lo parts
// (hi = x rounded to TF32, lo = x - hi rounded to TF32, so hi + lo carries
// 22 significant bits) and each term is the three products hi*hi + hi*lo +
// lo*hi.  The tensor core's accumulation into tensor memory does not round
// to nearest, and its error grows with the number of MMAs accumulated into
// one accumulator; so the MMAs of each chunk of stages (about 60 MMAs)
// accumulate into one of two tensor-memory buffers, and the epilogue warps
// add each chunk into f32 registers (round to nearest) while the next chunk
// runs in the other buffer.  One CTA computes 128 output channels x 256
// positions (one phase of a transposed convolution).
//
// A pipeline stage holds BK input channels (BK / 4 K groups of 4): 16 for
// pointwise convolutions (their stages are short, so fewer, longer stages
// keep the converters' per-stage round trip off the tensor cores), 8
// otherwise.  Operands in shared memory, canonical K-major layout without
// swizzle (8-row x 16-byte core matrices; rows 16 bytes apart, K groups of
// 4 TF32 values `LBO` apart):
//   A (weights) per stage and tap: [hi, lo][BK / 4 K groups][128 rows][4],
//     LBO 2048, arriving as one bulk copy per stage from an image prepared
//     on upload (tc_image below);
//   B (inputs) per stage: [hi, lo][BK / 4 K groups][256 + halo rows][4], LBO
//     16 * (256 + 56) (16 * 256 for pointwise convolutions), row n =
//     position j0 - halo + n, written by the converter warps (prologue
//     applied, hi / lo split).  Tap t reads rows t * dil .. t * dil + 255:
//     its descriptor starts t * dil * 16 bytes in; K step j (8 channels)
//     starts 2 j K groups in.
// Warp roles (544 threads): warps 0-15 stage B, add the chunks into
// registers (64 running sums per thread) and run the epilogue; warp 16
// allocates tensor memory and its lane 0 issues the A bulk copies and the
// MMAs (K = 8 per MMA).  Every wait is bounded (kDevTimeout, then a CTA-wide
// abort).
constexpr int kTcOc = 128;
constexpr int kTcPos = 256;
constexpr int kTcBK = 8;                              // channels per MMA (K = 8 TF32)
constexpr int kTcConvWarps = 16;
constexpr int kTcThreads = (kTcConvWarps + 1) * 32;
// tensor-core halo limit: 56 rows (the real decoder's largest is 6 x 9 = 54)
// keeps three 7-tap stages within the 227 KB of shared memory a CTA may use;
// a convolution with a longer halo runs on the CUDA-core kernel
constexpr int kTcMaxHalo = 56;
constexpr int kTcRowsB = kTcPos + kTcMaxHalo;
constexpr uint32_t kTcALbo = kTcOc * 16;              // 2048
// input channels per stage, and the layout sizes that follow from it
__host__ __device__ constexpr int tc_bk_of(int ks) { return ks == 1 ? 16 : 8; }
template <int KS> constexpr int tc_bk() { return tc_bk_of(KS); }
template <int KS> constexpr int tc_rows() { return KS == 1 ? kTcPos : kTcRowsB; }
template <int KS> constexpr uint32_t tc_atap() { return 2u * (tc_bk<KS>() / 4) * kTcALbo; }  // bytes per tap
template <int KS> constexpr uint32_t tc_blbo() { return (uint32_t)tc_rows<KS>() * 16u; }
template <int KS> constexpr uint32_t tc_bhalf() { return (uint32_t)(tc_bk<KS>() / 4) * tc_blbo<KS>(); }
template <int KS> constexpr uint32_t tc_bbytes() { return 2u * tc_bhalf<KS>(); }  // hi part, then lo part
constexpr uint32_t kTcTmemCols = 2 * kTcPos;          // two accumulators
constexpr size_t kTcMinSmem = 120 * 1024;             // one CTA per SM (all of tensor memory)
constexpr size_t kTcMaxSmem = 227 * 1024;             // dynamic + static shared memory of a CTA
constexpr size_t kTcAlign = 128;                      // stage buffers start 128-byte aligned
constexpr size_t kTcStatic = 256;                     // the kernel's barriers and flags, rounded up
template <int KS> constexpr uint32_t tc_stage_bytes() { return KS * tc_atap<KS>() + tc_bbytes<KS>(); }
// pipeline depth: as many stages as fit, up to 4 (7 taps: 3)
template <int KS> constexpr int tc_stages() {
    return (kTcMaxSmem - kTcAlign - kTcStatic) / tc_stage_bytes<KS>() < 4
               ? (int)((kTcMaxSmem - kTcAlign - kTcStatic) / tc_stage_bytes<KS>())
               : 4;
}
// stages per accumulation chunk: about 64 MMAs (3 per tap and 8 channels)
template <int KS> constexpr int tc_chunk() {
    return (64 / (3 * KS * (tc_bk<KS>() / kTcBK))) > 1 ? 64 / (3 * KS * (tc_bk<KS>() / kTcBK)) : 1;
}
template <int KS> constexpr size_t tc_smem() {
    return (size_t)tc_stages<KS>() * tc_stage_bytes<KS>() + kTcAlign > kTcMinSmem
               ? (size_t)tc_stages<KS>() * tc_stage_bytes<KS>() + kTcAlign
               : kTcMinSmem;
}
static_assert(tc_stages<7>() >= 3, "three 7-tap stages fit");
static_assert(tc_smem<7>() + kTcStatic <= kTcMaxSmem, "shared memory of a CTA");
static_assert(kTcRowsB % 8 == 0 && tc_stage_bytes<7>() % 16 == 0, "16-byte rows, 8-row core matrices");
static_assert(tc_stages<1>() == 4 && tc_smem<1>() + kTcStatic <= kTcMaxSmem, "four pointwise stages fit");
static_assert(tc_stage_bytes<1>() == 49152 && tc_stage_bytes<2>() == 36352 && tc_stage_bytes<7>() == 77312,
              "stage sizes");

__host__ __device__ constexpr uint32_t idesc_tf32_f32(int M, int N) {
    return (1u << 4)                     // D: f32
           | (2u << 7) | (2u << 10)      // A, B: TF32, both K-major
           | ((uint32_t)(N >> 3) << 17)  // N / 8
           | ((uint32_t)(M >> 4) << 24); // M / 16
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// x rounded to TF32 (nearest, ties away from zero), as a 32-bit pattern.
__device__ __forceinline__ uint32_t to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

template <int KS, int PRO, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1) k_dec_conv_tc(const ConvArgs a, const uint8_t *aimg) {
    constexpr int NS = tc_stages<KS>();
    constexpr int CH = tc_chunk<KS>();
    constexpr uint32_t SB = tc_stage_bytes<KS>();
    constexpr int BK = tc_bk<KS>(), KG = BK / 4;
    constexpr uint32_t ATAP = tc_atap<KS>(), BLBO = tc_blbo<KS>(), BHALF = tc_bhalf<KS>();
    constexpr uint32_t ABYTES = KS * ATAP;
    extern __shared__ uint8_t tc_raw[];
    __shared__ __align__(8) uint64_t a_full[NS], b_full[NS], s_empty[NS], d_full[2], d_empty[2];
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_s;
    uint8_t *sm = reinterpret_cast<uint8_t *>(((uintptr_t)tc_raw + (kTcAlign - 1)) & ~(uintptr_t)(kTcAlign - 1));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // one-dimensional grid, output-channel tile fastest, then phase, then
    // position tile: the CTAs that read the same input tile run together
    const int n_oct = (a.oc + kTcOc - 1) / kTcOc;
    const int oct = (int)(blockIdx.x % (unsigned)n_oct);
    const unsigned rest = blockIdx.x / (unsigned)n_oct;
    const int p = (int)(rest % (unsigned)a.phases);
    const int64_t j0 = (int64_t)(rest / (unsigned)a.phases) * kTcPos;
    const int oc0 = oct * kTcOc;
    const int halo = (KS - 1) * a.dil;
    const int nst = (a.ic + BK - 1) / BK;
    const uint8_t *aimg_t = aimg + ((int64_t)p * n_oct + oct) * nst * (int64_t)ABYTES;
    volatile int *abort_v = &abort_s;

    if (tid == 0) {
        for (int i = 0; i < NS; i++) {
            mbar_init(&a_full[i], 1);
            mbar_init(&b_full[i], kTcConvWarps);
            mbar_init(&s_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&d_full[i], 1);
            mbar_init(&d_empty[i], kTcConvWarps);
        }
        abort_s = 0;
        mbar_fence_init();
    }
    if (warp == kTcConvWarps) {
        tc::tmem_alloc(&tmem_slot, kTcTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (mbar_try_wait(bar, parity)) return true;
        const long long t0 = clock64();
        for (uint32_t i = 1;; i++) {
            if (mbar_try_wait(bar, parity)) return true;
            if ((i & 31) == 0) {
                if (*abort_v) return false;
                if (clock64() - t0 > (1ll << 31)) {
                    raise_error(a.err, kDevTimeout);
                    *abort_v = 1;
                    return false;
                }
            }
        }
    };

    if (warp == kTcConvWarps) {
        if (lane == 0) {
            // ------------------------------------------------ A copies + MMAs
            auto issue_a = [&](int s) {
                const int buf = s % NS;
                mbar_arrive_expect_tx(&a_full[buf], ABYTES);
                bulk_g2s(sm + buf * SB, aimg_t + (int64_t)s * ABYTES, ABYTES, &a_full[buf]);
            };
            int issued = 0, used = 0;
            for (; issued < min(NS, nst); issued++) issue_a(issued);
            constexpr uint32_t idesc = idesc_tf32_f32(kTcOc, kTcPos);
            for (int s = 0; s < nst; s++) {
                const int buf = s % NS, c = s / CH;
                const bool first = s % CH == 0;
                if (!wait(&a_full[buf], (s / NS) & 1)) break;
                used = s + 1;
                if (!wait(&b_full[buf], (s / NS) & 1)) break;
                // chunk c reuses the accumulator of chunk c - 2 once it is added up
                if (first && c >= 2 && !wait(&d_empty[c & 1], ((c >> 1) - 1) & 1)) break;
                tc::fence_after_sync();
                const uint32_t d = tmem + (uint32_t)(c & 1) * kTcPos;
                const uint32_t sA = smem_u32(sm + buf * SB), sB = sA + ABYTES;
#pragma unroll
                for (int t = 0; t < KS; t++) {
#pragma unroll
                    for (int j = 0; j < BK / kTcBK; j++) {
                        const uint32_t ak = sA + t * ATAP + j * 2 * kTcALbo;
                        const uint64_t ah = tc::smem_desc(ak, kTcALbo, 128);
                        const uint64_t al = tc::smem_desc(ak + ATAP / 2, kTcALbo, 128);
                        const uint32_t boff = (uint32_t)(t * a.dil) * 16u + (uint32_t)j * 2u * BLBO;
                        const uint64_t bh = tc::smem_desc(sB + boff, BLBO, 128);
                        const uint64_t bl = tc::smem_desc(sB + BHALF + boff, BLBO, 128);
                        mma_tf32(d, ah, bh, idesc, (first && t == 0 && j == 0) ? 0u : 1u);
                        mma_tf32(d, ah, bl, idesc, 1u);
                        mma_tf32(d, al, bh, idesc, 1u);
                    }
                }
                tc::commit(&s_empty[buf]);
                if (s % CH == CH - 1 || s == nst - 1) tc::commit(&d_full[c & 1]);
                // refill the previous stage's buffer once its MMAs are done
                // (the ones just issued queue behind them)
                if (s >= 1 && issued < nst) {
                    if (!wait(&s_empty[(s - 1) % NS], ((s - 1) / NS) & 1)) break;
                    issue_a(issued++);
                }
            }
            // every A copy issued lands before the CTA can exit
            for (int s = used; s < issued; s++) {
                const int buf = s % NS;
                const uint64_t t0 = global_ns();
                while (!mbar_try_wait(&a_full[buf], (s / NS) & 1) && global_ns() - t0 < 1000000000ull) {
                }
            }
        }
        __syncwarp();
    } else {
        // warp w owns tensor-memory lanes 32 (w % 4) .. + 31 (output channels)
        // and columns 64 (w / 4) .. + 63 (positions) of each accumulator
        constexpr int kCols = kTcPos / (kTcConvWarps / 4);
        const int lg = warp & 3, quarter = warp >> 2;
        float accr[kCols];
#pragma unroll
        for (int i = 0; i < kCols; i++) accr[i] = 0.0f;
        auto drain = [&](int c) {
            const bool ok = wait(&d_full[c & 1], (c >> 1) & 1);
            tc::fence_after_sync();
            if (ok) {
                const uint32_t base =
                    tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)(c & 1) * kTcPos + quarter * kCols;
#pragma unroll
                for (int q = 0; q < kCols / 32; q++) {
                    float v[32];
                    tc::ld_32x32b_x32(base + q * 32, v);
#pragma unroll
                    for (int i = 0; i < 32; i++) accr[q * 32 + i] += v[i];
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d_empty[c & 1]);
        };
        // ---------------------------------------------------- B staging
        // item (K group kg, row n): 4 input channels at one position.  A
        // thread's items are the same every stage, so their geometry is
        // worked out once; a stage's raw values are loaded into registers
        // one stage ahead, so their latency passes while the converters wait
        // for a free buffer.
        constexpr int kItems = (KG * tc_rows<KS>() + kTcConvWarps * 32 - 1) / (kTcConvWarps * 32);
        const int rows = kTcPos + halo;
        int it_kg[kItems], it_soff[kItems];
        int64_t it_pos[kItems];
        bool it_on[kItems], it_in[kItems];
#pragma unroll
        for (int q = 0; q < kItems; q++) {
            const int it = tid + q * kTcConvWarps * 32;
            const int kg = KG == 2 ? (it >= rows ? 1 : 0) : min(it / rows, KG - 1), n = it - kg * rows;
            it_on[q] = it < KG * rows;
            it_kg[q] = kg;
            it_soff[q] = kg * (int)BLBO + n * 16;
            it_pos[q] = j0 - halo + n;
            it_in[q] = it_on[q] && it_pos[q] >= 0 && it_pos[q] < a.len;
        }
        float raw[kItems][4];
        auto fetch = [&](int s) {
            const int ic0 = s * BK;
#pragma unroll
            for (int q = 0; q < kItems; q++) {
                const float *src = a.in + (int64_t)(ic0 + 4 * it_kg[q]) * a.len + it_pos[q];
#pragma unroll
                for (int u = 0; u < 4; u++)
                    raw[q][u] = (it_in[q] && ic0 + 4 * it_kg[q] + u < a.ic) ? __ldg(src + (int64_t)u * a.len) : 0.0f;
            }
        };
        fetch(0);
        for (int s = 0; s < nst; s++) {
            const int buf = s % NS;
            if (s >= NS && !wait(&s_empty[buf], ((s / NS) - 1) & 1)) break;
            uint8_t *B = sm + buf * SB + ABYTES;
            const int ic0 = s * BK;
            // the stage's per-channel prologue constants: all 8 channels of an
            // 8-channel stage, or the 4 of each item's K group of a 16-channel one
            constexpr bool kPerItem = KG > 2;
            float ca[kPerItem ? 1 : 8], cb[kPerItem ? 1 : 8];
            float ia[kPerItem ? kItems : 1][4], ib[kPerItem ? kItems : 1][4];
            if constexpr (kPerItem) {
#pragma unroll
                for (int q = 0; q < kItems; q++)
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int ic = min(ic0 + 4 * it_kg[q] + u, a.ic - 1);
                        ia[q][u] = (PRO == P_SNAKE || PRO == P_RMS || PRO == P_LN) ? __ldg(a.pa + ic) : 0.0f;
                        ib[q][u] = (PRO == P_SNAKE || PRO == P_LN) ? __ldg(a.pb + ic) : 0.0f;
                    }
            } else {
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const int ic = min(ic0 + u, a.ic - 1);
                    ca[u] = (PRO == P_SNAKE || PRO == P_RMS || PRO == P_LN) ? __ldg(a.pa + ic) : 0.0f;
                    cb[u] = (PRO == P_SNAKE || PRO == P_LN) ? __ldg(a.pb + ic) : 0.0f;
                }
            }
#pragma unroll
            for (int q = 0; q < kItems; q++) {
                if (!it_on[q]) continue;
                float ra = 0.0f, rb = 0.0f;
                if ((PRO == P_RMS || PRO == P_LN) && it_in[q]) {
                    ra = __ldg(a.ra + it_pos[q]);
                    if (PRO == P_LN) rb = __ldg(a.rb + it_pos[q]);
                }
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    float v = raw[q][u];
                    const int cu = 4 * it_kg[q] + u;
                    // positions outside the input are the convolution's zero padding
                    if (it_in[q] && ic0 + cu < a.ic) {
                        float pa, pb;
                        if constexpr (kPerItem) {
                            pa = ia[q][u];
                            pb = ib[q][u];
                        } else {
                            pa = it_kg[q] ? ca[4 + u] : ca[u];
                            pb = it_kg[q] ? cb[4 + u] : cb[u];
                        }
                        if constexpr (PRO == P_SNAKE) v = snake(v, pa, pb);
                        if constexpr (PRO == P_RMS) v = v * ra * pa;
                        if constexpr (PRO == P_LN) v = (v - ra) * rb * pa + pb;
                    }
                    hi[u] = to_tf32(v);
                    lo[u] = to_tf32(v - __uint_as_float(hi[u]));
                }
                *reinterpret_cast<uint4 *>(B + it_soff[q]) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4 *>(B + BHALF + it_soff[q]) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&b_full[buf]);
            if (s + 1 < nst) fetch(s + 1);
            // the previous chunk is added up while this one runs
            if (s > 0 && s % CH == 0) drain(s / CH - 1);
        }
        drain((nst - 1) / CH);
        // ---------------------------------------------------- epilogue
        // 32 columns at a time, transposed through shared memory (the stage
        // buffers are idle now) so that a warp's stores run along positions
        float *scr = reinterpret_cast<float *>(sm) + warp * (32 * 33);
        const int64_t out_len = a.len * a.phases;
#pragma unroll
        for (int q = 0; q < kCols / 32; q++) {
            const int col0 = quarter * kCols + q * 32;
#pragma unroll
            for (int i = 0; i < 32; i++) scr[lane * 33 + i] = accr[q * 32 + i];
            __syncwarp();
            const int64_t j = j0 + col0 + lane;
            // the residuals of the 32 rows are loaded together, then combined
            float rv[32];
#pragma unroll
            for (int rr = 0; rr < 32; rr++) {
                const int oc = oc0 + lg * 32 + rr;
                rv[rr] = 0.0f;
                if ((EPI == E_RESID || EPI == E_SCALE_RESID) && oc < a.oc && j < a.len)
                    rv[rr] = a.resid[(int64_t)oc * out_len + j * a.phases + p];
            }
#pragma unroll
            for (int rr = 0; rr < 32; rr++) {
                const int oc = oc0 + lg * 32 + rr;
                if (oc >= a.oc || j >= a.len) continue;
                const int64_t o = (int64_t)oc * out_len + j * a.phases + p;
                float x = scr[rr * 33 + lane];
                if (a.bias) x = __ldg(a.bias + oc) + x;
                if constexpr (EPI == E_RESID) x = x + rv[rr];
                if constexpr (EPI == E_SCALE_RESID) x = rv[rr] + x * __ldg(a.escale + oc);
                if constexpr (EPI == E_GELU) x = gelu_ref(x);
                a.out[o] = x;
            }
            __syncwarp();
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == kTcConvWarps) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTcTmemCols);
    }
}

}  // namespace
}  // namespace qora

// ====================================================================== host
namespace qora {
namespace {

struct DecLayer {
    DevBuf qkv_w, o_w, gu_w, down_w, in_norm, post_norm, attn_scale, mlp_scale;
};
// *_tc: the same weights as tensor-core images (tc_image)
struct DecUpsample {
    DevBuf ct_w, ct_b, dw_w, dw_b, ln_w, ln_b, pw1_w, pw1_b, pw2_w, pw2_b, gamma, ct_tc, pw1_tc, pw2_tc;
};
struct DecResidual {
    DevBuf a1, ib1, c1_w, c1_b, a2, ib2, c2_w, c2_b, c1_tc, c2_tc;
};
struct DecBlock {
    DevBuf pre_a, pre_ib, ct_w, ct_b, ct_tc;
    DecResidual res[3];
};

constexpr int kResDilations[3] = {1, 3, 9};  // loader.rs:622
constexpr int kPreTaps = 3, kVocosTaps = 7, kDwTaps = 7, kFinalTaps = 7;
constexpr int kUpKernel = 2, kUpStride = 2;   // loader.rs:587-588
constexpr float kDecEps = 1e-5f;              // decoder.rs:229, 288, 309, 346

int64_t round4(int64_t v) { return (v + 3) & ~int64_t(3); }

}  // namespace
}  // namespace qora

struct qora_decoder {
    qora::CtxRef ctx;
    qora_decoder_dims d{};
    std::map<std::string, std::vector<int64_t>> shapes;   // expected checkpoint tensors
    std::map<std::string, std::vector<float>> host;       // staged until finalize
    bool ready = false;
    int64_t hop = 0;                                       // samples per frame
    qora::DevBuf cb, vq_w0, vq_wr, pre_w, pre_b, in_w, in_b, norm_w, out_w, out_b, rope_cos, rope_sin;
    std::vector<qora::DecLayer> layers;
    std::vector<qora::DecUpsample> ups;
    qora::DevBuf init_w, init_b, init_tc, fin_a, fin_ib, fin_w, fin_b;
    int tc_mode = 1;   // tensor-core convolutions: 0 never, 1 when the grid fills the GPU, 2 always
    std::vector<qora::DecBlock> blocks;
    // workspace for `ws_frames` frames
    int64_t ws_frames = 0;
    qora::DevBuf e0, er, vq, pre, x, qkv, att, h, tfo, ra, rb, big[3];
    int64_t io_frames = 0, io_samples = 0;
    qora::DevBuf codes_dev, samples_dev;
};

namespace qora {
namespace {

int g_sms[64];   // SM count per device (set when a decoder is created)

template <int KS, int PRO, int EPI>
int launch_conv_t(const ConvArgs &a, int device, cudaStream_t st) {
    static std::atomic<uint64_t> attr_done{0};
    const int halo = (KS - 1) * a.dil;
    if (halo > cv_halo<KS>()) return set_error(QORA_ERR_UNSUPPORTED, "convolution halo %d > %d", halo, cv_halo<KS>());
    size_t smem = (size_t)cv_smem_floats<KS>(halo) * sizeof(float);
    if (a.ksplit > 1) smem = std::max<size_t>(smem, (size_t)kCvRecvFloats * sizeof(float));
    const uint64_t bit = 1ull << (device & 63);
    if (!(attr_done.load() & bit)) {
        const int max_smem = std::max(cv_smem_floats<KS>(cv_halo<KS>()), kCvRecvFloats) * (int)sizeof(float);
        QORA_CUDA(cudaFuncSetAttribute(k_dec_conv<KS, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       max_smem));
        attr_done.fetch_or(bit);
    }
    const int64_t gx = (a.len + kCvBN - 1) / kCvBN * a.phases;
    const int gy = (a.oc + kCvBM - 1) / kCvBM;
    if (gx > INT32_MAX || gy > 65535) return set_error(QORA_ERR_SHAPE, "convolution too long");
    if (a.ksplit == 1) {
        k_dec_conv<KS, PRO, EPI><<<dim3((unsigned)gx, gy, 1), kCvThreads, smem, st>>>(a);
    } else {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)gx, gy, a.ksplit);
        cfg.blockDim = dim3(kCvThreads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 1;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = a.ksplit;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        QORA_CUDA(cudaLaunchKernelEx(&cfg, k_dec_conv<KS, PRO, EPI>, a));
    }
    QORA_LAUNCH_CHECK();
    return QORA_OK;
}

// One k_dec_conv_tc launch: output-channel tiles x phases x position tiles,
// one CTA per SM (all of tensor memory each).
template <int KS, int PRO, int EPI>
int launch_conv_tc_t(const ConvArgs &a, int device, cudaStream_t st) {
    static std::atomic<uint64_t> attr_done{0};
    if ((KS - 1) * a.dil > kTcMaxHalo) return set_error(QORA_ERR_UNSUPPORTED, "convolution halo too large");
    const uint64_t bit = 1ull << (device & 63);
    if (!(attr_done.load() & bit)) {
        QORA_CUDA(cudaFuncSetAttribute(k_dec_conv_tc<KS, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)tc_smem<KS>()));
        attr_done.fetch_or(bit);
    }
    const int64_t gx = (a.len + kTcPos - 1) / kTcPos * a.phases;
    const int gy = (a.oc + kTcOc - 1) / kTcOc;
    if (gx > INT32_MAX || gy > 65535) return set_error(QORA_ERR_SHAPE, "convolution too long");
    if (gx * gy > INT32_MAX) return set_error(QORA_ERR_SHAPE, "convolution too long");
    k_dec_conv_tc<KS, PRO, EPI><<<dim3((unsigned)(gx * gy), 1, 1), kTcThreads, tc_smem<KS>(), st>>>(a, a.wtc);
    QORA_LAUNCH_CHECK();
    return QORA_OK;
}

// K split of a convolution whose tiles fill less than one wave of two CTAs
// per SM (the transformer's projections over a few hundred frames): the
// largest power of two up to 8 that keeps the grid within that wave and
// leaves each split at least two stages.
int choose_split(int taps, const ConvArgs &a, int sms) {
    if (a.phases != 1) return 1;
    const int bk = taps == 1 ? 16 : 8;
    const int64_t tiles = (a.len + kCvBN - 1) / kCvBN * ((a.oc + kCvBM - 1) / kCvBM);
    const int nall = (a.ic + bk - 1) / bk;
    int S = 1;
    while (S < kCvMaxSplit && tiles * 2 * S <= 2 * (int64_t)sms && nall >= 2 * 2 * S) S *= 2;
    return S;
}

int launch_conv(int taps, int pro, int epi, const ConvArgs &a0, int device, cudaStream_t st, int tc_mode, int *err) {
    ConvArgs a = a0;
    a.err = err;
    if (a.wtc && tc_mode != 0 && epi != E_SWIGLU && (taps - 1) * a.dil <= kTcMaxHalo) {
        // mode 1: the kernel with the smaller estimated time, from B200
        // measurements of both (tensor cores: about 2.0 + 0.12 x taps us per
        // 8 input channels per CTA, in waves of one CTA per SM; CUDA cores:
        // about 28 TFLOP/s (14 for pointwise convolutions, which stream
        // their input and residual) plus 10 us)
        const int sms = g_sms[device & 63];
        const int64_t tiles = (a.len + kTcPos - 1) / kTcPos * ((a.oc + kTcOc - 1) / kTcOc) * a.phases;
        const int64_t nst = (a.ic + kTcBK - 1) / kTcBK;
        const double t_tc = (double)((tiles + sms - 1) / sms) * (double)nst * (2.0 + 0.12 * taps);
        const double t_simt =
            2.0 * a.ic * taps * (double)a.oc * a.len * a.phases / (taps == 1 ? 14e6 : 28e6) + 10.0;
        if (tc_mode == 2 || t_tc < t_simt) {
#define QORA_TC_CASE(K, P, E) \
    if (taps == K && pro == P && epi == E) return launch_conv_tc_t<K, P, E>(a, device, st)
            QORA_TC_CASE(7, P_NONE, E_BIAS);      // Vocos input conv
            QORA_TC_CASE(1, P_NONE, E_BIAS);      // upsample transposed conv
            QORA_TC_CASE(1, P_LN, E_GELU);        // ConvNeXt pwconv1
            QORA_TC_CASE(1, P_NONE, E_SCALE_RESID);  // ConvNeXt pwconv2
            QORA_TC_CASE(1, P_SNAKE, E_BIAS);     // Vocos transposed conv (kernel = stride)
            QORA_TC_CASE(2, P_SNAKE, E_BIAS);     // Vocos transposed conv (kernel = 2 x stride)
            QORA_TC_CASE(7, P_SNAKE, E_BIAS);     // residual conv1
            QORA_TC_CASE(1, P_SNAKE, E_RESID);    // residual conv2
#undef QORA_TC_CASE
        }
    }
    a.wtc = nullptr;
    a.ksplit = choose_split(taps, a, g_sms[device & 63]);
#define QORA_CONV_CASE(K, P, E) \
    if (taps == K && pro == P && epi == E) return launch_conv_t<K, P, E>(a, device, st)
    QORA_CONV_CASE(1, P_NONE, E_BIAS);          // codebook projection, input projection
    QORA_CONV_CASE(1, P_NONE, E_RESID);         // second codebook projection
    QORA_CONV_CASE(3, P_NONE, E_BIAS);          // pre-conv
    QORA_CONV_CASE(1, P_RMS, E_BIAS);           // q/k/v, output projection
    QORA_CONV_CASE(1, P_NONE, E_SCALE_RESID);   // o / down (layer scale), ConvNeXt pwconv2 (gamma)
    QORA_CONV_CASE(1, P_RMS, E_SWIGLU);         // gate / up
    QORA_CONV_CASE(1, P_LN, E_GELU);            // ConvNeXt pwconv1
    QORA_CONV_CASE(7, P_NONE, E_BIAS);          // Vocos input conv
    QORA_CONV_CASE(1, P_SNAKE, E_BIAS);         // Vocos transposed conv (kernel = stride)
    QORA_CONV_CASE(2, P_SNAKE, E_BIAS);         // Vocos transposed conv (kernel = 2 x stride)
    QORA_CONV_CASE(7, P_SNAKE, E_BIAS);         // residual conv1
    QORA_CONV_CASE(1, P_SNAKE, E_RESID);        // residual conv2
#undef QORA_CONV_CASE
    return set_error(QORA_ERR_UNSUPPORTED, "decoder convolution taps=%d prologue=%d epilogue=%d", taps, pro, epi);
}

// ------------------------------------------------------------ weight layouts
// Conv1d [oc][ic][k] -> [ic][k][oc_pad] (a row of output channels per (ic, tap)).
std::vector<float> conv_layout(const float *w, int64_t oc, int64_t ic, int64_t k) {
    const int64_t ocp = round4(oc);
    std::vector<float> o((size_t)(ic * k * ocp), 0.0f);
    for (int64_t a = 0; a < oc; a++)
        for (int64_t b = 0; b < ic; b++)
            for (int64_t t = 0; t < k; t++) o[(size_t)((b * k + t) * ocp + a)] = w[(a * ic + b) * k + t];
    return o;
}

// ConvTranspose1d [ic][oc][k] with k = m * s, no padding, right-cropped by
// k - s (decoder.rs:462-474): phase p of output o = s j + p sums, for ic
// ascending, input positions i = j - m + 1 .. j ascending of
// in[ic][i] * w[ic][oc][p + s (j - i)]; as a causal conv of m taps, tap
// q = 0..m-1 reads in[j - (m - 1) + q] with weight w[..][p + s (m - 1 - q)].
// Layout [s][ic][m][oc_pad].
std::vector<float> convt_layout(const float *w, int64_t ic, int64_t oc, int64_t k, int64_t s) {
    const int64_t m = k / s, ocp = round4(oc);
    std::vector<float> o((size_t)(s * ic * m * ocp), 0.0f);
    for (int64_t p = 0; p < s; p++)
        for (int64_t b = 0; b < ic; b++)
            for (int64_t q = 0; q < m; q++)
                for (int64_t a = 0; a < oc; a++)
                    o[(size_t)(((p * ic + b) * m + q) * ocp + a)] = w[(b * oc + a) * k + p + s * (m - 1 - q)];
    return o;
}

// f32 -> TF32 (nearest, ties away from zero) as the f32 it represents;
// infinities and NaNs unchanged.
float tf32_rna(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0x1000u) & 0xFFFFE000u;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

// Tensor-core image of a convolution's weights wl [phases][ic][taps][oc_pad]
// (conv_layout / convt_layout): per (phase, 128-channel tile, stage of BK
// input channels, tap) the A operand of k_dec_conv_tc as it lies in shared
// memory, [hi, lo][BK / 4 K groups][128 rows][4 values], zero outside the
// weights; a stage's taps are contiguous, so one bulk copy loads a stage.
std::vector<float> tc_image(const std::vector<float> &wl, int64_t phases, int64_t ic, int64_t oc, int64_t ks) {
    const int bk = tc_bk_of((int)ks), kgs = bk / 4;
    const int64_t ocp = round4(oc), tiles = (oc + kTcOc - 1) / kTcOc, nst = (ic + bk - 1) / bk;
    std::vector<float> img((size_t)(phases * tiles * nst * ks * 2 * kgs * kTcOc * 4), 0.0f);
    size_t idx = 0;
    for (int64_t p = 0; p < phases; p++)
        for (int64_t ot = 0; ot < tiles; ot++)
            for (int64_t st = 0; st < nst; st++)
                for (int64_t t = 0; t < ks; t++)
                    for (int h = 0; h < 2; h++)
                        for (int kg = 0; kg < kgs; kg++)
                            for (int64_t row = 0; row < kTcOc; row++)
                                for (int u = 0; u < 4; u++, idx++) {
                                    const int64_t c = st * bk + 4 * kg + u, o = ot * kTcOc + row;
                                    if (c >= ic || o >= oc) continue;
                                    const float w = wl[(size_t)(((p * ic + c) * ks + t) * ocp + o)];
                                    const float hi = tf32_rna(w);
                                    img[idx] = h == 0 ? hi : tf32_rna(w - hi);
                                }
    return img;
}

int upload(DevBuf &buf, const std::vector<float> &v) {
    QORA_TRY(buf.alloc(v.size() * sizeof(float)));
    if (!v.empty()) QORA_CUDA(cudaMemcpy(buf.p, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice));
    return QORA_OK;
}

void add_shape(qora_decoder *dec, const std::string &name, std::vector<int64_t> shape) {
    dec->shapes[name] = std::move(shape);
}

// The checkpoint tensors load_speech_decoder reads (loader.rs:503-716).
void build_shapes(qora_decoder *dec) {
    const qora_decoder_dims &d = dec->d;
    const std::string q = "decoder.quantizer.";
    const int64_t HD = (int64_t)d.num_heads * d.head_dim;
    add_shape(dec, q + "rvq_first.vq.layers.0._codebook.embedding_sum", {d.codebook_size, d.codebook_dim});
    add_shape(dec, q + "rvq_first.vq.layers.0._codebook.cluster_usage", {d.codebook_size});
    add_shape(dec, q + "rvq_first.output_proj.weight", {d.vq_dim, d.codebook_dim, 1});
    for (int g = 0; g < d.num_quantizers - 1; g++) {
        const std::string c = q + "rvq_rest.vq.layers." + std::to_string(g) + "._codebook.";
        add_shape(dec, c + "embedding_sum", {d.codebook_size, d.codebook_dim});
        add_shape(dec, c + "cluster_usage", {d.codebook_size});
    }
    add_shape(dec, q + "rvq_rest.output_proj.weight", {d.vq_dim, d.codebook_dim, 1});
    add_shape(dec, "decoder.pre_conv.conv.weight", {d.latent, d.vq_dim, kPreTaps});
    add_shape(dec, "decoder.pre_conv.conv.bias", {d.latent});
    const std::string t = "decoder.pre_transformer.";
    add_shape(dec, t + "input_proj.weight", {d.hidden, d.latent});
    add_shape(dec, t + "input_proj.bias", {d.hidden});
    add_shape(dec, t + "output_proj.weight", {d.latent, d.hidden});
    add_shape(dec, t + "output_proj.bias", {d.latent});
    add_shape(dec, t + "norm.weight", {d.hidden});
    for (int i = 0; i < d.num_layers; i++) {
        const std::string l = t + "layers." + std::to_string(i) + ".";
        for (const char *n : {"q_proj", "k_proj", "v_proj"}) add_shape(dec, l + "self_attn." + n + ".weight", {HD, d.hidden});
        add_shape(dec, l + "self_attn.o_proj.weight", {d.hidden, HD});
        add_shape(dec, l + "mlp.gate_proj.weight", {d.intermediate, d.hidden});
        add_shape(dec, l + "mlp.up_proj.weight", {d.intermediate, d.hidden});
        add_shape(dec, l + "mlp.down_proj.weight", {d.hidden, d.intermediate});
        add_shape(dec, l + "input_layernorm.weight", {d.hidden});
        add_shape(dec, l + "post_attention_layernorm.weight", {d.hidden});
        add_shape(dec, l + "self_attn_layer_scale.scale", {d.hidden});
        add_shape(dec, l + "mlp_layer_scale.scale", {d.hidden});
    }
    for (int i = 0; i < d.upsample_stages; i++) {
        const std::string ct = "decoder.upsample." + std::to_string(i) + ".0.conv.";
        const std::string cn = "decoder.upsample." + std::to_string(i) + ".1.";
        add_shape(dec, ct + "weight", {d.latent, d.latent, kUpKernel});
        add_shape(dec, ct + "bias", {d.latent});
        add_shape(dec, cn + "dwconv.conv.weight", {d.latent, 1, kDwTaps});
        add_shape(dec, cn + "dwconv.conv.bias", {d.latent});
        add_shape(dec, cn + "norm.weight", {d.latent});
        add_shape(dec, cn + "norm.bias", {d.latent});
        add_shape(dec, cn + "pwconv1.weight", {d.upsample_inner, d.latent});
        add_shape(dec, cn + "pwconv1.bias", {d.upsample_inner});
        add_shape(dec, cn + "pwconv2.weight", {d.latent, d.upsample_inner});
        add_shape(dec, cn + "pwconv2.bias", {d.latent});
        add_shape(dec, cn + "gamma", {d.latent});
    }
    add_shape(dec, "decoder.decoder.0.conv.weight", {d.vocos_channels[0], d.latent, kVocosTaps});
    add_shape(dec, "decoder.decoder.0.conv.bias", {d.vocos_channels[0]});
    for (int b = 0; b < d.vocos_blocks; b++) {
        const std::string p = "decoder.decoder." + std::to_string(b + 1) + ".block.";
        const int64_t ci = d.vocos_channels[b], co = d.vocos_channels[b + 1];
        add_shape(dec, p + "0.alpha", {ci});
        add_shape(dec, p + "0.beta", {ci});
        add_shape(dec, p + "1.conv.weight", {ci, co, d.vocos_kernels[b]});
        add_shape(dec, p + "1.conv.bias", {co});
        for (int r = 0; r < 3; r++) {
            const std::string u = p + std::to_string(r + 2) + ".";
            add_shape(dec, u + "act1.alpha", {co});
            add_shape(dec, u + "act1.beta", {co});
            add_shape(dec, u + "conv1.conv.weight", {co, co, kVocosTaps});
            add_shape(dec, u + "conv1.conv.bias", {co});
            add_shape(dec, u + "act2.alpha", {co});
            add_shape(dec, u + "act2.beta", {co});
            add_shape(dec, u + "conv2.conv.weight", {co, co, 1});
            add_shape(dec, u + "conv2.conv.bias", {co});
        }
    }
    const int64_t cl = d.vocos_channels[d.vocos_blocks];
    const std::string f = "decoder.decoder." + std::to_string(d.vocos_blocks + 1) + ".";
    const std::string o = "decoder.decoder." + std::to_string(d.vocos_blocks + 2) + ".conv.";
    add_shape(dec, f + "alpha", {cl});
    add_shape(dec, f + "beta", {cl});
    add_shape(dec, o + "weight", {1, cl, kFinalTaps});
    add_shape(dec, o + "bias", {1});
}

const float *tensor_of(qora_decoder *dec, const std::string &name) { return dec->host.at(name).data(); }

// snake_beta's per-channel constants (conv.rs:628-629): exp(alpha), exp(-beta)
// in f32 on the host, as the reference computes them.
int upload_snake(qora_decoder *dec, const std::string &prefix, DevBuf &a, DevBuf &ib) {
    const std::vector<float> &al = dec->host.at(prefix + "alpha"), &be = dec->host.at(prefix + "beta");
    std::vector<float> ea(al.size()), eb(be.size());
    for (size_t i = 0; i < al.size(); i++) ea[i] = std::exp(al[i]);
    for (size_t i = 0; i < be.size(); i++) eb[i] = std::exp(-be[i]);
    QORA_TRY(upload(a, ea));
    return upload(ib, eb);
}

int upload_raw(qora_decoder *dec, const std::string &name, DevBuf &buf) { return upload(buf, dec->host.at(name)); }

int finalize(qora_decoder *dec) {
    const qora_decoder_dims &d = dec->d;
    const int64_t HD = (int64_t)d.num_heads * d.head_dim;
    // codebooks: ema_codebook (loader.rs:488-501): embedding_sum / max(usage, 1e-8)
    {
        const int64_t per = (int64_t)d.codebook_size * d.codebook_dim;
        std::vector<float> cb((size_t)(per * d.num_quantizers));
        for (int g = 0; g < d.num_quantizers; g++) {
            const std::string c = g == 0 ? "decoder.quantizer.rvq_first.vq.layers.0._codebook."
                                         : "decoder.quantizer.rvq_rest.vq.layers." + std::to_string(g - 1) + "._codebook.";
            const float *s = tensor_of(dec, c + "embedding_sum"), *u = tensor_of(dec, c + "cluster_usage");
            for (int64_t i = 0; i < d.codebook_size; i++) {
                const float us = std::fmax(u[i], 1e-8f);
                for (int64_t j = 0; j < d.codebook_dim; j++)
                    cb[(size_t)(g * per + i * d.codebook_dim + j)] = s[i * d.codebook_dim + j] / us;
            }
        }
        QORA_TRY(upload(dec->cb, cb));
    }
    QORA_TRY(upload(dec->vq_w0, conv_layout(tensor_of(dec, "decoder.quantizer.rvq_first.output_proj.weight"), d.vq_dim,
                                            d.codebook_dim, 1)));
    QORA_TRY(upload(dec->vq_wr, conv_layout(tensor_of(dec, "decoder.quantizer.rvq_rest.output_proj.weight"), d.vq_dim,
                                            d.codebook_dim, 1)));
    QORA_TRY(upload(dec->pre_w, conv_layout(tensor_of(dec, "decoder.pre_conv.conv.weight"), d.latent, d.vq_dim, kPreTaps)));
    QORA_TRY(upload_raw(dec, "decoder.pre_conv.conv.bias", dec->pre_b));
    const std::string t = "decoder.pre_transformer.";
    QORA_TRY(upload(dec->in_w, conv_layout(tensor_of(dec, t + "input_proj.weight"), d.hidden, d.latent, 1)));
    QORA_TRY(upload_raw(dec, t + "input_proj.bias", dec->in_b));
    QORA_TRY(upload(dec->out_w, conv_layout(tensor_of(dec, t + "output_proj.weight"), d.latent, d.hidden, 1)));
    QORA_TRY(upload_raw(dec, t + "output_proj.bias", dec->out_b));
    QORA_TRY(upload_raw(dec, t + "norm.weight", dec->norm_w));
    dec->layers.clear();
    dec->layers.resize(d.num_layers);
    for (int i = 0; i < d.num_layers; i++) {
        const std::string l = t + "layers." + std::to_string(i) + ".";
        DecLayer &L = dec->layers[i];
        // q, k, v stacked as one [3 HD][hidden] projection
        std::vector<float> qkv((size_t)(3 * HD * d.hidden));
        const char *names[3] = {"q_proj", "k_proj", "v_proj"};
        for (int j = 0; j < 3; j++)
            std::memcpy(qkv.data() + (size_t)j * HD * d.hidden, tensor_of(dec, l + "self_attn." + names[j] + ".weight"),
                        sizeof(float) * (size_t)(HD * d.hidden));
        QORA_TRY(upload(L.qkv_w, conv_layout(qkv.data(), 3 * HD, d.hidden, 1)));
        QORA_TRY(upload(L.o_w, conv_layout(tensor_of(dec, l + "self_attn.o_proj.weight"), d.hidden, HD, 1)));
        // gate / up interleaved in 64-row halves of 128-row tiles: tile b holds
        // gate rows 64b .. 64b+63, then up rows 64b .. 64b+63
        std::vector<float> gu((size_t)(2 * d.intermediate * d.hidden));
        const float *g = tensor_of(dec, l + "mlp.gate_proj.weight"), *u = tensor_of(dec, l + "mlp.up_proj.weight");
        for (int64_t r = 0; r < 2 * (int64_t)d.intermediate; r++) {
            const int64_t b = r / 128, w = r % 128;
            const float *src = (w < 64 ? g : u) + (b * 64 + (w % 64)) * d.hidden;
            std::memcpy(gu.data() + (size_t)(r * d.hidden), src, sizeof(float) * (size_t)d.hidden);
        }
        QORA_TRY(upload(L.gu_w, conv_layout(gu.data(), 2 * (int64_t)d.intermediate, d.hidden, 1)));
        QORA_TRY(upload(L.down_w, conv_layout(tensor_of(dec, l + "mlp.down_proj.weight"), d.hidden, d.intermediate, 1)));
        QORA_TRY(upload_raw(dec, l + "input_layernorm.weight", L.in_norm));
        QORA_TRY(upload_raw(dec, l + "post_attention_layernorm.weight", L.post_norm));
        QORA_TRY(upload_raw(dec, l + "self_attn_layer_scale.scale", L.attn_scale));
        QORA_TRY(upload_raw(dec, l + "mlp_layer_scale.scale", L.mlp_scale));
    }
    dec->ups.clear();
    dec->ups.resize(d.upsample_stages);
    for (int i = 0; i < d.upsample_stages; i++) {
        const std::string ct = "decoder.upsample." + std::to_string(i) + ".0.conv.";
        const std::string cn = "decoder.upsample." + std::to_string(i) + ".1.";
        DecUpsample &U = dec->ups[i];
        {
            const std::vector<float> l = convt_layout(tensor_of(dec, ct + "weight"), d.latent, d.latent, kUpKernel, kUpStride);
            QORA_TRY(upload(U.ct_w, l));
            QORA_TRY(upload(U.ct_tc, tc_image(l, kUpStride, d.latent, d.latent, kUpKernel / kUpStride)));
        }
        QORA_TRY(upload_raw(dec, ct + "bias", U.ct_b));
        QORA_TRY(upload_raw(dec, cn + "dwconv.conv.weight", U.dw_w));
        QORA_TRY(upload_raw(dec, cn + "dwconv.conv.bias", U.dw_b));
        QORA_TRY(upload_raw(dec, cn + "norm.weight", U.ln_w));
        QORA_TRY(upload_raw(dec, cn + "norm.bias", U.ln_b));
        {
            const std::vector<float> l = conv_layout(tensor_of(dec, cn + "pwconv1.weight"), d.upsample_inner, d.latent, 1);
            QORA_TRY(upload(U.pw1_w, l));
            QORA_TRY(upload(U.pw1_tc, tc_image(l, 1, d.latent, d.upsample_inner, 1)));
        }
        QORA_TRY(upload_raw(dec, cn + "pwconv1.bias", U.pw1_b));
        {
            const std::vector<float> l = conv_layout(tensor_of(dec, cn + "pwconv2.weight"), d.latent, d.upsample_inner, 1);
            QORA_TRY(upload(U.pw2_w, l));
            QORA_TRY(upload(U.pw2_tc, tc_image(l, 1, d.upsample_inner, d.latent, 1)));
        }
        QORA_TRY(upload_raw(dec, cn + "pwconv2.bias", U.pw2_b));
        QORA_TRY(upload_raw(dec, cn + "gamma", U.gamma));
    }
    {
        const std::vector<float> l = conv_layout(tensor_of(dec, "decoder.decoder.0.conv.weight"), d.vocos_channels[0],
                                                 d.latent, kVocosTaps);
        QORA_TRY(upload(dec->init_w, l));
        QORA_TRY(upload(dec->init_tc, tc_image(l, 1, d.latent, d.vocos_channels[0], kVocosTaps)));
    }
    QORA_TRY(upload_raw(dec, "decoder.decoder.0.conv.bias", dec->init_b));
    dec->blocks.clear();
    dec->blocks.resize(d.vocos_blocks);
    for (int b = 0; b < d.vocos_blocks; b++) {
        const std::string p = "decoder.decoder." + std::to_string(b + 1) + ".block.";
        const int64_t ci = d.vocos_channels[b], co = d.vocos_channels[b + 1];
        DecBlock &B = dec->blocks[b];
        QORA_TRY(upload_snake(dec, p + "0.", B.pre_a, B.pre_ib));
        {
            const int s = d.vocos_strides[b];
            const std::vector<float> l = convt_layout(tensor_of(dec, p + "1.conv.weight"), ci, co, d.vocos_kernels[b], s);
            QORA_TRY(upload(B.ct_w, l));
            QORA_TRY(upload(B.ct_tc, tc_image(l, s, ci, co, d.vocos_kernels[b] / s)));
        }
        QORA_TRY(upload_raw(dec, p + "1.conv.bias", B.ct_b));
        for (int r = 0; r < 3; r++) {
            const std::string u = p + std::to_string(r + 2) + ".";
            DecResidual &R = B.res[r];
            QORA_TRY(upload_snake(dec, u + "act1.", R.a1, R.ib1));
            {
                const std::vector<float> l = conv_layout(tensor_of(dec, u + "conv1.conv.weight"), co, co, kVocosTaps);
                QORA_TRY(upload(R.c1_w, l));
                QORA_TRY(upload(R.c1_tc, tc_image(l, 1, co, co, kVocosTaps)));
            }
            QORA_TRY(upload_raw(dec, u + "conv1.conv.bias", R.c1_b));
            QORA_TRY(upload_snake(dec, u + "act2.", R.a2, R.ib2));
            {
                const std::vector<float> l = conv_layout(tensor_of(dec, u + "conv2.conv.weight"), co, co, 1);
                QORA_TRY(upload(R.c2_w, l));
                QORA_TRY(upload(R.c2_tc, tc_image(l, 1, co, co, 1)));
            }
            QORA_TRY(upload_raw(dec, u + "conv2.conv.bias", R.c2_b));
        }
    }
    const std::string f = "decoder.decoder." + std::to_string(d.vocos_blocks + 1) + ".";
    const std::string o = "decoder.decoder." + std::to_string(d.vocos_blocks + 2) + ".conv.";
    QORA_TRY(upload_snake(dec, f, dec->fin_a, dec->fin_ib));
    QORA_TRY(upload_raw(dec, o + "weight", dec->fin_w));
    QORA_TRY(upload_raw(dec, o + "bias", dec->fin_b));
    // RoPE tables (loader.rs:668-682): f64 angles, f32 cos / sin
    {
        const int half = d.head_dim / 2;
        std::vector<float> c((size_t)d.rope_max_pos * half), s(c.size());
        for (int i = 0; i < half; i++) {
            const double freq = 1.0 / std::pow(d.rope_theta, (double)(2 * i) / (double)d.head_dim);
            for (int pos = 0; pos < d.rope_max_pos; pos++) {
                const double ang = (double)pos * freq;
                c[(size_t)pos * half + i] = (float)std::cos(ang);
                s[(size_t)pos * half + i] = (float)std::sin(ang);
            }
        }
        QORA_TRY(upload(dec->rope_cos, c));
        QORA_TRY(upload(dec->rope_sin, s));
    }
    QORA_CUDA(cudaDeviceSynchronize());
    return QORA_OK;
}

// Positions after the upsample stages, and the largest [channels][positions]
// tensor from there on (per frame).
int64_t big_per_frame(const qora_decoder_dims &d) {
    int64_t L = 1;
    int64_t m = 0;
    for (int i = 0; i < d.upsample_stages; i++) {
        L *= kUpStride;
        m = std::max<int64_t>(m, std::max<int64_t>(d.latent, d.upsample_inner) * L);
    }
    m = std::max<int64_t>(m, (int64_t)d.vocos_channels[0] * L);
    for (int b = 0; b < d.vocos_blocks; b++) {
        L *= d.vocos_strides[b];
        m = std::max<int64_t>(m, (int64_t)d.vocos_channels[b + 1] * L);
    }
    return m;
}

int ensure_workspace(qora_decoder *dec, int64_t F) {
    if (F <= dec->ws_frames) return QORA_OK;
    const qora_decoder_dims &d = dec->d;
    const int64_t HD = (int64_t)d.num_heads * d.head_dim;
    const size_t f4 = sizeof(float) * (size_t)F;
    QORA_TRY(dec->e0.alloc(f4 * d.codebook_dim));
    QORA_TRY(dec->er.alloc(f4 * d.codebook_dim));
    QORA_TRY(dec->vq.alloc(f4 * d.vq_dim));
    QORA_TRY(dec->pre.alloc(f4 * d.latent));
    QORA_TRY(dec->x.alloc(f4 * d.hidden));
    QORA_TRY(dec->qkv.alloc(f4 * 3 * HD));
    QORA_TRY(dec->att.alloc(f4 * HD));
    QORA_TRY(dec->h.alloc(f4 * d.intermediate));
    QORA_TRY(dec->tfo.alloc(f4 * d.latent));
    const int64_t lmax = F << d.upsample_stages;
    QORA_TRY(dec->ra.alloc(sizeof(float) * (size_t)lmax));
    QORA_TRY(dec->rb.alloc(sizeof(float) * (size_t)lmax));
    for (int i = 0; i < 3; i++) QORA_TRY(dec->big[i].alloc(f4 * big_per_frame(d)));
    dec->ws_frames = F;
    return QORA_OK;
}

ConvArgs conv_args(const float *in, int64_t len, const DevBuf &w, const float *bias, float *out, int ic, int oc,
                   int dil = 1, int phases = 1) {
    ConvArgs a;
    a.in = in;
    a.len = len;
    a.w = w.as<float>();
    a.bias = bias;
    a.out = out;
    a.ic = ic;
    a.oc = oc;
    a.oc_pad = (int)round4(oc);
    a.dil = dil;
    a.phases = phases;
    return a;
}

int attn_attr(int device) {
    static std::atomic<uint64_t> done{0};
    const uint64_t bit = 1ull << (device & 63);
    if (done.load() & bit) return QORA_OK;
    const int nk = kAttQ + kAttMaxWindow - 1;
    const int bytes = (int)sizeof(float) * (kAttQ * kAttRow + 2 * nk * kAttRow + kAttQ * kAttMaxWindow);
    QORA_CUDA(cudaFuncSetAttribute(k_dec_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.fetch_or(bit);
    return QORA_OK;
}

int grid_for(int64_t n, int sms) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8)); }

// decode_to_audio (decoder.rs:395-582) on device codes [nq][F] (warm-up
// frames included); samples before `skip` are dropped; `out` receives
// F * hop - skip samples.
int run(qora_decoder *dec, const uint32_t *codes, int64_t F, int64_t skip, float *out, cudaStream_t st,
        int *launches) {
    const qora_decoder_dims &d = dec->d;
    const int dev = dec->ctx->device, sms = dec->ctx->num_sms;
    const int64_t HD = (int64_t)d.num_heads * d.head_dim;
    int n = 0;
    QORA_TRY(ensure_workspace(dec, F));
    float *e0 = dec->e0.as<float>(), *er = dec->er.as<float>(), *vq = dec->vq.as<float>();
    float *pre = dec->pre.as<float>(), *x = dec->x.as<float>(), *qkv = dec->qkv.as<float>();
    float *att = dec->att.as<float>(), *h = dec->h.as<float>(), *tfo = dec->tfo.as<float>();
    float *ra = dec->ra.as<float>(), *rb = dec->rb.as<float>();
    float *big[3] = {dec->big[0].as<float>(), dec->big[1].as<float>(), dec->big[2].as<float>()};
    int *err = dec->ctx->err.as<int>();

    // 1. codebook lookup (decoder.rs:142-193)
    k_dec_vq<<<grid_for((int64_t)d.codebook_dim * F, sms), 256, 0, st>>>(
        codes, F, d.num_quantizers, dec->cb.as<float>(), d.codebook_size, d.codebook_dim, e0, er, err);
    QORA_LAUNCH_CHECK();
    n++;
    QORA_TRY(launch_conv(1, P_NONE, E_BIAS, conv_args(e0, F, dec->vq_w0, nullptr, vq, d.codebook_dim, d.vq_dim), dev, st, dec->tc_mode, err));
    {
        ConvArgs a = conv_args(er, F, dec->vq_wr, nullptr, vq, d.codebook_dim, d.vq_dim);
        a.resid = vq;
        QORA_TRY(launch_conv(1, P_NONE, E_RESID, a, dev, st, dec->tc_mode, err));
    }
    // 2. pre-conv (decoder.rs:433)
    QORA_TRY(launch_conv(kPreTaps, P_NONE, E_BIAS,
                         conv_args(vq, F, dec->pre_w, dec->pre_b.as<float>(), pre, d.vq_dim, d.latent), dev, st, dec->tc_mode, err));
    n += 3;
    // 3. transformer (decoder.rs:196-333)
    QORA_TRY(launch_conv(1, P_NONE, E_BIAS, conv_args(pre, F, dec->in_w, dec->in_b.as<float>(), x, d.latent, d.hidden),
                         dev, st, dec->tc_mode, err));
    n++;
    const float scale = 1.0f / std::sqrt((float)d.head_dim);
    const int gs = (int)((F + 31) / 32);
    for (int i = 0; i < d.num_layers; i++) {
        const DecLayer &L = dec->layers[i];
        k_dec_colstats<false><<<gs, 256, 0, st>>>(x, d.hidden, F, kDecEps, ra, nullptr);
        QORA_LAUNCH_CHECK();
        ConvArgs a = conv_args(x, F, L.qkv_w, nullptr, qkv, d.hidden, (int)(3 * HD));
        a.pa = L.in_norm.as<float>();
        a.ra = ra;
        QORA_TRY(launch_conv(1, P_RMS, E_BIAS, a, dev, st, dec->tc_mode, err));
        const int nk = kAttQ + d.sliding_window - 1;
        const size_t asmem = sizeof(float) * (size_t)(kAttQ * kAttRow + 2 * nk * kAttRow + kAttQ * d.sliding_window);
        QORA_TRY(attn_attr(dev));
        k_dec_attn<<<dim3((unsigned)((F + kAttQ - 1) / kAttQ), d.num_heads), 256, asmem, st>>>(
            qkv, F, d.num_heads, d.sliding_window, scale, dec->rope_cos.as<float>(), dec->rope_sin.as<float>(),
            d.rope_max_pos, att);
        QORA_LAUNCH_CHECK();
        a = conv_args(att, F, L.o_w, nullptr, x, (int)HD, d.hidden);
        a.resid = x;
        a.escale = L.attn_scale.as<float>();
        QORA_TRY(launch_conv(1, P_NONE, E_SCALE_RESID, a, dev, st, dec->tc_mode, err));
        k_dec_colstats<false><<<gs, 256, 0, st>>>(x, d.hidden, F, kDecEps, ra, nullptr);
        QORA_LAUNCH_CHECK();
        a = conv_args(x, F, L.gu_w, nullptr, h, d.hidden, 2 * d.intermediate);
        a.pa = L.post_norm.as<float>();
        a.ra = ra;
        QORA_TRY(launch_conv(1, P_RMS, E_SWIGLU, a, dev, st, dec->tc_mode, err));
        a = conv_args(h, F, L.down_w, nullptr, x, d.intermediate, d.hidden);
        a.resid = x;
        a.escale = L.mlp_scale.as<float>();
        QORA_TRY(launch_conv(1, P_NONE, E_SCALE_RESID, a, dev, st, dec->tc_mode, err));
        n += 7;
    }
    k_dec_colstats<false><<<gs, 256, 0, st>>>(x, d.hidden, F, kDecEps, ra, nullptr);
    QORA_LAUNCH_CHECK();
    {
        ConvArgs a = conv_args(x, F, dec->out_w, dec->out_b.as<float>(), tfo, d.hidden, d.latent);
        a.pa = dec->norm_w.as<float>();
        a.ra = ra;
        QORA_TRY(launch_conv(1, P_RMS, E_BIAS, a, dev, st, dec->tc_mode, err));
    }
    n += 2;
    // 4. upsample: ConvTranspose k=2 s=2 + ConvNeXt (decoder.rs:450-482, 337-382)
    const float *cur = tfo;
    int ci = -1;
    int64_t L = F;
    for (int i = 0; i < d.upsample_stages; i++) {
        const DecUpsample &U = dec->ups[i];
        const int ui = (ci + 1) % 3, di = (ui + 1) % 3, pi = (ui + 2) % 3;
        float *u = big[ui], *dw = big[di], *p1 = big[pi];
        ConvArgs a = conv_args(cur, L, U.ct_w, U.ct_b.as<float>(), u, d.latent, d.latent, 1, kUpStride);
        a.wtc = U.ct_tc.as<uint8_t>();
        QORA_TRY(launch_conv(kUpKernel / kUpStride, P_NONE, E_BIAS, a, dev, st, dec->tc_mode, err));
        L *= kUpStride;
        k_dec_dwconv<<<grid_for((int64_t)d.latent * L, sms), 256, 0, st>>>(u, U.dw_w.as<float>(), U.dw_b.as<float>(),
                                                                            d.latent, kDwTaps, L, dw);
        QORA_LAUNCH_CHECK();
        k_dec_colstats<true><<<(unsigned)((L + 31) / 32), 256, 0, st>>>(dw, d.latent, L, kDecEps, ra, rb);
        QORA_LAUNCH_CHECK();
        a = conv_args(dw, L, U.pw1_w, U.pw1_b.as<float>(), p1, d.latent, d.upsample_inner);
        a.wtc = U.pw1_tc.as<uint8_t>();
        a.pa = U.ln_w.as<float>();
        a.pb = U.ln_b.as<float>();
        a.ra = ra;
        a.rb = rb;
        QORA_TRY(launch_conv(1, P_LN, E_GELU, a, dev, st, dec->tc_mode, err));
        a = conv_args(p1, L, U.pw2_w, U.pw2_b.as<float>(), u, d.upsample_inner, d.latent);
        a.wtc = U.pw2_tc.as<uint8_t>();
        a.resid = u;
        a.escale = U.gamma.as<float>();
        QORA_TRY(launch_conv(1, P_NONE, E_SCALE_RESID, a, dev, st, dec->tc_mode, err));
        cur = u;
        ci = ui;
        n += 5;
    }
    // 5. Vocos input conv (decoder.rs:485)
    {
        const int ni = (ci + 1) % 3;
        ConvArgs a = conv_args(cur, L, dec->init_w, dec->init_b.as<float>(), big[ni], d.latent, d.vocos_channels[0]);
        a.wtc = dec->init_tc.as<uint8_t>();
        QORA_TRY(launch_conv(kVocosTaps, P_NONE, E_BIAS, a, dev, st, dec->tc_mode, err));
        cur = big[ni];
        ci = ni;
        n++;
    }
    // 6. Vocos blocks (decoder.rs:491-535)
    for (int b = 0; b < d.vocos_blocks; b++) {
        const DecBlock &B = dec->blocks[b];
        const int cin = d.vocos_channels[b], co = d.vocos_channels[b + 1], s = d.vocos_strides[b];
        const int ni = (ci + 1) % 3, ti = (ci + 2) % 3;
        float *sig = big[ni], *tmp = big[ti];
        ConvArgs a = conv_args(cur, L, B.ct_w, B.ct_b.as<float>(), sig, cin, co, 1, s);
        a.wtc = B.ct_tc.as<uint8_t>();
        a.pa = B.pre_a.as<float>();
        a.pb = B.pre_ib.as<float>();
        QORA_TRY(launch_conv(d.vocos_kernels[b] / s, P_SNAKE, E_BIAS, a, dev, st, dec->tc_mode, err));
        L *= s;
        n++;
        for (int r = 0; r < 3; r++) {
            const DecResidual &R = B.res[r];
            a = conv_args(sig, L, R.c1_w, R.c1_b.as<float>(), tmp, co, co, kResDilations[r]);
            a.wtc = R.c1_tc.as<uint8_t>();
            a.pa = R.a1.as<float>();
            a.pb = R.ib1.as<float>();
            QORA_TRY(launch_conv(kVocosTaps, P_SNAKE, E_BIAS, a, dev, st, dec->tc_mode, err));
            a = conv_args(tmp, L, R.c2_w, R.c2_b.as<float>(), sig, co, co);
            a.wtc = R.c2_tc.as<uint8_t>();
            a.pa = R.a2.as<float>();
            a.pb = R.ib2.as<float>();
            a.resid = sig;
            QORA_TRY(launch_conv(1, P_SNAKE, E_RESID, a, dev, st, dec->tc_mode, err));
            n += 2;
        }
        cur = sig;
        ci = ni;
    }
    // 7. SnakeBeta + conv to one channel + clamp, warm-up trimmed (decoder.rs:541-552)
    const int cl = d.vocos_channels[d.vocos_blocks];
    k_dec_final<<<(unsigned)((L + kFinT - 1) / kFinT), kFinT, 0, st>>>(
        cur, cl, L, dec->fin_a.as<float>(), dec->fin_ib.as<float>(), dec->fin_w.as<float>(), dec->fin_b.as<float>(),
        kFinalTaps, skip, out);
    QORA_LAUNCH_CHECK();
    n++;
    if (launches) *launches = n;
    return QORA_OK;
}

int check_dims(const qora_decoder_dims &d) {
    auto pos = [](int64_t v) { return v > 0; };
    if (!pos(d.codebook_dim) || !pos(d.codebook_size) || d.num_quantizers < 2 || !pos(d.vq_dim) || !pos(d.latent) ||
        !pos(d.hidden) || !pos(d.num_heads) || !pos(d.intermediate) || d.num_layers < 0 || !pos(d.sliding_window) ||
        d.upsample_stages < 0 || !pos(d.upsample_inner) || d.vocos_blocks < 1 || d.vocos_blocks > 7 ||
        !pos(d.rope_max_pos) || !(d.rope_theta > 0.0))
        return set_error(QORA_ERR_INVALID, "qora_decoder_dims: a dimension is not positive");
    if (d.head_dim != kAttD)
        return set_error(QORA_ERR_UNSUPPORTED, "decoder head_dim %d (the attention kernel takes %d)", d.head_dim, kAttD);
    if (d.sliding_window > kAttMaxWindow)
        return set_error(QORA_ERR_UNSUPPORTED, "decoder sliding window %d > %d", d.sliding_window, kAttMaxWindow);
    if (d.intermediate % 64)
        return set_error(QORA_ERR_UNSUPPORTED, "decoder intermediate size %d (a multiple of 64)", d.intermediate);
    for (int b = 0; b <= d.vocos_blocks; b++)
        if (d.vocos_channels[b] <= 0) return set_error(QORA_ERR_INVALID, "vocos channel count %d", d.vocos_channels[b]);
    if (d.vocos_channels[d.vocos_blocks] > 4096)
        return set_error(QORA_ERR_UNSUPPORTED, "output stage channels %d", d.vocos_channels[d.vocos_blocks]);
    for (int b = 0; b < d.vocos_blocks; b++) {
        const int k = d.vocos_kernels[b], s = d.vocos_strides[b];
        if (s <= 0 || k < s || k % s || k / s > 2)
            return set_error(QORA_ERR_UNSUPPORTED, "vocos block %d: transposed conv kernel %d stride %d "
                             "(kernel = stride or 2 x stride)", b, k, s);
    }
    return QORA_OK;
}

}  // namespace
}  // namespace qora

using namespace qora;

extern "C" {

int qora_decoder_create(qora_ctx *ctx, const qora_decoder_dims *dims, qora_decoder **out) {
    if (!ctx || !dims || !out) return set_error(QORA_ERR_INVALID, "qora_decoder_create: null argument");
    *out = nullptr;
    QORA_TRY(check_dims(*dims));
    auto *dec = new qora_decoder();
    dec->ctx = ctx;
    g_sms[ctx->device & 63] = ctx->num_sms;
    dec->d = *dims;
    int64_t hop = (int64_t)1 << dims->upsample_stages;
    for (int b = 0; b < dims->vocos_blocks; b++) hop *= dims->vocos_strides[b];
    dec->hop = hop;
    build_shapes(dec);
    *out = dec;
    return QORA_OK;
}

void qora_decoder_destroy(qora_decoder *dec) {
    if (!dec) return;
    DeviceGuard g;
    g.set(dec->ctx->device);
    delete dec;
}

int qora_decoder_set_tensor(qora_decoder *dec, const char *name, const float *data, int64_t count) {
    if (!dec || !name || (!data && count)) return set_error(QORA_ERR_INVALID, "qora_decoder_set_tensor: null argument");
    auto it = dec->shapes.find(name);
    if (it == dec->shapes.end()) return set_error(QORA_ERR_INVALID, "decoder tensor '%s' is not one the decoder reads", name);
    int64_t n = 1;
    for (int64_t v : it->second) n *= v;
    if (count != n)
        return set_error(QORA_ERR_SHAPE, "decoder tensor '%s': %lld values, expected %lld", name, (long long)count,
                         (long long)n);
    dec->host[name].assign(data, data + count);
    dec->ready = false;
    return QORA_OK;
}

int qora_decoder_finalize(qora_decoder *dec) {
    if (!dec) return set_error(QORA_ERR_INVALID, "qora_decoder_finalize: null decoder");
    for (const auto &kv : dec->shapes)
        if (!dec->host.count(kv.first))
            return set_error(QORA_ERR_INVALID, "decoder tensor '%s' was not set", kv.first.c_str());
    DeviceGuard g;
    QORA_TRY(g.set(dec->ctx->device));
    QORA_TRY(finalize(dec));
    dec->host.clear();
    dec->ready = true;
    return QORA_OK;
}

int qora_decoder_get_dims(const qora_decoder *dec, qora_decoder_dims *dims) {
    if (!dec || !dims) return set_error(QORA_ERR_INVALID, "qora_decoder_get_dims: bad argument");
    *dims = dec->d;
    return QORA_OK;
}

int qora_decoder_use_tensor_cores(qora_decoder *dec, int32_t mode) {
    if (!dec || mode < 0 || mode > 2) return set_error(QORA_ERR_INVALID, "qora_decoder_use_tensor_cores: bad argument");
    dec->tc_mode = mode;
    return QORA_OK;
}

int qora_decoder_samples(const qora_decoder *dec, int64_t frames, int64_t *samples) {
    if (!dec || !samples || frames < 0) return set_error(QORA_ERR_INVALID, "qora_decoder_samples: bad argument");
    *samples = frames * dec->hop;
    return QORA_OK;
}

int qora_decode_to_audio_device(qora_decoder *dec, const uint32_t *codes, int64_t frames, int64_t warmup_frames,
                                float *samples, int32_t *launches, void *stream) {
    if (!dec || frames < 0 || warmup_frames < 0 || (frames > 0 && (!codes || !samples)))
        return set_error(QORA_ERR_INVALID, "qora_decode_to_audio_device: bad argument");
    if (!dec->ready) return set_error(QORA_ERR_INVALID, "decoder weights not finalized");
    if (launches) *launches = 0;
    if (frames == 0) return QORA_OK;  // decoder.rs:401-404
    DeviceGuard g;
    QORA_TRY(g.set(dec->ctx->device));
    const int64_t F = frames + warmup_frames;
    // warmup_trim_len (decoder.rs:649-656): Tv / (Tv + T) of F * hop samples
    const int64_t skip = std::min(warmup_frames * (F * dec->hop) / F, F * dec->hop);
    int n = 0;
    QORA_TRY(run(dec, codes, F, skip, samples, as_stream(stream), &n));
    if (launches) *launches = n;
    return QORA_OK;
}

int qora_decode_to_audio(qora_decoder *dec, const uint32_t *codes_host, int64_t frames,
                         const uint32_t *warmup_host, int64_t warmup_frames, float *samples_host, int64_t capacity,
                         int64_t *n_samples, void *stream) {
    if (!dec || !n_samples || frames < 0 || (frames > 0 && (!codes_host || !samples_host)))
        return set_error(QORA_ERR_INVALID, "qora_decode_to_audio: bad argument");
    if (!dec->ready) return set_error(QORA_ERR_INVALID, "decoder weights not finalized");
    *n_samples = 0;
    if (frames == 0) return QORA_OK;
    // the warm-up is used only when it is a non-empty [nq][Tv] block (decoder.rs:412-430)
    const int64_t tv = (warmup_host && warmup_frames > 0) ? warmup_frames : 0;
    const int64_t F = frames + tv, nq = dec->d.num_quantizers;
    const int64_t total = F * dec->hop;
    const int64_t skip = std::min(tv * total / F, total);
    if (capacity < total - skip)
        return set_error(QORA_ERR_SHAPE, "sample buffer holds %lld values, %lld needed", (long long)capacity,
                         (long long)(total - skip));
    DeviceGuard g;
    QORA_TRY(g.set(dec->ctx->device));
    cudaStream_t st = as_stream(stream);
    if (F > dec->io_frames) {
        QORA_TRY(dec->codes_dev.alloc(sizeof(uint32_t) * (size_t)(F * nq)));
        dec->io_frames = F;
    }
    if (total > dec->io_samples) {
        QORA_TRY(dec->samples_dev.alloc(sizeof(float) * (size_t)total));
        dec->io_samples = total;
    }
    // [nq][Tv + T]: each quantizer's warm-up codes, then its codes (decoder.rs:420-428)
    uint32_t *cd = dec->codes_dev.as<uint32_t>();
    for (int64_t q = 0; q < nq; q++) {
        if (tv)
            QORA_CUDA(cudaMemcpyAsync(cd + q * F, warmup_host + q * tv, sizeof(uint32_t) * (size_t)tv,
                                      cudaMemcpyHostToDevice, st));
        QORA_CUDA(cudaMemcpyAsync(cd + q * F + tv, codes_host + q * frames, sizeof(uint32_t) * (size_t)frames,
                                  cudaMemcpyHostToDevice, st));
    }
    QORA_TRY(run(dec, cd, F, skip, dec->samples_dev.as<float>(), st, nullptr));
    QORA_CUDA(cudaMemcpyAsync(samples_host, dec->samples_dev.p, sizeof(float) * (size_t)(total - skip),
                              cudaMemcpyDeviceToHost, st));
    QORA_CUDA(cudaStreamSynchronize(st));
    *n_samples = total - skip;
    return QORA_OK;
}

}  // extern "C"
