// Q4 GEMV kernels for sm_100a (CUDA cores, packed f32x2 FMA).
//
// Replaces the reference's gemv/gemm (gemv.rs:149-162, 290-412) and its
// AVX-512 inner kernel (simd.rs:203-269).  Math per output column j:
//     y[j] = sum_k  (f32(scale[k][g]) * x[k]) * (q[k][j] - 8)
// The per-row product s = scale * x is formed exactly as gemv.rs:265 does;
// the per-weight multiply-add is one fused f32 FMA (the reference rounds the
// product and the sum separately; the difference is within the 1e-3
// chunk-assembly tolerance the reference itself accepts, gemv.rs:806-809).
//
// Work decomposition: the weight is stored column-group-major (see Q4Dev), a
// warp owns one 32-column group and 128 rows (4 per lane, lanes = consecutive
// rows, so every load instruction reads 512 contiguous bytes).  Lane partials
// are combined by a butterfly reduce-scatter (lane l ends with column l),
// then across the CTA's warps in fixed order, then across the K-split CTAs
// of one thread-block cluster by rank 0 over distributed shared memory, in
// rank order.  The result is deterministic.
//
// Launch: programmatic dependent launch.  Each CTA fetches its first weight
// tile (immutable) before griddepcontrol.wait, so weight traffic and launch
// latency overlap the previous kernel.
#include <algorithm>
#include <cmath>

#include "gemv_impl.cuh"

namespace qora {

namespace {

using namespace gemv_detail;

constexpr int kRowsPerLane = 4;

// Register caps per batch tile so a whole GEMV grid is resident in one wave
// (B = 1: 64 registers, 4 CTAs of 256 threads per SM).
template <int B>
struct GemvOcc {
    static constexpr int kMinBlocks = B == 1 ? 4 : (B == 2 ? 2 : 1);
};

template <int B, int XM, int EM>
__global__ void __launch_bounds__(256, GemvOcc<B>::kMinBlocks) k_gemv(const GemvArgs a) {
    constexpr int CPC = (EM == E_SWIGLU) ? 2 : 1;
    constexpr int R = kRowsPerLane;
    __shared__ float red[8][B][32];
    __shared__ float cta_red[kRowsPerZ][CPC][32];
    __shared__ int last_flag;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int WR = a.WR;
    const int cc = warp / WR, wr = warp % WR;
    const int64_t c = (int64_t)blockIdx.x * CPC + cc;
    const int s = blockIdx.y, z = blockIdx.z;
    const int64_t k = a.w.k;
    const int64_t k_begin = (int64_t)s * a.rows_per_cta_k;
    const int64_t k_end = min(k, k_begin + (int64_t)a.rows_per_cta_k);
    const int64_t wrow0 = k_begin + (int64_t)wr * 32 * R * a.NSUB;
    const int r_begin = z * a.rows_per_z;
    const int r_end = min(a.rows, r_begin + a.rows_per_z);

    const uint4 *nibc = a.w.nib + c * a.w.kpad;
    const __half *sclc = a.w.scl + c * a.w.kpad;
    const bool write_side = (XM == X_RMSNORM) && a.side && blockIdx.x == 0 && cc == 0;

    // Weights are immutable: fetch the first tile before waiting on the
    // kernel that produces x, so the fetch overlaps that kernel's tail.
    uint4 wv[R];
    float sc[R];
#pragma unroll
    for (int i = 0; i < R; i++) {
        const int64_t kr = wrow0 + lane + 32 * i;
        const bool ok = kr < k_end;
        wv[i] = ok ? ldg_stream(nibc + kr) : make_uint4(0u, 0u, 0u, 0u);
        sc[i] = ok ? __half2float(sclc[kr]) : 0.0f;
    }
    // Warm L2 with the next GEMV's weights (this grid's share of them).
    if (threadIdx.x == 0 && (a.pf0_bytes | a.pf1_bytes)) {
        const uint64_t nctas = (uint64_t)gridDim.x * gridDim.y * gridDim.z;
        const uint64_t id = ((uint64_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        l2_prefetch_share(a.pf0, a.pf0_bytes, id, nctas);
        l2_prefetch_share(a.pf1, a.pf1_bytes, id, nctas);
    }
    griddep_launch_dependents();
    griddep_wait();

    for (int r0 = r_begin; r0 < r_end; r0 += B) {
        // rms_norm_f16 (gemv.rs:445-454): inv = 1/sqrt(sum(x^2)/k + 1e-6), the
        // sum taken from the producer's per-32-column partials by a fixed
        // shuffle tree (same in every warp, so every CTA agrees)
        float inv[B];
#pragma unroll
        for (int b = 0; b < B; b++) {
            inv[b] = 1.0f;
            if constexpr (XM == X_RMSNORM) {
                const int r = r0 + b;
                float t = 0.0f;
                if (r < r_end)
                    for (int i = lane; i < a.ss_tiles; i += 32) t += __ldcg(a.ss + (int64_t)r * a.ldss + i);
                t = warp_sum(t);
                inv[b] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)k), 1e-6f)));
            }
        }
        uint64_t acc[B][16];
        float ssum[B];
#pragma unroll
        for (int b = 0; b < B; b++) {
            ssum[b] = 0.0f;
#pragma unroll
            for (int j = 0; j < 16; j++) acc[b][j] = 0ull;
        }
        for (int sb = 0; sb < a.NSUB; sb++) {
        const int64_t srow0 = wrow0 + (int64_t)sb * 32 * R;
        if (r0 != r_begin || sb != 0) {
#pragma unroll
            for (int i = 0; i < R; i++) {
                const int64_t kr = srow0 + lane + 32 * i;
                const bool ok = kr < k_end;
                wv[i] = ok ? ldg_stream(nibc + kr) : make_uint4(0u, 0u, 0u, 0u);
                sc[i] = ok ? __half2float(sclc[kr]) : 0.0f;
            }
        }
        float xs[R][B];
#pragma unroll
        for (int i = 0; i < R; i++) {
            const int64_t kr = srow0 + lane + 32 * i;
            const bool ok = kr < k_end;
#pragma unroll
            for (int b = 0; b < B; b++) {
                const int r = r0 + b;
                xs[i][b] = (ok && r < r_end) ? load_x<XM>(a, r, kr) : 0.0f;
            }
        }
        if constexpr (XM == X_RMSNORM) {
#pragma unroll
            for (int i = 0; i < R; i++) {
                const int64_t kr = srow0 + lane + 32 * i;
                const float g = kr < k_end ? __half2float(a.gamma[kr]) : 0.0f;
#pragma unroll
                for (int b = 0; b < B; b++) xs[i][b] = __fmul_rn(__fmul_rn(xs[i][b], inv[b]), g);
            }
        }
        if (write_side) {
#pragma unroll
            for (int i = 0; i < R; i++) {
                const int64_t kr = srow0 + lane + 32 * i;
#pragma unroll
                for (int b = 0; b < B; b++)
                    if (kr < k_end && r0 + b < r_end) a.side[(int64_t)(r0 + b) * a.ldside + kr] = xs[i][b];
            }
        }
        // Dequantise-and-accumulate.  A nibble at bit position 4p (p < 4) of a
        // 16-bit half-word, masked in place (v & 0xF<<4p), read as f32 bits is
        // exactly q * 2^(4p-149) (subnormal range: linear in q).  With
        // s' = scale * x * 2^75 (exact power-of-two scaling of gemv.rs:265's
        // product), fma(s', that, acc) adds s*q*2^(4p-74) with one rounding.
        // The -8 offset is applied once: sum_k s*(q-8) = sum_k s*q - 8*sum_k s.
#pragma unroll
        for (int i = 0; i < R; i++) {
            uint64_t s2[B];
#pragma unroll
            for (int b = 0; b < B; b++) {
                const float sp = __fmul_rn(sc[i], __fmul_rn(xs[i][b], 37778931862957161709568.0f));
                ssum[b] += sp;
                s2[b] = pk2(sp, sp);
            }
            const uint32_t words[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
#pragma unroll
            for (int q = 0; q < 4; q++) {
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    // nibbles 4h..4h+3 of the word (columns 8q+4h..8q+4h+3) at
                    // bit positions 0..15, where masked bits stay linear
                    const uint32_t v = h ? (words[q] >> 16) : words[q];
#pragma unroll
                    for (int pp = 0; pp < 4; pp += 2) {
                        const uint64_t qd = pk2(__uint_as_float(v & (0xFu << (4 * pp))),
                                                __uint_as_float(v & (0xFu << (4 * pp + 4))));
                        const int j = 4 * q + 2 * h + pp / 2;
#pragma unroll
                        for (int b = 0; b < B; b++) acc[b][j] = ffma2(s2[b], qd, acc[b][j]);
                    }
                }
            }
        }
        }  // sub-blocks
        // butterfly reduce-scatter: lane l ends with the warp total of column l
#pragma unroll
        for (int b = 0; b < B; b++) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 16; j++) upk2(acc[b][j], v[2 * j], v[2 * j + 1]);
#pragma unroll
            for (int sft = 16; sft >= 1; sft >>= 1) {
                const bool up = (lane & sft) != 0;
#pragma unroll
                for (int j = 0; j < sft; j++) {
                    const float send = up ? v[j] : v[j + sft];
                    const float keep = up ? v[j + sft] : v[j];
                    v[j] = keep + __shfl_xor_sync(0xffffffffu, send, sft);
                }
            }
            // undo the per-position scaling (column l sits at position l % 4 of
            // its half-word) and apply the offset: y = 2^(74-4p)*acc - 8*2^-75*sum(s')
            const float stot = warp_sum(ssum[b]);
            const float up = __int_as_float((127 + 74 - 4 * (lane & 3)) << 23);
            v[0] = __fsub_rn(__fmul_rn(v[0], up), __fmul_rn(stot, 2.117582368135751e-22f));  // 2^-72
            red[warp][b][lane] = v[0];
        }
        __syncthreads();
        // CTA total per (row, column group): warps summed in order
        for (int it = threadIdx.x; it < CPC * B * 32; it += blockDim.x) {
            const int l = it & 31;
            const int b = (it >> 5) % B;
            const int cc2 = (it >> 5) / B;
            float v = 0.0f;
            for (int w = 0; w < WR; w++) v += red[cc2 * WR + w][b][l];
            if (r0 + b < r_end) cta_red[r0 + b - r_begin][cc2][l] = v;
        }
        __syncthreads();
    }

    gemv_final<EM, CPC, kRowsPerZ>(a, cta_red, r_begin, r_end, last_flag);
}

template <int B, int XM, int EM>
int launch_one(const GemvArgs &a, const GemvPlan &p, cudaStream_t st) {
    return launch_ex(k_gemv<B, XM, EM>, p.grid, p.block, 0, st, (unsigned)p.S, a);
}

template <int B, int XM, int EM>
int allow_large_clusters() {
    QORA_CUDA(cudaFuncSetAttribute(k_gemv<B, XM, EM>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    return QORA_OK;
}

template <int XM, int EM>
int allow_large_clusters_b() {
    QORA_TRY((allow_large_clusters<1, XM, EM>()));
    QORA_TRY((allow_large_clusters<2, XM, EM>()));
    return allow_large_clusters<4, XM, EM>();
}

template <int XM>
int allow_large_clusters_e() {
    QORA_TRY((allow_large_clusters_b<XM, E_STORE>()));
    QORA_TRY((allow_large_clusters_b<XM, E_BIAS>()));
    QORA_TRY((allow_large_clusters_b<XM, E_RESID>()));
    return allow_large_clusters_b<XM, E_SWIGLU>();
}

template <int XM, int EM>
int launch_b(const GemvArgs &a, const GemvPlan &p, cudaStream_t st) {
    switch (p.B) {
        case 1: return launch_one<1, XM, EM>(a, p, st);
        case 2: return launch_one<2, XM, EM>(a, p, st);
        default: return launch_one<4, XM, EM>(a, p, st);
    }
}

template <int XM>
int launch_e(const GemvArgs &a, int emode, const GemvPlan &p, cudaStream_t st) {
    switch (emode) {
        case E_STORE: return launch_b<XM, E_STORE>(a, p, st);
        case E_BIAS: return launch_b<XM, E_BIAS>(a, p, st);
        case E_RESID: return launch_b<XM, E_RESID>(a, p, st);
        case E_SWIGLU: return launch_b<XM, E_SWIGLU>(a, p, st);
    }
    return set_error(QORA_ERR_INVALID, "bad epilogue mode %d", emode);
}

// ---------------------------------------------------------------- repack
__global__ void k_repack(const uint8_t *__restrict__ src, const __half *__restrict__ src_scl,
                         int64_t k, int64_t C, uint4 *__restrict__ dst, __half *__restrict__ dst_scl,
                         int64_t dst_k_stride, int64_t dst_off, int64_t dst_stride) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= k * C) return;
    const int64_t c = idx / k, kr = idx % k;  // consecutive threads: consecutive rows
    const uint4 *s16 = reinterpret_cast<const uint4 *>(src + (kr * C + c) * 16);
    const int64_t cd = dst_off + c * dst_stride;
    dst[cd * dst_k_stride + kr] = *s16;
    dst_scl[cd * dst_k_stride + kr] = src_scl[kr * C + c];
}

__global__ void k_embed_rows(EmbDev e, const uint32_t *__restrict__ tok, int64_t ldtok,
                             float *__restrict__ out, int64_t ldout, int *err) {
    griddep_launch_dependents();
    griddep_wait();
    const int i = blockIdx.x;
    const uint32_t t = __ldcg(tok + (int64_t)i * ldtok);
    if ((int64_t)t >= e.rows) {  // never read outside the table: zeros, and the flag
        if (threadIdx.x == 0) raise_error(err, kDevRange);
        for (int64_t j = threadIdx.x; j < e.n; j += blockDim.x) out[(int64_t)i * ldout + j] = 0.0f;
        return;
    }
    const uint8_t *p = e.packed + (int64_t)t * (e.n >> 1);
    const __half *s = e.scl + (int64_t)t * (e.n >> 5);
    for (int64_t j = threadIdx.x; j < e.n; j += blockDim.x) {
        const uint8_t byte = p[j >> 1];
        const int q = (j & 1) ? (byte >> 4) : (byte & 15);
        out[(int64_t)i * ldout + j] = __fmul_rn(__half2float(s[j >> 5]), (float)(q - 8));
    }
}

__global__ void k_copy_rowstats(const float *__restrict__ src, int64_t ldsrc, float *__restrict__ dst,
                                int64_t lddst, int n, float *__restrict__ ss, int64_t ldss) {
    griddep_launch_dependents();
    griddep_wait();
    const int r = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int g = warp; g * 32 < n; g += nw) {
        const int j = g * 32 + lane;
        const float v = j < n ? src[(int64_t)r * ldsrc + j] : 0.0f;
        if (j < n && dst) dst[(int64_t)r * lddst + j] = v;
        const float sq = warp_sum(__fmul_rn(v, v));
        if (lane == 0) ss[(int64_t)r * ldss + g] = sq;
    }
}

__global__ void k_rmsnorm_rows(const float *__restrict__ x, const __half *__restrict__ gamma,
                               int64_t n, float *__restrict__ out) {
    __shared__ float red[32];
    __shared__ float inv;
    griddep_launch_dependents();
    griddep_wait();
    const int r = blockIdx.x;
    const float *xr = x + (int64_t)r * n;
    float t = 0.0f;
    for (int64_t j = threadIdx.x; j < n; j += blockDim.x) t += __fmul_rn(xr[j], xr[j]);
    t = warp_sum(t);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = t;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += red[w];
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)n), 1e-6f)));
    }
    __syncthreads();
    for (int64_t j = threadIdx.x; j < n; j += blockDim.x)
        out[(int64_t)r * n + j] = __fmul_rn(__fmul_rn(xr[j], inv), __half2float(gamma[j]));
}

}  // namespace

// Clusters of up to kMaxSplit (16) CTAs exceed the portable size (8) and must
// be enabled per kernel; done once per device context, before any capture.
int gemv_init() {
    QORA_TRY(allow_large_clusters_e<X_PLAIN>());
    QORA_TRY(allow_large_clusters_e<X_RMSNORM>());
    QORA_TRY(allow_large_clusters_e<X_EMBED>());
    return gemv_mma_init();
}

GemvPlan plan_gemv_for(const GemvArgs &a, int xmode, int emode, int num_sms) {
    if (gemv_mma_eligible(a, xmode, emode)) return plan_gemv_mma(a.w.k, a.w.C, a.rows, emode, num_sms);
    return plan_gemv(a.w.k, a.w.C, a.rows, emode, num_sms);
}

GemvPlan plan_gemv(int64_t k, int64_t C, int rows, int emode, int num_sms) {
    GemvPlan p{};
    p.cpc = (emode == E_SWIGLU) ? 2 : 1;
    p.B = rows >= 3 ? 4 : rows;
    p.rows_per_z = std::min(rows, kRowsPerZ);
    p.Z = (rows + p.rows_per_z - 1) / p.rows_per_z;
    const int64_t tiles = C / p.cpc;
    const int64_t kp = pad_rows(k);
    // Resident warps per SM at this batch tile's register cap (GemvOcc); a
    // grid larger than ~90 % of that runs in waves, so long ones get more
    // 128-row sub-blocks per warp instead.
    const int warps_per_sm = p.B == 1 ? 32 : (p.B == 2 ? 16 : 8);
    const int64_t cap = (int64_t)num_sms * warps_per_sm * 9 / 10;
    const int64_t units = tiles * p.cpc * (kp / 128) * p.Z;
    int nsub = 1;
    while (nsub < 8 && units / nsub > cap) nsub *= 2;
    const int64_t wrows = 128LL * nsub;
    auto splits = [&](int wr) { return (kp + wr * wrows - 1) / (wr * wrows); };
    int WR = 8 / p.cpc;
    while (WR > 1 && splits(WR / 2) == splits(WR)) WR /= 2;  // not more warps than K needs
    // Smaller CTAs (more K-splits) until ~2 CTAs per SM, within one cluster.
    while (WR > 1 && splits(WR / 2) <= kMaxSplit && tiles * splits(WR) * p.Z < 2LL * num_sms) WR /= 2;
    while (splits(WR) > kMaxSplit && nsub < 64) {  // very long K: longer strips
        nsub *= 2;
        WR = 8 / p.cpc;
    }
    p.NSUB = nsub;
    p.WR = WR;
    p.S = (int)((kp + WR * 128LL * nsub - 1) / (WR * 128LL * nsub));
    p.rows_per_cta_k = WR * 128 * nsub;
    p.grid = dim3((unsigned)tiles, (unsigned)p.S, (unsigned)p.Z);
    p.block = dim3(32 * p.cpc * WR);
    return p;
}

int launch_gemv(GemvArgs a, int xmode, int emode, const GemvPlan &p, unsigned *gticket,
                cudaStream_t st) {
    if (a.rows <= 0 || a.rows > kMaxRows)
        return set_error(QORA_ERR_SHAPE, "gemv rows %d outside 1..%d", a.rows, kMaxRows);
    if (p.S > kMaxSplit)
        return set_error(QORA_ERR_UNSUPPORTED, "gemv k=%lld needs %d K-splits (max %d)",
                         (long long)a.w.k, p.S, kMaxSplit);
    if ((a.amax || a.adv_len) && !a.gticket) a.gticket = gticket;
    if ((a.amax || a.adv_len) && !a.gticket)
        return set_error(QORA_ERR_INVALID, "global stage needs a ticket");
    if (!(a.amax || a.adv_len)) a.gticket = nullptr;
    a.B = p.B;
    a.WR = p.WR;
    a.S = p.S;
    a.Z = p.Z;
    a.NSUB = p.NSUB;
    a.rows_per_cta_k = p.rows_per_cta_k;
    a.rows_per_z = p.rows_per_z;
    if (p.mma) {
        if (!gemv_mma_supported(a, xmode, emode))
            return set_error(QORA_ERR_INVALID, "tensor-core GEMV plan for an unsupported launch");
        return launch_gemv_mma(a, xmode, emode, p, st);
    }
    switch (xmode) {
        case X_PLAIN: return launch_e<X_PLAIN>(a, emode, p, st);
        case X_RMSNORM: return launch_e<X_RMSNORM>(a, emode, p, st);
        case X_EMBED: return launch_e<X_EMBED>(a, emode, p, st);
    }
    return set_error(QORA_ERR_INVALID, "bad prologue mode %d", xmode);
}

int repack_q4(const uint8_t *src_packed, const __half *src_scl, int64_t k, int64_t n,
              uint4 *dst_nib, __half *dst_scl, int64_t dst_k_stride, int64_t dst_off,
              int64_t dst_stride, cudaStream_t stream) {
    const int64_t C = n / kGroup;
    const int64_t total = k * C;
    if (total == 0) return QORA_OK;
    const int threads = 256;
    const int64_t blocks = (total + threads - 1) / threads;
    k_repack<<<(unsigned)blocks, threads, 0, stream>>>(src_packed, src_scl, k, C, dst_nib, dst_scl,
                                                       dst_k_stride, dst_off, dst_stride);
    QORA_LAUNCH_CHECK();
    return QORA_OK;
}

int launch_embed_rows(const EmbDev &e, const uint32_t *tok, int64_t ldtok, int count, float *out,
                      int64_t ldout, int *err, cudaStream_t stream) {
    if (count <= 0) return QORA_OK;
    return launch_ex(k_embed_rows, dim3(count), dim3(256), 0, stream, 1u, e, tok, ldtok, out, ldout,
                     err);
}

int launch_copy_rowstats(const float *src, int64_t ldsrc, float *dst, int64_t lddst, int rows,
                         int n, float *ss, int64_t ldss, cudaStream_t stream) {
    if (rows <= 0) return QORA_OK;
    return launch_ex(k_copy_rowstats, dim3(rows), dim3(256), 0, stream, 1u, src, ldsrc, dst, lddst,
                     n, ss, ldss);
}

int launch_rmsnorm_rows(const float *x, const __half *gamma, int64_t n, int rows, float *out,
                        cudaStream_t stream) {
    if (rows <= 0) return QORA_OK;
    return launch_ex(k_rmsnorm_rows, dim3(rows), dim3(256), 0, stream, 1u, x, gamma, n, out);
}

// Exponent E of the tensor-core operand scaling: the largest E in [0, 15] with
// max|scale| * 2^E <= 2^12, so every (q - 8) * scale * 2^E (|q - 8| <= 8) stays
// within 2^15 in f16 while small scales move away from the f16 subnormals.
// -1 when a scale is not finite or too large for the f16 operands.
// Value of a finite, non-negative f16 bit pattern (exact).
static float f16_magnitude(uint16_t mx) {
    const int ex = mx >> 10;
    return ex ? (1.0f + (float)(mx & 0x3FF) / 1024.0f) * std::ldexp(1.0f, ex - 15)
              : (float)(mx & 0x3FF) * std::ldexp(1.0f, -24);
}

static int mma_scale_exponent(const qora_q4_host *parts, int nparts) {
    uint16_t mx = 0;  // |scale| bits: ordered like the values for finite f16
    for (int i = 0; i < nparts; i++) {
        const int64_t cnt = parts[i].k * (parts[i].n / kGroup);
        for (int64_t j = 0; j < cnt; j++) mx = std::max<uint16_t>(mx, parts[i].scales[j] & 0x7FFFu);
    }
    if (mx >= 0x7C00u) return -1;  // inf / NaN
    const float m = f16_magnitude(mx);
    if (m == 0.0f) return 15;
    if (m > 4096.0f) return -1;
    int e = 15;
    while (e > 0 && m * std::ldexp(1.0f, e) > 4096.0f) e--;
    return e;
}

// Upload reference-layout parts of one fused weight (all with the same k) into
// a column-group-major buffer of C_total groups: part i's group c lands at
// group offs[i] + c * strides[i].
int upload_q4_parts(const qora_q4_host *parts, const int64_t *offs, const int64_t *strides,
                    int nparts, int64_t k, int64_t C_total, DevBuf &nib, DevBuf &scl, Q4Dev &out,
                    cudaStream_t stream) {
    const int64_t kp = pad_rows(k);
    QORA_TRY(nib.alloc((size_t)(C_total * kp) * 16));
    QORA_TRY(scl.alloc((size_t)(C_total * kp) * 2));
    QORA_CUDA(cudaMemsetAsync(nib.p, 0, nib.bytes, stream));   // pad rows: q = 0, scale = 0
    QORA_CUDA(cudaMemsetAsync(scl.p, 0, scl.bytes, stream));
    for (int i = 0; i < nparts; i++) {
        const qora_q4_host &h = parts[i];
        if (!h.packed || !h.scales) return set_error(QORA_ERR_INVALID, "null weight part");
        if (h.k != k || h.n % kGroup != 0)
            return set_error(QORA_ERR_SHAPE, "weight part %d: k=%lld n=%lld (need k=%lld, n%%32==0)",
                             i, (long long)h.k, (long long)h.n, (long long)k);
        const int64_t C = h.n / kGroup;
        DevBuf tp, ts;
        QORA_TRY(tp.alloc((size_t)(k * C) * 16));
        QORA_TRY(ts.alloc((size_t)(k * C) * 2));
        QORA_CUDA(cudaMemcpyAsync(tp.p, h.packed, tp.bytes, cudaMemcpyHostToDevice, stream));
        QORA_CUDA(cudaMemcpyAsync(ts.p, h.scales, ts.bytes, cudaMemcpyHostToDevice, stream));
        QORA_TRY(repack_q4(tp.as<uint8_t>(), ts.as<__half>(), k, h.n, nib.as<uint4>(),
                           scl.as<__half>(), kp, offs[i], strides[i], stream));
        QORA_CUDA(cudaStreamSynchronize(stream));
    }
    out.nib = nib.as<uint4>();
    out.scl = scl.as<__half>();
    out.k = k;
    out.kpad = kp;
    out.mma_exp = mma_scale_exponent(parts, nparts);
    out.C = C_total;
    out.n = C_total * kGroup;
    return QORA_OK;
}

int upload_emb(const qora_q4_host &h, DevBuf &packed, DevBuf &scl, EmbDev &out) {
    if (!h.packed || !h.scales) return set_error(QORA_ERR_INVALID, "null embedding");
    if (h.n % kGroup != 0) return set_error(QORA_ERR_SHAPE, "embedding n %% 32 != 0");
    QORA_TRY(packed.alloc((size_t)(h.k * h.n / 2)));
    QORA_TRY(scl.alloc((size_t)(h.k * (h.n / kGroup)) * 2));
    QORA_CUDA(cudaMemcpy(packed.p, h.packed, packed.bytes, cudaMemcpyHostToDevice));
    QORA_CUDA(cudaMemcpy(scl.p, h.scales, scl.bytes, cudaMemcpyHostToDevice));
    out.packed = packed.as<uint8_t>();
    out.scl = scl.as<__half>();
    out.rows = h.k;
    out.n = h.n;
    uint16_t mx = 0;  // the largest |scale|: rows are scale * (q - 8), |q - 8| <= 8
    const int64_t cnt = h.k * (h.n / kGroup);
    for (int64_t j = 0; j < cnt; j++) mx = std::max<uint16_t>(mx, h.scales[j] & 0x7FFFu);
    out.absmax = mx >= 0x7C00u ? INFINITY : 8.0f * f16_magnitude(mx);
    return QORA_OK;
}

}  // namespace qora
