// GQA decode attention with fused qk-norm, RoPE and KV append (sm_100a).
//
// Replaces the per-layer attention block of the talker and the predictor
// (talker.rs:285-331, code_predictor.rs:461-498, prefill variants
// talker.rs:402-458 and code_predictor.rs:369-414):
//   * apply_qk_norm (talker.rs:89-99): per-head RMS norm, eps 1e-6, f16 gamma;
//   * split / rotate-half RoPE (rope.rs:79-92, code_predictor.rs:97-121);
//   * KV append at the stream's cache length (extend_from_slice);
//   * scores (q.k) * 1/sqrt(hd), softmax, weighted V sum.
// One CTA handles one (kv head, position split, query row) and all G query
// heads sharing that kv head, so every K/V byte is read once per row.  Splits
// are merged flash-decoding style by the last-arriving CTA in split order.
#include "attention_impl.cuh"
#include "tc.cuh"

namespace qora {

namespace {

using attn::kTile;
using attn::norm_rope_head;
using attn::rope_rows;

constexpr int kThreads = 128;

template <int HD>
__global__ void __launch_bounds__(kThreads) k_qkv_post(const AttnArgs a) {
    constexpr int J = HD / 32;
    griddep_launch_dependents();
    griddep_wait();
    const int r = blockIdx.x;
    const int b = r / a.T, t = r % a.T;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int L0 = __ldcg(a.len + b);
    if (L0 + a.T > a.kv.max_pos) {
        if (threadIdx.x == 0) raise_error(a.err, kDevRange);
        return;
    }
    const float *cr, *sr;
    if (!rope_rows<HD>(a, b, t, L0, cr, sr)) {
        if (threadIdx.x == 0) raise_error(a.err, kDevRange);
        return;
    }
    float *row = a.qkv + (int64_t)r * a.ldqkv;
    const int nitems = a.heads + 2 * a.kv_heads;
    for (int it = warp; it < nitems; it += kThreads / 32) {
        float v[J];
        const float *src = row + (int64_t)it * HD;  // q heads, then k heads, then v heads
#pragma unroll
        for (int j = 0; j < J; j++) v[j] = src[lane + 32 * j];
        if (it < a.heads) {
            norm_rope_head<HD>(v, a.q_gamma, cr, sr, true, lane);
#pragma unroll
            for (int j = 0; j < J; j++) row[(int64_t)it * HD + lane + 32 * j] = v[j];
        } else if (it < a.heads + a.kv_heads) {
            const int h = it - a.heads;
            norm_rope_head<HD>(v, a.k_gamma, cr, sr, true, lane);
            float *dst = a.kv.k + a.kv.row(b, h, L0 + t);
#pragma unroll
            for (int j = 0; j < J; j++) dst[lane + 32 * j] = v[j];
        } else {
            const int h = it - a.heads - a.kv_heads;
            float *dst = a.kv.v + a.kv.row(b, h, L0 + t);
#pragma unroll
            for (int j = 0; j < J; j++) dst[lane + 32 * j] = v[j];
        }
    }
}

template <int HD, int G>
__global__ void __launch_bounds__(kThreads) k_attention(const AttnArgs a) {
    __shared__ attn::AttnSmem<HD, G, kThreads> sm;
    griddep_launch_dependents();
    griddep_wait();
    attn::attn_item<HD, G, kThreads, 0>(a, blockIdx.x, blockIdx.y, blockIdx.z, threadIdx.x, sm);
}

// ------------------------------------------------------------------------
// Causal prefill attention, tiled (the causal attention of
// prefill_talker_raw_from, talker.rs:425-458): T new rows per stream at
// positions L0 .. L0+T-1 (q normed and roped in place, K/V already appended
// by k_qkv_post) attend to cache positions 0 .. their own.  One CTA takes a
// block of kPfM query vectors (kPfM / G tokens x the G query heads of one kv
// head) and walks the key positions in tiles of kPfBK, double-buffered with
// cp.async, keeping a running max / sum per query (online softmax), so each
// K/V byte is read once per query block instead of once per query row.
// Exact f32 arithmetic; scores are (q.k) * 1/sqrt(hd) with the dot product
// accumulated in head-dimension order.  Every row's result depends only on
// its own query and keys (the key tiles start at position 0 whatever the
// block), so a row comes out with the same bits in any prefill chunk.
constexpr int kPfM = 64;        // query vectors per CTA
constexpr int kPfBK = 32;       // key positions per tile
constexpr int kPfThreads = 256;

template <int HD>
struct PfSmem {
    float q[kPfM][HD + 4];          // +4: rows fall on different banks
    float k[2][kPfBK][HD + 4];
    float v[2][kPfBK][HD + 4];
    float p[kPfM][kPfBK + 1];       // scores, then unnormalised probabilities
    float mx[kPfM], l[kPfM], corr[kPfM];
};

__device__ __forceinline__ void pf_cp16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}

template <int HD, int G>
__global__ void __launch_bounds__(kPfThreads, 2) k_prefill_attn(const AttnArgs a) {
    constexpr int BQ = kPfM / G;    // tokens per CTA
    constexpr int D4 = HD / 4;
    constexpr int DJ = HD / 64;     // float4 columns per thread in P.V
    extern __shared__ float4 pf_dyn[];
    PfSmem<HD> &sm = *reinterpret_cast<PfSmem<HD> *>(pf_dyn);
    griddep_launch_dependents();
    griddep_wait();
    const int qb = gridDim.x - 1 - blockIdx.x;  // the longest query blocks first
    const int h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int L0 = __ldcg(a.len + b);
    if (L0 + a.T > a.kv.max_pos) {
        if (tid == 0 && qb == 0 && h == 0) raise_error(a.err, kDevRange);
        return;
    }
    const int t0 = qb * BQ;
    const int nq = min(BQ, a.T - t0);
    if (nq <= 0) return;
    const int kend = L0 + t0 + nq;  // keys [0, kend) are visible to some row of the block
    const int ntiles = (kend + kPfBK - 1) / kPfBK;
    auto load_tile = [&](int kt, int buf) {
        const int k0 = kt * kPfBK;
        // a tile starts at a multiple of kPfBK, which divides the page size:
        // its rows are one contiguous block of the cache
        const float *kbase = a.kv.k + a.kv.row(b, h, k0);
        const float *vbase = a.kv.v + a.kv.row(b, h, k0);
        for (int i = tid; i < kPfBK * D4; i += kPfThreads) {
            const int n = i / D4, d4 = i % D4;
            float *kd = &sm.k[buf][n][4 * d4];
            float *vd = &sm.v[buf][n][4 * d4];
            if (k0 + n < kend) {
                pf_cp16(kd, kbase + (int64_t)n * HD + 4 * d4);
                pf_cp16(vd, vbase + (int64_t)n * HD + 4 * d4);
            } else {  // never visible: zeros (unwritten cache memory may hold anything)
                *reinterpret_cast<float4 *>(kd) = make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<float4 *>(vd) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    load_tile(0, 0);
    // query vectors: m = token * G + head within the kv head's group
    for (int i = tid; i < kPfM * D4; i += kPfThreads) {
        const int m = i / D4, d4 = i % D4;
        const int tl = m / G, g = m % G;
        float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tl < nq) {
            const float *row = a.qkv + (int64_t)(b * a.T + t0 + tl) * a.ldqkv + (int64_t)(h * G + g) * HD;
            q = __ldcg(reinterpret_cast<const float4 *>(row) + d4);
        }
        *reinterpret_cast<float4 *>(&sm.q[m][4 * d4]) = q;
    }
    if (tid < kPfM) {
        sm.mx[tid] = -INFINITY;
        sm.l[tid] = 0.0f;
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));  // talker.rs:305
    // thread tiles: rows tm*4 .. +3; scores for keys tn + 16 j; P.V columns 4 td + 64 jj
    const int tm = (warp >> 1) * 4 + (lane >> 3);
    const int tn = (warp & 1) * 8 + (lane & 7);
    float o[4][DJ][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int jj = 0; jj < DJ; jj++) o[i][jj][0] = o[i][jj][1] = o[i][jj][2] = o[i][jj][3] = 0.0f;

    for (int kt = 0; kt < ntiles; kt++) {
        const int buf = kt & 1;
        if (kt + 1 < ntiles) load_tile(kt + 1, buf ^ 1);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();
        // ---- scores S = Q K^T for this thread's 4 rows x 2 keys
        float s[4][2];
#pragma unroll
        for (int i = 0; i < 4; i++) s[i][0] = s[i][1] = 0.0f;
#pragma unroll 4
        for (int d4 = 0; d4 < D4; d4++) {
            float4 qv[4], kv[2];
#pragma unroll
            for (int i = 0; i < 4; i++) qv[i] = *reinterpret_cast<const float4 *>(&sm.q[tm * 4 + i][4 * d4]);
#pragma unroll
            for (int j = 0; j < 2; j++) kv[j] = *reinterpret_cast<const float4 *>(&sm.k[buf][tn + 16 * j][4 * d4]);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    float t = s[i][j];
                    t = __fmaf_rn(qv[i].x, kv[j].x, t);
                    t = __fmaf_rn(qv[i].y, kv[j].y, t);
                    t = __fmaf_rn(qv[i].z, kv[j].z, t);
                    t = __fmaf_rn(qv[i].w, kv[j].w, t);
                    s[i][j] = t;
                }
        }
        const int k0 = kt * kPfBK;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int m = tm * 4 + i, tl = m / G;
            const int qpos = L0 + t0 + tl;
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int n = tn + 16 * j;
                const bool vis = tl < nq && k0 + n <= qpos;
                sm.p[m][n] = vis ? __fmul_rn(s[i][j], scale) : -INFINITY;
            }
        }
        __syncthreads();
        // ---- online softmax: 4 threads per row, 8 keys each
        {
            const int row = tid >> 2, part = tid & 3;
            float v[8];
            float rmax = -INFINITY;
#pragma unroll
            for (int e = 0; e < 8; e++) {
                v[e] = sm.p[row][part * 8 + e];
                rmax = fmaxf(rmax, v[e]);
            }
            rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 1));
            rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 2));
            const float m_old = sm.mx[row];
            const float m_new = fmaxf(m_old, rmax);
            float psum = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const float pe = m_new == -INFINITY ? 0.0f : expf(v[e] - m_new);
                sm.p[row][part * 8 + e] = pe;
                psum += pe;
            }
            psum += __shfl_xor_sync(0xffffffffu, psum, 1);
            psum += __shfl_xor_sync(0xffffffffu, psum, 2);
            __syncwarp();
            if (part == 0) {
                const float c = m_new == -INFINITY ? 1.0f : expf(m_old - m_new);  // exp(-inf) = 0
                sm.corr[row] = c;
                sm.l[row] = __fmaf_rn(sm.l[row], c, psum);
                sm.mx[row] = m_new;
            }
        }
        __syncthreads();
        // ---- O = O * corr + P V
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float c = sm.corr[tm * 4 + i];
#pragma unroll
            for (int jj = 0; jj < DJ; jj++) {
                o[i][jj][0] = __fmul_rn(o[i][jj][0], c);
                o[i][jj][1] = __fmul_rn(o[i][jj][1], c);
                o[i][jj][2] = __fmul_rn(o[i][jj][2], c);
                o[i][jj][3] = __fmul_rn(o[i][jj][3], c);
            }
        }
#pragma unroll 4
        for (int n = 0; n < kPfBK; n++) {
            float pr[4];
#pragma unroll
            for (int i = 0; i < 4; i++) pr[i] = sm.p[tm * 4 + i][n];
#pragma unroll
            for (int jj = 0; jj < DJ; jj++) {
                const float4 vv = *reinterpret_cast<const float4 *>(&sm.v[buf][n][4 * tn + 64 * jj]);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    o[i][jj][0] = __fmaf_rn(pr[i], vv.x, o[i][jj][0]);
                    o[i][jj][1] = __fmaf_rn(pr[i], vv.y, o[i][jj][1]);
                    o[i][jj][2] = __fmaf_rn(pr[i], vv.z, o[i][jj][2]);
                    o[i][jj][3] = __fmaf_rn(pr[i], vv.w, o[i][jj][3]);
                }
            }
        }
        __syncthreads();  // the next iteration's prefetch overwrites this buffer
    }
    // ---- out = O / l
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int m = tm * 4 + i, tl = m / G, g = m % G;
        if (tl >= nq) continue;
        const float l = sm.l[m];
        float *dst = a.out + (int64_t)(b * a.T + t0 + tl) * a.ldout + (int64_t)(h * G + g) * HD;
#pragma unroll
        for (int jj = 0; jj < DJ; jj++) {
            float4 r;
            r.x = __fdiv_rn(o[i][jj][0], l);
            r.y = __fdiv_rn(o[i][jj][1], l);
            r.z = __fdiv_rn(o[i][jj][2], l);
            r.w = __fdiv_rn(o[i][jj][3], l);
            *reinterpret_cast<float4 *>(dst + 4 * tn + 64 * jj) = r;
        }
    }
}

// ------------------------------------------------------------------------
// Causal prefill attention on the tensor cores (head_dim 128): the same
// computation as k_prefill_attn, with Q K^T and P V as tcgen05 MMAs.
// A pair of CTAs takes 128 query vectors (128 / G tokens x the G query heads
// of one kv head: vector m = head (m / BQ), token (m % BQ)) = the MMA's M
// rows; the key positions go in tiles of 64 that start at multiples of 64
// (absolute positions), the even tiles to one CTA and the odd ones to the
// other, whose two online-softmax states are merged at the end in a fixed
// order (so every row's result has the same bits in any prefill chunk).
// Per tile:
//   * the K / V rows of the tile come from the cache (row addressing: slab
//     or paged) into an f32 staging buffer with cp.async, issued while the
//     previous tile computes; K goes to B[key][d] and V transposed to
//     B[d][key], both split into f16 hi + lo (x = xh + xl to ~22 bits) in
//     the canonical K-major layout;
//   * S = Qh Kh + Qh Kl + Ql Kh (the dropped Ql Kl is ~2^-22 relative),
//     accumulated in f32 in tensor memory; Q and K are scaled by powers of
//     two fixed per launch (from the qk-norm bounds sqrt(128) max |gamma|),
//     undone exactly in the softmax;
//   * an online softmax on S (row m in TMEM lane m; two threads per row,
//     each half the keys, the halves' max and sum combined in shared memory;
//     exp as the hardware exponential);
//   * O_tile = Ph Vh + Ph Vl + Pl Vh (P in [0, 1] as f16 hi + lo), added by
//     the CUDA cores into the row's running output: O = O * corr + O_tile.
// One thread issues the MMAs; completion comes through mbarriers.  V values
// beyond the f16 range raise kDevF16Range.
constexpr int kTcM = 128;        // query vectors per CTA (MMA M)
constexpr int kTcN = 64;         // keys per tile
constexpr int kTcThreads = 256;
constexpr uint32_t kTcTmemCols = 256;  // S: 64 columns, O_tile: 128
// shared memory (bytes): Q hi / lo [128 x 128], K hi / lo [64 x 128] (P hi /
// lo [128 x 64] in the same slots once S is computed), V^T hi / lo [128 x 64],
// all f16 K-major core matrices; then the f32 K / V rows of the next tile
// (cp.async staging, rows padded by 16 bytes so that 8 consecutive rows fall
// on different banks)
constexpr int kTcSRow = 128 + 4;  // staging row stride (floats)
constexpr int kTcQ = 0, kTcQl = 32768, kTcK = 65536, kTcKl = 81920, kTcV = 98304, kTcVl = 114688,
              kTcP = kTcK, kTcPl = kTcKl, kTcSK = 131072, kTcSV = kTcSK + 64 * kTcSRow * 4,
              kTcBytes = kTcSV + 64 * kTcSRow * 4;

// Byte offset of (row r, 8-element K block kb) in a K-major operand whose
// rows have `nkb` K blocks: core matrices of 8 rows x 16 bytes, K blocks
// adjacent (LBO 128), 8-row blocks nkb * 128 apart (SBO).
__device__ __forceinline__ int tc_off(int r, int kb, int nkb) { return ((r >> 3) * nkb + kb) * 128 + (r & 7) * 16; }

__device__ __forceinline__ uint32_t tc_h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// hi / lo f16 pairs of 8 values (already scaled), as two 16-byte rows
__device__ __forceinline__ bool tc_split8(const float (&x)[8], uint4 &hi, uint4 &lo) {
    uint32_t h[4], l[4];
    bool big = false;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        big |= fabsf(x[2 * i]) > 65504.0f || fabsf(x[2 * i + 1]) > 65504.0f;
        const __half2 hh = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
        const float2 hf = __half22float2(hh);
        h[i] = tc_h2u(hh);
        l[i] = tc_h2u(__floats2half2_rn(__fsub_rn(x[2 * i], hf.x), __fsub_rn(x[2 * i + 1], hf.y)));
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
    return big;
}

// Exponent e with (bound * 2^e) in [2^14, 2^15) (0 for a zero or non-finite
// bound; clamped to [-60, 60], so that 2^-(eq + ek) is a normal float).
__device__ __forceinline__ int tc_exponent(float m) {
    if (!(m > 0.0f) || !(m <= 3.4e38f)) return 0;
    const int ex = (int)((__float_as_uint(m) >> 23) & 0xFF) - 127;
    return max(-60, min(60, 14 - ex));
}

template <int G>
__global__ void __launch_bounds__(kTcThreads, 1) k_prefill_attn_tc(const AttnArgs a) {
    constexpr int HD = 128;
    constexpr int BQ = kTcM / G;    // tokens per CTA
    extern __shared__ __align__(1024) uint8_t tc_dyn[];
    uint8_t *sm = tc_dyn;
    __shared__ __align__(8) uint64_t bar_s, bar_o;
    __shared__ uint32_t tmem_slot;
    __shared__ float red_s[8];
    __shared__ float red_m[2][kTcM], red_l[2][kTcM];  // per-half row max / sum of a tile
    __shared__ int last_flag;
    const int qb = gridDim.x - 1 - blockIdx.x;  // the longest query blocks first
    const int h = blockIdx.y, b = blockIdx.z >> 1;
    const int sp = blockIdx.z & 1;               // this CTA's key tiles: kt = sp mod 2
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        mbar_init(&bar_s, 1);
        mbar_init(&bar_o, 1);
        mbar_fence_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(&tmem_slot, kTcTmemCols);
        tc::tmem_relinquish();
    }
    // power-of-two operand scales from the qk-norm bounds (immutable gammas):
    // |q|, |k| <= sqrt(128) max |gamma| after the norm and the rotation
    {
        float m = 0.0f;
        if (tid < HD) m = fabsf(__half2float(a.q_gamma[tid]));
        else m = fabsf(__half2float(a.k_gamma[tid - HD]));
        m = warp_max(m);
        if (lane == 0) red_s[warp] = m;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    float gq = 0.0f, gk = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; w++) {
        gq = fmaxf(gq, red_s[w]);
        gk = fmaxf(gk, red_s[4 + w]);
    }
    const float sq = __fmul_rn(__fsqrt_rn((float)HD), 1.0009765625f);
    const int eq = tc_exponent(__fmul_rn(sq, gq)), ek = tc_exponent(__fmul_rn(sq, gk));
    const float qs = __int_as_float((127 + eq) << 23), ks = __int_as_float((127 + ek) << 23);
    const float unscale = __int_as_float((127 - eq - ek) << 23);

    griddep_launch_dependents();
    griddep_wait();
    const int L0 = __ldcg(a.len + b);
    bool bad = L0 + a.T > a.kv.max_pos;
    if (bad && tid == 0 && qb == 0 && h == 0) raise_error(a.err, kDevRange);
    const int t0 = qb * BQ;
    const int nq = min(BQ, a.T - t0);
    const int kend = L0 + t0 + max(nq, 0);  // keys [0, kend) are visible to some row
    const bool run = !bad && nq > 0;
    const int ntiles = run ? (kend + kTcN - 1) / kTcN : 0;
    bool big = false;
    // f32 K / V rows of tile kt -> staging (16-byte cp.async pieces; rows past
    // kend are zeros: never visible, and unwritten cache memory may hold anything)
    auto stage_tile = [&](int kt) {
        const int k0 = kt * kTcN;
        for (int i = tid; i < kTcN * (HD / 4); i += kTcThreads) {
            const int n = i >> 5, d4 = i & 31;
            float *kd = reinterpret_cast<float *>(sm + kTcSK) + n * kTcSRow + 4 * d4;
            float *vd = reinterpret_cast<float *>(sm + kTcSV) + n * kTcSRow + 4 * d4;
            if (k0 + n < kend) {
                const int64_t row = a.kv.row(b, h, k0 + n);
                pf_cp16(kd, a.kv.k + row + 4 * d4);
                pf_cp16(vd, a.kv.v + row + 4 * d4);
            } else {
                *reinterpret_cast<float4 *>(kd) = make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<float4 *>(vd) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (sp < ntiles) stage_tile(sp);

    // ---- Q (A operand of S): vector m = head g = m / BQ, token m % BQ
    // thread -> (row, 8-d block) with 8 consecutive rows per 8 lanes: each
    // quarter-warp's 16-byte stores fill distinct bank slots
    for (int i = tid; i < kTcM * (HD / 8); i += kTcThreads) {
        const int m = (i & 7) | ((i >> 7) << 3), kb = (i >> 3) & 15;
        const int g = m / BQ, tl = m % BQ;
        float x[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (tl < nq) {
            const float4 *src = reinterpret_cast<const float4 *>(
                a.qkv + (int64_t)(b * a.T + t0 + tl) * a.ldqkv + (int64_t)(h * G + g) * HD + 8 * kb);
            const float4 u0 = __ldcg(src), u1 = __ldcg(src + 1);
            x[0] = u0.x; x[1] = u0.y; x[2] = u0.z; x[3] = u0.w;
            x[4] = u1.x; x[5] = u1.y; x[6] = u1.z; x[7] = u1.w;
        }
#pragma unroll
        for (int e = 0; e < 8; e++) x[e] = __fmul_rn(x[e], qs);
        uint4 hi, lo;
        big |= tc_split8(x, hi, lo);
        *reinterpret_cast<uint4 *>(sm + kTcQ + tc_off(m, kb, 16)) = hi;
        *reinterpret_cast<uint4 *>(sm + kTcQl + tc_off(m, kb, 16)) = lo;
    }

    // softmax role: row m = 32 (warp % 4) + lane (its TMEM lane), half hs =
    // warp / 4 of the row's keys for P and of the output columns
    const int mrow = 32 * (warp & 3) + lane, hs = warp >> 2;
    const int tl_r = mrow % BQ;
    const int qpos = L0 + t0 + tl_r;
    const bool rvalid = tl_r < nq;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));  // talker.rs:305
    float m_run = -INFINITY, l_run = 0.0f;
    float o[64];
#pragma unroll
    for (int i = 0; i < 64; i++) o[i] = 0.0f;
    const uint32_t t_lane = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    constexpr uint32_t id_s = tc::idesc_f16_f32(128, kTcN);
    constexpr uint32_t id_o = tc::idesc_f16_f32(128, HD);
    const uint32_t sbase = smem_u32(sm);

    for (int kt = sp, it = 0; kt < ntiles; kt += 2, it++) {
        const int k0 = kt * kTcN;
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();  // tile kt staged (every thread's pieces)
        const float *skf = reinterpret_cast<const float *>(sm + kTcSK);
        const float *svf = reinterpret_cast<const float *>(sm + kTcSV);
        // ---- K tile: B[key n][d]; thread -> (key, 8-d block) pairs
        for (int i = tid; i < kTcN * (HD / 8); i += kTcThreads) {
            const int n = (i & 7) | ((i >> 7) << 3), kb = (i >> 3) & 15;
            const float4 u0 = *reinterpret_cast<const float4 *>(skf + n * kTcSRow + 8 * kb);
            const float4 u1 = *reinterpret_cast<const float4 *>(skf + n * kTcSRow + 8 * kb + 4);
            float x[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int e = 0; e < 8; e++) x[e] = __fmul_rn(x[e], ks);
            uint4 hi, lo;
            big |= tc_split8(x, hi, lo);
            *reinterpret_cast<uint4 *>(sm + kTcK + tc_off(n, kb, 16)) = hi;
            *reinterpret_cast<uint4 *>(sm + kTcKl + tc_off(n, kb, 16)) = lo;
        }
        // ---- V tile transposed: B[d][key]; thread -> (d, four 8-key blocks):
        // consecutive lanes read consecutive words and store distinct slots
        {
            const int d = tid & 127, nb0 = (tid >> 7) * 4;
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int nb = nb0 + q;
                float x[8];
#pragma unroll
                for (int j = 0; j < 8; j++) x[j] = svf[(8 * nb + j) * kTcSRow + d];
                uint4 hi, lo;
                big |= tc_split8(x, hi, lo);
                *reinterpret_cast<uint4 *>(sm + kTcV + tc_off(d, nb, 8)) = hi;
                *reinterpret_cast<uint4 *>(sm + kTcVl + tc_off(d, nb, 8)) = lo;
            }
        }
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();
        __syncthreads();  // operands written, staging read
        if (kt + 2 < ntiles) stage_tile(kt + 2);  // lands while this tile computes
        // ---- S = Qh Kh + Qh Kl + Ql Kh
        if (tid == 0) {
            tc::fence_after_sync();
#pragma unroll
            for (int j = 0; j < HD / 16; j++) {
                const uint64_t qh = tc::smem_desc(sbase + kTcQ + 256 * j, 128, 2048);
                const uint64_t ql = tc::smem_desc(sbase + kTcQl + 256 * j, 128, 2048);
                const uint64_t kh = tc::smem_desc(sbase + kTcK + 256 * j, 128, 2048);
                const uint64_t kl = tc::smem_desc(sbase + kTcKl + 256 * j, 128, 2048);
                tc::mma_f16(tmem, qh, kh, id_s, j != 0 ? 1u : 0u);
                tc::mma_f16(tmem, qh, kl, id_s, 1u);
                tc::mma_f16(tmem, ql, kh, id_s, 1u);
            }
            tc::commit(&bar_s);
        }
        // bounded wait (phase kt of bar_s)
        {
            const long long tw = clock64();
            while (!mbar_try_wait(&bar_s, it & 1))
                if (clock64() - tw > (1ll << 31)) {
                    raise_error(a.err, kDevTimeout);
                    break;
                }
        }
        tc::fence_after_sync();
        // ---- online softmax: each of the row's two threads takes half the
        // keys; the halves' max and sum meet in shared memory (half 0 first)
        float sv[32];
        tc::ld_32x32b_x32(t_lane + 32 * hs, sv);
        float rmax = -INFINITY;
#pragma unroll
        for (int c = 0; c < 32; c++) {
            const bool vis = rvalid && k0 + 32 * hs + c <= qpos;
            sv[c] = vis ? __fmul_rn(__fmul_rn(sv[c], unscale), scale) : -INFINITY;
            rmax = fmaxf(rmax, sv[c]);
        }
        red_m[hs][mrow] = rmax;
        __syncthreads();
        const float m_new = fmaxf(m_run, fmaxf(red_m[0][mrow], red_m[1][mrow]));
        float psum = 0.0f;
#pragma unroll
        for (int c = 0; c < 32; c++) {
            sv[c] = m_new == -INFINITY ? 0.0f : __expf(sv[c] - m_new);
            psum += sv[c];
        }
        red_l[hs][mrow] = psum;
        // P (A operand of O): row mrow, keys 32 hs .. +31
#pragma unroll
        for (int kb = 0; kb < 4; kb++) {
            float x[8];
#pragma unroll
            for (int e = 0; e < 8; e++) x[e] = sv[8 * kb + e];
            uint4 hi, lo;
            tc_split8(x, hi, lo);
            *reinterpret_cast<uint4 *>(sm + kTcP + tc_off(mrow, 4 * hs + kb, 8)) = hi;
            *reinterpret_cast<uint4 *>(sm + kTcPl + tc_off(mrow, 4 * hs + kb, 8)) = lo;
        }
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();
        __syncthreads();
        // ---- O_tile = Ph Vh + Ph Vl + Pl Vh
        if (tid == 0) {
            tc::fence_after_sync();
#pragma unroll
            for (int j = 0; j < kTcN / 16; j++) {
                const uint64_t ph = tc::smem_desc(sbase + kTcP + 256 * j, 128, 1024);
                const uint64_t pl = tc::smem_desc(sbase + kTcPl + 256 * j, 128, 1024);
                const uint64_t vh = tc::smem_desc(sbase + kTcV + 256 * j, 128, 1024);
                const uint64_t vl = tc::smem_desc(sbase + kTcVl + 256 * j, 128, 1024);
                tc::mma_f16(tmem + kTcN, ph, vh, id_o, j != 0 ? 1u : 0u);
                tc::mma_f16(tmem + kTcN, ph, vl, id_o, 1u);
                tc::mma_f16(tmem + kTcN, pl, vh, id_o, 1u);
            }
            tc::commit(&bar_o);
        }
        const float corr = m_new == -INFINITY ? 1.0f : __expf(m_run - m_new);  // exp(-inf) = 0
        l_run = __fmaf_rn(l_run, corr, __fadd_rn(red_l[0][mrow], red_l[1][mrow]));
        m_run = m_new;
        {
            const long long tw = clock64();
            while (!mbar_try_wait(&bar_o, it & 1))
                if (clock64() - tw > (1ll << 31)) {
                    raise_error(a.err, kDevTimeout);
                    break;
                }
        }
        tc::fence_after_sync();
        {
            float u0[32], u1[32];
            tc::ld_32x32b_x32(t_lane + kTcN + 64 * hs, u0);
            tc::ld_32x32b_x32(t_lane + kTcN + 64 * hs + 32, u1);
#pragma unroll
            for (int c = 0; c < 32; c++) {
                o[c] = __fadd_rn(__fmul_rn(o[c], corr), u0[c]);
                o[32 + c] = __fadd_rn(__fmul_rn(o[32 + c], corr), u1[c]);
            }
        }
        tc::fence_before_sync();
        __syncthreads();  // shared operands and tensor memory are rewritten next
    }
    if (big) raise_error(a.err, kDevF16Range);
    // ---- the two CTAs' partial states (even and odd key tiles) meet in
    // global scratch; the second to finish merges them, split 0 first, and
    // writes out = O / l: row mrow, columns 64 hs .. +63.  The scratch is
    // indexed by the query vector itself ((stream, token) row x query head),
    // so it needs rows x heads x 2 x (128 + 2) floats whatever the block
    // shape: within attn_part_o_floats / attn_part_ml_floats of those rows.
    if (run) {
        const int64_t pair = ((int64_t)b * a.kv_heads + h) * gridDim.x + qb;
        const int64_t vec = (int64_t)(b * a.T + t0 + tl_r) * a.heads + h * G + mrow / BQ;
        if (rvalid) {
            float *po = a.part_o + (vec * 2 + sp) * HD + 64 * hs;
#pragma unroll
            for (int c = 0; c < 64; c += 4)
                __stcg(reinterpret_cast<float4 *>(po + c), make_float4(o[c], o[c + 1], o[c + 2], o[c + 3]));
            if (hs == 0) {
                __stcg(a.part_ml + (vec * 2 + sp) * 2, m_run);
                __stcg(a.part_ml + (vec * 2 + sp) * 2 + 1, l_run);
            }
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) last_flag = atomicAdd(&a.tickets[pair], 1u) == 1u;
        __syncthreads();
        if (last_flag && rvalid) {
            __threadfence();
            const float *p0 = a.part_o + (vec * 2) * HD + 64 * hs;
            const float *p1 = p0 + HD;
            const float *q0 = a.part_ml + (vec * 2) * 2;
            const float *q1 = q0 + 2;
            const float m0 = __ldcg(q0), l0 = __ldcg(q0 + 1), m1 = __ldcg(q1), l1 = __ldcg(q1 + 1);
            const float M = fmaxf(m0, m1);
            const float w0 = m0 == -INFINITY ? 0.0f : __expf(m0 - M);
            const float w1 = m1 == -INFINITY ? 0.0f : __expf(m1 - M);
            const float L = __fadd_rn(__fmul_rn(l0, w0), __fmul_rn(l1, w1));
            {
                const int g = mrow / BQ;
                float *dst = a.out + (int64_t)(b * a.T + t0 + tl_r) * a.ldout + (int64_t)(h * G + g) * HD + 64 * hs;
#pragma unroll
                for (int c = 0; c < 64; c += 4) {
                    const float4 u = __ldcg(reinterpret_cast<const float4 *>(p0 + c));
                    const float4 v = __ldcg(reinterpret_cast<const float4 *>(p1 + c));
                    float4 r;
                    r.x = __fdiv_rn(__fadd_rn(__fmul_rn(u.x, w0), __fmul_rn(v.x, w1)), L);
                    r.y = __fdiv_rn(__fadd_rn(__fmul_rn(u.y, w0), __fmul_rn(v.y, w1)), L);
                    r.z = __fdiv_rn(__fadd_rn(__fmul_rn(u.z, w0), __fmul_rn(v.z, w1)), L);
                    r.w = __fdiv_rn(__fadd_rn(__fmul_rn(u.w, w0), __fmul_rn(v.w, w1)), L);
                    *reinterpret_cast<float4 *>(dst + c) = r;
                }
            }
        }
        if (last_flag && tid == 0) a.tickets[pair] = 0u;
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTcTmemCols);
    }
}

// ------------------------------------------------------------------------
// Decode attention over a long cache, streamed (T = 1; the attention block of
// forward_with_embedding, talker.rs:285-331): one CTA per (kv head, position
// split, stream row) as k_attention.  A producer warp pulls the split's K and
// V rows into a ring of kDsStages shared-memory stages with cp.async.bulk
// (one contiguous copy per tile for K and one for V: a (stream, kv head)
// slab holds its positions back to back), completion on a "full" mbarrier per
// stage; eight compute warps each take every eighth position of a stage and
// keep their own running max / sum / weighted V sum per query head (online
// softmax), so no block-wide barrier falls inside the loop: a warp releases
// a stage on its "empty" mbarrier and moves on.  The warps' states merge once
// at the end, then the splits merge as in k_attention (last arriver, split
// order).  qk-norm + RoPE of the query heads and of the new key, and the
// append of the new K / V row at the cache length, are fused as in
// k_attention; the split that holds the new row reads it from shared memory
// (its bulk copy stops before that row).  Every mbarrier wait is bounded.
constexpr int kDsWarps = 8;                    // compute warps
constexpr int kDsThreads = (kDsWarps + 1) * 32; // + the producer warp
constexpr int kDsStages = 4;
constexpr int kDsTileBytes = 8192;             // K (and V) bytes per tile
constexpr int kDsMinChunk = 128;               // positions per split at least

template <int HD, int G>
struct DsSmem {
    static constexpr int TP = kDsTileBytes / (HD * 4);  // positions per tile
    float k[kDsStages][TP][HD];
    float v[kDsStages][TP][HD];
    float q[G][HD];
    float newk[HD], newv[HD];
    float wo[kDsWarps][G][HD];     // each warp's weighted V sums at the end
    float wm[kDsWarps][G], wl[kDsWarps][G];
    uint64_t full[kDsStages], empty[kDsStages];
    int last_flag;
    int abort;
};

template <int HD, int G>
__global__ void __launch_bounds__(kDsThreads, 2) k_attn_stream(const AttnArgs a) {
    using Sm = DsSmem<HD, G>;
    constexpr int TP = Sm::TP;
    constexpr int J = HD / 32;     // head-dimension values per lane (contiguous)
    extern __shared__ float4 ds_dyn[];
    Sm &sm = *reinterpret_cast<Sm *>(ds_dyn);
    const int kvh = blockIdx.x, split = blockIdx.y, r = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        for (int s = 0; s < kDsStages; s++) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], kDsWarps);
        }
        sm.abort = 0;
        mbar_fence_init();
    }
    __syncthreads();
    griddep_launch_dependents();
    griddep_wait();
    const int b = r;  // T = 1: one row per stream
    const int L0 = a.len_static >= 0 ? a.len_static : __ldcg(a.len + b);
    if (L0 + 1 > a.kv.max_pos) {
        if (tid == 0 && split == 0 && kvh == 0) raise_error(a.err, kDevRange);
        return;
    }
    const int Lq = L0 + 1;
    const int nsplit0 = min(kAttnMaxSplit, max(1, Lq / kDsMinChunk));
    const int chunk = ((Lq + nsplit0 - 1) / nsplit0 + TP - 1) / TP * TP;  // whole tiles
    const int nsplit = (Lq + chunk - 1) / chunk;
    if (split >= nsplit) return;
    const int p0 = split * chunk, p1 = min(Lq, p0 + chunk);
    const bool appender = (p1 == Lq);
    const int ntiles = (p1 - p0 + TP - 1) / TP;
    const float *cr = nullptr, *sr = nullptr;
    if (!rope_rows<HD>(a, b, 0, L0, cr, sr)) {
        if (tid == 0 && split == 0 && kvh == 0) raise_error(a.err, kDevRange);
        return;
    }
    if (warp == kDsWarps) {
        // ------------------------------------------------------ producer
        // tile i: positions [p0 + i TP, ..), its cached rows (< L0) by bulk copy
        if (lane == 0) {
            for (int i = 0; i < ntiles; i++) {
                const int s = i % kDsStages;
                if (i >= kDsStages &&
                    !mbar_wait_bounded(&sm.empty[s], ((i / kDsStages) + 1) & 1, a.err)) {
                    sm.abort = 1;
                    break;
                }
                if (*(volatile int *)&sm.abort) break;
                const int t0 = p0 + i * TP;
                const int nrow = max(0, min(min(t0 + TP, p1), L0) - t0);
                const uint32_t bytes = (uint32_t)nrow * HD * 4;
                mbar_arrive_expect_tx(&sm.full[s], 2 * bytes);
                if (bytes) {  // t0 is a multiple of TP, which divides the page size
                    bulk_g2s(&sm.k[s][0][0], a.kv.k + a.kv.row(b, kvh, t0), bytes, &sm.full[s]);
                    bulk_g2s(&sm.v[s][0][0], a.kv.v + a.kv.row(b, kvh, t0), bytes, &sm.full[s]);
                }
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------ compute warps
        // query heads (qk-norm + RoPE) and, on the appending split, the new row
        const float *row = a.qkv + (int64_t)r * a.ldqkv;
        for (int it = warp; it < G + 2; it += kDsWarps) {
            if (it >= G && !appender) continue;
            float v[J];
            const int64_t off = it < G ? (int64_t)(kvh * G + it) * HD
                                       : (it == G ? (int64_t)(a.heads + kvh) * HD
                                                  : (int64_t)(a.heads + a.kv_heads + kvh) * HD);
#pragma unroll
            for (int j = 0; j < J; j++) v[j] = __ldcg(row + off + lane + 32 * j);
            if (it < G) {
                norm_rope_head<HD>(v, a.q_gamma, cr, sr, true, lane);
#pragma unroll
                for (int j = 0; j < J; j++) sm.q[it][lane + 32 * j] = v[j];
            } else if (it == G) {
                norm_rope_head<HD>(v, a.k_gamma, cr, sr, true, lane);
                float *dst = a.kv.k + a.kv.row(b, kvh, L0);
#pragma unroll
                for (int j = 0; j < J; j++) {
                    sm.newk[lane + 32 * j] = v[j];
                    dst[lane + 32 * j] = v[j];
                }
            } else {
                float *dst = a.kv.v + a.kv.row(b, kvh, L0);
#pragma unroll
                for (int j = 0; j < J; j++) {
                    sm.newv[lane + 32 * j] = v[j];
                    dst[lane + 32 * j] = v[j];
                }
            }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kDsWarps * 32) : "memory");
        // lane holds head-dimension values J*lane .. J*lane + J - 1
        float qr[G][J], o[G][J], m[G], l[G];
#pragma unroll
        for (int g = 0; g < G; g++) {
#pragma unroll
            for (int j = 0; j < J; j++) {
                qr[g][j] = sm.q[g][J * lane + j];
                o[g][j] = 0.0f;
            }
            m[g] = -INFINITY;
            l[g] = 0.0f;
        }
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));  // talker.rs:305
        for (int i = 0; i < ntiles; i++) {
            const int s = i % kDsStages;
            const int t0 = p0 + i * TP;
            const int cnt = min(TP, p1 - t0);
            if (!mbar_wait_bounded(&sm.full[s], (i / kDsStages) & 1, a.err)) sm.abort = 1;
            if (*(volatile int *)&sm.abort) break;
            for (int pp = warp; pp < cnt; pp += kDsWarps) {
                const bool fresh = appender && t0 + pp == L0;
                const float *kr = fresh ? sm.newk : &sm.k[s][pp][0];
                const float *vr = fresh ? sm.newv : &sm.v[s][pp][0];
                float kk[J], vv[J];
                if constexpr (J % 4 == 0) {   // head_dim 128: 16-byte pieces
#pragma unroll
                    for (int j = 0; j < J; j += 4) {
                        const float4 k4 = *reinterpret_cast<const float4 *>(kr + J * lane + j);
                        const float4 v4 = *reinterpret_cast<const float4 *>(vr + J * lane + j);
                        kk[j] = k4.x; kk[j + 1] = k4.y; kk[j + 2] = k4.z; kk[j + 3] = k4.w;
                        vv[j] = v4.x; vv[j + 1] = v4.y; vv[j + 2] = v4.z; vv[j + 3] = v4.w;
                    }
                } else {                      // head_dim 64: 8-byte pieces
                    static_assert(J == 2, "head_dim 64 or 128");
                    const float2 k2 = *reinterpret_cast<const float2 *>(kr + J * lane);
                    const float2 v2 = *reinterpret_cast<const float2 *>(vr + J * lane);
                    kk[0] = k2.x; kk[1] = k2.y;
                    vv[0] = v2.x; vv[1] = v2.y;
                }
                float d[G];
#pragma unroll
                for (int g = 0; g < G; g++) {
                    float t = 0.0f;
#pragma unroll
                    for (int j = 0; j < J; j++) t = __fmaf_rn(qr[g][j], kk[j], t);
                    d[g] = t;
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                    for (int g = 0; g < G; g++) d[g] += __shfl_xor_sync(0xffffffffu, d[g], off);
#pragma unroll
                for (int g = 0; g < G; g++) {
                    const float sc = __fmul_rn(d[g], scale);
                    const float m_new = fmaxf(m[g], sc);
                    const float corr = expf(m[g] - m_new);   // exp(-inf) = 0 at the first position
                    const float pe = expf(sc - m_new);
                    l[g] = __fmaf_rn(l[g], corr, pe);
#pragma unroll
                    for (int j = 0; j < J; j++) o[g][j] = __fmaf_rn(pe, vv[j], __fmul_rn(o[g][j], corr));
                    m[g] = m_new;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[s]);
        }
        // this warp's state -> shared memory
#pragma unroll
        for (int g = 0; g < G; g++) {
#pragma unroll
            for (int j = 0; j < J; j++) sm.wo[warp][g][J * lane + j] = o[g][j];
            if (lane == 0) {
                sm.wm[warp][g] = m[g];
                sm.wl[warp][g] = l[g];
            }
        }
    }
    __syncthreads();
    if (sm.abort) {
        // copies still in flight land before the CTA exits (bounded)
        if (tid == 0)
            for (int i = max(0, ntiles - kDsStages); i < ntiles; i++)
                mbar_wait_bounded(&sm.full[i % kDsStages], (i / kDsStages) & 1, nullptr);
        __syncthreads();
        return;
    }
    // ---- merge the warps (fixed warp order): M = max m_w, L = sum l_w e^(m_w - M), O likewise
    const int64_t out_base = (int64_t)r * a.ldout + (int64_t)kvh * G * HD;
    const int64_t slot = ((int64_t)r * a.kv_heads + kvh) * kAttnMaxSplit;
    for (int o = tid; o < G * HD; o += kDsThreads) {
        const int g = o / HD, dd = o % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kDsWarps; w++) M = fmaxf(M, sm.wm[w][g]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < kDsWarps; w++) {
            const float e = sm.wl[w][g] > 0.0f ? expf(sm.wm[w][g] - M) : 0.0f;
            L = __fmaf_rn(sm.wl[w][g], e, L);
            O = __fmaf_rn(sm.wo[w][g][dd], e, O);
        }
        if (nsplit == 1) {
            a.out[out_base + o] = __fdiv_rn(O, L);
        } else {
            __stcg(a.part_o + (slot + split) * (G * HD) + o, O);
            if (dd == 0) {
                __stcg(a.part_ml + ((slot + split) * G + g) * 2 + 0, M);
                __stcg(a.part_ml + ((slot + split) * G + g) * 2 + 1, L);
            }
        }
    }
    if (nsplit == 1) return;
    // ---- split partials: the last split to arrive merges them in split order
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned tk = atomicAdd(&a.tickets[(int64_t)r * a.kv_heads + kvh], 1u);
        sm.last_flag = (tk == (unsigned)(nsplit - 1));
    }
    __syncthreads();
    if (!sm.last_flag) return;
    __threadfence();
    for (int o = tid; o < G * HD; o += kDsThreads) {
        const int g = o / HD;
        float M = -INFINITY;
        for (int sp = 0; sp < nsplit; sp++) M = fmaxf(M, __ldcg(a.part_ml + ((slot + sp) * G + g) * 2));
        float L = 0.0f, O = 0.0f;
        for (int sp = 0; sp < nsplit; sp++) {
            const float w = expf(__ldcg(a.part_ml + ((slot + sp) * G + g) * 2) - M);
            L = __fmaf_rn(__ldcg(a.part_ml + ((slot + sp) * G + g) * 2 + 1), w, L);
            O = __fmaf_rn(__ldcg(a.part_o + (slot + sp) * (G * HD) + o), w, O);
        }
        a.out[out_base + o] = __fdiv_rn(O, L);
    }
    if (tid == 0) a.tickets[(int64_t)r * a.kv_heads + kvh] = 0u;
}

template <int HD, int G>
int launch_attn_stream_g(const AttnArgs &a, cudaStream_t st) {
    // the kernel splits a row's positions into at most kAttnMaxSplit runs of
    // whole tiles, at least kDsMinChunk positions each: this bounds the grid
    const int ysplit = std::max(1, std::min(kAttnMaxSplit, a.kv.max_pos / kDsMinChunk));
    dim3 grid(a.kv_heads, ysplit, a.streams);
    constexpr size_t smem = sizeof(DsSmem<HD, G>);
    static bool attr_done[64] = {};  // per device, per instantiation
    int dev = 0;
    QORA_CUDA(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        QORA_CUDA(cudaFuncSetAttribute(k_attn_stream<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
        attr_done[dev] = true;
    }
    return launch_ex(k_attn_stream<HD, G>, grid, dim3(kDsThreads), smem, st, 1u, a);
}

template <int HD>
int launch_attn_stream_hd(const AttnArgs &a, cudaStream_t st) {
    switch (a.heads / a.kv_heads) {
        case 1: return launch_attn_stream_g<HD, 1>(a, st);
        case 2: return launch_attn_stream_g<HD, 2>(a, st);
        case 4: return launch_attn_stream_g<HD, 4>(a, st);
    }
    return set_error(QORA_ERR_UNSUPPORTED, "heads/kv_heads = %d", a.heads / a.kv_heads);
}

template <int HD, int G>
int launch_prefill_attn_g(const AttnArgs &a, cudaStream_t st) {
    constexpr int BQ = kPfM / G;
    static bool attr_done[64] = {};
    int dev = 0;
    QORA_CUDA(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        QORA_CUDA(cudaFuncSetAttribute(k_prefill_attn<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sizeof(PfSmem<HD>)));
        attr_done[dev] = true;
    }
    dim3 grid((a.T + BQ - 1) / BQ, a.kv_heads, a.streams);
    return launch_ex(k_prefill_attn<HD, G>, grid, dim3(kPfThreads), sizeof(PfSmem<HD>), st, 1u, a);
}

// Caches of at least this many positions decode on the streamed kernel and
// prefill on the tensor-core kernel.
constexpr int kStreamMinCapacity = 256;

// QORA_PREFILL_ATTN_TC=0 in the environment keeps head_dim-128 prefills on
// the CUDA-core kernel (for comparison).
bool prefill_attn_tc_disabled() {
    static const bool off = [] {
        const char *v = getenv("QORA_PREFILL_ATTN_TC");
        return v && v[0] == '0';
    }();
    return off;
}

template <int G>
int launch_prefill_attn_tc_g(const AttnArgs &a, cudaStream_t st) {
    constexpr int BQ = kTcM / G;
    static bool attr_done[64] = {};
    int dev = 0;
    QORA_CUDA(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        QORA_CUDA(cudaFuncSetAttribute(k_prefill_attn_tc<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcBytes));
        attr_done[dev] = true;
    }
    // two CTAs per query block (even and odd key tiles)
    dim3 grid((a.T + BQ - 1) / BQ, a.kv_heads, 2 * a.streams);
    return launch_ex(k_prefill_attn_tc<G>, grid, dim3(kTcThreads), (size_t)kTcBytes, st, 1u, a);
}

// The tensor-core kernel serves caches of kStreamMinCapacity positions or
// more (the talker's); short caches (the predictor's, whose per-op batched
// path prefills 2 tokens per stream) keep the f32 kernel, whose small CTAs
// suit them.  The choice depends on the cache only, so every prefill call
// into one cache uses the same kernel (same bits however a prompt is split).
template <int HD>
int launch_prefill_attn_hd(const AttnArgs &a, cudaStream_t st) {
    if (HD == 128 && a.kv.max_pos >= kStreamMinCapacity && !prefill_attn_tc_disabled()) {
        switch (a.heads / a.kv_heads) {
            case 1: return launch_prefill_attn_tc_g<1>(a, st);
            case 2: return launch_prefill_attn_tc_g<2>(a, st);
            case 4: return launch_prefill_attn_tc_g<4>(a, st);
        }
    }
    switch (a.heads / a.kv_heads) {
        case 1: return launch_prefill_attn_g<HD, 1>(a, st);
        case 2: return launch_prefill_attn_g<HD, 2>(a, st);
        case 4: return launch_prefill_attn_g<HD, 4>(a, st);
    }
    return set_error(QORA_ERR_UNSUPPORTED, "heads/kv_heads = %d", a.heads / a.kv_heads);
}

template <int HD>
int launch_attn_hd(const AttnArgs &a, cudaStream_t st) {
    const int G = a.heads / a.kv_heads;
    const int rows = a.streams * a.T;
    // position splits: the kernel uses min(16, ceil(positions / 32)) of them
    // and positions never exceed the cache capacity, so that bounds the grid
    // (a short cache such as the predictor's launches one split per row)
    const int ysplit = std::max(1, std::min(kAttnMaxSplit, (a.kv.max_pos + attn::kTile - 1) / attn::kTile));
    dim3 grid(a.kv_heads, ysplit, rows);
    switch (G) {
        case 1: return launch_ex(k_attention<HD, 1>, grid, dim3(kThreads), 0, st, 1u, a);
        case 2: return launch_ex(k_attention<HD, 2>, grid, dim3(kThreads), 0, st, 1u, a);
        case 4: return launch_ex(k_attention<HD, 4>, grid, dim3(kThreads), 0, st, 1u, a);
    }
    return set_error(QORA_ERR_UNSUPPORTED, "heads/kv_heads = %d", G);
}

}  // namespace

int launch_qkv_post(const AttnArgs &a, cudaStream_t st) {
    const int rows = a.streams * a.T;
    if (rows <= 0) return QORA_OK;
    switch (a.kv.head_dim) {
        case 64: return launch_ex(k_qkv_post<64>, dim3(rows), dim3(kThreads), 0, st, 1u, a);
        case 128: return launch_ex(k_qkv_post<128>, dim3(rows), dim3(kThreads), 0, st, 1u, a);
    }
    return set_error(QORA_ERR_UNSUPPORTED, "head_dim %d", a.kv.head_dim);
}


int launch_attention(const AttnArgs &a, cudaStream_t st) {
    if (!a.preappended && a.T != 1)
        return set_error(QORA_ERR_INVALID, "fused append needs T == 1");
    if (a.streams * a.T <= 0) return QORA_OK;
    // every pre-appended (prefill) run takes the tiled causal kernel, whatever
    // its length: a row's bits then do not depend on how a prompt was split
    // into prefill calls (prefix cache, generate_new.rs:320-322)
    if (a.preappended && a.len && a.pos_static < 0 && a.len_static < 0) {
        switch (a.kv.head_dim) {  // tiled causal prefill
            case 64: return launch_prefill_attn_hd<64>(a, st);
            case 128: return launch_prefill_attn_hd<128>(a, st);
        }
    }
    // decode over a long cache: the streamed kernel (a short cache such as
    // the predictor's, refilled every frame, keeps the per-tile kernel)
    if (!a.preappended && a.kv.max_pos >= kStreamMinCapacity && a.pos_static < 0 && a.stable_len < 0) {
        switch (a.kv.head_dim) {
            case 64: return launch_attn_stream_hd<64>(a, st);
            case 128: return launch_attn_stream_hd<128>(a, st);
        }
    }
    switch (a.kv.head_dim) {
        case 64: return launch_attn_hd<64>(a, st);
        case 128: return launch_attn_hd<128>(a, st);
    }
    return set_error(QORA_ERR_UNSUPPORTED, "head_dim %d", a.kv.head_dim);
}

}  // namespace qora
