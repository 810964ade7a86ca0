// Persistent frame kernel (sm_100a): one launch = one frame of the
// reference's per-frame loop (generate_new.rs:606-665) for one stream:
//   sample_token (generate_new.rs:771-862) -> generate_acoustic_codes
//   (code_predictor.rs:218-273: 16 single-token passes of the 5-layer
//   predictor, 15 heads + argmax) -> frame-input assembly
//   (generate_new.rs:639-654) -> forward_with_embedding (talker.rs:263-360).
//
// Why: at batch 1 the frame is ~570 dependent steps whose weights (~1.5 GB of
// Q4 passes) would stream in ~0.2 ms, but as separate launches every step
// costs a kernel boundary (~6 us).  Here one CTA per SM walks the same op
// list; op i starts on an SM once every SM has finished op i-1 (a per-op
// arrival counter in global memory, bounded spin), so a step costs one
// counter round trip instead of a launch.
//
// Weight streaming is decoupled from that chain.  Each SM's share of every
// GEMV is known in advance (item j of op i runs on SM (j + rot_i) % grid),
// so a producer warp walks the op list ahead of the compute warps and pulls
// the SM's weight slices into a ring of shared-memory slots with
// cp.async.bulk (no multicast), signalling an mbarrier per slot; the compute
// warps consume slots in the same order and release them.  Weights are
// immutable, so the stream never waits on activations: while the compute
// warps wait for op i-1 to finish everywhere, the ring is already filling
// with op i, i+1, ... weights.
//
// Every GEMV item is one column unit (32 output columns, or a gate/up pair)
// over all K rows, so it ends with final values and applies its epilogue
// itself: residual add (plus the per-32-column sum of squares the next
// RMSNorm needs), bias, or silu(gate) * up.  An SM that has items in an op
// reads that op's whole input vector (<= 6144 floats, from L2) into shared
// memory and applies the RMSNorm prologue from those sums of squares, summed
// in the same fixed order on every SM.  The attention and sampler ops run the
// same device code as the standalone kernels (attention_impl.cuh,
// sampler_impl.cuh).
//
// Every wait is bounded (~2 s of globaltimer); a timeout raises kDevTimeout,
// sets a global abort flag that every other waiter polls, and the kernel
// drains its own in-flight bulk copies before returning.
#include <algorithm>
#include <cstring>

#include "attention_impl.cuh"
#include "frame.cuh"
#include "sampler_impl.cuh"

namespace qora {
namespace fk {

namespace {

constexpr uint64_t kWaitNs = 2000000000ull;  // bounded waits: 2 s

template <int HD, int G>
using ASmem = attn::AttnSmem<HD, G, kNT>;

struct alignas(128) FrameSmem {
    uint8_t nib[kSlots][kSlotNib];
    uint8_t scl[kSlots][kSlotScl];
    union U {
        float xs[kXMax];
        ASmem<128, 1> a128_1;
        ASmem<128, 2> a128_2;
        ASmem<128, 4> a128_4;
        ASmem<64, 1> a64_1;
        ASmem<64, 2> a64_2;
        ASmem<64, 4> a64_4;
        samp::SampleSmem<kNT, 1> samp;
    } u;
    float red[2][kNT / 32][2][32];     // per-item cross-warp reduction (double buffered)
    float bred[kNT / 32];              // block reductions
    int bidx[kNT / 32];
    uint64_t full[kSlots], empty[kSlots];
    int abort;
    // the current op's descriptor, staged from global memory while thread 0
    // waits for the op's dependency
    union alignas(16) Desc {
        GemvDesc g;
        AttnArgs a;
        uint4 words[1];
    } desc;
};
static_assert(sizeof(GemvDesc) % 16 == 0 && sizeof(AttnArgs) % 16 == 0, "descriptor staging");

__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kNT) : "memory"); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_volatile(const int *p) {
    int v;
    asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ int first_item(int cta, int rot, int grid) {
    int j = (cta - rot) % grid;
    return j < 0 ? j + grid : j;
}

__device__ __forceinline__ void stamp(const FrameParams &P, int op, int field, bool on) {
    if (on) P.trace[(int64_t)op * kTraceFields + field] = global_ns();
}

// Sets the abort state everywhere after a failed or timed-out wait.
__device__ __forceinline__ void raise_abort(const FrameParams &P, FrameSmem &S, int code) {
    raise_error(P.err, code);
    atomicExch(P.abort_flag, 1);
    S.abort = 1;
}

// Bounded mbarrier wait that also gives up when the CTA aborted.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t *bar, uint32_t parity, FrameSmem &S,
                                                   const FrameParams &P) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (int it = 0;; it++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63) == 63) {
            if (*(volatile int *)&S.abort) return false;
            if (global_ns() - t0 > kWaitNs) {
                raise_abort(P, S, kDevTimeout);
                return false;
            }
        }
    }
}

// ------------------------------------------------------------- producer
// One lane walks every GEMV op this SM has items in and streams the items'
// weight rows into the slot ring, in the order the compute warps consume them.
__device__ void producer(const FrameParams &P, FrameSmem &S, int cta, int grid) {
    uint32_t q = 0;
    bool ok = true;
    for (int i = 0; i < P.n_ops && ok; i++) {
        const OpRef op = P.ops[i];
        if (op.type != OP_GEMV) continue;
        const GemvDesc &d = P.gemv[op.idx];
        const int G = d.G, kpad = d.kpad;
        const int CR = G == 1 ? 1024 : 512;
        for (int u = first_item(cta, op.rot, grid); u < op.n_items && ok; u += grid) {
            for (int c0 = 0; c0 < kpad; c0 += CR) {
                const int rows = min(CR, kpad - c0);
                const int slot = q % kSlots;
                if (q >= kSlots && !mbar_wait_or_abort(&S.empty[slot], ((q / kSlots) - 1) & 1, S, P)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&S.full[slot], (uint32_t)(G * rows * 18));
                for (int g = 0; g < G; g++) {
                    const int64_t grp = (int64_t)u * G + g;
                    bulk_g2s(S.nib[slot] + g * rows * 16, d.nib + grp * kpad + c0, (uint32_t)rows * 16,
                             &S.full[slot]);
                    bulk_g2s(S.scl[slot] + g * rows * 2, d.scl + grp * kpad + c0, (uint32_t)rows * 2,
                             &S.full[slot]);
                }
                q++;
            }
        }
    }
    if (!ok || *(volatile int *)&S.abort) {
        // the compute warps stopped early: wait (bounded) for this SM's copies
        // still in flight before the CTA exits
        const uint32_t q0 = q > (uint32_t)kSlots ? q - kSlots : 0;
        for (uint32_t qq = q0; qq < q; qq++) {
            const uint64_t t0 = global_ns();
            while (!mbar_try_wait(&S.full[qq % kSlots], (qq / kSlots) & 1))
                if (global_ns() - t0 > kWaitNs) break;
        }
    }
}

// ------------------------------------------------------------- consumers
// Sum of one value per thread over the kNT compute threads in a fixed order
// (xor tree in each warp, warps in order).
__device__ __forceinline__ float block_sum(float v, FrameSmem &S, int tid) {
    v = warp_sum(v);
    if ((tid & 31) == 0) S.bred[tid >> 5] = v;
    csync();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < kNT / 32; w++) t += S.bred[w];
    csync();
    return t;
}

// Argmax of src[0..n) (n a multiple of 4, <= 4096); ties keep the larger
// index (the last maximum, code_predictor.rs:336-339).  Identical on every SM.
__device__ int block_argmax(const FrameParams &P, const float *src, int n, FrameSmem &S, int tid) {
    constexpr int U = 4;  // float4s per thread: 4 * 4 * 256 = 4096
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    float4 v[U];
#pragma unroll
    for (int m = 0; m < U; m++) {
        const int i = tid + m * kNT;
        if (4 * i < n) v[m] = __ldcg(s4 + i);
    }
    float bv = -INFINITY;
    int bi = -1;
#pragma unroll
    for (int m = 0; m < U; m++) {
        const int i = tid + m * kNT;
        if (4 * i < n) {
            const float e[4] = {v[m].x, v[m].y, v[m].z, v[m].w};
#pragma unroll
            for (int c = 0; c < 4; c++) {
                if (e[c] != e[c]) raise_error(P.err, kDevNaN);
                if (bi < 0 || e[c] > bv || (e[c] == bv && 4 * i + c > bi)) {
                    bv = e[c];
                    bi = 4 * i + c;
                }
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi > bi))) {
            bv = ov;
            bi = oi;
        }
    }
    if ((tid & 31) == 0) {
        S.bred[tid >> 5] = bv;
        S.bidx[tid >> 5] = bi;
    }
    csync();
    float best = -INFINITY;
    int idx = -1;
#pragma unroll
    for (int w = 0; w < kNT / 32; w++) {
        const int oi = S.bidx[w];
        const float ov = S.bred[w];
        if (oi >= 0 && (idx < 0 || ov > best || (ov == best && oi > idx))) {
            best = ov;
            idx = oi;
        }
    }
    csync();
    return idx < 0 ? 0 : idx;
}

// The 8 values of columns 8w..8w+7 of embedding row `code`: nibble word w
// and its group scale, dequantised as embed_lookup_q4 (gemv.rs:425-433):
// scale * (q - 8).
struct EmbWord {
    uint32_t w;
    float sc;
};
__device__ __forceinline__ EmbWord emb_word(const EmbDev &e, uint32_t code, int w) {
    EmbWord r;
    r.w = __ldg(reinterpret_cast<const uint32_t *>(e.packed + (int64_t)code * (e.n >> 1)) + w);
    r.sc = __half2float(e.scl[(int64_t)code * (e.n >> 5) + (w >> 2)]);
    return r;
}
__device__ __forceinline__ float emb_at(const EmbWord &e, int c) {
    return __fmul_rn(e.sc, (float)((int)((e.w >> (4 * c)) & 15u) - 8));
}

// Writes this SM's slice of x (the participating SMs partition [0, K)).
__device__ __forceinline__ void save_slice(const GemvDesc &d, const float *xs, int j0, int n_items,
                                           int grid, int tid) {
    const int parts = min(n_items, grid);
    const int a = (int)((int64_t)j0 * d.K / parts), b = (int)((int64_t)(j0 + 1) * d.K / parts);
    for (int k = a + tid; k < b; k += kNT) __stcg(d.save + k, xs[k]);
}

// Builds the GEMV input x[0..kpad) in shared memory (rows >= K are zero).
__device__ void build_input(const FrameParams &P, const GemvDesc &d, FrameSmem &S, int tid,
                            bool leader, int j0, int n_items, int grid) {
    float *xs = S.u.xs;
    const int K = d.K;
    switch (d.in_mode) {
        case IN_VEC: {
            // x in 8-float chunks (K is a multiple of 32); every load of the
            // thread (x, gamma, one sum-of-squares partial) in flight together
            constexpr int U = kXMax / 8 / kNT;
            const float4 *src = reinterpret_cast<const float4 *>(d.in);
            const uint4 *gm = reinterpret_cast<const uint4 *>(d.gamma);
            const int K8 = K >> 3;
            float4 v[U][2];
            uint4 gv[U];
#pragma unroll
            for (int m = 0; m < U; m++) {
                const int w = tid + m * kNT;
                if (w < K8) {
                    v[m][0] = __ldcg(src + 2 * w);
                    v[m][1] = __ldcg(src + 2 * w + 1);
                    if (d.gamma) gv[m] = __ldg(gm + w);
                }
            }
            const float ssp = (d.gamma && tid < (K >> 5)) ? __ldcg(d.ss_in + tid) : 0.0f;
            float inv = 1.0f;
            if (d.gamma) {
                // the producer's per-32-column sums of squares (K / 32 <= kNT of
                // them), summed by the fixed block tree: rms_norm_f16's
                // inv = 1 / sqrt(sum(x^2) / K + 1e-6)
                const float ssum = block_sum(ssp, S, tid);
                inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ssum, (float)K), 1e-6f)));
            }
            const bool pre_save = d.save && !d.save_normed;
#pragma unroll
            for (int m = 0; m < U; m++) {
                const int w = tid + m * kNT;
                if (w < K8) {
                    float e[8] = {v[m][0].x, v[m][0].y, v[m][0].z, v[m][0].w,
                                  v[m][1].x, v[m][1].y, v[m][1].z, v[m][1].w};
                    if (pre_save) {
                        // this SM's slice of the un-normalised input
                        const int parts = min(n_items, grid);
                        const int lo = (int)((int64_t)j0 * K / parts), hi = (int)((int64_t)(j0 + 1) * K / parts);
#pragma unroll
                        for (int c = 0; c < 8; c++)
                            if (8 * w + c >= lo && 8 * w + c < hi) __stcg(d.save + 8 * w + c, e[c]);
                    }
                    if (d.gamma) {
                        const __half *gh = reinterpret_cast<const __half *>(&gv[m]);
#pragma unroll
                        for (int c = 0; c < 8; c++) e[c] = __fmul_rn(__fmul_rn(e[c], inv), __half2float(gh[c]));
                    }
                    reinterpret_cast<float4 *>(xs)[2 * w] = make_float4(e[0], e[1], e[2], e[3]);
                    reinterpret_cast<float4 *>(xs)[2 * w + 1] = make_float4(e[4], e[5], e[6], e[7]);
                }
            }
            for (int k = K + tid; k < d.kpad; k += kNT) xs[k] = 0.0f;
            csync();
            if (d.save && d.save_normed) save_slice(d, xs, j0, n_items, grid, tid);
            return;
        }
        case IN_EMB: {
            uint32_t code;
            if (d.amax_src) {
                code = (uint32_t)block_argmax(P, d.amax_src, d.amax_n, S, tid);
                if (leader && tid == 0 && d.code_dst) __stcg(d.code_dst, code);
            } else {
                code = __ldcg(d.code_src);
            }
            for (int w = tid; w < (d.kpad >> 3); w += kNT) {
                float o[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                if (8 * w < K) {
                    const EmbWord e = emb_word(d.emb, code, w);
#pragma unroll
                    for (int c = 0; c < 8; c++) o[c] = emb_at(e, c);
                }
                reinterpret_cast<float4 *>(xs)[2 * w] = make_float4(o[0], o[1], o[2], o[3]);
                reinterpret_cast<float4 *>(xs)[2 * w + 1] = make_float4(o[4], o[5], o[6], o[7]);
            }
            break;
        }
        case IN_FRAME: {
            const FrameEmbed &fe = P.fe;
            const uint32_t last = (uint32_t)block_argmax(P, d.amax_src, d.amax_n, S, tid);
            if (leader && tid == 0) {
                __stcg(fe.codes + fe.ngroups, last);
                for (int g = 1; g < fe.ngroups; g++) __stcg(fe.prev + g, __ldcg(fe.codes + g));
                __stcg(fe.prev + fe.ngroups, last);
            }
            const uint32_t c0 = __ldcg(fe.codes);
            for (int w = tid; w < (d.kpad >> 3); w += kNT) {
                float o[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                if (8 * w < K) {
                    // every load of the 8 columns in flight before the sums
                    EmbWord e[kMaxEmbedGroups];
#pragma unroll
                    for (int g = 0; g < kMaxEmbedGroups; g++) {
                        if (g < fe.ngroups) {
                            const uint32_t cg = g + 1 < fe.ngroups ? __ldcg(fe.codes + g + 1) : last;
                            e[g] = emb_word(fe.pred[g], cg, w);
                        }
                    }
                    const EmbWord et = emb_word(fe.talker, c0, w);
                    const float4 t0 = __ldcg(reinterpret_cast<const float4 *>(P.text) + 2 * w);
                    const float4 t1 = __ldcg(reinterpret_cast<const float4 *>(P.text) + 2 * w + 1);
                    const float tx[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        // (E_talker[c0] + (sum_g E_g[c_{g+1}])) + text, as the engine's frame embed
                        float acc = 0.0f;
#pragma unroll
                        for (int g = 0; g < kMaxEmbedGroups; g++)
                            if (g < fe.ngroups) acc = __fadd_rn(acc, emb_at(e[g], c));
                        acc = __fadd_rn(emb_at(et, c), acc);
                        o[c] = __fadd_rn(acc, tx[c]);
                    }
                }
                reinterpret_cast<float4 *>(xs)[2 * w] = make_float4(o[0], o[1], o[2], o[3]);
                reinterpret_cast<float4 *>(xs)[2 * w + 1] = make_float4(o[4], o[5], o[6], o[7]);
            }
            break;
        }
    }
    csync();
    if (d.save && !d.save_normed) save_slice(d, xs, j0, n_items, grid, tid);
    if (d.gamma) {
        constexpr int U = kXMax / 8 / kNT;
        const uint4 *gm = reinterpret_cast<const uint4 *>(d.gamma);
        uint4 gv[U];
#pragma unroll
        for (int m = 0; m < U; m++)
            if (tid + m * kNT < (K >> 3)) gv[m] = __ldg(gm + tid + m * kNT);
        float t = 0.0f;
        for (int k = tid; k < K; k += kNT) t += __fmul_rn(xs[k], xs[k]);
        const float ss = block_sum(t, S, tid);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), 1e-6f)));
#pragma unroll
        for (int m = 0; m < U; m++) {
            const int w = tid + m * kNT;
            if (w < (K >> 3)) {
                const __half *gh = reinterpret_cast<const __half *>(&gv[m]);
#pragma unroll
                for (int c = 0; c < 8; c++) xs[8 * w + c] = __fmul_rn(__fmul_rn(xs[8 * w + c], inv), __half2float(gh[c]));
            }
        }
        csync();
    }
    if (d.save && d.save_normed) save_slice(d, xs, j0, n_items, grid, tid);
}

// One weight row of one 32-column group: acc += s' * nibbles, with
// s' = f32(scale) * x * 2^75 (gemv.rs:265 times an exact power of two).  A
// nibble at bit 4p of a half-word, read as f32 bits, is q * 2^(4p-149):
// linear in q, so one packed FMA handles two columns.
__device__ __forceinline__ void row_fma(uint64_t (&acc)[16], float &ssum, float sp, const uint4 wv) {
    ssum += sp;
    const uint64_t s2 = pk2(sp, sp);
    const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int w4 = 0; w4 < 4; w4++) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t v = h ? (words[w4] >> 16) : words[w4];
#pragma unroll
            for (int pp = 0; pp < 4; pp += 2) {
                const uint64_t qd = pk2(__uint_as_float(v & (0xFu << (4 * pp))),
                                        __uint_as_float(v & (0xFu << (4 * pp + 4))));
                const int jj = 4 * w4 + 2 * h + pp / 2;
                acc[jj] = ffma2(s2, qd, acc[jj]);
            }
        }
    }
}

// The items of one GEMV op on this SM, G groups per unit, all K rows each.
template <int G>
__device__ void gemv_items(const FrameParams &P, const GemvDesc &d, const OpRef &op, FrameSmem &S,
                           int tid, int cta, int grid, uint32_t &q, int &rbuf, bool tr, int op_i) {
    uint64_t waited = 0, slots = 0, comp = 0, redc = 0;
    const int lane = tid & 31, warp = tid >> 5;
    constexpr int CR = G == 1 ? 1024 : 512;
    const float *xs = S.u.xs;
    for (int u = first_item(cta, op.rot, grid); u < op.n_items; u += grid) {
        // the epilogue's residual / bias values, fetched while the item computes
        float pre = 0.0f;
        if (G == 1 && warp == 0) {
            const int64_t col = (int64_t)u * 32 + lane;
            if (d.out_mode == OUT_RESID) pre = __ldcg(d.resid + col);
            else if (d.bias) pre = __ldg(d.bias + col);
        }
        uint64_t acc[G][16];
        float ssum[G];
#pragma unroll
        for (int g = 0; g < G; g++) {
            ssum[g] = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; i++) acc[g][i] = 0ull;
        }
        for (int c0 = 0; c0 < d.kpad; c0 += CR) {
            const int rows = min(CR, d.kpad - c0);
            const int slot = q % kSlots;
            // on a failed wait the thread skips the slot but keeps to the
            // block's barrier sequence; the op ends with a uniform abort check
            const long long tw = tr ? clock64() : 0;
            const bool ok = mbar_wait_or_abort(&S.full[slot], (q / kSlots) & 1, S, P);
            long long tc = 0;
            if (tr) {
                tc = clock64();
                waited += (uint64_t)(tc - tw);
                slots++;
            }
            const uint4 *nb = reinterpret_cast<const uint4 *>(S.nib[slot]);
            const __half *sb = reinterpret_cast<const __half *>(S.scl[slot]);
            for (int lr = tid; ok && lr < rows; lr += kNT) {
                const float x75 = __fmul_rn(xs[c0 + lr], 37778931862957161709568.0f);
#pragma unroll
                for (int g = 0; g < G; g++)
                    row_fma(acc[g], ssum[g], __fmul_rn(__half2float(sb[g * rows + lr]), x75), nb[g * rows + lr]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[slot]);
            if (tr) comp += (uint64_t)(clock64() - tc);
            q++;
        }
        const long long tr0 = tr ? clock64() : 0;
        // butterfly reduce-scatter: lane l ends with the warp's total of column l
#pragma unroll
        for (int g = 0; g < G; g++) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 16; i++) upk2(acc[g][i], v[2 * i], v[2 * i + 1]);
#pragma unroll
            for (int sft = 16; sft >= 1; sft >>= 1) {
                const bool upper = (lane & sft) != 0;
#pragma unroll
                for (int i = 0; i < sft; i++) {
                    const float send = upper ? v[i] : v[i + sft];
                    const float keep = upper ? v[i + sft] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, sft);
                }
            }
            // column l sits at nibble position l % 4: y = 2^(74-4p) acc - 8 * 2^-75 * sum(s')
            const float stot = warp_sum(ssum[g]);
            const float up = __int_as_float((127 + 74 - 4 * (lane & 3)) << 23);
            S.red[rbuf][warp][g][lane] = __fsub_rn(__fmul_rn(v[0], up), __fmul_rn(stot, 2.117582368135751e-22f));
        }
        csync();
        if (warp == 0) {
            float y[G];
#pragma unroll
            for (int g = 0; g < G; g++) {
                float t = 0.0f;
#pragma unroll
                for (int w = 0; w < kNT / 32; w++) t += S.red[rbuf][w][g][lane];
                y[g] = t;
            }
            if constexpr (G == 2) {
                // SwiGLU unit: group 2u is gate, 2u+1 is up (talker.rs:341-345)
                __stcg(d.out + (int64_t)u * 32 + lane, __fmul_rn(silu_ref(y[0]), y[1]));
            } else {
                const int64_t col = (int64_t)u * 32 + lane;
                float o = y[0];
                if (d.out_mode == OUT_RESID) o = __fadd_rn(pre, o);  // x += attn / mlp
                else if (d.bias) o = __fadd_rn(o, pre);
                __stcg(d.out + col, o);
                if (d.ss_out) {
                    const float sq = warp_sum(__fmul_rn(o, o));
                    if (lane == 0) __stcg(d.ss_out + u, sq);
                }
            }
        }
        rbuf ^= 1;
        if (tr) redc += (uint64_t)(clock64() - tr0);
    }
    if (tr) {
        P.trace[(int64_t)op_i * kTraceFields + 4] = waited;
        P.trace[(int64_t)op_i * kTraceFields + 5] = comp;
        P.trace[(int64_t)op_i * kTraceFields + 6] = redc;
        P.trace[(int64_t)op_i * kTraceFields + 7] = slots;
    }
}

template <int HD, int G>
__device__ __forceinline__ void attn_items(const AttnArgs &a, const OpRef &op, ASmem<HD, G> &sm,
                                           int tid, int cta, int grid) {
    const int per_head = op.n_items / a.kv_heads;
    for (int j = first_item(cta, op.rot, grid); j < op.n_items; j += grid) {
        attn::attn_item<HD, G, kNT, 1>(a, j / per_head, j % per_head, 0, tid, sm);
        csync();
    }
}

__device__ void run_attn(const FrameParams &P, const OpRef &op, FrameSmem &S, int tid, int cta,
                         int grid) {
    const AttnArgs &a = S.desc.a;
    const int G = a.heads / a.kv_heads;
    if (a.kv.head_dim == 128) {
        if (G == 1) attn_items<128, 1>(a, op, S.u.a128_1, tid, cta, grid);
        else if (G == 2) attn_items<128, 2>(a, op, S.u.a128_2, tid, cta, grid);
        else attn_items<128, 4>(a, op, S.u.a128_4, tid, cta, grid);
    } else {
        if (G == 1) attn_items<64, 1>(a, op, S.u.a64_1, tid, cta, grid);
        else if (G == 2) attn_items<64, 2>(a, op, S.u.a64_2, tid, cta, grid);
        else attn_items<64, 4>(a, op, S.u.a64_4, tid, cta, grid);
    }
}

__device__ void consumer(const FrameParams &P, FrameSmem &S, int tid, int cta, int grid) {
    const unsigned target = (unsigned)grid;
    uint32_t q = 0;
    int rbuf = 0;
    for (int i = 0; i < P.n_ops; i++) {
        const OpRef op = P.ops[i];
        const int j0 = first_item(cta, op.rot, grid);
        const bool tr = P.trace && j0 == 0 && tid == 0;
        if (j0 < op.n_items) {
            // stage the descriptor (immutable) while thread 0 polls below;
            // the barrier after the poll publishes it
            if (op.type != OP_SAMPLE) {
                const uint4 *src = op.type == OP_GEMV ? reinterpret_cast<const uint4 *>(P.gemv + op.idx)
                                                      : reinterpret_cast<const uint4 *>(P.attn + op.idx);
                const int nw = (op.type == OP_GEMV ? (int)sizeof(GemvDesc) : (int)sizeof(AttnArgs)) / 16;
                if (tid >= 32 && tid - 32 < nw) S.desc.words[tid - 32] = __ldg(src + (tid - 32));
            }
            if (i > 0) {
                // every SM has finished op i-1 (bounded wait, abort-aware)
                if (tid == 0) {
                    const uint64_t t0 = global_ns();
                    for (int it = 0; ld_acquire(P.done + i - 1) < target; it++) {
                        if ((it & 31) == 31) {
                            if (ld_volatile(P.abort_flag)) {
                                S.abort = 1;
                                break;
                            }
                            if (global_ns() - t0 > kWaitNs) {
                                raise_abort(P, S, kDevTimeout);
                                break;
                            }
                        }
                    }
                }
            }
            csync();
            if (*(volatile int *)&S.abort) return;
            stamp(P, i, 0, tr);
            if (op.type == OP_GEMV) {
                const GemvDesc &d = S.desc.g;
                build_input(P, d, S, tid, j0 == 0, j0, op.n_items, grid);
                stamp(P, i, 1, tr);
                if (d.G == 1) gemv_items<1>(P, d, op, S, tid, cta, grid, q, rbuf, tr, i);
                else gemv_items<2>(P, d, op, S, tid, cta, grid, q, rbuf, tr, i);
                csync();
                if (*(volatile int *)&S.abort) return;
                if (d.adv_len && j0 == 0 && tid == 0) {
                    // end of the talker step: the cache and RoPE position advance
                    d.adv_len[0] += 1;
                    d.adv_pos[0] += 1;
                }
            } else if (op.type == OP_ATTN) {
                stamp(P, i, 1, tr);
                run_attn(P, op, S, tid, cta, grid);
            } else {
                stamp(P, i, 1, tr);
                samp::sample_row<kNT, 1>(P.sample, 0, tid, S.u.samp);
            }
            stamp(P, i, 2, tr);
        }
        csync();
        if (tid == 0) {
            __threadfence();
            atomicAdd(P.done + i, 1u);
        }
        stamp(P, i, 3, tr);
    }
}

__global__ void __launch_bounds__(kThreads, 1) k_frame(const __grid_constant__ FrameParams P) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    FrameSmem &S = *reinterpret_cast<FrameSmem *>(smem_raw);
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int i = 0; i < kSlots; i++) {
            mbar_init(&S.full[i], 1);
            mbar_init(&S.empty[i], kNT / 32);
        }
        S.abort = 0;
        mbar_fence_init();
    }
    __syncthreads();
    if (tid >= kNT) {
        if (tid == kNT) producer(P, S, blockIdx.x, gridDim.x);
        return;
    }
    consumer(P, S, tid, blockIdx.x, gridDim.x);
}

}  // namespace
}  // namespace fk

// =====================================================================
// host: program builder
// =====================================================================
using namespace fk;

bool frame_supported(const qora_engine *e) {
    const qora_talker *t = e->t;
    const qora_predictor *p = e->p;
    auto hd_ok = [](int hd) { return hd == 64 || hd == 128; };
    auto g_ok = [](int h, int kv) {
        return kv > 0 && h % kv == 0 && (h / kv == 1 || h / kv == 2 || h / kv == 4);
    };
    return e->B == 1 && p->has_proj && hd_ok(t->hd) && hd_ok(p->hd) && g_ok(t->heads, t->kvh) &&
           g_ok(p->heads, p->kvh) && t->H <= kXMax && t->ffn <= kXMax && t->qd() <= kXMax &&
           p->H <= kXMax && p->ffn <= kXMax && (int64_t)p->heads * p->hd <= kXMax &&
           p->Ht <= kXMax && t->vocab <= samp::kSampleMaxV && p->groups + 1 <= 16 &&
           p->groups <= kMaxEmbedGroups && e->params.top_k <= kMaxSurvivors &&
           !(e->params.top_k <= 0 && e->params.top_p > 0.0f && e->params.top_p < 1.0f);
}

namespace {

struct Builder {
    FrameProgram *fp;
    int grid;
    int64_t items_total = 0;

    void push(int type, int idx, int n_items) {
        OpRef r;
        r.type = type;
        r.idx = idx;
        r.n_items = n_items;
        r.rot = (int)(items_total % grid);
        items_total += n_items;
        fp->ops.push_back(r);
    }
    void gemv(GemvDesc d, const Q4Dev &w, int G) {
        d.nib = w.nib;
        d.scl = w.scl;
        d.kpad = (int)w.kpad;
        d.K = (int)w.k;
        d.G = G;
        d.units = (int)(w.C / G);
        fp->gemv.push_back(d);
        push(OP_GEMV, (int)fp->gemv.size() - 1, d.units);
    }
    void attn(const AttnArgs &a, int per_head) {
        fp->attn.push_back(a);
        push(OP_ATTN, (int)fp->attn.size() - 1, a.kv_heads * per_head);
    }
};

}  // namespace

int frame_build(qora_engine *e, FrameProgram **out) {
    qora_talker *t = e->t;
    qora_predictor *p = e->p;
    qora_ctx *ctx = t->ctx;
    auto *fp = new FrameProgram();
    fp->grid = ctx->num_sms;
    fp->smem = sizeof(FrameSmem);
    int rc = QORA_OK;

    // ---- activation buffers (one allocation, 256-byte aligned pieces)
    const int Hm = std::max(t->H, p->H);
    const int qkvm = (int)std::max(t->qkvn(), (int64_t)(p->heads + 2 * p->kvh) * p->hd);
    const int qdm = (int)std::max(t->qd(), (int64_t)p->heads * p->hd);
    const int ffm = std::max(t->ffn, p->ffn);
    const int kvh_m = std::max(t->kvh, p->kvh);
    size_t off = 0;
    auto take = [&](size_t floats) {
        const size_t o = off;
        off += (floats * 4 + 255) / 256 * 256;
        return o;
    };
    const size_t o_qkv = take(qkvm), o_attn = take(qdm), o_xa = take(Hm), o_xb = take(Hm),
                 o_ssa = take(Hm / 32), o_ssb = take(Hm / 32), o_h = take(ffm),
                 o_head = take(p->vocab),
                 o_apo = take(std::max(attn_part_o_floats(1, t->kvh, t->heads, t->hd),
                                       attn_part_o_floats(1, p->kvh, p->heads, p->hd))),
                 o_apml = take(std::max(attn_part_ml_floats(1, t->kvh, t->heads),
                                        attn_part_ml_floats(1, p->kvh, p->heads))),
                 o_atk = take(kvh_m);
    rc = fp->bufs.alloc(off);
    if (rc == QORA_OK) rc = fp->bufs.zero();
    if (rc != QORA_OK) {
        delete fp;
        return rc;
    }
    char *base = fp->bufs.as<char>();
    float *qkv = (float *)(base + o_qkv), *attn_out = (float *)(base + o_attn);
    float *xa = (float *)(base + o_xa), *xb = (float *)(base + o_xb);
    float *ssa = (float *)(base + o_ssa), *ssb = (float *)(base + o_ssb);
    float *hbuf = (float *)(base + o_h), *head = (float *)(base + o_head);
    float *apo = (float *)(base + o_apo), *apml = (float *)(base + o_apml);
    unsigned *atk = (unsigned *)(base + o_atk);

    Builder B{fp, fp->grid};
    uint32_t *codes = e->codes.as<uint32_t>();
    uint32_t *prev = e->prev.as<uint32_t>();
    float *hidden = p->x2.as<float>();  // row 0: the talker's final-normed hidden

    // ---- op 0: code 0 = sample_token(logits)
    SampleArgs sa;
    sa.logits = e->logits.as<float>();
    sa.ldlogits = t->vocab;
    sa.V = t->vocab;
    sa.prev = prev;
    sa.ldprev = 16;
    sa.n_prev = 16;
    sa.rng = e->rng.as<uint64_t>();
    sa.params = e->params;
    sa.out = codes;
    sa.ldout = 16;
    sa.prev_update = prev;
    sa.ldprev_update = 16;
    sa.err = ctx->err.as<int>();
    B.push(OP_SAMPLE, 0, 1);

    // One decoder layer (talker.rs:275-349).  The residual stream enters in xa
    // (sums of squares in ssa) unless `first` supplies the QKV input itself;
    // attention adds into xb (ssb), the MLP back into xa (ssa).
    auto layer = [&](const LayerDev &ld, int H, int heads, int kvh, int hd, const GemvDesc *first,
                     AttnArgs at, int per_head) {
        const int qkvn = (heads + 2 * kvh) * hd;
        GemvDesc q = first ? *first : GemvDesc();
        if (!first) {
            q.in = xa;
            q.ss_in = ssa;
        }
        q.gamma = ld.in_norm.as<__half>();
        q.out = qkv;
        B.gemv(q, ld.qkv, 1);
        at.qkv = qkv;
        at.ldqkv = qkvn;
        at.heads = heads;
        at.kv_heads = kvh;
        at.T = 1;
        at.streams = 1;
        at.q_gamma = ld.q_norm.as<__half>();
        at.k_gamma = ld.k_norm.as<__half>();
        at.out = attn_out;
        at.ldout = (int64_t)heads * hd;
        at.part_o = apo;
        at.part_ml = apml;
        at.tickets = atk;
        at.err = ctx->err.as<int>();
        B.attn(at, per_head);
        GemvDesc o;
        o.in = attn_out;
        o.out_mode = OUT_RESID;
        o.resid = xa;
        o.out = xb;
        o.ss_out = ssb;
        B.gemv(o, ld.o, 1);
        GemvDesc gu;
        gu.in = xb;
        gu.ss_in = ssb;
        gu.gamma = ld.post_norm.as<__half>();
        gu.out_mode = OUT_SWIGLU;
        gu.out = hbuf;
        B.gemv(gu, ld.gu, 2);
        GemvDesc dn;
        dn.in = hbuf;
        dn.out_mode = OUT_RESID;
        dn.resid = xb;
        dn.out = xa;
        dn.ss_out = ssa;
        B.gemv(dn, ld.dn, 1);
        (void)H;
    };

    // ---- predictor: 16 single-token passes (hidden, semantic, codes 1..14);
    // the reference's 2-token prefill (code_predictor.rs:345-438) is causal, so
    // its two tokens are the first two passes
    AttnArgs pat;
    pat.rope_cos = p->rope_cos.as<float>();
    pat.rope_sin = p->rope_sin.as<float>();
    pat.rope_max_pos = p->rope_max;
    for (int tk = 0; tk <= p->groups; tk++) {
        GemvDesc pr;  // project_input (code_predictor.rs:51-61) into the residual stream
        if (tk == 0) {
            pr.in_mode = IN_VEC;
            pr.in = hidden;
        } else if (tk == 1) {
            pr.in_mode = IN_EMB;
            pr.code_src = codes;
            pr.emb = t->codec_emb;
        } else {
            pr.in_mode = IN_EMB;
            pr.amax_src = head;
            pr.amax_n = p->vocab;
            pr.code_dst = codes + (tk - 1);
            pr.emb = p->embs[tk - 2];
        }
        pr.out = xa;
        pr.ss_out = ssa;
        pr.bias = p->proj_bias.as<float>();
        B.gemv(pr, p->proj, 1);
        for (int l = 0; l < p->L; l++) {
            AttnArgs at = pat;
            at.kv = e->pkv->layer(l);
            at.pos_static = tk;
            at.len_static = tk;
            layer(p->layers[l], p->H, p->heads, p->kvh, p->hd, nullptr, at, 1);
        }
        if (tk >= 1) {
            GemvDesc hd;
            hd.in = xa;
            hd.ss_in = ssa;
            hd.gamma = p->final_norm.as<__half>();
            hd.out = head;
            B.gemv(hd, p->heads_w[tk - 1], 1);
        }
    }

    // ---- talker step
    AttnArgs tat;
    tat.rope_cos = t->rope_cos.as<float>();
    tat.rope_sin = t->rope_sin.as<float>();
    tat.rope_max_pos = t->rope_max;
    tat.pos = e->pos.as<int>();
    tat.len = e->tkv->lens();
    for (int l = 0; l < t->L; l++) {
        AttnArgs at = tat;
        at.kv = e->tkv->layer(l);
        if (l == 0) {
            GemvDesc fr;
            fr.in_mode = IN_FRAME;
            fr.amax_src = head;
            fr.amax_n = p->vocab;
            fr.save = xa;  // the frame input is the residual stream for layer 0's attention add
            layer(t->layers[l], t->H, t->heads, t->kvh, t->hd, &fr, at, kAttnMaxSplit);
        } else {
            layer(t->layers[l], t->H, t->heads, t->kvh, t->hd, nullptr, at, kAttnMaxSplit);
        }
    }
    {
        GemvDesc hd;  // final norm + apply_codec_head (talker.rs:353-359, 647-649)
        hd.in = xa;
        hd.ss_in = ssa;
        hd.gamma = t->final_norm.as<__half>();
        hd.save = hidden;
        hd.save_normed = 1;
        hd.out = e->logits.as<float>();
        hd.adv_len = e->tkv->lens();
        hd.adv_pos = e->pos.as<int>();
        B.gemv(hd, t->head, 1);
    }

    FrameEmbed fe;
    fe.talker = t->codec_emb;
    for (int g = 0; g < p->groups; g++) fe.pred[g] = p->embs[g];
    fe.ngroups = p->groups;
    fe.n = t->H;
    fe.codes = codes;
    fe.prev = prev;

    // ---- device copies
    const size_t nops = fp->ops.size();
    rc = fp->d_ops.alloc(nops * sizeof(OpRef));
    if (rc == QORA_OK) rc = fp->d_gemv.alloc(fp->gemv.size() * sizeof(GemvDesc));
    if (rc == QORA_OK) rc = fp->d_attn.alloc(fp->attn.size() * sizeof(AttnArgs));
    if (rc == QORA_OK) rc = fp->d_done.alloc((nops + 1) * sizeof(unsigned));
    if (rc == QORA_OK) rc = fp->d_trace.alloc(nops * kTraceFields * sizeof(unsigned long long));
    if (rc == QORA_OK && (cudaMemcpy(fp->d_ops.p, fp->ops.data(), nops * sizeof(OpRef), cudaMemcpyHostToDevice) ||
                          cudaMemcpy(fp->d_gemv.p, fp->gemv.data(), fp->gemv.size() * sizeof(GemvDesc),
                                     cudaMemcpyHostToDevice) ||
                          cudaMemcpy(fp->d_attn.p, fp->attn.data(), fp->attn.size() * sizeof(AttnArgs),
                                     cudaMemcpyHostToDevice)))
        rc = set_error(QORA_ERR_CUDA, "frame program upload failed");
    if (rc == QORA_OK &&
        cudaFuncSetAttribute(k_frame, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fp->smem) != cudaSuccess)
        rc = set_error(QORA_ERR_CUDA, "frame kernel needs %zu bytes of shared memory", fp->smem);
    if (rc == QORA_OK) {
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_frame, kThreads, fp->smem) != cudaSuccess ||
            per_sm < 1)
            rc = set_error(QORA_ERR_UNSUPPORTED, "frame kernel does not fit one SM");
    }
    if (rc != QORA_OK) {
        delete fp;
        return rc;
    }
    FrameParams &P = fp->params;
    P.ops = fp->d_ops.as<OpRef>();
    P.n_ops = (int)nops;
    P.gemv = fp->d_gemv.as<GemvDesc>();
    P.attn = fp->d_attn.as<AttnArgs>();
    P.sample = sa;
    P.fe = fe;
    P.done = fp->d_done.as<unsigned>();
    P.abort_flag = reinterpret_cast<int *>(fp->d_done.as<unsigned>() + nops);
    P.err = ctx->err.as<int>();
    *out = fp;
    return QORA_OK;
}

int frame_launch(FrameProgram *fp, const float *text, cudaStream_t st) {
    FrameParams P = fp->params;
    P.text = text;
    P.trace = fp->trace ? fp->d_trace.as<unsigned long long>() : nullptr;
    // counters and the abort flag start each frame at zero
    QORA_CUDA(cudaMemsetAsync(fp->d_done.p, 0, fp->d_done.bytes, st));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(fp->grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = fp->smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident (they wait on each other)
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    QORA_CUDA(cudaLaunchKernelEx(&cfg, k_frame, P));
    return QORA_OK;
}

void frame_program_destroy(FrameProgram *p) { delete p; }

}  // namespace qora
