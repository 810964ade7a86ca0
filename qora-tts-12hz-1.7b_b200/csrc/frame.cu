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
// list and the steps are chained through the data itself: every activation
// an op publishes is a tagged 64-bit word (value | tag << 32, tag unique to
// the op and the launch), and a consumer polls exactly the words it needs
// until they carry its producer's tag.  A step then costs one store-to-load
// trip through L2 - no counters, no separate flag, no per-op fence of its
// own.  The only plain data read back within a launch is the K/V cache: an
// attention op fences (release) between its K/V append and its tagged
// output, and fences (acquire) after polling its q/k/v, before it reads the
// cache through L2.  Every op consumes its producer's whole
// output (or, for attention, its head's q/k/v, whose consumer needs all of
// attention's output), so by the time any SM overwrites a buffer every
// reader of its previous contents has finished.  The one op whose data does
// not reach back to its predecessor (the semantic pass's projection needs
// only the sampled code) waits on the previous pass's output explicitly.
//
// Weight streaming is decoupled from that chain.  Each SM's share of every
// GEMV is known in advance (item j of op i runs on SM (rot_i + j % avail_i)
// % grid), so a producer warp walks the op list ahead of the compute warps and pulls
// the SM's weight slices into a ring of shared-memory slots with
// cp.async.bulk (no multicast), signalling an mbarrier per slot; the compute
// warps consume slots in the same order and release them.  Weights are
// immutable, so the stream never waits on activations.
//
// Every GEMV item is one column unit (32 output columns, or a gate/up pair)
// over all K rows, so it ends with final values and applies its epilogue
// itself: residual add (plus the per-32-column sum of squares the next
// RMSNorm needs), bias, or silu(gate) * up.  An SM that has items in an op
// polls that op's whole input vector (<= 6144 values) into shared memory and
// applies the RMSNorm prologue from those sums of squares, summed in the
// same fixed order on every SM.  The attention and sampler ops run the same
// device code as the standalone kernels (attention_impl.cuh,
// sampler_impl.cuh).  Each op's descriptor is staged into shared memory with
// cp.async while the previous op runs.
//
// Every wait is bounded (~2 s of globaltimer); a timeout raises kDevTimeout,
// sets a global abort flag that every other waiter polls, and the kernel
// drains its own in-flight bulk copies before returning.
#include <algorithm>
#include <cstddef>
#include <cstring>

#include "attention_impl.cuh"
#include "frame.cuh"
#include "sampler_impl.cuh"

namespace qora {
namespace fk {

namespace {

constexpr uint64_t kWaitNs = 2000000000ull;  // bounded waits: 2 s

constexpr int kMaxOps = 640;                 // op table held in shared memory
constexpr int kChunkRows = kSlotNib / 16;    // weight rows of one group per slot
constexpr int kDescWords = 24;               // 384-byte descriptor slots

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
    float red[2][kNT / 32][32];        // per-group cross-warp reduction (double buffered)
    float bred[kNT / 32];              // block reductions
    int bidx[kNT / 32];
    uint64_t full[kSlots], empty[kSlots];
    int abort;
    uint32_t codes_s[kMaxEmbedGroups];  // the frame's codes (talker frame input)
    // two descriptor slots: the current op's and the next op's (staged with
    // cp.async while the current op runs)
    union alignas(16) Desc {
        GemvDesc g;
        AttnArgs a;
        uint4 words[kDescWords];
    } desc[2];
    OpRef ops[kMaxOps];
};
static_assert(sizeof(GemvDesc) <= 16 * kDescWords && sizeof(AttnArgs) <= 16 * kDescWords,
              "descriptor staging slots");
static_assert(sizeof(OpRef) == 16, "op table staging");

__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kNT) : "memory"); }
// csync that also ORs a flag over the compute threads: every thread gets the
// same answer (an abort the producer warp raises mid-op may reach the threads
// at different times; this makes them leave together).
__device__ __forceinline__ bool csync_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kNT)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ int ld_volatile(const int *p) {
    int v;
    asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
}

// This SM's first item of `op` (op.n_items if it has none); its further
// items follow every op.avail.  (rot is kept in [0, grid) by the builder, so
// no division is needed: this sits on the path between two ops, where an
// integer division is measurable.)
__device__ __forceinline__ int first_item(int cta, const OpRef &op, int grid) {
    int j = cta - op.rot;
    if (j < 0) j += grid;
    return j < op.avail ? j : op.n_items;
}

// Across SMs: field 0 keeps the earliest time (stored complemented, so a
// max does it), fields 1-3 the latest.
__device__ __forceinline__ void stamp_all(const FrameParams &P, int op, int field, bool on) {
    if (!on) return;
    const unsigned long long t = global_ns();
    atomicMax(P.trace + (int64_t)op * kTraceFields + field, field == 0 ? ~t : t);
}

// Sets the abort state everywhere after a failed or timed-out wait.
__device__ __forceinline__ void raise_abort(const FrameParams &P, FrameSmem &S, int code) {
    raise_error(P.err, code);
    atomicExch(P.abort_flag, 1);
    S.abort = 1;
}

// Bounded mbarrier wait that also gives up when the CTA or the grid aborted.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t *bar, uint32_t parity, FrameSmem &S,
                                                   const FrameParams &P) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (int it = 0;; it++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63) == 63) {
            if (*(volatile int *)&S.abort || ld_volatile(P.abort_flag)) {
                S.abort = 1;
                return false;
            }
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
        const OpRef op = S.ops[i];
        if (op.type != OP_GEMV) continue;
        const int u0 = first_item(cta, op, grid);
        if (u0 >= op.n_items) continue;
        const GemvDesc &d = P.gemv[op.idx];
        const int G = d.G, kpad = d.kpad;
        const uint4 *nib = d.nib;
        const __half *scl = d.scl;
        for (int u = u0; u < op.n_items && ok; u += op.avail) {
            for (int g = 0; g < G && ok; g++) {  // a unit's groups one after the other
                const int64_t grp = (int64_t)u * G + g;
                for (int c0 = 0; c0 < kpad; c0 += kChunkRows) {
                    const int rows = min(kChunkRows, kpad - c0);
                    const int slot = q % kSlots;
                    if (q >= kSlots && !mbar_wait_or_abort(&S.empty[slot], ((q / kSlots) - 1) & 1, S, P)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&S.full[slot], (uint32_t)(rows * 18));
                    bulk_g2s(S.nib[slot], nib + grp * kpad + c0, (uint32_t)rows * 16, &S.full[slot]);
                    bulk_g2s(S.scl[slot], scl + grp * kpad + c0, (uint32_t)rows * 2, &S.full[slot]);
                    q++;
                }
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

// Polls dst[i] = value of src[i] for i = i0 + tid + m * kNT (m < U, i < n)
// until every word carries `tag` (bounded; on failure the CTA aborts after
// its barrier sequence).  GEMV inputs are all tagged, so no fence follows.
// Every attempt reloads all of the thread's pending words (one L2 round trip
// per attempt), so the values are in hand in the attempt that sees them.
template <int U>
__device__ __forceinline__ void poll_to_smem(const FrameParams &P, FrameSmem &S, const uint64_t *src,
                                             int i0, int n, uint32_t tag, float *dst, int tid) {
    uint32_t pending = 0;
#pragma unroll
    for (int m = 0; m < U; m++)
        if (i0 + tid + m * kNT < n) pending |= 1u << m;
    uint64_t t0 = global_ns();
    for (int it = 0; pending; it++) {
        uint64_t v[U];
#pragma unroll
        for (int m = 0; m < U; m++)
            if (pending & (1u << m)) v[m] = ld_relaxed_u64(src + i0 + tid + m * kNT);
#pragma unroll
        for (int m = 0; m < U; m++) {
            if ((pending & (1u << m)) && (uint32_t)(v[m] >> 32) == tag) {
                dst[i0 + tid + m * kNT] = __uint_as_float((uint32_t)v[m]);
                pending &= ~(1u << m);
            }
        }
        if (!pending) break;
        if ((it & 15) == 15) {
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

// A tagged word loaded early (w) or, if it did not carry `tag` yet, polled
// until it does.
__device__ __forceinline__ float settle_word(const FrameParams &P, FrameSmem &S, const uint64_t *p,
                                             uint64_t w, uint32_t tag) {
    if ((uint32_t)(w >> 32) == tag) return __uint_as_float((uint32_t)w);
    float v[1] = {0.0f};
    const bool pr[1] = {true};
    if (!poll_tagged<1>(p, 0, tag, v, pr, P.err, P.abort_flag)) S.abort = 1;
    return v[0];
}

// Polls the tagged vector src[0..n) (n <= kXMax) into dst.
__device__ __forceinline__ void poll_vector(const FrameParams &P, FrameSmem &S, const uint64_t *src,
                                            int n, uint32_t tag, float *dst, int tid) {
    constexpr int UH = kXMax / kNT / 2;  // two rounds of loads at most
    poll_to_smem<UH>(P, S, src, 0, n, tag, dst, tid);
    if (n > UH * kNT) poll_to_smem<UH>(P, S, src, UH * kNT, n, tag, dst, tid);
}

// Argmax over the tagged logits src[0..n) (n <= kXMax, staged through xs);
// ties keep the larger index (the last maximum, code_predictor.rs:336-339).
// Identical on every SM.
__device__ int block_argmax(const FrameParams &P, const uint64_t *src, int n, uint32_t tag,
                            FrameSmem &S, int tid) {
    float *xs = S.u.xs;
    poll_vector(P, S, src, n, tag, xs, tid);
    float bv = -INFINITY;
    int bi = -1;
    for (int i = tid; i < n; i += kNT) {
        const float v = xs[i];
        if (v != v) raise_error(P.err, kDevNaN);
        if (bi < 0 || v > bv || (v == bv && i > bi)) {
            bv = v;
            bi = i;
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

// This SM's slice of [0, K) (the SMs with items in the op partition it).
__device__ __forceinline__ void my_slice(int K, int j0, int n_items, int avail, int &lo, int &hi) {
    const int parts = min(n_items, avail);
    lo = (int)((int64_t)j0 * K / parts);
    hi = (int)((int64_t)(j0 + 1) * K / parts);
}

constexpr int kGammaPre = 8;  // gamma values per thread fetched before the input wait

// Applies rms_norm_f16 (gemv.rs:445-454) to xs[0..K) in place:
// x * (1 / sqrt(ss / K + 1e-6)) * gamma.  The first kGammaPre values per
// thread come from gm[] (prefetched by the caller).
__device__ __forceinline__ void norm_strided(float *xs, const __half *gamma, int K, float ss,
                                             const float (&gm)[kGammaPre], int tid) {
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), 1e-6f)));
#pragma unroll
    for (int m = 0; m < kGammaPre; m++) {
        const int k = tid + m * kNT;
        if (k < K) xs[k] = __fmul_rn(__fmul_rn(xs[k], inv), gm[m]);
    }
    for (int k = tid + kGammaPre * kNT; k < K; k += kNT)
        xs[k] = __fmul_rn(__fmul_rn(xs[k], inv), __half2float(__ldg(gamma + k)));
}

// Whether an op's input may be built without block-wide waits: a tagged
// vector that nothing else reads back (no saved copy, no ordering input).
// Every thread then uses only the input values it polled itself (the rows
// tid + 256 m it processes in every chunk), so it starts on them as soon as
// they arrive; the RMSNorm's 1 / rms is applied to the column totals instead
// (y = inv * sum_k W x gamma), from the sum of squares the item's reduction
// gathers anyway.
__device__ __forceinline__ bool streamed_input(const GemvDesc &d) {
    return d.in_mode == IN_VEC && d.in && !d.in_plain && !d.save && !d.save_plain && !d.dep;
}

// Streamed inputs (streamed_input): x * gamma per thread, no barrier; returns
// this thread's share of the sum of squares (0 without gamma).  Inlined into
// the op loop: it is the input path of almost every op, and an out-of-line
// call saves and restores the caller's live registers through local memory,
// which the L1 left beside the weight ring cannot hold.
__device__ __forceinline__ float build_streamed(const FrameParams &P, const GemvDesc &d, FrameSmem &S,
                                                int tid) {
    float *xs = S.u.xs;
    const int K = d.K;
    const bool has_ss = d.gamma && tid < (K >> 5);
    const uint64_t ssw = has_ss ? ld_relaxed_u64(d.ss_in + tid) : 0ull;
    // gamma is immutable: its loads go out before the wait
    float gm[kGammaPre];
#pragma unroll
    for (int m = 0; m < kGammaPre; m++) {
        const int k = tid + m * kNT;
        gm[m] = (d.gamma && k < K) ? __half2float(__ldg(d.gamma + k)) : 0.0f;
    }
    for (int k = K + tid; k < d.kpad; k += kNT) xs[k] = 0.0f;
    poll_vector(P, S, d.in, K, P.tag_base + d.in_tag, xs, tid);
    if (d.gamma) {
#pragma unroll
        for (int m = 0; m < kGammaPre; m++) {
            const int k = tid + m * kNT;
            if (k < K) xs[k] = __fmul_rn(xs[k], gm[m]);
        }
        for (int k = tid + kGammaPre * kNT; k < K; k += kNT)
            xs[k] = __fmul_rn(xs[k], __half2float(__ldg(d.gamma + k)));
    }
    return has_ss ? settle_word(P, S, d.ss_in + tid, ssw, P.tag_base + d.ss_tag) : 0.0f;
}

// Builds the GEMV input x[0..kpad) in shared memory (rows >= K are zero) for
// the ops whose input is not streamed: plain vectors, embeddings, the frame
// input, saved or ordered inputs.
__device__ __noinline__ void build_input(const FrameParams &P, const GemvDesc &d, FrameSmem &S, int tid,
                            bool leader, int j0, int n_items, int avail) {
    float *xs = S.u.xs;
    const int K = d.K;
    // gamma is immutable: its first loads go out before any wait
    float gm[kGammaPre];
#pragma unroll
    for (int m = 0; m < kGammaPre; m++) {
        const int k = tid + m * kNT;
        gm[m] = (d.gamma && k < K) ? __half2float(__ldg(d.gamma + k)) : 0.0f;
    }
    if (d.dep) {
        // ordering only: the values land in xs and are overwritten below
        poll_vector(P, S, d.dep, d.dep_n, P.tag_base + d.dep_tag, xs, tid);
        csync();
    }
    for (int k = K + tid; k < d.kpad; k += kNT) xs[k] = 0.0f;
    float ss = 0.0f;
    switch (d.in_mode) {
        case IN_VEC: {
            float ssp = 0.0f;
            // the sum-of-squares word goes out with the input loads
            const bool has_ss = d.gamma && tid < (K >> 5);
            const uint64_t ssw = has_ss ? ld_relaxed_u64(d.ss_in + tid) : 0ull;
            if (d.in_plain) {
                for (int k = tid; k < K; k += kNT) xs[k] = __ldcg(d.in_plain + k);
            } else {
                poll_vector(P, S, d.in, K, P.tag_base + d.in_tag, xs, tid);
            }
            if (has_ss) ssp = settle_word(P, S, d.ss_in + tid, ssw, P.tag_base + d.ss_tag);
            csync();
            if (d.gamma) ss = block_sum(ssp, S, tid);
            break;
        }
        case IN_EMB: {
            uint32_t code;
            if (d.amax_src) {
                code = (uint32_t)block_argmax(P, d.amax_src, d.amax_n, P.tag_base + d.amax_tag, S, tid);
                if (leader && tid == 0 && d.code_dst) {
                    st_relaxed_u64(d.code_dst, tag_pack(__uint_as_float(code), P.tag_base + d.out_tag));
                }
            } else {
                float c[1] = {0.0f};
                const bool pr[1] = {true};
                if (!poll_tagged<1>(d.code_src, 0, P.tag_base + d.code_tag, c, pr, P.err, P.abort_flag))
                    S.abort = 1;
                code = __float_as_uint(c[0]);
            }
            // an aborted wait leaves no code: row 0 keeps the reads in the table
            if (code >= (uint32_t)d.emb.rows) {
                raise_error(P.err, kDevRange);
                code = 0;
            }
            for (int w = tid; w < (K >> 3); w += kNT) {
                const EmbWord e = emb_word(d.emb, code, w);
                float o[8];
#pragma unroll
                for (int c = 0; c < 8; c++) o[c] = emb_at(e, c);
                reinterpret_cast<float4 *>(xs)[2 * w] = make_float4(o[0], o[1], o[2], o[3]);
                reinterpret_cast<float4 *>(xs)[2 * w + 1] = make_float4(o[4], o[5], o[6], o[7]);
            }
            break;
        }
        case IN_FRAME: {
            const FrameEmbed &fe = P.fe;
            const uint32_t last =
                (uint32_t)block_argmax(P, d.amax_src, d.amax_n, P.tag_base + d.amax_tag, S, tid);
            // codes 0 .. ngroups-1, each tagged by the op that produced it:
            // thread g polls code g
            if (tid < fe.ngroups) {
                const uint32_t tg = P.tag_base + fe.code_tag[tid];
                const uint64_t t0 = global_ns();
                for (int it = 0;; it++) {
                    const uint64_t w = ld_relaxed_u64(fe.codes_t + tid);
                    if ((uint32_t)(w >> 32) == tg) {
                        S.codes_s[tid] = (uint32_t)w;
                        break;
                    }
                    if ((it & 15) == 15 && (ld_volatile(P.abort_flag) || global_ns() - t0 > kWaitNs)) {
                        raise_abort(P, S, kDevTimeout);
                        S.codes_s[tid] = 0;
                        break;
                    }
                }
            }
            csync();
            uint32_t cg[kMaxEmbedGroups];
#pragma unroll
            for (int g = 0; g < kMaxEmbedGroups; g++) cg[g] = g < fe.ngroups ? S.codes_s[g] : 0u;
            if (leader && tid == 0) {
                // the frame's codes for the host and the repetition-penalty window
                for (int g = 0; g < fe.ngroups; g++) fe.codes[g] = cg[g];
                fe.codes[fe.ngroups] = last;
                for (int g = 1; g < fe.ngroups; g++) fe.prev[g] = cg[g];
                fe.prev[fe.ngroups] = last;
            }
            for (int w = tid; w < (K >> 3); w += kNT) {
                const EmbWord et = emb_word(fe.talker, cg[0], w);
                const float4 t0v = __ldcg(reinterpret_cast<const float4 *>(P.text) + 2 * w);
                const float4 t1v = __ldcg(reinterpret_cast<const float4 *>(P.text) + 2 * w + 1);
                float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                // (E_talker[c0] + (sum_g E_g[c_{g+1}])) + text, as the engine's
                // frame embed; tables in two halves, each half's loads in flight together
#pragma unroll
                for (int h = 0; h < kMaxEmbedGroups; h += kMaxEmbedGroups / 2) {
                    EmbWord e[kMaxEmbedGroups / 2];
#pragma unroll
                    for (int g = 0; g < kMaxEmbedGroups / 2; g++)
                        if (h + g < fe.ngroups)
                            e[g] = emb_word(fe.pred[h + g], h + g + 1 < fe.ngroups ? cg[h + g + 1] : last, w);
#pragma unroll
                    for (int g = 0; g < kMaxEmbedGroups / 2; g++)
                        if (h + g < fe.ngroups)
#pragma unroll
                            for (int c = 0; c < 8; c++) acc[c] = __fadd_rn(acc[c], emb_at(e[g], c));
                }
                const float tx[8] = {t0v.x, t0v.y, t0v.z, t0v.w, t1v.x, t1v.y, t1v.z, t1v.w};
                float o[8];
#pragma unroll
                for (int c = 0; c < 8; c++) o[c] = __fadd_rn(__fadd_rn(emb_at(et, c), acc[c]), tx[c]);
                reinterpret_cast<float4 *>(xs)[2 * w] = make_float4(o[0], o[1], o[2], o[3]);
                reinterpret_cast<float4 *>(xs)[2 * w + 1] = make_float4(o[4], o[5], o[6], o[7]);
            }
            break;
        }
    }
    csync();
    if (d.in_mode != IN_VEC && d.gamma) {
        float t = 0.0f;
        for (int k = tid; k < K; k += kNT) t += __fmul_rn(xs[k], xs[k]);
        ss = block_sum(t, S, tid);
    }
    if (d.save) {
        // this SM's slice of the un-normalised input, published as tagged words
        int lo, hi;
        my_slice(K, j0, n_items, avail, lo, hi);
        for (int k = lo + tid; k < hi; k += kNT) st_relaxed_u64(d.save + k, tag_pack(xs[k], P.tag_base + d.out_tag));
    }
    if (d.gamma) {
        csync();  // the save above read xs before it is normalised
        norm_strided(xs, d.gamma, K, ss, gm, tid);
        csync();
    }
    if (d.save_plain) {
        int lo, hi;
        my_slice(K, j0, n_items, avail, lo, hi);
        for (int k = lo + tid; k < hi; k += kNT) __stcg(d.save_plain + k, xs[k]);
    }
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

// The items of one GEMV op on this SM: each unit's G groups (1, or the
// gate / up pair) in turn, all K rows each.
__device__ void gemv_items(const FrameParams &P, const GemvDesc &d, const OpRef &op, FrameSmem &S,
                           int tid, int cta, int grid, uint32_t &q, int &rbuf, bool tr, int op_i,
                           float ssp) {
    uint64_t waited = 0, slots = 0, comp = 0, redc = 0;
    const int lane = tid & 31, warp = tid >> 5;
    const float *xs = S.u.xs;
    const uint32_t otag = P.tag_base + d.out_tag;
    // streamed RMSNorm input: 1 / rms multiplies the column totals; the sum of
    // squares rides on the first reduction's barrier (fixed warp order)
    const bool defer_norm = streamed_input(d) && d.gamma;
    float inv = 1.0f;
    bool have_inv = !defer_norm;
    const float ssw = defer_norm ? warp_sum(ssp) : 0.0f;
    for (int u = first_item(cta, op, grid); u < op.n_items; u += op.avail) {
        // the epilogue's residual / bias value, fetched while the item computes
        float pre = 0.0f;
        uint64_t prew = 0;
        if (warp == 0) {
            const int64_t col = (int64_t)u * 32 + lane;
            if (d.out_mode == OUT_RESID) prew = ld_relaxed_u64(d.resid + col);  // checked at the epilogue
            else if (d.bias) pre = __ldg(d.bias + col);
        }
        float y[2] = {0.0f, 0.0f};  // warp 0: the unit's group totals, lane = column
        for (int g = 0; g < d.G; g++) {
            uint64_t acc[16];
            float ssum = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; i++) acc[i] = 0ull;
            for (int c0 = 0; c0 < d.kpad; c0 += kChunkRows) {
                const int rows = min(kChunkRows, d.kpad - c0);
                const int slot = q % kSlots;
                const long long tw = tr ? clock64() : 0;
                // on a failed wait the thread skips the slot but keeps to the
                // block's barrier sequence; the op ends with a uniform abort check
                const bool ok = mbar_wait_or_abort(&S.full[slot], (q / kSlots) & 1, S, P);
                long long tc = 0;
                if (tr) {
                    tc = clock64();
                    waited += (uint64_t)(tc - tw);
                    slots++;
                }
                const uint4 *nb = reinterpret_cast<const uint4 *>(S.nib[slot]);
                const __half *sb = reinterpret_cast<const __half *>(S.scl[slot]);
                int lr = tid;
                if (ok) {
                    // four rows' operands loaded before their FMAs (the
                    // thread's rows in the same order: the same bits)
                    for (; lr + 3 * kNT < rows; lr += 4 * kNT) {
                        float xv[4], sv[4];
                        uint4 wv[4];
#pragma unroll
                        for (int u = 0; u < 4; u++) {
                            xv[u] = xs[c0 + lr + u * kNT];
                            sv[u] = __half2float(sb[lr + u * kNT]);
                            wv[u] = nb[lr + u * kNT];
                        }
#pragma unroll
                        for (int u = 0; u < 4; u++)
                            row_fma(acc, ssum, __fmul_rn(sv[u], __fmul_rn(xv[u], 37778931862957161709568.0f)), wv[u]);
                    }
                    for (; lr < rows; lr += kNT) {
                        const float x75 = __fmul_rn(xs[c0 + lr], 37778931862957161709568.0f);
                        row_fma(acc, ssum, __fmul_rn(__half2float(sb[lr]), x75), nb[lr]);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.empty[slot]);
                if (tr) comp += (uint64_t)(clock64() - tc);
                q++;
            }
            const long long tr0 = tr ? clock64() : 0;
            // butterfly reduce-scatter: lane l ends with the warp's total of column l
            float v[32];
#pragma unroll
            for (int i = 0; i < 16; i++) upk2(acc[i], v[2 * i], v[2 * i + 1]);
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
            const float stot = warp_sum(ssum);
            const float up = __int_as_float((127 + 74 - 4 * (lane & 3)) << 23);
            S.red[rbuf][warp][lane] = __fsub_rn(__fmul_rn(v[0], up), __fmul_rn(stot, 2.117582368135751e-22f));
            if (!have_inv && lane == 0) S.bred[warp] = ssw;
            csync();
            if (!have_inv) {
                // rms_norm_f16 (gemv.rs:445-454): 1 / sqrt(ss / K + 1e-6)
                float ss = 0.0f;
#pragma unroll
                for (int w = 0; w < kNT / 32; w++) ss += S.bred[w];
                inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)d.K), 1e-6f)));
                have_inv = true;
            }
            if (warp == 0) {
                float t = 0.0f;
#pragma unroll
                for (int w = 0; w < kNT / 32; w++) t += S.red[rbuf][w][lane];
                if (defer_norm) t = __fmul_rn(t, inv);
                if (g == 0) y[0] = t;
                else y[1] = t;
            }
            rbuf ^= 1;
            if (tr) redc += (uint64_t)(clock64() - tr0);
        }
        if (warp == 0) {
            if (d.out_mode == OUT_SWIGLU) {
                // SwiGLU unit: group 2u is gate, 2u+1 is up (talker.rs:341-345)
                st_relaxed_u64(d.out + (int64_t)u * 32 + lane, tag_pack(__fmul_rn(silu_ref(y[0]), y[1]), otag));
            } else {
                const int64_t col = (int64_t)u * 32 + lane;
                float o = y[0];
                if (d.out_mode == OUT_RESID)  // x += attn / mlp
                    o = __fadd_rn(settle_word(P, S, d.resid + col, prew, P.tag_base + d.resid_tag), o);
                else if (d.bias)
                    o = __fadd_rn(o, pre);
                if (d.out) st_relaxed_u64(d.out + col, tag_pack(o, otag));
                else __stcg(d.out_plain + col, o);
                if (d.ss_out) {
                    const float sq = warp_sum(__fmul_rn(o, o));
                    if (lane == 0) st_relaxed_u64(d.ss_out + u, tag_pack(sq, otag));
                }
            }
        }
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
                                           int tid, int cta, int grid, bool stable_all) {
    const int per_head = op.n_items / a.kv_heads;
    // Early reads of rows written in this launch: the SM learned that their
    // writer is complete through relaxed polls only, so an acquire fence
    // (which also drops any L1 line of the cache, read with cp.async.ca)
    // comes before the first of those reads.
    if (stable_all && first_item(cta, op, grid) < op.n_items) fence_acq_rel_gpu();
    for (int j = first_item(cta, op, grid); j < op.n_items; j += op.avail) {
        attn::attn_item<HD, G, kNT, 1>(a, j / per_head, j % per_head, 0, tid, sm, stable_all);
        csync();
    }
}

// last_gemv: the latest GEMV op whose whole input this SM has waited for.
// Each op's items wait for the previous op's whole output, so every op before
// last_gemv is complete; if that includes the writer of the cache's last row
// (its K/V stores precede its release fence and tagged outputs), all cached
// rows are final and the item may read them before its own inputs arrive.
// (This SM reads those rows only once they are final, so its L1 holds no
// stale copy of them.)
__device__ __noinline__ void run_attn(const AttnArgs &a, const OpRef &op, FrameSmem &S, int tid, int cta,
                                     int grid, int last_gemv) {
    const bool stable_all = a.stable_writer >= 0 && last_gemv > a.stable_writer;
    const int G = a.heads / a.kv_heads;
    if (a.kv.head_dim == 128) {
        if (G == 1) attn_items<128, 1>(a, op, S.u.a128_1, tid, cta, grid, stable_all);
        else if (G == 2) attn_items<128, 2>(a, op, S.u.a128_2, tid, cta, grid, stable_all);
        else attn_items<128, 4>(a, op, S.u.a128_4, tid, cta, grid, stable_all);
    } else {
        if (G == 1) attn_items<64, 1>(a, op, S.u.a64_1, tid, cta, grid, stable_all);
        else if (G == 2) attn_items<64, 2>(a, op, S.u.a64_2, tid, cta, grid, stable_all);
        else attn_items<64, 4>(a, op, S.u.a64_4, tid, cta, grid, stable_all);
    }
}

// The sampler op (kept out of line: cold code, its own register budget).
__device__ __noinline__ void run_sample(const FrameParams &P, FrameSmem &S, int tid) {
    samp::sample_row<kNT, 1>(P.sample, 0, tid, S.u.samp);
}

// Next op after `i` that has items on this SM (n_ops if none).
__device__ __forceinline__ int next_op(const FrameSmem &S, int i, int n_ops, int cta, int grid) {
    for (int k = i + 1; k < n_ops; k++)
        if (first_item(cta, S.ops[k], grid) < S.ops[k].n_items) return k;
    return n_ops;
}

// Threads 32.. start copying op i's descriptor into slot b (cp.async).
__device__ __forceinline__ void stage_issue(const FrameParams &P, FrameSmem &S, int i, int b, int tid) {
    const OpRef &op = S.ops[i];
    if (op.type == OP_SAMPLE) return;
    const uint4 *src = op.type == OP_GEMV ? reinterpret_cast<const uint4 *>(P.gemv + op.idx)
                                          : reinterpret_cast<const uint4 *>(P.attn + op.idx);
    const int nw = (op.type == OP_GEMV ? (int)sizeof(GemvDesc) : (int)sizeof(AttnArgs)) / 16;
    const int k = tid - 32;
    if (k >= 0 && k < nw) cp_async16(&S.desc[b].words[k], src + k);
}

// The staging threads wait for their copies; attention descriptors get this
// launch's tag base (the thread that copied that word patches it).
__device__ __forceinline__ void stage_wait(const FrameParams &P, FrameSmem &S, int i, int b, int tid) {
    const OpRef &op = S.ops[i];
    if (op.type == OP_SAMPLE) return;
    const int nw = (op.type == OP_GEMV ? (int)sizeof(GemvDesc) : (int)sizeof(AttnArgs)) / 16;
    const int k = tid - 32;
    if (k >= 0 && k < nw) {
        cp_async_commit_wait();
        if (op.type == OP_ATTN && k == (int)(offsetof(AttnArgs, tag_base) / 16))
            S.desc[b].a.tag_base = P.tag_base;
    }
}

__device__ void consumer(const FrameParams &P, FrameSmem &S, int tid, int cta, int grid) {
    uint32_t q = 0;
    int rbuf = 0, b = 0, last_gemv = -1;
    int i = next_op(S, -1, P.n_ops, cta, grid);
    if (i < P.n_ops) {
        stage_issue(P, S, i, b, tid);
        stage_wait(P, S, i, b, tid);
    }
    csync();
    // One barrier per op: it ends op i (every thread is done with the shared
    // buffers it used), publishes op i+1's staged descriptor and carries the
    // abort decision.
    while (i < P.n_ops) {
        const OpRef op = S.ops[i];
        const int j0 = first_item(cta, op, grid);
        const bool tr = P.trace && j0 == 0 && tid == 0;
        const bool ta = P.trace && tid == 0;  // every SM: across-SM stamps
        const int nx = next_op(S, i, P.n_ops, cta, grid);
        if (nx < P.n_ops) stage_issue(P, S, nx, b ^ 1, tid);  // lands while op i runs
        stamp_all(P, i, 3, ta);
        if (op.type == OP_GEMV) {
            const GemvDesc &d = S.desc[b].g;
            float ssp = 0.0f;
            if (streamed_input(d)) ssp = build_streamed(P, d, S, tid);
            else build_input(P, d, S, tid, j0 == 0, j0, op.n_items, op.avail);
            last_gemv = i;
            stamp_all(P, i, 0, ta);
            stamp_all(P, i, 1, ta);
            gemv_items(P, d, op, S, tid, cta, grid, q, rbuf, tr, i, ssp);
            if (d.adv_len && j0 == 0 && tid == 0) {
                // end of the talker step: the cache and RoPE position advance
                d.adv_len[0] += 1;
                d.adv_pos[0] += 1;
            }
        } else if (op.type == OP_ATTN) {
            stamp_all(P, i, 0, ta);  // (the q/k/v wait is inside the items)
            stamp_all(P, i, 1, ta);
            run_attn(S.desc[b].a, op, S, tid, cta, grid, last_gemv);
        } else {
            stamp_all(P, i, 0, ta);
            stamp_all(P, i, 1, ta);
            run_sample(P, S, tid);
            if (tid == 0) {
                // code 0 for the predictor's semantic pass, tagged
                st_relaxed_u64(P.code0_t, tag_pack(__uint_as_float((uint32_t)S.u.samp.out_code), P.tag_base + i + 1));
            }
        }
        if (nx < P.n_ops) stage_wait(P, S, nx, b ^ 1, tid);
        const bool stop = csync_or(*(volatile int *)&S.abort != 0);
        stamp_all(P, i, 2, ta);
        if (stop) return;
        b ^= 1;
        i = nx;
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
    for (int i = tid; i < P.n_ops; i += kThreads)
        reinterpret_cast<uint4 *>(S.ops)[i] = __ldg(reinterpret_cast<const uint4 *>(P.ops) + i);
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

    int last_rot = 0, last_used = 0;  // the SM window of the previous op

    // appends an op; returns its tag (op index + 1, relative to the launch).
    // Items go round the SMs continuing where the previous op's ended; with
    // avail > 0 they are instead spread over the `avail` SMs right after the
    // previous op's window (which must then be grid - last_used wide).
    uint32_t push(int type, int idx, int n_items, int avail = 0) {
        OpRef r;
        r.type = (int16_t)type;
        r.idx = idx;
        r.n_items = n_items;
        if (avail > 0) {
            r.rot = (last_rot + last_used) % grid;
            r.avail = (int16_t)avail;
            items_total = (int64_t)r.rot + avail;
        } else {
            r.rot = (int)(items_total % grid);
            r.avail = (int16_t)grid;
            items_total += n_items;
        }
        last_rot = r.rot;
        last_used = std::min(n_items, (int)r.avail);
        fp->ops.push_back(r);
        return (uint32_t)fp->ops.size();
    }
    uint32_t next_tag() const { return (uint32_t)fp->ops.size() + 1; }
    uint32_t gemv(GemvDesc d, const Q4Dev &w, int G) {
        d.nib = w.nib;
        d.scl = w.scl;
        d.kpad = (int)w.kpad;
        d.K = (int)w.k;
        d.G = G;
        d.units = (int)(w.C / G);
        d.out_tag = next_tag();
        fp->gemv.push_back(d);
        // Small single-group items that would spill onto the SMs still
        // finishing the previous op (whose inputs then arrive late there) go
        // two to an SM on the free SMs instead: a second item of K <= 1024 rows
        // costs less than the late start (the predictor's QKV after its down
        // projection).
        const int free_sms = grid - last_used;
        const bool avoid = G == 1 && d.K <= 1024 && !d.save && !d.save_plain && free_sms > 0 &&
                           d.units > free_sms && d.units <= 2 * free_sms;
        return push(OP_GEMV, (int)fp->gemv.size() - 1, d.units, avoid ? free_sms : 0);
    }
    uint32_t attn(AttnArgs a, int per_head) {
        a.out_tag = next_tag();
        fp->attn.push_back(a);
        return push(OP_ATTN, (int)fp->attn.size() - 1, a.kv_heads * per_head);
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

    // ---- tagged activation buffers (8 bytes per value) and attention scratch
    const int Hm = std::max(t->H, p->H);
    const int qkvm = (int)std::max(t->qkvn(), (int64_t)(p->heads + 2 * p->kvh) * p->hd);
    const int qdm = (int)std::max(t->qd(), (int64_t)p->heads * p->hd);
    const int ffm = std::max(t->ffn, p->ffn);
    const int kvh_m = std::max(t->kvh, p->kvh);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) / 256 * 256;
        return o;
    };
    const size_t o_qkv = take(8 * qkvm), o_attn = take(8 * qdm), o_xa = take(8 * Hm),
                 o_xb = take(8 * Hm), o_ssa = take(8 * (Hm / 32)), o_ssb = take(8 * (Hm / 32)),
                 o_h = take(8 * ffm), o_head = take(8 * p->vocab), o_codes = take(8 * 16),
                 o_apo = take(4 * std::max(attn_part_o_floats(1, t->kvh, t->heads, t->hd),
                                           attn_part_o_floats(1, p->kvh, p->heads, p->hd))),
                 o_apml = take(4 * std::max(attn_part_ml_floats(1, t->kvh, t->heads),
                                            attn_part_ml_floats(1, p->kvh, p->heads))),
                 o_atk = take(4 * kvh_m);
    rc = fp->bufs.alloc(off);
    if (rc == QORA_OK) rc = fp->bufs.zero();  // tag 0 never matches
    if (rc != QORA_OK) {
        delete fp;
        return rc;
    }
    char *base = fp->bufs.as<char>();
    uint64_t *qkv = (uint64_t *)(base + o_qkv), *attn_out = (uint64_t *)(base + o_attn);
    uint64_t *xa = (uint64_t *)(base + o_xa), *xb = (uint64_t *)(base + o_xb);
    uint64_t *ssa = (uint64_t *)(base + o_ssa), *ssb = (uint64_t *)(base + o_ssb);
    uint64_t *hbuf = (uint64_t *)(base + o_h), *head = (uint64_t *)(base + o_head);
    uint64_t *codes_t = (uint64_t *)(base + o_codes);
    float *apo = (float *)(base + o_apo), *apml = (float *)(base + o_apml);
    unsigned *atk = (unsigned *)(base + o_atk);
    rc = fp->d_abort.alloc(16);
    if (rc == QORA_OK) rc = fp->d_abort.zero();
    if (rc != QORA_OK) {
        delete fp;
        return rc;
    }
    int *abort_flag = fp->d_abort.as<int>();

    Builder B{fp, fp->grid};
    uint32_t *codes = e->codes.as<uint32_t>();
    uint32_t *prev = e->prev.as<uint32_t>();
    float *hidden = p->x2.as<float>();  // row 0: the talker's final-normed hidden

    // the op that last wrote each tagged buffer (its tag)
    uint32_t tag_xa = 0, tag_ssa = 0;
    uint32_t code_tag[16] = {};

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
    code_tag[0] = B.push(OP_SAMPLE, 0, 1);

    // One decoder layer (talker.rs:275-349).  The residual stream enters in xa
    // (sums of squares in ssa) unless `first` supplies the QKV input itself;
    // attention adds into xb (ssb), the MLP back into xa (ssa).
    int last_attn_op = -1;  // op index of the latest attention op (set by layer())
    auto layer = [&](const LayerDev &ld, int heads, int kvh, int hd, const GemvDesc *first, AttnArgs at,
                     int per_head) {
        const int qkvn = (heads + 2 * kvh) * hd;
        GemvDesc q = first ? *first : GemvDesc();
        if (!first) {
            q.in = xa;
            q.in_tag = tag_xa;
            q.ss_in = ssa;
            q.ss_tag = tag_ssa;
        }
        q.gamma = ld.in_norm.as<__half>();
        q.out = qkv;
        const uint32_t tag_qkv = B.gemv(q, ld.qkv, 1);
        if (first && first->save == xa) tag_xa = tag_qkv;  // the frame input, saved by this op
        at.qkv = nullptr;
        at.qkv_t = qkv;
        at.qkv_tag = tag_qkv;
        at.ldqkv = qkvn;
        at.heads = heads;
        at.kv_heads = kvh;
        at.T = 1;
        at.streams = 1;
        at.q_gamma = ld.q_norm.as<__half>();
        at.k_gamma = ld.k_norm.as<__half>();
        at.out = nullptr;
        at.out_t = attn_out;
        at.ldout = (int64_t)heads * hd;
        at.part_o = apo;
        at.part_ml = apml;
        at.tickets = atk;
        at.err = ctx->err.as<int>();
        at.abort_flag = abort_flag;
        const uint32_t tag_attn = B.attn(at, per_head);
        last_attn_op = (int)tag_attn - 1;
        GemvDesc o;
        o.in = attn_out;
        o.in_tag = tag_attn;
        o.out_mode = OUT_RESID;
        o.resid = xa;
        o.resid_tag = tag_xa;
        o.out = xb;
        o.ss_out = ssb;
        const uint32_t tag_xb = B.gemv(o, ld.o, 1);
        GemvDesc gu;
        gu.in = xb;
        gu.in_tag = tag_xb;
        gu.ss_in = ssb;
        gu.ss_tag = tag_xb;
        gu.gamma = ld.post_norm.as<__half>();
        gu.out_mode = OUT_SWIGLU;
        gu.out = hbuf;
        const uint32_t tag_h = B.gemv(gu, ld.gu, 2);
        GemvDesc dn;
        dn.in = hbuf;
        dn.in_tag = tag_h;
        dn.out_mode = OUT_RESID;
        dn.resid = xb;
        dn.resid_tag = tag_xb;
        dn.out = xa;
        dn.ss_out = ssa;
        tag_xa = tag_ssa = B.gemv(dn, ld.dn, 1);
    };

    // ---- predictor: 16 single-token passes (hidden, semantic, codes 1..14);
    // the reference's 2-token prefill (code_predictor.rs:345-438) is causal, so
    // its two tokens are the first two passes
    AttnArgs pat;
    pat.rope_cos = p->rope_cos.as<float>();
    pat.rope_sin = p->rope_sin.as<float>();
    pat.rope_max_pos = p->rope_max;
    uint32_t tag_head = 0;
    std::vector<int> prev_attn_op((size_t)p->L, -1);
    for (int tk = 0; tk <= p->groups; tk++) {
        GemvDesc pr;  // project_input (code_predictor.rs:51-61) into the residual stream
        if (tk == 0) {
            pr.in_mode = IN_VEC;
            pr.in_plain = hidden;
        } else if (tk == 1) {
            pr.in_mode = IN_EMB;
            pr.code_src = codes_t;
            pr.code_tag = code_tag[0];
            pr.emb = t->codec_emb;
            // this pass needs only code 0, so it waits for the first pass's last
            // output before reusing its buffers and its cache position
            pr.dep = xa;
            pr.dep_tag = tag_xa;
            pr.dep_n = p->H;
        } else {
            pr.in_mode = IN_EMB;
            pr.amax_src = head;
            pr.amax_tag = tag_head;
            pr.amax_n = p->vocab;
            pr.code_dst = codes_t + (tk - 1);
            pr.emb = p->embs[tk - 2];
        }
        pr.out = xa;
        pr.ss_out = ssa;
        pr.bias = p->proj_bias.as<float>();
        const uint32_t tg = B.gemv(pr, p->proj, 1);
        if (tk >= 2) code_tag[tk - 1] = tg;
        tag_xa = tag_ssa = tg;
        for (int l = 0; l < p->L; l++) {
            AttnArgs at = pat;
            at.kv = e->pkv->layer(l);
            at.pos_static = tk;
            at.len_static = tk;
            at.stable_len = 0;  // the predictor cache is refilled within this launch:
            // its rows [0, tk) are final once the previous pass's attention op
            // of this layer (the writer of row tk - 1) is
            at.stable_writer = tk >= 1 ? prev_attn_op[(size_t)l] : -1;
            layer(p->layers[l], p->heads, p->kvh, p->hd, nullptr, at, 1);
            prev_attn_op[(size_t)l] = last_attn_op;
        }
        if (tk >= 1) {
            GemvDesc hd;
            hd.in = xa;
            hd.in_tag = tag_xa;
            hd.ss_in = ssa;
            hd.ss_tag = tag_ssa;
            hd.gamma = p->final_norm.as<__half>();
            hd.out = head;
            tag_head = B.gemv(hd, p->heads_w[tk - 1], 1);
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
            fr.amax_tag = tag_head;
            fr.amax_n = p->vocab;
            fr.save = xa;  // the frame input is the residual stream for layer 0's attention add
            layer(t->layers[l], t->heads, t->kvh, t->hd, &fr, at, kAttnMaxSplit);
        } else {
            layer(t->layers[l], t->heads, t->kvh, t->hd, nullptr, at, kAttnMaxSplit);
        }
    }
    {
        GemvDesc hd;  // final norm + apply_codec_head (talker.rs:353-359, 647-649)
        hd.in = xa;
        hd.in_tag = tag_xa;
        hd.ss_in = ssa;
        hd.ss_tag = tag_ssa;
        hd.gamma = t->final_norm.as<__half>();
        hd.save_plain = hidden;
        hd.out_plain = e->logits.as<float>();
        hd.adv_len = e->tkv->lens();
        hd.adv_pos = e->pos.as<int>();
        B.gemv(hd, t->head, 1);
    }

    FrameEmbed fe;
    fe.talker = t->codec_emb;
    for (int g = 0; g < p->groups; g++) fe.pred[g] = p->embs[g];
    fe.ngroups = p->groups;
    fe.n = t->H;
    fe.codes_t = codes_t;
    for (int g = 0; g < 16; g++) fe.code_tag[g] = code_tag[g];
    fe.codes = codes;
    fe.prev = prev;

    // ---- device copies
    const size_t nops = fp->ops.size();
    if (nops > (size_t)kMaxOps || nops + 1 >= kTagStride) {
        delete fp;
        return set_error(QORA_ERR_UNSUPPORTED, "frame program has %zu ops (max %d)", nops, kMaxOps);
    }
    rc = fp->d_ops.alloc(nops * sizeof(OpRef));
    if (rc == QORA_OK) rc = fp->d_gemv.alloc(fp->gemv.size() * sizeof(GemvDesc));
    if (rc == QORA_OK) rc = fp->d_attn.alloc(fp->attn.size() * sizeof(AttnArgs));
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
    P.code0_t = codes_t;
    P.fe = fe;
    P.abort_flag = abort_flag;
    P.err = ctx->err.as<int>();
    *out = fp;
    return QORA_OK;
}

int frame_launch(FrameProgram *fp, const float *text, cudaStream_t st) {
    FrameParams P = fp->params;
    P.text = text;
    P.trace = fp->trace ? fp->d_trace.as<unsigned long long>() : nullptr;
    // Each launch bakes its tags into its parameters, so a captured launch
    // replayed from a graph would accept the previous replay's words as its
    // own: capture is refused (the per-op path is the one to capture).
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    QORA_CUDA(cudaStreamIsCapturing(st, &cs));
    if (cs != cudaStreamCaptureStatusNone)
        return set_error(QORA_ERR_UNSUPPORTED,
                         "the persistent frame kernel cannot be captured in a CUDA graph "
                         "(qora_engine_use_persistent(e, 0) selects the capturable per-op path)");
    // tags unique to this launch (a stale word from an earlier launch never
    // matches).  tag_base = epoch * kTagStride stays below 2^32; before the
    // epochs start over, every tagged word is cleared back to tag 0, which no
    // launch uses, so a word left over from an earlier cycle cannot match.
    fp->epoch++;
    if ((uint64_t)fp->epoch * kTagStride >= (1ull << 32)) {
        QORA_CUDA(cudaMemsetAsync(fp->bufs.p, 0, fp->bufs.bytes, st));
        fp->epoch = 1;
    }
    P.tag_base = fp->epoch * kTagStride;
    QORA_CUDA(cudaMemsetAsync(fp->d_abort.p, 0, 4, st));
    if (fp->trace) QORA_CUDA(cudaMemsetAsync(fp->d_trace.p, 0, fp->d_trace.bytes, st));
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

// The sampler's arguments travel in the launch parameters, so the next launch
// picks the new temperature up.
void frame_program_set_temperature(FrameProgram *p, float temperature) {
    p->params.sample.params.temperature = temperature;
}

}  // namespace qora
