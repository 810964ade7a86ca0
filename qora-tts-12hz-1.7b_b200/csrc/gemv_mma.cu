// Tensor-core Q4 GEMV for batched rows (sm_100a, tcgen05).
//
// The batched step of the reference's gemv / gemm (gemv.rs:149-162, 290-412)
// is a dense contraction once 8 or more rows share the weights:
//     y[r][j] = sum_k x[r][k] * (q[k][j] - 8) * scale[k][j/32]
// One CTA computes a 128-column tile (four 32-column groups) for 32 rows over
// a slice of K, as D[column][row] = A[column][k] * B[row][k]: A = the
// dequantised weights, written by the CUDA cores straight into tensor memory;
// B = the input rows, in shared memory; D accumulated in tensor memory.
//
// Exactness of the operands (f16, kind::f16, f32 accumulate):
//   * the scale is pre-multiplied by 2^E (E per weight matrix, chosen at
//     upload so that 8 * scale * 2^E <= 2^15) and split as s = sa + sb, sa
//     the top 8 significant bits and sb the 3-bit remainder; (q - 8) * sa and
//     (q - 8) * sb are then exact f16 values (<= 11 and <= 6 significant bits),
//     so A1 + A2 = 2^E (q - 8) scale exactly;
//   * each input row is scaled by a power of two 2^e_r (its largest value
//     over the CTA's K slice lands in [2^14, 2^15), so any magnitude fits
//     the f16 operands) and split as xh = f16(x), xl = f16(x - xh) (22
//     significant bits); the epilogue multiplies by 2^-e_r;
//   * D = A1 [xh; xl] (one N = 64 MMA: the xh and xl products side by side)
//     + A2 xh (A2 xl, ~2^-19 relative, is dropped); the epilogue adds the two
//     halves and multiplies by 2^-E.
// The relative error per product is ~2^-17: far inside the 1e-3 tolerance the
// reference accepts for its own chunked summation (gemv.rs:806-809).
//
// Warp roles (192 threads):
//   warps 0-3  warp g converts column group g (TMEM lanes 32 g ..): raw nibbles
//              + scales -> A1 / A2 in tensor memory; and x rows 8 g .. 8 g + 7
//              -> B (hi / lo) in shared memory, RMSNorm prologue applied; then
//              reads the accumulator back and sends it to its K-split owner;
//   warp 4     streams raw weights and x rows into a 4-stage ring with
//              16-byte cp.async copies (weights are immutable and issued before
//              the wait on the previous kernel);
//   warp 5     allocates tensor memory and issues the MMAs (one thread).
// K-split: the S CTAs of one cluster each own a slice of the outputs; every
// CTA sends its partial sums for a slice into the owner's shared memory with
// asynchronous stores that complete on the owner's mbarrier, and the owner,
// once its bytes are in, sums the S partials in rank order and applies the
// epilogue.  Every mbarrier wait is bounded.
#include "gemv_impl.cuh"
#include "tc.cuh"

namespace qora {

namespace {

using namespace gemv_detail;

constexpr int kMmaRows = 32;                 // batch rows per CTA (MMA N = 2 x 32: hi / lo)
constexpr int kMmaGroups = 4;                // 32-column groups per CTA (MMA M = 128)
constexpr int kStageK = 32;                  // K rows per pipeline stage (two K = 16 MMAs)
constexpr int kRawStages = 4;
constexpr int kOpStages = 4;
constexpr int kConvGroups = 2;               // converter groups: group c takes stages t = c mod 2
constexpr int kConvWarps = 4 * kConvGroups;
constexpr int kProdWarp = kConvWarps;
constexpr int kMmaWarp = kConvWarps + 1;
constexpr int kMmaThreads = (kConvWarps + 2) * 32;
// tensor memory columns: D (64: hi then lo products), then per operand stage
// A1 (16 columns: 32 f16 K values) and A2 (16)
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kTmemA = 64;
constexpr uint32_t kTmemAStage = 32;

// raw stage (bytes): per-group nibble rows and scales, then x rows; strides
// padded by 16 bytes so that the groups / rows fall on different banks
constexpr int kNibGroupStride = kStageK * 16 + 16;
constexpr int kSclGroupStride = kStageK * 2 + 16;
constexpr int kXRowStride = kStageK * 4 + 16;
constexpr int kRawNib = 0;
constexpr int kRawScl = kRawNib + kMmaGroups * kNibGroupStride;
constexpr int kRawX = kRawScl + kMmaGroups * kSclGroupStride;
constexpr int kRawGamma = kRawX + kMmaRows * kXRowStride;   // RMSNorm gamma of the stage (f16)
constexpr int kRawBytes = kRawGamma + kStageK * 2;
// operand stage: B = [xh rows; xl rows] (64 x 32 f16) in the canonical K-major
// layout without swizzle.  Core matrix (8 rows x 8 k) = 128 contiguous bytes;
// core (row block rb, k block kc) at (rb * 4 + kc) * 128, so LBO (along K) =
// 128 and SBO (along rows) = 512; the xl rows are row blocks 4-7.
constexpr int kBTile = kMmaRows * kStageK * 2;  // one of xh / xl
constexpr int kOpBytes = 2 * kBTile;
constexpr uint32_t kLBO = 128, kSBO = 512;
// K-split reduction: 16 units per CTA tile, unit = (output group, chunk of
// rows); rank q of S owns units u with u % S == q.  Receive buffer: [unit slot
// u / S][source rank][partial][column][padded chunk rows] (rows padded by 4:
// 16-byte remote stores): ceil(16 / S) * S (slot, source) pairs, at most
// kSlotPairs for the splits the planner uses (S <= 12 or S == 16).
constexpr int kUnits = 16;
constexpr int kSlotPairs = 24;
constexpr bool split_ok(int S) { return S >= 1 && (S <= 12 || S == 16); }
constexpr int kRecvFloats = kSlotPairs * 2 * 32 * 8 > kSlotPairs * 32 * 12 ? kSlotPairs * 2 * 32 * 8
                                                                           : kSlotPairs * 32 * 12;
static_assert(split_ok(kMaxSplit), "the largest cluster split");
constexpr size_t kMmaSmem =
    128 + (size_t)kOpStages * kOpBytes + (size_t)kRawStages * kRawBytes + (size_t)kRecvFloats * 4;

static_assert(kOpBytes % 128 == 0 && kRawBytes % 16 == 0, "stage alignment");
static_assert(kMmaRows == 32 && kConvWarps == kConvGroups * kMmaGroups, "one converter warp per column group");

// 16-byte asynchronous copy global -> shared (L2 only), both addresses 16-byte aligned.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// One arrival on `bar` (counted in its init count) once every cp.async this
// thread issued before has landed.
__device__ __forceinline__ void cp_async_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait that also gives up when another role of this CTA aborted.
// The spin is try_wait alone (it suspends in hardware for a while before
// failing); the bound (2^31 SM cycles, about a second) and the abort flag
// are looked at every 32 attempts, with the SM's own cycle counter.
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort_s,
                                              int *err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t i = 1;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 31) == 0) {
            if (*abort_s) return false;
            if (clock64() - t0 > (1ll << 31)) {
                raise_error(err, kDevTimeout);
                *abort_s = 1;
                return false;
            }
        }
    }
}

// Shared-memory address of `local` (this CTA) in cluster rank `rank`'s shared memory.
__device__ __forceinline__ uint32_t cluster_addr(const void *local, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c),
                 "f"(d)
                 : "memory");
}
// Asynchronous 16-byte store into a cluster peer's shared memory; its bytes
// complete on the peer's mbarrier `bar` (a shared::cluster address too).
__device__ __forceinline__ void st_async_v4(uint32_t addr, float a, float b, float c, float d, uint32_t bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                     addr),
                 "f"(a), "f"(b), "f"(c), "f"(d), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

// Exponent e for which m * 2^e lies in [2^14, 2^15) (m > 0 finite; the
// result is clamped to [-100, 100], so 2^e and 2^-e are normal floats);
// 0 for m == 0 or a non-finite m.
__device__ __forceinline__ int operand_exponent(float m) {
    if (!(m > 0.0f) || !(m <= 3.4e38f)) return 0;
    const int ex = (int)((__float_as_uint(m) >> 23) & 0xFF) - 127;  // floor(log2 m); subnormal: -127
    return max(-100, min(100, 14 - ex));
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

template <int XM, int EM>
__global__ void __maxnreg__(80) k_gemv_mma(const GemvArgs a) {
    constexpr int CO = (EM == E_SWIGLU) ? kMmaGroups / 2 : kMmaGroups;  // output groups per CTA
    constexpr int P = (EM == E_SWIGLU) ? 2 : 1;      // partials per output (gate, up)
    constexpr int RC = kMmaRows * CO / kUnits;       // rows per reduction unit (8, or 4 for SwiGLU)
    constexpr int RPAD = RC + 4;                     // padded chunk row stride in the receive buffer
    constexpr int NCH = kMmaRows / RC;               // row chunks per output group
    extern __shared__ uint8_t mma_dyn[];
    __shared__ __align__(8) uint64_t raw_full[kRawStages], raw_empty[kRawStages];
    __shared__ __align__(8) uint64_t op_full[kOpStages], op_empty[kOpStages], d_full, recv_full;
    __shared__ uint32_t tmem_slot;
    __shared__ float inv_s[kMmaRows];
    __shared__ int rexp_s[kMmaRows];      // B operand of row r is x * 2^rexp_s[r]
    __shared__ float red_s[kConvWarps];
    __shared__ int abort_s;
    __shared__ int last_flag;

    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)mma_dyn + 127) & ~(uintptr_t)127);
    uint8_t *op_base = smem;
    uint8_t *raw_base = smem + kOpStages * kOpBytes;
    float *recv = reinterpret_cast<float *>(raw_base + kRawStages * kRawBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t c0 = (int64_t)blockIdx.x * kMmaGroups;
    const int T = (int)(a.w.k / kStageK);
    const int t_begin = (int)((int64_t)blockIdx.y * T / a.S);
    const int t_end = (int)((int64_t)(blockIdx.y + 1) * T / a.S);
    const int nst = t_end - t_begin;
    const int r_begin = blockIdx.z * kMmaRows;
    const int r_end = min(a.rows, r_begin + kMmaRows);
    const int nvalid = r_end - r_begin;
    volatile int *abort_v = &abort_s;
    cg::cluster_group cluster = cg::this_cluster();
    const int S = a.S;
    const int rank = (S == 1) ? 0 : (int)cluster.block_rank();

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRawStages; i++) {
            mbar_init(&raw_full[i], 32);  // one cp.async arrival per producer lane
            mbar_init(&raw_empty[i], 4);  // the converter group of the stage
        }
        for (int i = 0; i < kOpStages; i++) {
            mbar_init(&op_full[i], 4);
            mbar_init(&op_empty[i], 1);
        }
        mbar_init(&d_full, 1);
        mbar_init(&recv_full, 1);  // this rank's K-split partials (expect_tx below)
        static_assert(kOpStages % kConvGroups == 0, "a converter group keeps its operand stages");
        abort_s = 0;
        mbar_fence_init();
    }
    if (warp == kMmaWarp) {
        tc::tmem_alloc(&tmem_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    // K-split: the cluster's ranks send partial sums into each other's
    // receive buffers; a rank's mbarriers must be initialised before a peer
    // stores, which this arrive (released here, waited on before the first
    // remote store) guarantees.  This rank expects every byte of its units.
    if (S > 1) {
        cluster_arrive();
        if (threadIdx.x == 0) {
            uint32_t bytes = 0;
            for (int slot = 0; slot * S + rank < kUnits; slot++)
                if (((slot * S + rank) % NCH) * RC < nvalid) bytes += (uint32_t)(S * P * 32 * RC * 4);
            mbar_arrive_expect_tx(&recv_full, bytes);
        }
    }

    if (warp == kProdWarp) {
        // ---------------------------------------------------------- producer
        // 16-byte cp.async per lane (a stage is ~13 coalesced copies per lane);
        // each lane's arrival on raw_full[b] fires when its copies have landed
        auto issue_w = [&](int t) {
            uint8_t *raw = raw_base + (t % kRawStages) * kRawBytes;
            const int64_t k0 = (int64_t)(t_begin + t) * kStageK;
#pragma unroll
            for (int g = 0; g < kMmaGroups; g++)  // row `lane` of each group
                cp_async16(raw + kRawNib + g * kNibGroupStride + lane * 16, a.w.nib + (c0 + g) * a.w.kpad + k0 + lane);
            if (lane < kMmaGroups * 4) {  // 64 bytes of scales per group
                const int g = lane >> 2, part = lane & 3;
                cp_async16(raw + kRawScl + g * kSclGroupStride + part * 16,
                           reinterpret_cast<const uint8_t *>(a.w.scl + (c0 + g) * a.w.kpad + k0) + part * 16);
            }
            if constexpr (XM == X_RMSNORM) {  // the stage's 32 gamma values (immutable)
                if (lane >= 28) cp_async16(raw + kRawGamma + (lane - 28) * 16, a.gamma + k0 + (lane - 28) * 8);
            }
        };
        // X_EMBED: the token of row `lane` (tokens come from earlier kernels)
        uint32_t tok = 0;
        auto issue_x = [&](int t) {
            const int b = t % kRawStages;
            uint8_t *raw = raw_base + b * kRawBytes;
            const int64_t k0 = (int64_t)(t_begin + t) * kStageK;
            if constexpr (XM == X_EMBED) {
                // row `lane`: the stage's 16 bytes of nibbles and the 16-byte
                // block holding its scale (embed_lookup_q4, gemv.rs:425-433)
                if (lane < nvalid) {
                    cp_async16(raw + kRawX + lane * kXRowStride, a.emb.packed + (int64_t)tok * (a.emb.n >> 1) + (k0 >> 1));
                    const int64_t si = (int64_t)tok * (a.emb.n >> 5) + (k0 >> 5);
                    cp_async16(raw + kRawX + lane * kXRowStride + 16, a.emb.scl + (si & ~(int64_t)7));
                }
            } else {
                for (int i = lane; i < nvalid * 8; i += 32) {  // 8 x 16 bytes per row
                    const int r = i >> 3, part = i & 7;
                    cp_async16(raw + kRawX + r * kXRowStride + part * 16,
                               a.x + (int64_t)(r_begin + r) * a.ldx + k0 + part * 4);
                }
            }
            cp_async_arrive(&raw_full[b]);
        };
        if (lane == 0 && (a.pf0_bytes | a.pf1_bytes)) {
            const uint64_t nctas = (uint64_t)gridDim.x * gridDim.y * gridDim.z;
            const uint64_t id = ((uint64_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
            l2_prefetch_share(a.pf0, a.pf0_bytes, id, nctas);
            l2_prefetch_share(a.pf1, a.pf1_bytes, id, nctas);
        }
        // weights of the first stages before the wait on the previous kernel
        const int pre = min(nst, kRawStages);
        for (int t = 0; t < pre; t++) issue_w(t);
        griddep_launch_dependents();
        griddep_wait();
        if constexpr (XM == X_EMBED) {
            if (lane < nvalid) tok = __ldcg(a.tok + (int64_t)(r_begin + lane) * a.ldtok);
            if ((int64_t)tok >= a.emb.rows) {  // never read outside the table
                raise_error(a.err, kDevRange);
                tok = 0;
            }
        }
        for (int t = 0; t < pre; t++) issue_x(t);
        for (int t = pre; t < nst; t++) {
            const int b = t % kRawStages;
            bool ok = true;
            if (lane == 0) ok = wait_or_abort(&raw_empty[b], ((t / kRawStages) & 1) ^ 1, abort_v, a.err);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            issue_w(t);
            issue_x(t);
        }
        // every copy this CTA issued lands before the CTA can exit
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncwarp();
        if (S > 1) cluster_wait();
    } else if (warp == kMmaWarp) {
        // ---------------------------------------------------------- MMA issue
        griddep_launch_dependents();
        griddep_wait();
        if (lane == 0) {
            constexpr uint32_t id64 = tc::idesc_f16_f32(128, 2 * kMmaRows);
            constexpr uint32_t id32 = tc::idesc_f16_f32(128, kMmaRows);
            for (int t = 0; t < nst; t++) {
                const int o = t % kOpStages;
                if (!wait_or_abort(&op_full[o], (t / kOpStages) & 1, abort_v, a.err)) break;
                tc::fence_after_sync();
                const uint32_t bbase = smem_u32(op_base + o * kOpBytes);
                const uint32_t abase = tmem + kTmemA + (uint32_t)o * kTmemAStage;
#pragma unroll
                for (int j = 0; j < kStageK / 16; j++) {
                    // K = 16: two 8-k core columns of B, 8 TMEM columns of A
                    const uint64_t bhl = tc::smem_desc(bbase + (uint32_t)j * 256, kLBO, kSBO);  // xh; xl
                    tc::mma_f16_ts(tmem, abase + 8 * j, bhl, id64, (t | j) != 0 ? 1u : 0u);
                    tc::mma_f16_ts(tmem, abase + 16 + 8 * j, bhl, id32, 1u);      // A2 * xh
                }
                tc::commit(&op_empty[o]);
            }
            tc::commit(&d_full);
        }
        __syncwarp();
        if (S > 1) cluster_wait();
    } else {
        // ---------------------------------------------------------- converters
        float gmax = 0.0f;
        if constexpr (XM == X_RMSNORM) {
            // gamma is immutable: its largest magnitude over this CTA's K slice
            // is known before the previous kernel is done
            for (int i = threadIdx.x; i < nst * kStageK; i += kConvWarps * 32)
                gmax = fmaxf(gmax, fabsf(__half2float(a.gamma[(int64_t)t_begin * kStageK + i])));
        }
        griddep_launch_dependents();
        griddep_wait();
        const int64_t k = a.w.k;
        if constexpr (XM == X_RMSNORM) {
            // rms_norm_f16 (gemv.rs:445-454): inv from the producer's
            // per-32-column sums of squares, summed as k_gemv sums them
            for (int rr = warp; rr < kMmaRows; rr += kConvWarps) {
                const int r = r_begin + rr;
                float t = 0.0f;
                if (r < r_end)
                    for (int i = lane; i < a.ss_tiles; i += 32) t += __ldcg(a.ss + (int64_t)r * a.ldss + i);
                t = warp_sum(t);
                if (lane == 0) inv_s[rr] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)k), 1e-6f)));
            }
        }
        // ---- per-row power-of-two scale of the B operand: the row's values
        // over this CTA's K slice are multiplied by 2^e (exact) so that the
        // largest lies in [2^14, 2^15): no value can leave the f16 range and
        // small ones keep the precision of the hi / lo split.  The epilogue
        // multiplies by 2^-e (exact), so in-range inputs give the same bits
        // as without the scale.  Bound of the row's largest value:
        //   X_PLAIN   max |x| over the slice, read here (8 threads per row);
        //   X_RMSNORM sqrt(k) * max |gamma|: a normalised row has
        //             sum (x * inv)^2 <= k, so |x * inv| <= sqrt(k);
        //   X_EMBED   8 * the table's largest scale (set at upload).
        {
            const int rr = threadIdx.x >> 3, part = threadIdx.x & 7;
            float m = 0.0f;
            if constexpr (XM == X_PLAIN) {
                if (r_begin + rr < r_end) {
                    // eight 16-byte loads in flight per thread (the row's 8
                    // threads read 128 contiguous bytes per step), so a slice
                    // of up to 256 values costs one round trip, overlapped
                    // with the producer's first stage
                    const float4 *xr = reinterpret_cast<const float4 *>(
                        a.x + (int64_t)(r_begin + rr) * a.ldx + (int64_t)t_begin * kStageK);
                    const int n4 = nst * (kStageK / 4);
                    for (int i0 = part; i0 < n4; i0 += 64) {
                        float4 v[8];
#pragma unroll
                        for (int u = 0; u < 8; u++)
                            v[u] = i0 + 8 * u < n4 ? __ldcg(xr + i0 + 8 * u) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (int u = 0; u < 8; u++)
                            m = fmaxf(m, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)),
                                               fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
                    }
                }
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
            } else if constexpr (XM == X_RMSNORM) {
                gmax = warp_max(gmax);
                if (lane == 0) red_s[warp] = gmax;
                asm volatile("bar.sync 1, %0;" ::"n"(kConvWarps * 32) : "memory");
#pragma unroll
                for (int w = 0; w < kConvWarps; w++) m = fmaxf(m, red_s[w]);
                // (1 + 2^-10) covers the rounding of inv and of the products
                m = __fmul_rn(__fmul_rn(__fsqrt_rn((float)k), m), 1.0009765625f);
            } else {
                m = a.emb.absmax;
            }
            if (part == 0) rexp_s[rr] = (r_begin + rr < r_end) ? operand_exponent(m) : 0;
            asm volatile("bar.sync 1, %0;" ::"n"(kConvWarps * 32) : "memory");
        }
        // Converter group cgp = warp / 4 takes stages t = cgp, cgp + 2, ...
        // A role: column 32 g + lane of the tile (TMEM lane 32 g + lane), all
        // K rows of the stage.  The nibble pair of K rows (2p, 2p+1) is
        // gathered into one 32-bit word (byte perm) and biased into f16 as
        // 1024 + q (low nibble) or 1024 + 16 q (high nibble); one f16 FMA gives
        // q - 8 exactly.
        const int g = warp & 3, cgp = warp >> 2;
        const int cq = lane & 7;
        const uint32_t sel = (uint32_t)(cq >> 1) | ((uint32_t)(4 + (cq >> 1)) << 8);
        const uint32_t nmask = (cq & 1) ? 0x00F000F0u : 0x000F000Fu;
        const __half2 m1 = __float2half2_rn((cq & 1) ? 0.0625f : 1.0f);
        const __half2 c1 = __float2half2_rn((cq & 1) ? -72.0f : -1032.0f);
        const int E = a.w.mma_exp;
        const __half2 pw = __float2half2_rn(__int_as_float((127 + E) << 23));
        const uint32_t a_lane = tmem + ((uint32_t)(32 * g) << 16) + kTmemA;
        // B role: row r = 8 g + lane % 8, K block kc = lane / 8 (8 values)
        const bool write_side = (XM == X_RMSNORM) && a.side && blockIdx.x == 0;
        const int r = 8 * g + (lane & 7), kc = lane >> 3;
        const bool rvalid = r < nvalid;
        uint32_t tok_r = 0;  // X_EMBED: the token of row r
        if constexpr (XM == X_EMBED) {
            if (rvalid) tok_r = __ldcg(a.tok + (int64_t)(r_begin + r) * a.ldtok);
            if ((int64_t)tok_r >= a.emb.rows) tok_r = 0;  // (reported by the producer)
        }
        float inv_r = 1.0f;
        if constexpr (XM == X_RMSNORM) inv_r = inv_s[r];
        const float rscale = __int_as_float((127 + rexp_s[r]) << 23);

        for (int t = cgp; t < nst; t += kConvGroups) {
            const int b = t % kRawStages, o = t % kOpStages;
            if (!wait_or_abort(&raw_full[b], (t / kRawStages) & 1, abort_v, a.err)) break;
            if (!wait_or_abort(&op_empty[o], ((t / kOpStages) & 1) ^ 1, abort_v, a.err)) break;
            const uint8_t *raw = raw_base + b * kRawBytes;
            uint8_t *op = op_base + o * kOpBytes;
            const int64_t k0 = (int64_t)(t_begin + t) * kStageK;

            // ---- A1 / A2 -> tensor memory
            const uint8_t *nibg = raw + kRawNib + g * kNibGroupStride + (lane >> 3) * 4;
            uint4 sc4[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
                sc4[i] = *reinterpret_cast<const uint4 *>(raw + kRawScl + g * kSclGroupStride + 16 * i);
            uint32_t A1[16], A2[16];
#pragma unroll
            for (int p = 0; p < 16; p++) {
                const uint32_t w0 = *reinterpret_cast<const uint32_t *>(nibg + (2 * p) * 16);
                const uint32_t w1 = *reinterpret_cast<const uint32_t *>(nibg + (2 * p + 1) * 16);
                const uint32_t sw = (p & 3) == 0 ? sc4[p >> 2].x
                                  : (p & 3) == 1 ? sc4[p >> 2].y
                                  : (p & 3) == 2 ? sc4[p >> 2].z : sc4[p >> 2].w;
                const __half2 s2 = __hmul2(u2h(sw), pw);            // exact (power of two)
                const __half2 sa = u2h(h2u(s2) & 0xFFF8FFF8u);      // top 8 significant bits
                const __half2 sb = __hsub2(s2, sa);                 // exact remainder
                const uint32_t pr = __byte_perm(w0, w1, sel);
                const __half2 q8 = __hfma2(u2h((pr & nmask) | 0x64006400u), m1, c1);
                A1[p] = h2u(__hmul2(q8, sa));
                A2[p] = h2u(__hmul2(q8, sb));
            }
            tc::st_32x32b_x16(a_lane + (uint32_t)o * kTmemAStage, A1);
            tc::st_32x32b_x16(a_lane + (uint32_t)o * kTmemAStage + 16, A2);

            // ---- B (hi / lo): row r, k = k0 + 8 kc .. + 7
            float xv[8];
            if constexpr (XM == X_EMBED) {
                // x = scale * (q - 8) (gemv.rs:425-433): exact in f32, and
                // exact as the f16 hi + lo pair below
                const uint32_t nb = *reinterpret_cast<const uint32_t *>(raw + kRawX + r * kXRowStride + 4 * kc);
                const int64_t si = (int64_t)tok_r * (a.emb.n >> 5) + (k0 >> 5);
                const float sc = __half2float(
                    *reinterpret_cast<const __half *>(raw + kRawX + r * kXRowStride + 16 + 2 * (int)(si & 7)));
#pragma unroll
                for (int i = 0; i < 8; i++) xv[i] = __fmul_rn(sc, (float)((int)((nb >> (4 * i)) & 15u) - 8));
            } else {
                const float4 *xp = reinterpret_cast<const float4 *>(raw + kRawX + r * kXRowStride + kc * 32);
                const float4 u0 = xp[0], u1 = xp[1];
                xv[0] = u0.x; xv[1] = u0.y; xv[2] = u0.z; xv[3] = u0.w;
                xv[4] = u1.x; xv[5] = u1.y; xv[6] = u1.z; xv[7] = u1.w;
            }
            if (!rvalid) {
#pragma unroll
                for (int i = 0; i < 8; i++) xv[i] = 0.0f;
            }
            if constexpr (XM == X_RMSNORM) {
                const uint4 gq = *reinterpret_cast<const uint4 *>(raw + kRawGamma + 16 * kc);
                const uint32_t gw[4] = {gq.x, gq.y, gq.z, gq.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float2 gf = __half22float2(u2h(gw[i]));
                    xv[2 * i] = __fmul_rn(__fmul_rn(xv[2 * i], inv_r), gf.x);
                    xv[2 * i + 1] = __fmul_rn(__fmul_rn(xv[2 * i + 1], inv_r), gf.y);
                }
                if (write_side && rvalid) {
                    float *sp = a.side + (int64_t)(r_begin + r) * a.ldside + k0 + 8 * kc;
#pragma unroll
                    for (int i = 0; i < 8; i++) sp[i] = xv[i];
                }
            }
            uint32_t bh[4], bl[4];
            bool big = false;
#pragma unroll
            for (int i = 0; i < 8; i++) xv[i] = __fmul_rn(xv[i], rscale);  // exact: a power of two
#pragma unroll
            for (int i = 0; i < 4; i++) {
                // after the scale only an infinite input can exceed the range
                big |= fabsf(xv[2 * i]) > 65504.0f || fabsf(xv[2 * i + 1]) > 65504.0f;
                const __half2 hh = __floats2half2_rn(xv[2 * i], xv[2 * i + 1]);
                const float2 hf = __half22float2(hh);
                bh[i] = h2u(hh);
                bl[i] = h2u(__floats2half2_rn(__fsub_rn(xv[2 * i], hf.x), __fsub_rn(xv[2 * i + 1], hf.y)));
            }
            if (big) raise_error(a.err, kDevF16Range);
            {
                const int off = ((r >> 3) * 4 + kc) * 128 + (r & 7) * 16;
                *reinterpret_cast<uint4 *>(op + off) = make_uint4(bh[0], bh[1], bh[2], bh[3]);
                *reinterpret_cast<uint4 *>(op + kBTile + off) = make_uint4(bl[0], bl[1], bl[2], bl[3]);
            }
            tc::fence_proxy_async_smem();   // B: generic-proxy writes -> tensor-core reads
            tc::fence_before_sync();        // A: tensor-memory stores -> the MMA thread
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&raw_empty[b]);
                mbar_arrive(&op_full[o]);
            }
        }
        if (cgp != 0 && S > 1) cluster_wait();
        if (cgp == 0) {
            // ---- accumulator (column 32 g + lane; xh and xl halves), scaled back
            // by 2^-E -> the owners of its units
            const bool ok = wait_or_abort(&d_full, 0, abort_v, a.err);
            tc::fence_after_sync();
            float vh[32], vl[32];
            if (ok) {
                tc::ld_32x32b_x32(tmem + ((uint32_t)(32 * g) << 16), vh);
                tc::ld_32x32b_x32(tmem + ((uint32_t)(32 * g) << 16) + kMmaRows, vl);
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) vh[i] = vl[i] = 0.0f;
            }
            const float unscale = __int_as_float((127 - E) << 23);
#pragma unroll
            for (int n = 0; n < kMmaRows; n++)
                vh[n] = __fmul_rn(__fmul_rn(__fadd_rn(vh[n], vl[n]), unscale),
                                  __int_as_float((127 - rexp_s[n]) << 23));
            const int cc2 = (EM == E_SWIGLU) ? (g >> 1) : g;
            const int hp = (EM == E_SWIGLU) ? (g & 1) : 0;
            if (S > 1) cluster_wait();  // every rank's mbarriers are initialised
#pragma unroll
            for (int c = 0; c < NCH; c++) {
                if (c * RC < nvalid) {
                    const int u = cc2 * NCH + c;
                    const int owner = u % S, slot = u / S;
                    const float *dst = recv + (((slot * S + rank) * P + hp) * 32 + lane) * RPAD;
                    if (S == 1) {
                        const uint32_t da = smem_u32(dst);
#pragma unroll
                        for (int i = 0; i < RC / 4; i++)
                            st_cluster_v4(da + 16 * i, vh[c * RC + 4 * i], vh[c * RC + 4 * i + 1],
                                          vh[c * RC + 4 * i + 2], vh[c * RC + 4 * i + 3]);
                    } else {
                        const uint32_t da = cluster_addr(dst, owner), ba = cluster_addr(&recv_full, owner);
#pragma unroll
                        for (int i = 0; i < RC / 4; i++)
                            st_async_v4(da + 16 * i, vh[c * RC + 4 * i], vh[c * RC + 4 * i + 1],
                                        vh[c * RC + 4 * i + 2], vh[c * RC + 4 * i + 3], ba);
                    }
                }
            }
        }
    }
    // the residual of this rank's first outputs does not depend on the
    // partial sums: load it while the cluster barrier completes
    constexpr int kPre = 4;
    float yres[kPre];
    if constexpr (EM == E_RESID) {
#pragma unroll
        for (int m = 0; m < kPre; m++) {
            yres[m] = 0.0f;
            const int slot = 0;  // the first unit of this rank covers the prefetched items
            const int u = slot * S + rank;
            const int it = threadIdx.x + m * blockDim.x;
            if (u < kUnits) {
                const int cc2 = u / NCH, c = u % NCH;
                const int nrow = min(RC, nvalid - c * RC);
                if (it < nrow * 32) {
                    const int64_t col = ((int64_t)blockIdx.x * CO + cc2) * 32 + (it & 31);
                    yres[m] = __ldcg(a.y + (int64_t)(r_begin + c * RC + (it >> 5)) * a.ldy + col);
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();  // tensor memory read back (S == 1: partials in place)
    if (warp == kMmaWarp) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
    // ---- S > 1: every partial of this rank's units has arrived
    if (S > 1) wait_or_abort(&recv_full, 0, abort_v, a.err);
    // ---- finish this rank's units: rank-order sums, epilogue
    const int64_t n_out = (EM == E_SWIGLU) ? (a.w.C / 2) * 32 : a.w.n;
    for (int slot = 0; slot * S + rank < kUnits; slot++) {
        const int u = slot * S + rank;
        const int cc2 = u / NCH, c = u % NCH;
        const int nrow = min(RC, nvalid - c * RC);
        for (int it = threadIdx.x, m = 0; it < nrow * 32; it += blockDim.x, m++) {  // whole rows per warp
            const int l = it & 31, rr = it >> 5;
            float vsum = 0.0f, usum = 0.0f;
            for (int j = 0; j < S; j++) {
                const float *src = recv + (((slot * S + j) * P) * 32 + l) * RPAD + rr;
                vsum += src[0];
                if constexpr (EM == E_SWIGLU) usum += src[32 * RPAD];
            }
            const int row = c * RC + rr;
            const int64_t grp = (int64_t)blockIdx.x * CO + cc2;
            if constexpr (EM == E_RESID) {
                // x[j] += attn_out[j] (talker.rs:334-336)
                float yr = 0.0f;
                bool have = false;
#pragma unroll
                for (int q = 0; q < kPre; q++)
                    if (slot == 0 && m == q) {
                        yr = yres[q];
                        have = true;
                    }
                if (!have) yr = __ldcg(a.y + (int64_t)(r_begin + row) * a.ldy + grp * 32 + l);
                finalize_resid(a, r_begin + row, grp, l, __fadd_rn(yr, vsum));
            } else {
                finalize_group<EM>(a, r_begin + row, grp, l, vsum, usum, n_out, CO);
            }
        }
    }
    // tail columns beyond the last full group stay zero (gemv.rs:846-861)
    if (EM == E_STORE && a.w.n > a.w.C * 32 && blockIdx.x == 0 && rank == 0) {
        for (int rr = r_begin; rr < r_end; rr++)
            for (int64_t col = a.w.C * 32 + threadIdx.x; col < a.w.n; col += blockDim.x)
                a.y[(int64_t)rr * a.ldy + col] = 0.0f;
    }
    gemv_global_stage(a, last_flag, gridDim.x * CO);
}

// ======================================================================
// Prefill GEMM: the same contraction for many rows (a prompt chunk of up to
// kMaxRows rows), one CTA per 128-column x RT-row tile over all of K
// (RT = 128, or 64 when 128-row tiles would leave SMs idle).
// k_gemv_mma converts each weight tile once per 32 rows and the input rows
// once per column tile; here
//   * k_row_prep finds each row's RMSNorm factor and power-of-two operand
//     exponent (one CTA per row),
//   * k_b_convert writes the B operand of every (128-row tile, 32-K stage)
//     once, in the MMA's shared-memory layout (xh rows, then xl rows; 16 KB
//     for a 128-row tile) in global memory,
//   * k_gemm_mma streams those B tiles with one bulk copy per stage, converts
//     only its weights (A1 / A2 into tensor memory), and issues one N = 2 RT
//     MMA (RT rows, xh and xl side by side) plus one N = RT MMA (A2 xh) per
//     16 K rows.
// The operands, the K order of the accumulation and the epilogue arithmetic
// are those of k_gemv_mma without a K split (the split its prefill plan uses
// at the 1.7B dims), so every output has the same bits as there, whatever
// the rows of the launch.
//
// k_gemm_mma warp roles (320 threads):
//   warps 0..  kGGroups converter groups of four (group c takes stages
//              t = c mod kGGroups; warp g of a group: column group g, TMEM
//              lanes 32 g ..), then the epilogue (warp w: column group w % 4,
//              rows 32 (w / 4) .. + 31 of the row tile);
//   next warp  streams each stage's weights (bulk copies into a raw ring) and
//              B tile (one bulk copy into the operand ring);
//   last warp  allocates tensor memory and issues the MMAs (one thread).
constexpr int kGGroups = 4;                    // converter groups (four warps each)
constexpr int kGConvWarps = 4 * kGGroups;
constexpr int kGProdWarp = kGConvWarps;
constexpr int kGMmaWarp = kGConvWarps + 1;
constexpr int kGThreads = 32 * (kGConvWarps + 2);
constexpr int kGRawSlots = 3;                  // weight slots per converter group (own stages)
constexpr int kGOpStages = 8;
constexpr int kGRawNib = 0;
constexpr int kGRawScl = kGRawNib + kMmaGroups * kNibGroupStride;
constexpr int kGRawBytes = kGRawScl + kMmaGroups * kSclGroupStride;
// Row tiles of RT = 128 or 64 rows (64 when 128-row tiles would leave many
// SMs idle).  One B tile: xh rows then xl rows, RT x 32 K each (f16), in the
// same layout in global and shared memory.
constexpr int gbtile(int RT) { return RT * kStageK * 2; }
constexpr int gopbytes(int RT) { return 2 * gbtile(RT); }
constexpr uint32_t kGTmemCols = 512;           // D: 256 (xh rows, then xl rows), A: 8 stages x 32
constexpr uint32_t kGTmemA = 256;
constexpr uint32_t kGTmemAStage = 32;
constexpr size_t gsmem(int RT) {
    return 128 + (size_t)kGOpStages * gopbytes(RT) + (size_t)kGGroups * kGRawSlots * kGRawBytes;
}
static_assert(kGRawScl % 16 == 0 && kGRawBytes % 16 == 0 && gopbytes(64) % 128 == 0, "bulk-copy alignment");
static_assert(kGOpStages * gopbytes(64) >= 4 * 64 * 32 * 4, "SwiGLU exchange fits the operand stages");

// Byte offset of element (row r, k) of a B tile (K-major core matrices of
// 8 rows x 8 K, 128 contiguous bytes; 4 per row block along K), hi half.
__device__ __forceinline__ int btile_off(int r, int kc) { return ((r >> 3) * 4 + kc) * 128 + (r & 7) * 16; }

// Per-row prologue constants of a prefill GEMM input (one CTA per row):
//   rexp[r]  operand exponent: of max |x[r][0..k)| (X_PLAIN, the value
//            k_gemv_mma finds over an unsplit K), or of the bound
//            sqrt(k) max |gamma| (1 + 2^-10) (X_RMSNORM);
//   rinv[r]  X_RMSNORM: 1 / sqrt(ss / k + 1e-6) (rms_norm_f16, gemv.rs:445-454)
//            from the per-32-column sums of squares, summed as k_gemv_mma sums them.
template <int XM>
__global__ void __launch_bounds__(256) k_row_prep(const GemvArgs a, int *rexp, float *rinv) {
    __shared__ float red[8];
    const int r = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t k = a.w.k;
    float m = 0.0f;
    if constexpr (XM == X_RMSNORM) {
        for (int64_t i = threadIdx.x; i < k; i += 256) m = fmaxf(m, fabsf(__half2float(a.gamma[i])));
    }
    griddep_launch_dependents();
    griddep_wait();
    if constexpr (XM == X_PLAIN) {
        const float4 *xr = reinterpret_cast<const float4 *>(a.x + (int64_t)r * a.ldx);
        for (int64_t i = threadIdx.x; i < k / 4; i += 256) {
            const float4 v = __ldcg(xr + i);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    } else {
        if (warp == 0) {
            float t = 0.0f;
            for (int i = lane; i < a.ss_tiles; i += 32) t += __ldcg(a.ss + (int64_t)r * a.ldss + i);
            t = warp_sum(t);
            if (lane == 0) rinv[r] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)k), 1e-6f)));
        }
    }
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++) t = fmaxf(t, red[w]);
        if constexpr (XM == X_RMSNORM) t = __fmul_rn(__fmul_rn(__fsqrt_rn((float)k), t), 1.0009765625f);
        rexp[r] = operand_exponent(t);
    }
}

// B tiles of a prefill GEMM: block (row tile of RT rows, group of 4
// stages), thread (row r = tid % RT, stages tid / RT + 256 / RT j).  Row r's 32 K values
// of a stage: x (normalised: (x * inv) * gamma), times 2^rexp, split as
// xh = f16(x), xl = f16(x - xh), exactly as k_gemv_mma forms its B operand;
// rows past `rows` are zero.
template <int XM, int RT>
__global__ void __launch_bounds__(256) k_b_convert(const GemvArgs a, const int *rexp, const float *rinv,
                                                   uint8_t *bop) {
    constexpr int SL = 256 / RT;  // threads per row: stage slots of the block's 4 stages
    const int rt = blockIdx.x, r = threadIdx.x % RT;
    const int row = rt * RT + r;
    const bool rvalid = row < a.rows;
    const int nst = (int)(a.w.k / kStageK);
    griddep_launch_dependents();
    griddep_wait();
    const float rscale = __int_as_float((127 + (rvalid ? __ldcg(rexp + row) : 0)) << 23);
    float inv_r = 1.0f;
    if constexpr (XM == X_RMSNORM) inv_r = rvalid ? __ldcg(rinv + row) : 1.0f;
    bool big = false;
    for (int s = threadIdx.x / RT; s < 4; s += SL) {
        const int t = blockIdx.y * 4 + s;
        if (t >= nst) break;
        const int64_t k0 = (int64_t)t * kStageK;
        uint8_t *tile = bop + ((int64_t)rt * nst + t) * gopbytes(RT);
#pragma unroll
        for (int kc = 0; kc < 4; kc++) {
            float xv[8];
            if (rvalid) {
                const float4 *xp = reinterpret_cast<const float4 *>(a.x + (int64_t)row * a.ldx + k0 + 8 * kc);
                const float4 u0 = __ldcg(xp), u1 = __ldcg(xp + 1);
                xv[0] = u0.x; xv[1] = u0.y; xv[2] = u0.z; xv[3] = u0.w;
                xv[4] = u1.x; xv[5] = u1.y; xv[6] = u1.z; xv[7] = u1.w;
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) xv[i] = 0.0f;
            }
            if constexpr (XM == X_RMSNORM) {
                const uint4 gq = __ldg(reinterpret_cast<const uint4 *>(a.gamma + k0 + 8 * kc));
                const uint32_t gw[4] = {gq.x, gq.y, gq.z, gq.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float2 gf = __half22float2(u2h(gw[i]));
                    xv[2 * i] = __fmul_rn(__fmul_rn(xv[2 * i], inv_r), gf.x);
                    xv[2 * i + 1] = __fmul_rn(__fmul_rn(xv[2 * i + 1], inv_r), gf.y);
                }
            }
            uint32_t bh[4], bl[4];
#pragma unroll
            for (int i = 0; i < 8; i++) xv[i] = __fmul_rn(xv[i], rscale);  // exact: a power of two
#pragma unroll
            for (int i = 0; i < 4; i++) {
                big |= fabsf(xv[2 * i]) > 65504.0f || fabsf(xv[2 * i + 1]) > 65504.0f;
                const __half2 hh = __floats2half2_rn(xv[2 * i], xv[2 * i + 1]);
                const float2 hf = __half22float2(hh);
                bh[i] = h2u(hh);
                bl[i] = h2u(__floats2half2_rn(__fsub_rn(xv[2 * i], hf.x), __fsub_rn(xv[2 * i + 1], hf.y)));
            }
            const int off = btile_off(r, kc);
            __stcg(reinterpret_cast<uint4 *>(tile + off), make_uint4(bh[0], bh[1], bh[2], bh[3]));
            __stcg(reinterpret_cast<uint4 *>(tile + gbtile(RT) + off), make_uint4(bl[0], bl[1], bl[2], bl[3]));
        }
    }
    if (big) raise_error(a.err, kDevF16Range);
}

template <int XM, int EM, int RT>
__global__ void __launch_bounds__(kGThreads, 1) k_gemm_mma(const GemvArgs a) {
    constexpr int CO = (EM == E_SWIGLU) ? kMmaGroups / 2 : kMmaGroups;  // output groups per CTA
    constexpr int kGOpBytes = gopbytes(RT);
    extern __shared__ uint8_t gm_dyn[];
    __shared__ __align__(8) uint64_t b_full[kGOpStages], a_full[kGOpStages], op_empty[kGOpStages], d_full;
    __shared__ uint32_t tmem_slot;
    __shared__ int rexp_s[RT];
    __shared__ int abort_s;
    __shared__ int grp_go[kGGroups];  // a converter group's decision for its current stage

    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)gm_dyn + 127) & ~(uintptr_t)127);
    uint8_t *op_base = smem;
    uint8_t *raw_base = smem + kGOpStages * kGOpBytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t c0 = (int64_t)blockIdx.x * kMmaGroups;
    const int nst = (int)(a.w.k / kStageK);
    const int r_begin = blockIdx.y * RT;
    const int nvalid = min(RT, a.rows - r_begin);
    volatile int *abort_v = &abort_s;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kGOpStages; i++) {
            mbar_init(&b_full[i], 1);     // expect_tx arrival (+ the B tile's bytes)
            mbar_init(&a_full[i], 4);     // the converter group: A in tensor memory
            mbar_init(&op_empty[i], 1);   // the MMAs of the stage (commit)
        }
        mbar_init(&d_full, 1);
        abort_s = 0;
        mbar_fence_init();
    }
    if (warp == kGMmaWarp) {
        tc::tmem_alloc(&tmem_slot, kGTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;

    if (warp == kGProdWarp) {
        // ---------------------------------------------------------- producer
        // one bulk copy per stage: the stage's B tile, once the MMAs of the
        // stage that last used its operand slot are done
        auto issue_b = [&](int t) {
            if (lane == 0) {
                const int o = t % kGOpStages;
                mbar_arrive_expect_tx(&b_full[o], kGOpBytes);
                bulk_g2s(op_base + o * kGOpBytes, a.bop + ((int64_t)blockIdx.y * nst + t) * kGOpBytes, kGOpBytes,
                         &b_full[o]);
            }
        };
        if (lane == 0 && (a.pf0_bytes | a.pf1_bytes)) {
            const uint64_t nctas = (uint64_t)gridDim.x * gridDim.y;
            const uint64_t id = (uint64_t)blockIdx.y * gridDim.x + blockIdx.x;
            l2_prefetch_share(a.pf0, a.pf0_bytes, id, nctas);
            l2_prefetch_share(a.pf1, a.pf1_bytes, id, nctas);
        }
        griddep_launch_dependents();
        griddep_wait();
        const int preb = min(nst, kGOpStages);
        for (int t = 0; t < preb; t++) issue_b(t);
        int issued_b = preb;
        for (int t = 0; t + kGOpStages < nst; t++) {
            bool ok = true;
            if (lane == 0) ok = wait_or_abort(&op_empty[t % kGOpStages], (t / kGOpStages) & 1, abort_v, a.err);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            issue_b(t + kGOpStages);
            issued_b = t + kGOpStages + 1;
        }
        // the copies of the last stages land before the CTA may exit (bounded)
        if (lane == 0) {
            for (int t = max(0, issued_b - kGOpStages); t < issued_b; t++) {
                const long long t0 = clock64();
                while (!mbar_try_wait(&b_full[t % kGOpStages], (t / kGOpStages) & 1))
                    if (clock64() - t0 > (1ll << 31)) break;
            }
        }
        __syncwarp();
    } else if (warp == kGMmaWarp) {
        // ---------------------------------------------------------- MMA issue
        if (lane == 0) {
            constexpr uint32_t id256 = tc::idesc_f16_f32(128, 2 * RT);  // xh and xl rows
            constexpr uint32_t id128 = tc::idesc_f16_f32(128, RT);      // xh rows
            for (int t = 0; t < nst; t++) {
                const int o = t % kGOpStages;
                if (!wait_or_abort(&a_full[o], (t / kGOpStages) & 1, abort_v, a.err)) break;
                if (!wait_or_abort(&b_full[o], (t / kGOpStages) & 1, abort_v, a.err)) break;
                tc::fence_after_sync();
                const uint32_t bbase = smem_u32(op_base + o * kGOpBytes);
                const uint32_t abase = tmem + kGTmemA + (uint32_t)o * kGTmemAStage;
#pragma unroll
                for (int j = 0; j < kStageK / 16; j++) {
                    // K = 16: two 8-k core columns of B (rows: 128 xh, then 128 xl)
                    const uint64_t bhl = tc::smem_desc(bbase + (uint32_t)j * 256, kLBO, kSBO);
                    tc::mma_f16_ts(tmem, abase + 8 * j, bhl, id256, (t | j) != 0 ? 1u : 0u);
                    tc::mma_f16_ts(tmem, abase + 16 + 8 * j, bhl, id128, 1u);  // A2 * xh
                }
                tc::commit(&op_empty[o]);
            }
            tc::commit(&d_full);
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------- converters
        // Converter group cgp = warp / 4 takes stages t = cgp + kGGroups j and
        // streams their weights itself: 16-byte cp.async pieces (thread
        // (g, lane): row `lane` of column group g; lanes 0-3 also a quarter of
        // the group's scales) into its own ring of kGRawSlots slots, one
        // cp.async group per stage, issued kGRawSlots - 1 stages ahead.
        const int g = warp & 3, cgp = warp >> 2;
        const int nj = nst > cgp ? (nst - cgp + kGGroups - 1) / kGGroups : 0;
        uint8_t *raw_grp = raw_base + cgp * kGRawSlots * kGRawBytes;
        auto prefetch = [&](int j) {  // weights of the group's j-th stage (immutable)
            if (j < nj) {
                uint8_t *raw = raw_grp + (j % kGRawSlots) * kGRawBytes;
                const int64_t k0 = (int64_t)(cgp + kGGroups * j) * kStageK;
                cp_async16(raw + kGRawNib + g * kNibGroupStride + lane * 16, a.w.nib + (c0 + g) * a.w.kpad + k0 + lane);
                if (lane < 4)
                    cp_async16(raw + kGRawScl + g * kSclGroupStride + lane * 16,
                               reinterpret_cast<const uint8_t *>(a.w.scl + (c0 + g) * a.w.kpad + k0) + lane * 16);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        };
        auto group_sync = [&]() { asm volatile("bar.sync %0, 128;" ::"r"(2 + cgp) : "memory"); };
        for (int j = 0; j < kGRawSlots; j++) prefetch(j);
        griddep_launch_dependents();
        griddep_wait();
        if (threadIdx.x < RT)
            rexp_s[threadIdx.x] = (int)threadIdx.x < nvalid ? __ldcg(a.rexp + r_begin + threadIdx.x) : 0;
        // A role: column 32 g + lane of the tile, as in k_gemv_mma
        const int cq = lane & 7;
        const uint32_t sel = (uint32_t)(cq >> 1) | ((uint32_t)(4 + (cq >> 1)) << 8);
        const uint32_t nmask = (cq & 1) ? 0x00F000F0u : 0x000F000Fu;
        const __half2 m1 = __float2half2_rn((cq & 1) ? 0.0625f : 1.0f);
        const __half2 c1 = __float2half2_rn((cq & 1) ? -72.0f : -1032.0f);
        const int E = a.w.mma_exp;
        const __half2 pw = __float2half2_rn(__int_as_float((127 + E) << 23));
        const uint32_t a_lane = tmem + ((uint32_t)(32 * g) << 16) + kGTmemA;

        for (int j = 0; j < nj; j++) {
            const int t = cgp + kGGroups * j, o = t % kGOpStages;
            // one thread waits until tensor-memory stage o is free (the MMAs of
            // stage t - kGOpStages are done) and decides for the group, which
            // leaves the loop as a whole (its barriers stay matched)
            if (g == 0 && lane == 0) {
                bool ok = t < kGOpStages || wait_or_abort(&op_empty[o], ((t / kGOpStages) & 1) ^ 1, abort_v, a.err);
                grp_go[cgp] = ok && !*abort_v;
            }
            // this thread's pieces of stage j have landed; the group's barrier
            // makes every piece (and the decision) visible to the group
            asm volatile("cp.async.wait_group %0;" ::"n"(kGRawSlots - 1) : "memory");
            group_sync();
            if (!*reinterpret_cast<volatile int *>(&grp_go[cgp])) break;
            tc::fence_after_sync();
            const uint8_t *raw = raw_grp + (j % kGRawSlots) * kGRawBytes;
            const uint8_t *nibg = raw + kGRawNib + g * kNibGroupStride + (lane >> 3) * 4;
            uint4 sc4[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
                sc4[i] = *reinterpret_cast<const uint4 *>(raw + kGRawScl + g * kSclGroupStride + 16 * i);
            uint32_t A1[16], A2[16];
#pragma unroll
            for (int p = 0; p < 16; p++) {
                const uint32_t w0 = *reinterpret_cast<const uint32_t *>(nibg + (2 * p) * 16);
                const uint32_t w1 = *reinterpret_cast<const uint32_t *>(nibg + (2 * p + 1) * 16);
                const uint32_t sw = (p & 3) == 0 ? sc4[p >> 2].x
                                  : (p & 3) == 1 ? sc4[p >> 2].y
                                  : (p & 3) == 2 ? sc4[p >> 2].z : sc4[p >> 2].w;
                const __half2 s2 = __hmul2(u2h(sw), pw);            // exact (power of two)
                const __half2 sa = u2h(h2u(s2) & 0xFFF8FFF8u);      // top 8 significant bits
                const __half2 sb = __hsub2(s2, sa);                 // exact remainder
                const uint32_t pr = __byte_perm(w0, w1, sel);
                const __half2 q8 = __hfma2(u2h((pr & nmask) | 0x64006400u), m1, c1);
                A1[p] = h2u(__hmul2(q8, sa));
                A2[p] = h2u(__hmul2(q8, sb));
            }
            tc::st_32x32b_x16(a_lane + (uint32_t)o * kGTmemAStage, A1);
            tc::st_32x32b_x16(a_lane + (uint32_t)o * kGTmemAStage + 16, A2);
            tc::fence_before_sync();  // tensor-memory stores -> the MMA thread
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[o]);
            group_sync();        // every thread of the group is done with this slot
            prefetch(j + kGRawSlots);
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
        asm volatile("bar.sync 1, %0;" ::"n"(kGConvWarps * 32) : "memory");  // rexp_s

        // ---------------------------------------------------------- epilogue
        // warp w: column group w % 4 (its TMEM lanes), rows 32 (w / 4) .. + 31
        // (converter groups past RT / 32 have no rows)
        bool ok = wait_or_abort(&d_full, 0, abort_v, a.err);
        ok = __all_sync(0xffffffffu, ok);
        tc::fence_after_sync();
        const float unscale = __int_as_float((127 - E) << 23);
        const int64_t n_out = (EM == E_SWIGLU) ? (a.w.C / 2) * 32 : a.w.n;
        float *xch = reinterpret_cast<float *>(op_base);  // SwiGLU: [group][row][column]
#pragma unroll 1
        for (int ch = cgp; ch < RT / 32; ch += kGGroups) {
            const int n0 = 32 * ch;
            float vh[32], vl[32];
            if (ok) {
                tc::ld_32x32b_x32(tmem + ((uint32_t)(32 * g) << 16) + (uint32_t)n0, vh);
                tc::ld_32x32b_x32(tmem + ((uint32_t)(32 * g) << 16) + (uint32_t)(RT + n0), vl);
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) vh[i] = vl[i] = 0.0f;
            }
#pragma unroll
            for (int n = 0; n < 32; n++)
                vh[n] = __fmul_rn(__fmul_rn(__fadd_rn(vh[n], vl[n]), unscale),
                                  __int_as_float((127 - rexp_s[n0 + n]) << 23));
            if constexpr (EM == E_SWIGLU) {
#pragma unroll
                for (int n = 0; n < 32; n++) xch[(g * RT + n0 + n) * 32 + lane] = vh[n];
            } else {
                const int64_t grp = c0 + g;
#pragma unroll 4
                for (int n = 0; n < 32; n++) {
                    const int row = n0 + n;
                    if (row < nvalid) {
                        if constexpr (EM == E_RESID) {
                            // x[j] += attn_out / mlp (talker.rs:334-336, 347-349)
                            const float yr = __ldcg(a.y + (int64_t)(r_begin + row) * a.ldy + grp * 32 + lane);
                            finalize_resid(a, r_begin + row, grp, lane, __fadd_rn(yr, vh[n]));
                        } else {
                            finalize_group<EM>(a, r_begin + row, grp, lane, vh[n], 0.0f, n_out, CO);
                        }
                    }
                }
            }
        }
        if constexpr (EM == E_SWIGLU) {
            // silu(gate) * up (talker.rs:341-345): group 2u is gate, 2u + 1 up
            asm volatile("bar.sync 1, %0;" ::"n"(kGConvWarps * 32) : "memory");
            constexpr int RW = 2 * RT / kGConvWarps;  // rows per warp (two units)
            const int u = warp & 1, rb = (warp >> 1) * RW;
            for (int n = 0; n < RW; n++) {
                const int row = rb + n;
                if (row < nvalid)
                    finalize_group<EM>(a, r_begin + row, c0 / 2 + u, lane, xch[((2 * u) * RT + row) * 32 + lane],
                                       xch[((2 * u + 1) * RT + row) * 32 + lane], n_out, CO);
            }
        }
        // tail columns beyond the last full group stay zero (gemv.rs:846-861)
        if (EM == E_STORE && a.w.n > a.w.C * 32 && blockIdx.x == 0) {
            for (int rr = 0; rr < nvalid; rr++)
                for (int64_t col = a.w.C * 32 + threadIdx.x; col < a.w.n; col += kGConvWarps * 32)
                    a.y[(int64_t)(r_begin + rr) * a.ldy + col] = 0.0f;
        }
    }
    tc::fence_before_sync();
    __syncthreads();  // tensor memory read back
    if (warp == kGMmaWarp) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kGTmemCols);
    }
}

template <int XM, int EM>
int gemm_attrs() {
    QORA_CUDA(cudaFuncSetAttribute(k_gemm_mma<XM, EM, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)gsmem(128)));
    QORA_CUDA(cudaFuncSetAttribute(k_gemm_mma<XM, EM, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)gsmem(64)));
    return QORA_OK;
}

template <int XM, int RT>
int launch_gemm_e(const GemvArgs &a, int emode, dim3 grid, cudaStream_t st) {
    const dim3 block(kGThreads);
    switch (emode) {
        case E_STORE: return launch_ex(k_gemm_mma<XM, E_STORE, RT>, grid, block, gsmem(RT), st, 1u, a);
        case E_BIAS: return launch_ex(k_gemm_mma<XM, E_BIAS, RT>, grid, block, gsmem(RT), st, 1u, a);
        case E_RESID: return launch_ex(k_gemm_mma<XM, E_RESID, RT>, grid, block, gsmem(RT), st, 1u, a);
        case E_SWIGLU: return launch_ex(k_gemm_mma<XM, E_SWIGLU, RT>, grid, block, gsmem(RT), st, 1u, a);
    }
    return set_error(QORA_ERR_INVALID, "bad epilogue mode %d", emode);
}

// Row prologue, B tiles and GEMM of one prefill GEMM with RT-row tiles.
template <int XM, int RT>
int launch_gemm_rt(const GemvArgs &a, int emode, const GemmScratch &sc, cudaStream_t st) {
    const int rt = (a.rows + RT - 1) / RT, nst = (int)(a.w.k / kStageK);
    const dim3 grid((unsigned)(a.w.C / kMmaGroups), (unsigned)rt);
    const dim3 cgrid((unsigned)rt, (unsigned)((nst + 3) / 4));
    QORA_TRY(launch_ex(k_row_prep<XM>, dim3((unsigned)a.rows), dim3(256), 0, st, 1u, a, sc.rexp, sc.rinv));
    QORA_TRY(launch_ex(k_b_convert<XM, RT>, cgrid, dim3(256), 0, st, 1u, a, (const int *)sc.rexp,
                       (const float *)sc.rinv, sc.bop));
    return launch_gemm_e<XM, RT>(a, emode, grid, st);
}

template <int XM, int EM>
int mma_attrs() {
    QORA_CUDA(cudaFuncSetAttribute(k_gemv_mma<XM, EM>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    QORA_CUDA(cudaFuncSetAttribute(k_gemv_mma<XM, EM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kMmaSmem));
    // two CTAs per SM need the shared-memory carveout at its maximum
    QORA_CUDA(cudaFuncSetAttribute(k_gemv_mma<XM, EM>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                   (int)cudaSharedmemCarveoutMaxShared));
    return QORA_OK;
}

template <int XM>
int mma_attrs_e() {
    QORA_TRY((mma_attrs<XM, E_STORE>()));
    QORA_TRY((mma_attrs<XM, E_BIAS>()));
    QORA_TRY((mma_attrs<XM, E_RESID>()));
    return mma_attrs<XM, E_SWIGLU>();
}

template <int XM>
int launch_mma_e(const GemvArgs &a, int emode, const GemvPlan &p, cudaStream_t st) {
    switch (emode) {
        case E_STORE: return launch_ex(k_gemv_mma<XM, E_STORE>, p.grid, p.block, kMmaSmem, st, (unsigned)p.S, a);
        case E_BIAS: return launch_ex(k_gemv_mma<XM, E_BIAS>, p.grid, p.block, kMmaSmem, st, (unsigned)p.S, a);
        case E_RESID: return launch_ex(k_gemv_mma<XM, E_RESID>, p.grid, p.block, kMmaSmem, st, (unsigned)p.S, a);
        case E_SWIGLU: return launch_ex(k_gemv_mma<XM, E_SWIGLU>, p.grid, p.block, kMmaSmem, st, (unsigned)p.S, a);
    }
    return set_error(QORA_ERR_INVALID, "bad epilogue mode %d", emode);
}

bool mma_disabled_by_env() {
    static const bool off = [] {
        const char *v = getenv("QORA_MMA");
        return v && v[0] == '0';
    }();
    return off;
}

// Clusters of S CTAs (S = 1..16) that can be resident at once, per device:
// a grid with more clusters than this runs in waves.
constexpr int kMaxDevices = 64;
int g_max_clusters[kMaxDevices][kMaxSplit + 1];

// cudaOccupancyMaxActiveClusters counts one CTA of this kernel per SM.  Two
// fit when each SM sub-partition can hold the registers of the warps two CTAs
// place on it (the 10 warps of a CTA go 3/3/2/2 over the four 16K-register
// sub-partitions: 6 warps at most), and then twice as many clusters are
// resident (measured on 148 SMs: 14 clusters of 16 CTAs where the query
// reports 7).  Only a performance bound: more clusters than this run in waves.
int query_max_clusters(int dev) {
    cudaFuncAttributes fa;
    QORA_CUDA(cudaFuncGetAttributes(&fa, k_gemv_mma<X_RMSNORM, E_SWIGLU>));
    const int regs_warp = ((fa.numRegs + 7) / 8) * 8 * 32;
    const int warps_smsp = 2 * ((kMmaThreads / 32 + 3) / 4);
    const int per_sm = (warps_smsp * regs_warp <= 16384) ? 2 : 1;
    for (int S = 1; S <= kMaxSplit; S++) {
        g_max_clusters[dev][S] = 0;
        if (!split_ok(S)) continue;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(64, (unsigned)S, 1);
        cfg.blockDim = dim3(kMmaThreads);
        cfg.dynamicSmemBytes = kMmaSmem;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = 1;
        attr.val.clusterDim.y = (unsigned)S;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        QORA_CUDA(cudaOccupancyMaxActiveClusters(&n, k_gemv_mma<X_RMSNORM, E_SWIGLU>, &cfg));
        g_max_clusters[dev][S] = n * per_sm;
    }
    return QORA_OK;
}

}  // namespace

int gemv_mma_init() {
    QORA_TRY((gemm_attrs<X_PLAIN, E_STORE>()));
    QORA_TRY((gemm_attrs<X_PLAIN, E_BIAS>()));
    QORA_TRY((gemm_attrs<X_PLAIN, E_RESID>()));
    QORA_TRY((gemm_attrs<X_PLAIN, E_SWIGLU>()));
    QORA_TRY((gemm_attrs<X_RMSNORM, E_STORE>()));
    QORA_TRY((gemm_attrs<X_RMSNORM, E_BIAS>()));
    QORA_TRY((gemm_attrs<X_RMSNORM, E_RESID>()));
    QORA_TRY((gemm_attrs<X_RMSNORM, E_SWIGLU>()));
    QORA_TRY(mma_attrs_e<X_PLAIN>());
    QORA_TRY(mma_attrs_e<X_RMSNORM>());
    QORA_TRY(mma_attrs_e<X_EMBED>());
    int dev = 0;
    QORA_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return set_error(QORA_ERR_UNSUPPORTED, "device id %d", dev);
    return query_max_clusters(dev);
}

bool gemv_mma_eligible(const GemvArgs &a, int xmode, int emode) {
    return a.rows >= kMmaMinRows && gemv_mma_supported(a, xmode, emode);
}

bool gemv_mma_supported(const GemvArgs &a, int xmode, int emode) {
    if (mma_disabled_by_env()) return false;
    if (xmode != X_PLAIN && xmode != X_RMSNORM && xmode != X_EMBED) return false;
    if (emode < E_STORE || emode > E_SWIGLU) return false;
    if (a.w.mma_exp < 0 || a.w.k % kStageK != 0 || a.w.C % kMmaGroups != 0) return false;
    if (xmode == X_EMBED) {
        // nibble rows and scale rows must be whole 16-byte blocks
        if (a.emb.n != a.w.k || a.emb.n % 256 != 0 || ((uintptr_t)a.emb.packed & 15) != 0 ||
            ((uintptr_t)a.emb.scl & 15) != 0 || !a.tok)
            return false;
    } else if (a.ldx % 4 != 0 || ((uintptr_t)a.x & 15) != 0) {
        return false;
    }
    if (xmode == X_RMSNORM && ((uintptr_t)a.gamma & 15) != 0) return false;
    return true;
}

GemvPlan plan_gemv_mma(int64_t k, int64_t C, int rows, int emode, int num_sms) {
    GemvPlan p{};
    p.mma = true;
    p.cpc = kMmaGroups;
    p.B = kMmaRows;
    p.rows_per_z = kMmaRows;
    p.Z = (rows + kMmaRows - 1) / kMmaRows;
    const int64_t tiles = C / kMmaGroups;
    const int64_t stages = k / kStageK;
    // about two CTAs per SM: K-split CTAs (one cluster) fill what the column
    // and row tiles leave
    const int64_t want = (2LL * num_sms) / std::max<int64_t>(1, tiles * p.Z);
    int dev = 0;
    cudaGetDevice(&dev);
    const int *maxc = (dev >= 0 && dev < kMaxDevices) ? g_max_clusters[dev] : nullptr;
    // the largest split up to `want` whose clusters all stay resident at once
    int64_t S = 1;
    for (int s = 2; s <= std::min<int64_t>(std::min<int64_t>(want, kMaxSplit), stages); s++)
        if (split_ok(s) && (!maxc || maxc[s] <= 0 || tiles * p.Z <= maxc[s])) S = s;
    p.S = (int)S;
    p.WR = kConvWarps;
    p.NSUB = 1;
    p.rows_per_cta_k = (int)((stages + S - 1) / S * kStageK);
    p.grid = dim3((unsigned)tiles, (unsigned)p.S, (unsigned)p.Z);
    p.block = dim3(kMmaThreads);
    (void)emode;
    return p;
}

// QORA_PREFILL_GEMM=0 in the environment sends prefill GEMMs back to
// k_gemv_mma (the same bits, for comparison).
bool prefill_gemm_disabled_by_env() {
    static const bool off = [] {
        const char *v = getenv("QORA_PREFILL_GEMM");
        return v && v[0] == '0';
    }();
    return off;
}

bool gemm_mma_supported(const GemvArgs &a, int xmode, int emode) {
    if (prefill_gemm_disabled_by_env()) return false;
    if (xmode != X_PLAIN && xmode != X_RMSNORM) return false;
    if (!gemv_mma_supported(a, xmode, emode)) return false;
    // no normalised side copy and no global stage (argmax, cache advance)
    if (a.side || a.tbest_v || a.amax || a.adv_len) return false;
    return a.rows >= 1 && a.rows <= kMaxRows;
}

int launch_gemm_mma(GemvArgs a, int xmode, int emode, const GemmScratch &sc, cudaStream_t st, int *launches) {
    if (!gemm_mma_supported(a, xmode, emode))
        return set_error(QORA_ERR_INVALID, "prefill GEMM: unsupported launch");
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // 64-row tiles when 128-row tiles would fill under three quarters of the SMs
    const int64_t tiles128 = (a.w.C / kMmaGroups) * ((a.rows + 127) / 128);
    const int RT = (a.rows <= 64 || tiles128 * 4 < 3LL * sms) ? 64 : 128;
    const int nst = (int)(a.w.k / kStageK);
    const size_t need = (size_t)((a.rows + RT - 1) / RT) * nst * gopbytes(RT);
    if (!sc.rexp || !sc.rinv || !sc.bop || a.rows > sc.rows || need > sc.bop_bytes)
        return set_error(QORA_ERR_INVALID, "prefill GEMM: scratch too small (%d rows, k %lld)", a.rows,
                         (long long)a.w.k);
    a.S = 1;
    a.gticket = nullptr;
    a.rexp = sc.rexp;
    a.bop = sc.bop;
    if (xmode == X_PLAIN) {
        QORA_TRY(RT == 64 ? (launch_gemm_rt<X_PLAIN, 64>(a, emode, sc, st)) : (launch_gemm_rt<X_PLAIN, 128>(a, emode, sc, st)));
    } else {
        QORA_TRY(RT == 64 ? (launch_gemm_rt<X_RMSNORM, 64>(a, emode, sc, st))
                          : (launch_gemm_rt<X_RMSNORM, 128>(a, emode, sc, st)));
    }
    if (launches) *launches += 3;
    return QORA_OK;
}

int launch_gemv_mma(const GemvArgs &a, int xmode, int emode, const GemvPlan &p, cudaStream_t st) {
    switch (xmode) {
        case X_PLAIN: return launch_mma_e<X_PLAIN>(a, emode, p, st);
        case X_RMSNORM: return launch_mma_e<X_RMSNORM>(a, emode, p, st);
        case X_EMBED: return launch_mma_e<X_EMBED>(a, emode, p, st);
    }
    return set_error(QORA_ERR_INVALID, "tensor-core GEMV: prologue mode %d unsupported", xmode);
}

}  // namespace qora
