// Device helpers shared by the Q4 GEMV kernels (CUDA-core k_gemv and the
// tensor-core k_gemv_mma): input prologue, output epilogue and the K-split /
// global final stage.
#pragma once

#include <cooperative_groups.h>

#include "gemv.cuh"

namespace qora {
namespace gemv_detail {

namespace cg = cooperative_groups;
// Input element x[r][kr] before the RMSNorm scaling (applied by the caller).
template <int XM>
__device__ __forceinline__ float load_x(const GemvArgs &a, int r, int64_t kr) {
    if constexpr (XM == X_PLAIN || XM == X_RMSNORM) {
        return __ldcg(a.x + (int64_t)r * a.ldx + kr);
    } else {
        // embed_lookup_q4 (gemv.rs:425-433): scale * (q - 8)
        const uint32_t t = __ldcg(a.tok + (int64_t)r * a.ldtok);
        const uint8_t byte = a.emb.packed[(int64_t)t * (a.emb.n >> 1) + (kr >> 1)];
        const int q = (kr & 1) ? (byte >> 4) : (byte & 15);
        const float sc = __half2float(a.emb.scl[(int64_t)t * (a.emb.n >> 5) + (kr >> 5)]);
        return __fmul_rn(sc, (float)(q - 8));
    }
}

// Epilogue value for one (row, column) result.
template <int EM>
__device__ __forceinline__ float epilogue_value(const GemvArgs &a, int r, int64_t col, float v) {
    if constexpr (EM == E_BIAS) return __fadd_rn(v, a.bias[col]);
    if constexpr (EM == E_RESID) return __fadd_rn(__ldcg(a.y + (int64_t)r * a.ldy + col), v);
    return v;
}

// Stores a finished residual-stream value and its sum-of-squares partial.
__device__ __forceinline__ void finalize_resid(const GemvArgs &a, int r, int64_t out_group, int lane,
                                               float y) {
    a.y[(int64_t)r * a.ldy + out_group * 32 + lane] = y;
    if (a.ss_out) {
        const float sq = warp_sum(__fmul_rn(y, y));
        if (lane == 0) a.ss_out[(int64_t)r * a.ldss_out + out_group] = sq;
    }
}

// Writes the final values for one warp-group (32 columns of one row).
// For E_SWIGLU, v is the gate sum and u the up sum (silu(gate) * up, talker.rs:344).
// n_tile_groups: output groups per CTA (the per-group argmax table has
// gridDim.x * n_tile_groups entries per row).
template <int EM>
__device__ __forceinline__ void finalize_group(const GemvArgs &a, int r, int64_t out_group,
                                               int lane, float v, float u, int64_t n_out,
                                               int n_tile_groups) {
    const int64_t col = out_group * 32 + lane;
    float y;
    if constexpr (EM == E_SWIGLU) {
        y = __fmul_rn(silu_ref(v), u);
    } else {
        y = epilogue_value<EM>(a, r, col, v);
    }
    if (col < n_out) a.y[(int64_t)r * a.ldy + col] = y;
    if (a.ss_out) {
        const float sq = warp_sum(__fmul_rn(y, y));
        if (lane == 0) a.ss_out[(int64_t)r * a.ldss_out + out_group] = sq;
    }
    if (a.tbest_v) {
        // per-tile argmax, last index on ties (code_predictor.rs:336-339)
        float bv = y;
        int bi = (int)col;
        if (y != y) raise_error(a.err, kDevNaN);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi > bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {  // one entry per output group: [rows][groups]
            const int64_t ng = (int64_t)gridDim.x * n_tile_groups;
            a.tbest_v[(int64_t)r * ng + out_group] = bv;
            a.tbest_i[(int64_t)r * ng + out_group] = bi;
        }
    }
}

// Bulk L2 prefetch of CTA `id`'s share (16-byte aligned pieces) of [p, p+bytes).
__device__ __forceinline__ void l2_prefetch_share(const void *p, uint64_t bytes, uint64_t id,
                                                  uint64_t nctas) {
    if (!p || bytes == 0) return;
    const uint64_t per = ((bytes + nctas - 1) / nctas + 15) & ~15ull;
    uint64_t off = id * per;
    if (off >= bytes) return;
    uint64_t len = per < bytes - off ? per : bytes - off;
    const char *base = static_cast<const char *>(p) + off;
    while (len >= 16) {
        const uint64_t whole = len & ~15ull;
        const uint32_t piece = (uint32_t)(whole < (1ull << 20) ? whole : (1ull << 20));
        prefetch_l2_bulk(base, piece);
        base += piece;
        len -= piece;
    }
}

// The global stage of a GEMV grid: every CTA takes a ticket; the last one
// (all other CTAs' outputs visible) runs the argmax over the per-group maxima
// and the cache-length advance.  `n_groups` = output groups (argmax table width).
__device__ __forceinline__ void gemv_global_stage(const GemvArgs &a, int &last_flag, unsigned n_groups) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (!a.gticket) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned t = atomicAdd(a.gticket, 1u);
        last_flag = (t == (unsigned)(gridDim.x * gridDim.y * gridDim.z - 1));
    }
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    if (a.amax) {
        // argmax over the column groups, one warp per row: lanes take groups
        // lane, lane+32, ...; ties keep the larger index (the last maximum,
        // code_predictor.rs:336-339)
        const int nwarps = blockDim.x >> 5;
        for (int r = warp; r < a.rows; r += nwarps) {
            float bv = -INFINITY;
            int bi = -1;
            for (unsigned t = lane; t < n_groups; t += 32) {
                const float v = __ldcg(a.tbest_v + (int64_t)r * n_groups + t);
                const int i = __ldcg(a.tbest_i + (int64_t)r * n_groups + t);
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
            if (lane == 0) a.amax[(int64_t)r * a.ldamax] = (uint32_t)bi;
        }
    }
    if (a.adv_len) {
        for (int st = threadIdx.x; st < a.adv_streams; st += blockDim.x) {
            a.adv_len[st] += a.adv_T;
            if (a.adv_pos) a.adv_pos[st] += a.adv_T;
        }
    }
    if (threadIdx.x == 0) *a.gticket = 0u;
}

// The end of a k_gemv CTA.  cta_red holds this
// CTA's partial sums for rows r_begin..r_end-1 (RPZ rows), CPC column groups.
// The S K-split CTAs of one cluster share the finishing work: rank q takes a
// 1/S slice of the (row, 32-column group) blocks, sums the S partials of each
// output over distributed shared memory in rank order (eight loads in flight
// at a time), and applies the epilogue (store / bias / residual + sum of squares
// / SwiGLU, per-group argmax).  The last CTA of the grid to finish runs the
// global stage (argmax over groups, cache-length advance).
template <int EM, int CPC, int RPZ>
__device__ __forceinline__ void gemv_final(const GemvArgs &a, float (&cta_red)[RPZ][CPC][32], int r_begin,
                                           int r_end, int &last_flag) {
    const int64_t C = a.w.C;
    const int64_t n32 = C * 32;
    const int64_t n_out = (EM == E_SWIGLU) ? (C / 2) * 32 : a.w.n;
    cg::cluster_group cluster = cg::this_cluster();
    const int S = a.S;
    const int rank = (S == 1) ? 0 : (int)cluster.block_rank();
    // output column groups per CTA; SwiGLU pairs (gate, up) sit at groups
    // (2i, 2i+1) of the tile
    constexpr int CO = (EM == E_SWIGLU) ? CPC / 2 : CPC;
    constexpr int kPre = 4;  // residual values prefetched per thread
    const int nblk = (r_end - r_begin) * CO;
    const int per = (nblk + S - 1) / S;
    const int it_begin = min(nblk, rank * per) * 32;
    const int it_end = min(nblk, (rank + 1) * per) * 32;
    float yres[kPre];
    if constexpr (EM == E_RESID) {
        // the residual does not depend on the K-split partials: load it while
        // the cluster barrier completes
#pragma unroll
        for (int m = 0; m < kPre; m++) {
            const int it = it_begin + threadIdx.x + m * blockDim.x;
            if (it < it_end) {
                const int l = it & 31, q = it >> 5;
                const int64_t col = ((int64_t)blockIdx.x * CPC + q % CO) * 32 + l;
                yres[m] = __ldcg(a.y + (int64_t)(r_begin + q / CO) * a.ldy + col);
            }
        }
    }
    if (S > 1) cluster.sync();
    auto finish = [&](int it, float yr, bool have_yr) {
        const int l = it & 31;
        const int q = it >> 5;
        const int row = q / CO, cc2 = q % CO;
        const int off = (row * CPC + ((EM == E_SWIGLU) ? 2 * cc2 : cc2)) * 32 + l;
        // rank-order sum; peer loads issued eight at a time
        float v = 0.0f, u = 0.0f;
        for (int r8 = 0; r8 < S; r8 += 8) {
            float pv[8], pu[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (r8 + j < S) {
                    const float *p = (S == 1) ? &cta_red[0][0][0]
                                              : cluster.map_shared_rank(&cta_red[0][0][0], r8 + j);
                    pv[j] = p[off];
                    if constexpr (EM == E_SWIGLU) pu[j] = p[off + 32];
                }
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (r8 + j < S) {
                    v += pv[j];
                    if constexpr (EM == E_SWIGLU) u += pu[j];
                }
            }
        }
        const int64_t grp = (int64_t)blockIdx.x * CO + cc2;
        if constexpr (EM == E_RESID) {
            // x[j] += attn_out[j] (talker.rs:334-336)
            if (!have_yr) yr = __ldcg(a.y + (int64_t)(r_begin + row) * a.ldy + grp * 32 + l);
            finalize_resid(a, r_begin + row, grp, l, __fadd_rn(yr, v));
        } else {
            finalize_group<EM>(a, r_begin + row, grp, l, v, u, n_out, CO);
        }
    };
    // items come in whole 32-column blocks per warp (epilogue warp sums)
#pragma unroll
    for (int m = 0; m < kPre; m++) {
        const int it = it_begin + threadIdx.x + m * blockDim.x;
        if (it < it_end) finish(it, (EM == E_RESID) ? yres[m] : 0.0f, true);
    }
    for (int it = it_begin + threadIdx.x + kPre * blockDim.x; it < it_end; it += blockDim.x)
        finish(it, 0.0f, false);
    // tail columns beyond the last full group stay zero (gemv.rs:846-861)
    if (EM == E_STORE && a.w.n > n32 && blockIdx.x == 0 && rank == 0) {
        for (int r = r_begin; r < r_end; r++)
            for (int64_t col = n32 + threadIdx.x; col < a.w.n; col += blockDim.x)
                a.y[(int64_t)r * a.ldy + col] = 0.0f;
    }
    if (S > 1) cluster.sync();  // peers keep their shared memory until every rank is done

    gemv_global_stage(a, last_flag, gridDim.x * CO);
}

}  // namespace gemv_detail
}  // namespace qora
