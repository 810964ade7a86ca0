// Q4 GEMV engine: kernel arguments, launch planning and launchers.
#pragma once

#include "common.cuh"

namespace qora {

enum XMode : int { X_PLAIN = 0, X_RMSNORM = 1, X_EMBED = 2 };
enum EMode : int { E_STORE = 0, E_BIAS = 1, E_RESID = 2, E_SWIGLU = 3 };

// One fused GEMV launch:  y[r] = epilogue( prologue(x[r]) @ W )  for rows r.
struct GemvArgs {
    Q4Dev w;
    int rows = 0;
    // ---- input prologue
    const float *x = nullptr;
    int64_t ldx = 0;
    const __half *gamma = nullptr;  // X_RMSNORM: f16 gamma[k]
    const float *ss = nullptr;      // X_RMSNORM: per-row sum-of-squares partials
    int64_t ldss = 0;
    int ss_tiles = 0;
    EmbDev emb;                     // X_EMBED: x[r] = dequantised emb row tok[r*ldtok]
    const uint32_t *tok = nullptr;
    int64_t ldtok = 1;
    float *side = nullptr;          // X_RMSNORM: also write the normalised rows here
    int64_t ldside = 0;
    // ---- output epilogue
    float *y = nullptr;
    int64_t ldy = 0;
    const float *bias = nullptr;    // E_BIAS
    float *ss_out = nullptr;        // per-row, per-32-column sum of squares of y
    int64_t ldss_out = 0;
    // ---- global final stage (one CTA after all column tiles are done)
    float *tbest_v = nullptr;       // [rows][tiles] per-tile max (argmax)
    int *tbest_i = nullptr;
    uint32_t *amax = nullptr;       // argmax output per row (last index on ties)
    int64_t ldamax = 1;
    int *adv_len = nullptr;         // len[s] += adv_T for s < adv_streams
    int *adv_pos = nullptr;         // pos[s] += adv_T
    int adv_T = 0, adv_streams = 0;
    int *err = nullptr;
    // ---- L2 prefetch of the weights the next kernel will stream (issued
    // before griddepcontrol.wait; spread over the grid's CTAs)
    const void *pf0 = nullptr, *pf1 = nullptr;
    uint64_t pf0_bytes = 0, pf1_bytes = 0;
    const int *rexp = nullptr;      // prefill GEMM: per-row operand exponent
    const uint8_t *bop = nullptr;   // prefill GEMM: B tiles (k_b_convert)
    // ---- filled by plan_gemv
    int B = 1, WR = 1, S = 1, Z = 1, NSUB = 1;
    int rows_per_cta_k = 128, rows_per_z = 0;
    unsigned *gticket = nullptr;    // [1] arrival counter of the global final stage
};

constexpr int kRowsPerZ = 16;       // rows one CTA carries through the K loop
constexpr int kMaxSplit = 16;       // CTAs of one cluster along K

// Tiling of one GEMV: column groups x K-splits (one cluster) x row groups.
struct GemvPlan {
    int B, WR, S, Z, NSUB, rows_per_cta_k, rows_per_z, cpc;
    bool mma;                       // k_gemv_mma (tensor cores, batches of kMmaMinRows rows or more)
    dim3 grid, block;
};

constexpr int kMmaMinRows = 8;      // from this many rows on, the tensor-core kernel serves batches

// Point a GEMV's L2 prefetch at the weights of the GEMV that follows it.
inline void prefetch_next(GemvArgs &a, const Q4Dev &next) {
    a.pf0 = next.nib;
    a.pf0_bytes = (uint64_t)next.C * next.kpad * 16;
    a.pf1 = next.scl;
    a.pf1_bytes = (uint64_t)next.C * next.kpad * 2;
}

// Per-device one-time kernel attribute setup (large clusters).
int gemv_init();

// Chooses tiling so that at least ~2 CTAs per SM are launched (CUDA-core kernel).
GemvPlan plan_gemv(int64_t k, int64_t C, int rows, int emode, int num_sms);

// Tensor-core kernel (gemv_mma.cu): whether a launch qualifies (rows >=
// kMmaMinRows, plain or RMSNorm input, aligned rows, k % 32 == 0, C % 4 == 0,
// weight scales within the f16 operand range), its tiling, its launcher.
int gemv_mma_init();
bool gemv_mma_eligible(const GemvArgs &a, int xmode, int emode);
// The same conditions apart from the row count (any 1..kMaxRows rows run correctly).
bool gemv_mma_supported(const GemvArgs &a, int xmode, int emode);
GemvPlan plan_gemv_mma(int64_t k, int64_t C, int rows, int emode, int num_sms);
int launch_gemv_mma(const GemvArgs &a, int xmode, int emode, const GemvPlan &p, cudaStream_t st);
// Scratch of the prefill GEMM: per-row exponent and RMSNorm factor (`rows`
// entries) and the B tiles (rows rounded up to 128, times k, times 4 bytes).
struct GemmScratch {
    int *rexp = nullptr;
    float *rinv = nullptr;
    uint8_t *bop = nullptr;
    int rows = 0;
    size_t bop_bytes = 0;
};
// Prefill GEMM (tensor cores, 128-column x 128-row tiles over all of K, any
// row count up to kMaxRows): the bits of k_gemv_mma without a K split.
// Three kernels (row prologue, B tiles, GEMM); *launches is increased by 3.
bool gemm_mma_supported(const GemvArgs &a, int xmode, int emode);
int launch_gemm_mma(GemvArgs a, int xmode, int emode, const GemmScratch &sc, cudaStream_t st, int *launches);

// The plan for one launch: the tensor-core kernel where it qualifies, else
// the CUDA-core kernel.
GemvPlan plan_gemv_for(const GemvArgs &a, int xmode, int emode, int num_sms);

// Launches the fused GEMV; `gticket` backs the global final stage (argmax /
// length advance) when `a` asks for one.
int launch_gemv(GemvArgs a, int xmode, int emode, const GemvPlan &plan, unsigned *gticket,
                cudaStream_t stream);

// Repack reference-layout Q4 rows (device copy) into column-group-major
// chunks at destination chunk index dst_off + c * dst_stride.
int repack_q4(const uint8_t *src_packed, const __half *src_scl, int64_t k, int64_t n,
              uint4 *dst_nib, __half *dst_scl, int64_t dst_k_stride, int64_t dst_off,
              int64_t dst_stride, cudaStream_t stream);

// A token outside the table gives a zero row and raises kDevRange on `err`.
int launch_embed_rows(const EmbDev &e, const uint32_t *tok, int64_t ldtok, int count, float *out,
                      int64_t ldout, int *err, cudaStream_t stream);

// Copy rows and write their per-32-column sum-of-squares partials.
int launch_copy_rowstats(const float *src, int64_t ldsrc, float *dst, int64_t lddst, int rows,
                         int n, float *ss, int64_t ldss, cudaStream_t stream);

int launch_rmsnorm_rows(const float *x, const __half *gamma, int64_t n, int rows, float *out,
                        cudaStream_t stream);

// Host-side helpers shared by the model code.
int upload_q4_parts(const qora_q4_host *parts, const int64_t *offs, const int64_t *strides,
                    int nparts, int64_t k, int64_t C_total, DevBuf &nib, DevBuf &scl,
                    Q4Dev &out, cudaStream_t stream);
int upload_emb(const qora_q4_host &h, DevBuf &packed, DevBuf &scl, EmbDev &out);

}  // namespace qora
