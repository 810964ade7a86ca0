// Persistent frame kernel: one launch runs a whole frame of the reference's
// per-frame loop (generate_new.rs:606-665) for one stream as a fixed program
// of ops, each op a slice of work for every SM.  See frame.cu.
#pragma once

#include "attention.cuh"
#include "model.cuh"
#include "sampler.cuh"

namespace qora {
namespace fk {

constexpr int kNT = 256;               // consumer threads (8 warps)
constexpr int kThreads = kNT + 32;     // + one producer warp
constexpr int kSlots = 9;              // weight ring slots per SM
constexpr int kSlotNib = 16384;        // nibble bytes per slot (1024 rows of one group)
constexpr int kSlotScl = 2048;         // scale bytes per slot
constexpr int kXMax = 6144;            // widest GEMV input (talker down projection)
constexpr int kTraceFields = 8;

enum OpType : int { OP_GEMV = 0, OP_ATTN = 1, OP_SAMPLE = 2 };
enum InMode : int {
    IN_VEC = 0,     // x = in[0..K)  (RMSNorm from the producer's sum-of-squares partials)
    IN_EMB = 1,     // x = dequantised embedding row of a code (argmax of logits or a stored code)
    IN_FRAME = 2,   // x = (E_talker[c0] + sum_g E_g[c_{g+1}]) + text  (talker layer-0 input)
};
enum OutMode : int {
    OUT_STORE = 0,  // y (+ bias)
    OUT_RESID = 1,  // y + resid  (residual stream)
    OUT_SWIGLU = 2, // silu(gate) * up of the unit's two groups (talker.rs:341-345)
};

// One GEMV op: y = epilogue(prologue(x) @ W) over `units` column units of G
// 32-column groups each; item j = unit j covers all K rows, so every output
// is final when its item ends.
struct alignas(16) GemvDesc {
    const uint4 *nib = nullptr;
    const __half *scl = nullptr;
    int kpad = 0, K = 0, units = 0, G = 1;
    // input
    int in_mode = IN_VEC;
    const float *in = nullptr;
    const __half *gamma = nullptr;       // RMSNorm prologue (rms_norm_f16, gemv.rs:445-454)
    const float *ss_in = nullptr;        // IN_VEC + gamma: per-32-column sums of squares of `in`
    float *save = nullptr;               // materialise x (before, or after the norm)
    int save_normed = 0;
    const float *amax_src = nullptr;     // IN_EMB / IN_FRAME: logits for the argmax
    int amax_n = 0;
    uint32_t *code_dst = nullptr;        // where the argmax code is stored
    const uint32_t *code_src = nullptr;  // IN_EMB without amax_src: the code to look up
    EmbDev emb;                          // IN_EMB table
    // output
    int out_mode = OUT_STORE;
    float *out = nullptr;
    const float *resid = nullptr;        // OUT_RESID
    const float *bias = nullptr;         // optional, OUT_STORE
    float *ss_out = nullptr;             // per-32-column sums of squares of the output
    int *adv_len = nullptr;              // end of frame: len[0] += 1, pos[0] += 1
    int *adv_pos = nullptr;
};

// Talker frame-input assembly (generate_new.rs:639-654, code_predictor.rs:287-300).
struct FrameEmbed {
    EmbDev talker;                       // E_talker (semantic row of code 0)
    EmbDev pred[kMaxEmbedGroups];        // acoustic tables
    int ngroups = 0;
    int64_t n = 0;
    uint32_t *codes = nullptr;           // [16]: code 0 .. code ngroups
    uint32_t *prev = nullptr;            // [16]: previous-code window (repetition penalty)
};

struct OpRef {
    int type = OP_GEMV;
    int idx = 0;        // into the gemv / attn arrays
    int n_items = 0;
    int rot = 0;        // item j runs on SM (j + rot) % grid
};

struct FrameParams {
    const OpRef *ops = nullptr;
    int n_ops = 0;
    const GemvDesc *gemv = nullptr;
    const AttnArgs *attn = nullptr;
    SampleArgs sample;
    FrameEmbed fe;
    const float *text = nullptr;         // [hidden] text row of this frame
    unsigned *done = nullptr;            // [n_ops] completion counters (zeroed per launch)
    int *abort_flag = nullptr;
    int *err = nullptr;
    unsigned long long *trace = nullptr; // optional [n_ops][8] of each op's item-0 SM: globaltimer
                                         // stamps (dependency met, input built, items done,
                                         // signalled); thread 0's SM cycles waiting for weight
                                         // slots, computing, reducing; slots consumed
};

}  // namespace fk

// Host-side program of the frame kernel for one engine (B = 1).
struct FrameProgram {
    std::vector<fk::OpRef> ops;
    std::vector<fk::GemvDesc> gemv;
    std::vector<AttnArgs> attn;
    DevBuf d_ops, d_gemv, d_attn, d_done, bufs, d_trace;
    fk::FrameParams params;
    int grid = 0;
    size_t smem = 0;
    bool trace = false;
};

// Whether the engine's model fits the frame kernel (B = 1, supported dims).
bool frame_supported(const qora_engine *e);
int frame_build(qora_engine *e, FrameProgram **out);
int frame_launch(FrameProgram *p, const float *text, cudaStream_t st);

}  // namespace qora
