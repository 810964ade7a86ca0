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
// Weight ring slots per SM.  Four keep every slot filled before its op's
// input arrives, and leave ~120 KB of the SM's 256 KB of L1 + shared memory
// to the data cache, which holds the kernel's stack (register saves around
// the out-of-line op bodies); with nine slots the L1 kept ~28 KB and a frame
// took 6 % longer.
constexpr int kSlots = 4;
constexpr int kSlotNib = 16384;        // nibble bytes per slot (1024 rows of one group)
constexpr int kSlotScl = 2048;         // scale bytes per slot
constexpr int kXMax = 6144;            // widest GEMV input (talker down projection)
constexpr int kTraceFields = 8;
constexpr uint32_t kTagStride = 2048;  // tags per launch (ops + 1 <= kTagStride)

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
// is final when its item ends.  Activations passed between ops are tagged
// words (value | tag << 32, tag = the producing op's tag); a consumer polls
// the words it needs until they carry the producer's tag.
struct alignas(16) GemvDesc {
    const uint4 *nib = nullptr;
    const __half *scl = nullptr;
    int kpad = 0, K = 0, units = 0, G = 1;
    // input
    int in_mode = IN_VEC;
    const uint64_t *in = nullptr;        // IN_VEC: tagged x[K]
    const float *in_plain = nullptr;     // IN_VEC: plain x[K] written by an earlier launch
    uint32_t in_tag = 0;
    const __half *gamma = nullptr;       // RMSNorm prologue (rms_norm_f16, gemv.rs:445-454)
    const uint64_t *ss_in = nullptr;     // with gamma: tagged per-32-column sums of squares of x
    uint32_t ss_tag = 0;
    uint64_t *save = nullptr;            // materialise x as tagged words (before the norm)
    float *save_plain = nullptr;         // materialise x plain (after the norm)
    const uint64_t *amax_src = nullptr;  // IN_EMB / IN_FRAME: tagged logits for the argmax
    int amax_n = 0;
    uint32_t amax_tag = 0;
    uint64_t *code_dst = nullptr;        // tagged slot for the argmax code
    const uint64_t *code_src = nullptr;  // IN_EMB without amax_src: tagged code to look up
    uint32_t code_tag = 0;
    EmbDev emb;                          // IN_EMB table
    const uint64_t *dep = nullptr;       // extra ordering input: wait until dep[0..dep_n) carry
    uint32_t dep_tag = 0;                // dep_tag before writing (an op whose data input does
    int dep_n = 0;                       // not already imply its predecessors are done)
    // output
    int out_mode = OUT_STORE;
    uint64_t *out = nullptr;             // tagged output
    float *out_plain = nullptr;          // plain output (read by the next launch)
    uint32_t out_tag = 0;
    const uint64_t *resid = nullptr;     // OUT_RESID: tagged residual stream
    uint32_t resid_tag = 0;
    const float *bias = nullptr;         // optional, OUT_STORE
    uint64_t *ss_out = nullptr;          // tagged per-32-column sums of squares of the output
    int *adv_len = nullptr;              // end of frame: len[0] += 1, pos[0] += 1
    int *adv_pos = nullptr;
};

// Talker frame-input assembly (generate_new.rs:639-654, code_predictor.rs:287-300).
struct FrameEmbed {
    EmbDev talker;                       // E_talker (semantic row of code 0)
    EmbDev pred[kMaxEmbedGroups];        // acoustic tables
    int ngroups = 0;
    int64_t n = 0;
    const uint64_t *codes_t = nullptr;   // [16] tagged codes 0 .. ngroups-1
    uint32_t code_tag[16] = {};          // the tag of each tagged code
    uint32_t *codes = nullptr;           // [16]: plain codes of the frame (for the host)
    uint32_t *prev = nullptr;            // [16]: previous-code window (repetition penalty)
};

struct OpRef {
    int16_t type = OP_GEMV;
    int16_t avail = 0;  // SMs the items are spread over (the window starting at rot)
    int idx = 0;        // into the gemv / attn arrays
    int n_items = 0;
    int rot = 0;        // item j runs on SM (j % avail + rot) % grid
};

struct FrameParams {
    const OpRef *ops = nullptr;
    int n_ops = 0;
    const GemvDesc *gemv = nullptr;
    const AttnArgs *attn = nullptr;
    SampleArgs sample;
    uint64_t *code0_t = nullptr;         // tagged code 0 (the sampler's output)
    FrameEmbed fe;
    const float *text = nullptr;         // [hidden] text row of this frame
    uint32_t tag_base = 0;               // op i of this launch tags its outputs tag_base + i + 1
    int *abort_flag = nullptr;
    int *err = nullptr;
    unsigned long long *trace = nullptr; // optional [n_ops][8] (zeroed per launch): globaltimer
                                         // ns over the SMs with items: ~earliest input ready, latest
                                         // input ready, latest done, latest start; then on the
                                         // item-0 SM: cycles waiting for weight slots, computing,
                                         // reducing, and slots consumed
};

}  // namespace fk

// Host-side program of the frame kernel for one engine (B = 1).
struct FrameProgram {
    std::vector<fk::OpRef> ops;
    std::vector<fk::GemvDesc> gemv;
    std::vector<AttnArgs> attn;
    DevBuf d_ops, d_gemv, d_attn, d_abort, bufs, d_trace;
    uint32_t epoch = 0;                  // launches so far (tags of launch e start at e * kTagStride)
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
