// Allocation-free KV append + attend (qora_kv_attend_noalloc).
//
// Some callers cannot let a library call cudaMalloc: a real-time audio loop
// that must not stall (cudaMalloc can wait on device-wide work for an
// unbounded time, and the TTS frame loop runs against a playback deadline),
// or a host application whose own memory manager has already reserved the
// GPU's memory, so a driver allocation would fail.  qora_kv_attend sizes its
// split-merge scratch with cudaMalloc on its first call on a cache; this
// variant runs the same kernel with its scratch in a fixed array of this
// library's static device memory instead.
//
// The array (g_attend_scratch, ~1.1 MB) exists on every GPU that loads the
// library and is held until the process exits.  Host code cannot use the
// array's name as a device address: the first call on each device looks the
// address up with cudaGetSymbolAddress (with that device current) and caches
// it.  Every call shares the one array and it keeps the last call's contents;
// the per-(stream, kv head) arrival counters are cleared by each call before
// its kernel runs.  Calls that overlap on the GPU (other streams, other host
// threads) race on the array: issue them on one stream, in order.
#include <mutex>

#include "kv.cuh"

namespace {

// Scratch limits (floats unless noted), checked before any launch:
//   split partial outputs  B * num_heads * head_dim * 16 <= kNaPartO
//   split max / sum pairs  B * num_heads * 16 * 2         <= kNaPartML
//   arrival counters       B * kv_heads (u32)             <= kNaTickets
// e.g. the talker (16 heads x 128) fits B <= 8 streams per call.
constexpr size_t kNaPartO = 262144;
constexpr size_t kNaPartML = 16384;
constexpr size_t kNaTickets = 512;

static __device__ __align__(256) float g_attend_scratch[kNaPartO + kNaPartML + kNaTickets];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
float *g_scratch_addr[kMaxDevices] = {};

// Device address of g_attend_scratch on `device` (looked up once per device).
int scratch_address(int device, float **out) {
    if (device < 0 || device >= kMaxDevices)
        return qora::set_error(QORA_ERR_INVALID, "device %d outside 0..%d", device, kMaxDevices - 1);
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[device]) {
        int cur = 0;
        QORA_CUDA(cudaGetDevice(&cur));
        QORA_CUDA(cudaSetDevice(device));
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attend_scratch);
        const cudaError_t e2 = cudaSetDevice(cur);
        if (e != cudaSuccess)
            return qora::set_error(QORA_ERR_CUDA, "cudaGetSymbolAddress(g_attend_scratch): %s",
                                   cudaGetErrorString(e));
        if (e2 != cudaSuccess)
            return qora::set_error(QORA_ERR_CUDA, "cudaSetDevice(%d): %s", cur, cudaGetErrorString(e2));
        g_scratch_addr[device] = static_cast<float *>(p);
    }
    *out = g_scratch_addr[device];
    return QORA_OK;
}

}  // namespace

using namespace qora;

extern "C" int qora_kv_attend_noalloc(qora_kv *kv, int32_t layer, const float *qkv,
                                      int32_t num_heads, const uint16_t *q_norm,
                                      const uint16_t *k_norm, const float *rope_cos,
                                      const float *rope_sin, int32_t rope_max_pos,
                                      const int32_t *positions, int32_t B, int32_t advance,
                                      float *out, void *stream) {
    AttnArgs at;
    QORA_TRY(kv_attend_args(kv, layer, qkv, num_heads, q_norm, k_norm, rope_cos, rope_sin,
                            rope_max_pos, positions, B, out, at));
    const size_t po = attn_part_o_floats(B, kv->kvh, num_heads, kv->hd);
    const size_t pml = attn_part_ml_floats(B, kv->kvh, num_heads);
    const size_t tk = (size_t)B * kv->kvh;
    if (po > kNaPartO || pml > kNaPartML || tk > kNaTickets)
        return set_error(QORA_ERR_UNSUPPORTED,
                         "qora_kv_attend_noalloc: B=%d x %d heads x head_dim %d needs %zu + %zu "
                         "floats and %zu counters of scratch; the static array holds %zu + %zu "
                         "and %zu (B * heads * head_dim <= 16384)",
                         B, num_heads, kv->hd, po, pml, tk, kNaPartO, kNaPartML, kNaTickets);
    // the cache's device is current for the look-up, the clear and the launch,
    // whatever device the calling thread had current (restored on return)
    DeviceGuard dg;
    QORA_TRY(dg.set(kv->ctx->device));
    float *base = nullptr;
    QORA_TRY(scratch_address(kv->ctx->device, &base));
    at.part_o = base;
    at.part_ml = base + kNaPartO;
    at.tickets = reinterpret_cast<unsigned *>(base + kNaPartO + kNaPartML);
    cudaStream_t st = as_stream(stream);
    QORA_TRY(kv_prepare(kv, 0, B, 1, st));  // paged caches: the append at each stream's length
    QORA_CUDA(cudaMemsetAsync(at.tickets, 0, tk * sizeof(unsigned), st));
    QORA_TRY(launch_attention(at, st));
    if (advance) {
        QORA_TRY(kv_advance(kv, B, st));
        kv_note_growth(kv, 0, B, 1);
    }
    return QORA_OK;
}
