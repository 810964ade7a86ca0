// Internal shared definitions of the QORA B200 engine (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <utility>
#include <vector>

#include "qora_cuda.h"

namespace qora {

constexpr int kGroup = 32;          // Q4 group width (gemv.rs:18)
constexpr int kMaxRows = 512;       // rows (streams x tokens) per GEMV launch
constexpr int kAttnMaxSplit = 16;   // position splits per (row, kv head)
constexpr int kEngineKernelsUnknown = -1;

// ------------------------------------------------------------------ errors
int set_error(int code, const char *fmt, ...);

#define QORA_TRY(expr)                   \
    do {                                 \
        int rc__ = (expr);               \
        if (rc__ != QORA_OK) return rc__; \
    } while (0)

#define QORA_CUDA(call)                                                                      \
    do {                                                                                     \
        cudaError_t e__ = (call);                                                            \
        if (e__ != cudaSuccess)                                                              \
            return ::qora::set_error(e__ == cudaErrorMemoryAllocation ? QORA_ERR_OOM         \
                                                                      : QORA_ERR_CUDA,       \
                                     "%s:%d %s: %s", __FILE__, __LINE__, #call,              \
                                     cudaGetErrorString(e__));                               \
    } while (0)

#define QORA_LAUNCH_CHECK() QORA_CUDA(cudaGetLastError())

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

// Makes a device current for the guard's lifetime and gives the caller's
// current device back afterwards (entry points that launch on an object's
// device whatever device the calling thread has current).
class DeviceGuard {
    int prev_ = -1;

  public:
    DeviceGuard() = default;
    DeviceGuard(const DeviceGuard &) = delete;
    DeviceGuard &operator=(const DeviceGuard &) = delete;
    int set(int device) {
        int cur = 0;
        QORA_CUDA(cudaGetDevice(&cur));
        if (cur == device) return QORA_OK;
        QORA_CUDA(cudaSetDevice(device));
        prev_ = cur;
        return QORA_OK;
    }
    ~DeviceGuard() {
        if (prev_ >= 0) cudaSetDevice(prev_);
    }
};

// Device error flag codes (written by kernels, read by the host).
enum DeviceError : int {
    kDevOk = 0,
    kDevRange = 1,   // position past the RoPE table or KV capacity
    kDevNaN = 2,     // NaN logits reached an argmax / sampler
    kDevTimeout = 3, // bounded wait expired
    kDevF16Range = 4,// an infinite input row value reached the tensor-core GEMV operands
};

// ------------------------------------------------------------ device memory
// Owning device buffer (freed on destruction).
struct DevBuf {
    void *p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    DevBuf(DevBuf &&o) noexcept : p(o.p), bytes(o.bytes) {
        o.p = nullptr;
        o.bytes = 0;
    }
    DevBuf &operator=(DevBuf &&o) noexcept {
        if (this != &o) {
            release();
            p = o.p;
            bytes = o.bytes;
            o.p = nullptr;
            o.bytes = 0;
        }
        return *this;
    }
    ~DevBuf() { release(); }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    int alloc(size_t n) {
        release();
        if (n == 0) return QORA_OK;
        cudaError_t e = cudaMalloc(&p, n);
        if (e != cudaSuccess) {
            p = nullptr;
            return set_error(QORA_ERR_OOM, "cudaMalloc(%zu): %s", n, cudaGetErrorString(e));
        }
        bytes = n;
        return QORA_OK;
    }
    int zero(cudaStream_t s = nullptr) {
        if (!p) return QORA_OK;
        QORA_CUDA(cudaMemsetAsync(p, 0, bytes, s));
        return QORA_OK;
    }
    template <class T>
    T *as() const { return reinterpret_cast<T *>(p); }
};

// ------------------------------------------------------------ device helpers
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// Packed 2-wide fp32 FMA / add (sm_100a): d = a * b + c lane-wise, one rounding.
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// 128-bit streaming load through the non-coherent path, no L1 allocation.
__device__ __forceinline__ uint4 ldg_stream(const uint4 *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// ---- shared-memory bulk copies completed on an mbarrier (no multicast) ----
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// dst (this CTA's shared memory) <- src (global), `bytes` a multiple of 16,
// both addresses 16-byte aligned; completion is signalled on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait for an mbarrier phase: gives up after ~1 s (raising
// kDevTimeout on `err`) instead of spinning forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > 1000000000ull) {
            if (err) atomicCAS(err, 0, 3);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---- tagged values: one 64-bit word = (tag << 32) | float bits, written and
// read with single-copy-atomic relaxed accesses.  A reader that sees the
// expected tag sees that writer's value (no separate flag, no counter).
__device__ __forceinline__ uint64_t tag_pack(float v, uint32_t tag) {
    return ((uint64_t)tag << 32) | __float_as_uint(v);
}
__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u64(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Orders this thread's earlier accesses before its later ones at GPU scope:
// after a poll it is the acquire half, before tagged stores the release half.
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ uint64_t global_ns_t() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits (bounded, ~2 s) until base[k * stride] carries `tag` for every k < N
// (pred[k] false skips an element) and returns the values in out[].  On
// timeout, or when *abort is set by another waiter, it raises kDevTimeout,
// sets *abort and returns what it has: the caller keeps to its barrier
// sequence and checks the abort state afterwards.  Every attempt reloads
// all pending words (one L2 round trip per attempt), so the values are in
// hand in the attempt that sees them.
// ACQ adds an acquire fence at the end, for callers that go on to read
// plain data the writers published before their tagged stores.
template <int N, bool ACQ = false>
__device__ __forceinline__ bool poll_tagged(const uint64_t *base, int64_t stride, uint32_t tag,
                                            float (&out)[N], const bool (&pred)[N], int *err,
                                            int *abort) {
    uint32_t pending = 0;
#pragma unroll
    for (int k = 0; k < N; k++)
        if (pred[k]) pending |= 1u << k;
    uint64_t t0 = 0;
    bool ok = true;
    for (int it = 0; pending; it++) {
        uint64_t v[N];
#pragma unroll
        for (int k = 0; k < N; k++)
            if (pending & (1u << k)) v[k] = ld_relaxed_u64(base + k * stride);
#pragma unroll
        for (int k = 0; k < N; k++) {
            if ((pending & (1u << k)) && (uint32_t)(v[k] >> 32) == tag) {
                out[k] = __uint_as_float((uint32_t)v[k]);
                pending &= ~(1u << k);
            }
        }
        if (!pending) break;
        if (it == 0) t0 = global_ns_t();
        if ((it & 15) == 15) {
            if (*(volatile int *)abort) {
                ok = false;
                break;
            }
            if (global_ns_t() - t0 > 2000000000ull) {
                if (err) atomicCAS(err, 0, 3);
                atomicExch(abort, 1);
                ok = false;
                break;
            }
        }
    }
    if (ACQ) fence_acq_rel_gpu();
    return ok;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float silu_ref(float x) {
    // gemv.rs:486-488: x / (1 + exp(-x))
    return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
}

__device__ __forceinline__ void raise_error(int *err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// Programmatic dependent launch: a kernel may start while its predecessor in
// the stream is still running.  Everything it reads or writes that another
// kernel produces or consumes must come after griddep_wait(); only immutable
// data (weights, norms, tables) may be touched before it.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Whether launches carry the programmatic-serialization attribute
// (QORA_PDL=0 in the environment turns it off).
bool pdl_enabled();

// Launch with cudaLaunchKernelEx: PDL attribute and an optional (1, cy, 1)
// thread-block cluster.
template <typename... KArgs, typename... Args>
int launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
              unsigned cluster_y, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    unsigned n = 0;
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    n++;
    if (cluster_y > 1) {
        attrs[n].id = cudaLaunchAttributeClusterDimension;
        attrs[n].val.clusterDim.x = 1;
        attrs[n].val.clusterDim.y = cluster_y;
        attrs[n].val.clusterDim.z = 1;
        n++;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = n;
    QORA_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
    return QORA_OK;
}

// ------------------------------------------------------------ weights
// Device Q4 weight: column-group-major copy of the reference layout.
//   nib[c][k] : 16 bytes = the 32 nibbles of group c in row k (byte j holds
//               columns 32c+2j (low) and 32c+2j+1 (high), as in gemv.rs)
//   scl[c][k] : f16 scale of group c in row k
// A warp reading rows k0..k0+31 of one group reads 512 contiguous bytes.
//   Each group's rows are padded with zeros to kpad = round_up(k, 128), so a
//   128-row chunk is always a whole, 16-byte-aligned bulk copy.
struct Q4Dev {
    const uint4 *nib = nullptr;
    const __half *scl = nullptr;
    int64_t k = 0, n = 0;  // n may exceed 32*C: the tail stays zero (gemv.rs:846-861)
    int64_t C = 0;         // full groups
    int64_t kpad = 0;      // row stride of one group in nib / scl
    int mma_exp = -1;      // tensor-core path: scales are used as scale * 2^mma_exp in f16
                           // (chosen at upload so 8 * max scale * 2^mma_exp <= 2^15); -1: unusable
};

constexpr int kChunkRows = 128;  // rows per bulk-copy chunk
inline int64_t pad_rows(int64_t k) { return (k + kChunkRows - 1) / kChunkRows * kChunkRows; }

// Row-major device copy of an embedding table in the reference layout
// (row = token): packed[tok][n/2], scales[tok][n/32].
struct EmbDev {
    const uint8_t *packed = nullptr;
    const __half *scl = nullptr;
    int64_t rows = 0, n = 0;
    float absmax = 0.0f;  // bound on |row value|: 8 * the table's largest scale
};

}  // namespace qora

// A context is reference counted: the caller's handle (released by
// qora_ctx_destroy) and every object created from it (weights, caches,
// models, text projections) each hold one reference, so destroying the
// context before its objects leaves it alive until the last one is gone.
struct qora_ctx {
    int device = 0;
    int num_sms = 148;
    qora::DevBuf err;       // device error flag
    std::atomic<int> refs{1};
};

namespace qora {
// An object's reference to its context (retained on assignment, released
// when the object is destroyed; the last release frees the context).
class CtxRef {
    qora_ctx *c_ = nullptr;
    static void release(qora_ctx *c) {
        if (c && c->refs.fetch_sub(1) == 1) delete c;
    }

  public:
    CtxRef() = default;
    CtxRef(const CtxRef &) = delete;
    CtxRef &operator=(const CtxRef &) = delete;
    ~CtxRef() { release(c_); }
    CtxRef &operator=(qora_ctx *c) {
        if (c) c->refs.fetch_add(1);
        release(c_);
        c_ = c;
        return *this;
    }
    operator qora_ctx *() const { return c_; }
    qora_ctx *operator->() const { return c_; }
    // Drops the caller's own reference (qora_ctx_destroy).
    static void drop(qora_ctx *c) { release(c); }
};
}  // namespace qora

struct qora_w4 {
    qora::CtxRef ctx;
    qora::DevBuf nib, scl, rowmajor_packed, rowmajor_scl;
    qora::Q4Dev dev;
    qora::EmbDev emb;  // valid after qora_q4_embed_rows first use (lazy)
    std::vector<uint8_t> host_packed;   // kept only until the row-major copy exists
    std::vector<uint16_t> host_scales;
};
