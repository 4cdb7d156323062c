// common.cuh — shared definitions of libmoearc_b200: the context, return codes, the block
// formats' element rules, and the launch bookkeeping every entry point uses.
#pragma once

#include <atomic>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <utility>
#include <vector>

#include "../../include/moearc.h"

namespace moearc {

// Return codes (crates/moearc-kernels/src/ffi.rs:8-10, kernels.cpp:470-476).
constexpr int OK = 0;
constexpr int ERR = -1;
constexpr int ERR_ARG = -2;

// GGUF type ids (reference.rs:21-40; crates/moearc-model/src/quant.rs:51-107).
constexpr unsigned T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_BF16 = 30, T_MXFP4 = 39;
constexpr unsigned T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14;  // 256-element super-blocks

// Largest k the router selects and largest matrix count one batched launch takes
// (kernels.cpp:451, 651): both bound by-value kernel arguments, not allocations.
constexpr int MAX_TOPK = 32;
constexpr int MAX_BATCHED_MATS = 32;

inline int block_bytes(unsigned t) {
    switch (t) {
    case T_F32: return 4;
    case T_F16: return 2;
    case T_BF16: return 2;
    case T_Q4_0: return 18;
    case T_Q8_0: return 34;
    case T_MXFP4: return 17;
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    default: return 0;
    }
}
inline int block_elems(unsigned t) {
    switch (t) {
    case T_F32:
    case T_F16:
    case T_BF16: return 1;
    case T_Q4_0:
    case T_Q8_0:
    case T_MXFP4: return 32;
    case T_Q4_K:
    case T_Q5_K:
    case T_Q6_K: return 256;
    default: return 0;
    }
}

struct kernel_time {
    std::string key;
    unsigned long long ns;
    unsigned long long calls;
};

struct pending_event {
    std::string key;
    cudaEvent_t start, stop;
};

}  // namespace moearc

// The context: one device, one in-order stream (kernels.cpp:804-828), a second stream for
// host-to-device expert staging, event profiling (kernels.cpp:736-872) and a scratch arena
// for kernels that need temporary device memory (split-K partials).
struct moearc_ctx {
    int device = 0;
    int sm_count = 148;
    cudaStream_t stream = nullptr;
    cudaStream_t copy_stream = nullptr;
    bool profiling = false;  // MOEARC_PROFILE_EVENTS=1
    bool sync_each = false;  // MOEARC_SYNC_EACH=1
    std::vector<moearc::pending_event> pending;
    std::vector<moearc::kernel_time> totals;
    void *scratch = nullptr;
    size_t scratch_bytes = 0;
    cudaEvent_t t0 = nullptr, t1 = nullptr;
};

namespace moearc {

// Bookkeeping around one launch: an event pair when profiling, a wait when MOEARC_SYNC_EACH
// is set, and the launch error (a bad configuration) turned into ERR.
struct launch_scope {
    moearc_ctx *c;
    const char *what;
    unsigned long rows;
    unsigned mats;
    cudaEvent_t e0 = nullptr;
    launch_scope(moearc_ctx *c_, const char *what_, unsigned long rows_, unsigned mats_)
        : c(c_), what(what_), rows(rows_), mats(mats_) {
        if (c->profiling) {
            cudaEventCreate(&e0);
            cudaEventRecord(e0, c->stream);
        }
    }
    int finish();
};

// A scratch buffer of at least `bytes`, owned by the context. Growing it waits for the
// stream (the old buffer may still be in use) and is not allowed during stream capture.
void *ctx_scratch(moearc_ctx *c, size_t bytes);

// ---- device-side element rules ----------------------------------------------------------

// ggml_e8m0_to_fp32_half: 2^(x-128); x < 2 is the subnormal arm (reference.rs:66-70).
__device__ __forceinline__ float e8m0_half(uint32_t x) {
    const uint32_t bits = (x < 2u) ? (0x00200000u << x) : ((x - 1u) << 23);
    return __uint_as_float(bits);
}

// The doubled E2M1 table (reference.rs:56) as a function: magnitudes {0,1,2,3,4,6,8,12} packed
// one per nibble, sign in bit 3 of the code. Index 8 is negative zero and decodes to 0.
__device__ __forceinline__ float kv_mxfp4(uint32_t code) {
    const int mag = (int)((0xC8643210u >> (4u * (code & 7u))) & 0xFu);
    return (float)((code & 8u) ? -mag : mag);
}

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
}
// f32 -> bf16 bits, round to nearest even; a NaN stays a (quiet) NaN.
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Two E2M1 codes (one byte: low nibble first) -> f16x2 of their true values, exactly.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
    uint32_t r;
    asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %1;\n"
        " cvt.rn.f16x2.e2m1x2 %0, b0;\n}" : "=r"(r) : "r"(byte));
    return r;
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

inline unsigned cdiv(unsigned long a, unsigned long b) { return (unsigned)((a + b - 1) / b); }

// ---- phase timestamps (compiled in only with -DMOEARC_TRACE) --------------------------------
// TRACE(slot) stores %globaltimer for thread 0 of each CTA at trace[trace_row * 32 + slot]
// (trace_row: the CTA's row, defined by the kernel as its block index plus a per-kernel base); the
// buffer is set per translation unit with moearc_trace_set_<unit>. A normal build has none.
#ifdef MOEARC_TRACE
static __device__ unsigned long long *g_trace;
#define TRACE(slot)                                                                      \
    do {                                                                                 \
        if (threadIdx.x == 0 && g_trace) {                                               \
            unsigned long long t_;                                                       \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                      \
            g_trace[(size_t)(trace_row) * 32 + (slot)] = t_;                             \
        }                                                                                \
    } while (0)
// TRACE_WARP(slot): the same for lane 0 of every warp (slot chosen per warp by the caller)
#define TRACE_WARP(slot)                                                                 \
    do {                                                                                 \
        if ((threadIdx.x & 31) == 0 && g_trace) {                                        \
            unsigned long long t_;                                                       \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                      \
            g_trace[(size_t)(trace_row) * 32 + (slot)] = t_;                             \
        }                                                                                \
    } while (0)
#define TRACE_SETTER(unit)                                                               \
    extern "C" int moearc_trace_set_##unit(void *p) {                                    \
        unsigned long long *v = static_cast<unsigned long long *>(p);                     \
        return cudaMemcpyToSymbol(g_trace, &v, sizeof(v)) == cudaSuccess ? 0 : -1;         \
    }
#else
#define TRACE(slot) \
    do {            \
    } while (0)
#define TRACE_WARP(slot) \
    do {                 \
    } while (0)
#define TRACE_SETTER(unit)
#endif

// Release / acquire fence at GPU scope, for the last-arriver reductions: each thread that
// wrote partials fences before its warp's arrival (an atomic), and the last arriver fences
// after seeing the count, before it reads them. Cheaper than __threadfence (fence.sc).
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;\n" ::: "memory"); }

// ---- partial slots polled by their reader ----------------------------------------------------
// A partial slot (of the expert and dense decode kernels) holds PART_EMPTY until its producer
// stores the partial, and is set back to PART_EMPTY by the warp that reads it, so a finished
// buffer is all PART_EMPTY again. The pattern is a NaN that no arithmetic produces (results that
// are NaN carry the canonical 0x7FFFFFFF). Slots are written and polled with relaxed gpu-scope
// accesses, and written in whole 32-byte sectors: a read of a sector that was only partly
// written waits for the L2 to fill the rest from DRAM.
constexpr uint32_t PART_EMPTY = 0xFFC0DEADu;
constexpr unsigned long long XPOLL_NS = 200000000ull;  // a poll on other CTAs gives up after 0.2 s

__device__ __forceinline__ uint32_t ld_part(const float *p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint4 ld_part4(const float *p) {
    uint4 v;
    asm volatile("ld.relaxed.gpu.global.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ void st_part(float *p, float x) {
    asm volatile("st.relaxed.gpu.global.f32 [%0], %1;" ::"l"(p), "f"(x) : "memory");
}
__device__ __forceinline__ void st_part4(float *p, float x, float y, float z, float w) {
    asm volatile("st.relaxed.gpu.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(x), "f"(y), "f"(z), "f"(w)
                 : "memory");
}
// Set the first used4 float4s of nrec consecutive records (rec floats apart) back to PART_EMPTY,
// whole sectors, the warp's lanes striding. Plain stores: a slot is next written in a later
// launch, after this kernel has completed, and read after that.
__device__ __forceinline__ void empty_recs(float *p, int nrec, int rec, int used4, int lane) {
    const uint4 e = make_uint4(PART_EMPTY, PART_EMPTY, PART_EMPTY, PART_EMPTY);
    for (int i = lane; i < nrec * used4; i += 32) {
        const int r = i / used4, k = i - r * used4;
        *reinterpret_cast<uint4 *>(p + (size_t)r * rec + k * 4) = e;
    }
}
__device__ __forceinline__ unsigned long long xnow() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Fill n 32-bit words with PART_EMPTY (stream-ordered).
void parts_empty(float *p, size_t n, cudaStream_t s, int sm_count);

// ---- programmatic dependent launch ---------------------------------------------------------
// A kernel launched with launch_pdl may begin while the kernel before it in the stream is
// still running. Everything it does before pdl_wait() must not read that kernel's outputs nor
// write anything another kernel reads (only static data: weights); pdl_wait() returns once the
// preceding kernel has completed and its writes are visible. pdl_trigger() lets the next
// kernel launch early. Both are no-ops in a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// Device slots of an offloaded MoE block: the routed experts' packed gate-up and down banks,
// one slot per distinct routed expert, filled from pinned host memory each step.
struct moe_offload {
    uint8_t *gu_stage, *dn_stage;
    // With a residency cache (slot_of non-null) the stage holds n_cache slots of the block's
    // own, and the experts stay there across steps: slot_of[e] is expert e's slot or -1,
    // owner[s] the expert in slot s or -1, stamp[s] the position slot s was last used at; each
    // step's plan lists the misses to fetch ([0] = count, then (expert, slot) pairs), and
    // fetched counts the experts copied over PCIe.
    int *slot_of = nullptr, *owner = nullptr, *stamp = nullptr, *plan = nullptr;
    unsigned long long *fetched = nullptr;
    const int *clock = nullptr;  // device position, advanced once a step: the cache's clock
    int n_cache = 0;
    const struct moe_host *host = nullptr;  // part of the block's experts on the host cores, or null
};

// Host execution of part of an offloaded block's experts, beside the device (moe.rs:2169-2211,
// 2389-2420), through a mailbox in pinned, device-mapped host memory. After the router a
// one-warp kernel splits the token's choices by the policy, leaves the device's mask in `hmask`,
// writes the host's share (block, experts, weights, the routed activation) into the mail and
// then, last, the next sequence number; a host thread polling the mail runs the pool on it and
// writes the result and the same number into `done`. The main stream meanwhile runs the
// device's share into `ffn`; the fold kernel waits (bounded) for `done` to show the number and
// adds h + (ffn + host share).
// Mail layout (bytes): [0] u64 sequence, [8] u32 experts n, [12] u32 block, [16] u32 experts[32],
// [144] f32 weights[32], [512] f32 x[n_embd]. Done layout: [0] u64 sequence, [64] f32 out[n_embd].
constexpr int MAIL_SEQ = 0, MAIL_N = 8, MAIL_BLOCK = 12, MAIL_IDS = 16, MAIL_WTS = 144, MAIL_X = 512;
constexpr int DONE_SEQ = 0, DONE_OUT = 64;

struct moe_host {
    int kind = 0;  // 0 off, 1 a fraction of the misses (rounded up), 2 the misses beyond `over`
    float frac = 0.f;
    int over = 0;
    int block = 0;                          // the block's index, for the host thread
    unsigned *hmask = nullptr;              // device word: the choices the host takes
    unsigned long long *seq = nullptr;      // device counter: the last sequence number issued
    uint8_t *mail = nullptr;                // device pointer of the pinned mail
    const uint8_t *done = nullptr;          // device pointer of the pinned done record
    float *ffn = nullptr;                   // device [n_embd]: the device's share
    unsigned long long wait_ns = 0;         // the fold's wait limit
    int *status = nullptr;                  // raised when the wait runs out
};

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Shared-memory limit of a kernel, with the SM's unified L1 / shared storage configured for
// the most shared memory. The carveout is per kernel: a kernel launched with a smaller one
// leaves its SMs unable to take a neighbouring kernel's CTA (PDL overlap needs both resident).
template <typename... KArgs>
inline cudaError_t set_smem(void (*kernel)(KArgs...), int max_dynamic) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_dynamic);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
}

// Kernel attributes such as the shared-memory limit belong to the device they were set on: a
// process driving two GPUs has to set them on each. once_per_device(done, f) runs f (which
// returns a cudaError_t) with the current device the first time that device asks, and again
// after a failure. Two threads asking at once may both run f; setting the same attribute to
// the same value twice is harmless.
constexpr int MOEARC_MAX_DEVICES = 64;

template <typename F>
inline cudaError_t once_per_device(std::atomic<bool> (&done)[MOEARC_MAX_DEVICES], F &&f) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= MOEARC_MAX_DEVICES) return f();
    if (done[dev].load(std::memory_order_acquire)) return cudaSuccess;
    e = f();
    if (e == cudaSuccess) done[dev].store(true, std::memory_order_release);
    return e;
}

// A cooperative launch (every CTA resident at once, so CTAs may wait on one another), with
// programmatic dependent launch when the runtime accepts both attributes together.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_coop(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                               Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
    if (e != cudaSuccess) {
        cudaGetLastError();
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    }
    return e;
}

}  // namespace moearc
