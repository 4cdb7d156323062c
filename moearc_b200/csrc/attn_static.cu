// attn_static.cu — decode attention whose split-K partials live in a fixed device array.
//
// moearc_attn_decode takes its partials from the context's scratch, which grows with
// cudaMalloc on first use. A host that must not allocate on its decode thread (a serving loop
// with a fixed memory budget measured at start-up, or one that enqueues work while another
// thread is capturing a CUDA graph, where an allocation would break the capture) cannot use
// that. This entry point does the same work with a file-scope device array of fixed size in
// place of the scratch, so a call makes no allocation of any kind.
#include <mutex>

#include "common.cuh"

namespace moearc {
size_t attn_scratch_bytes(size_t n_heads, size_t head_dim, int n_splits);
int attn_splits(moearc_ctx *c, size_t n_kv_heads, size_t n_heads, size_t span, bool mma, size_t *kps_out);
bool attn_mma_ok(size_t n_heads, size_t n_kv_heads, size_t head_dim, unsigned kv_type,
                 const void *kp, const void *vp);
int attn_launch(moearc_ctx *c, float *out, const float *q, const void *kp, const void *vp,
                const unsigned *table, const float *sinks, size_t n_heads, size_t n_kv_heads,
                size_t hd, size_t kv_begin, size_t n_kv, size_t pt, float scale, unsigned kv_type,
                float *scratch, size_t scratch_bytes, const int *dpos, int window, int max_splits,
                unsigned *ctr);
}  // namespace moearc

using namespace moearc;

namespace {

constexpr size_t STATIC_PARTIAL_BYTES = MOEARC_X_ATTN_STATIC_SCRATCH_BYTES;

// One copy per device (each device loads its own instance of this module). Every split writes
// its partial (max, sum, accumulator row) before the merge kernel that follows it on the same
// stream reads it, so nothing here has to start at zero.
//
// The address below is looked up once per device and kept for the life of the process. It is
// valid for as long as the device's primary context lives: after cudaDeviceReset (or a release
// and re-creation of the primary context) the module loads again at a new address, and a
// process that resets a device must not call this entry point on it again.
__device__ __align__(256) float g_attn_partials[STATIC_PARTIAL_BYTES / sizeof(float)];

constexpr int MAX_DEVICES = 64;
std::mutex g_addr_mu;
float *g_addr[MAX_DEVICES];

// The array's address on device `dev`, looked up once with that device current.
float *partials_on(int dev) {
    if (dev < 0 || dev >= MAX_DEVICES) return nullptr;
    std::lock_guard<std::mutex> lock(g_addr_mu);
    if (g_addr[dev]) return g_addr[dev];
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) return nullptr;
    if (prev != dev && cudaSetDevice(dev) != cudaSuccess) return nullptr;
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_partials);
    if (prev != dev) cudaSetDevice(prev);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    g_addr[dev] = static_cast<float *>(p);
    return g_addr[dev];
}

}  // namespace

extern "C" {

int moearc_x_attn_decode_static(moearc_ctx *c, float *out, const float *q, const void *k_pages,
                                const void *v_pages, const unsigned int *block_table, const float *sinks,
                                unsigned long n_heads, unsigned long n_kv_heads, unsigned long head_dim,
                                unsigned long kv_begin, unsigned long n_kv, unsigned long page_tokens,
                                float scale, unsigned int kv_type) {
    if (!c || !out || !q || !k_pages || !v_pages || !block_table) return ERR;
    if (kv_type != T_F32 && kv_type != T_F16 && kv_type != T_BF16) return ERR_ARG;
    if (n_heads == 0 || n_kv_heads == 0 || head_dim == 0 || n_kv == 0 || page_tokens == 0) return ERR_ARG;
    if (n_heads % n_kv_heads != 0) return ERR_ARG;
    if (kv_begin >= n_kv) return ERR_ARG;
    if (head_dim > 1024) return ERR_ARG;
    const bool mma = attn_mma_ok(n_heads, n_kv_heads, head_dim, kv_type, k_pages, v_pages);
    size_t kps = 0;
    const int n_splits = attn_splits(c, n_kv_heads, n_heads, n_kv - kv_begin, mma, &kps);
    float *scratch = nullptr;
    size_t sb = 0;
    if (n_splits > 1) {
        sb = attn_scratch_bytes(n_heads, head_dim, n_splits);
        // the fixed array bounds the problem: refuse before anything is enqueued
        if (sb > STATIC_PARTIAL_BYTES) return ERR_ARG;
        scratch = partials_on(c->device);
        if (!scratch) return ERR;
    }
    // attn_launch checks each of its own launches, so an unrelated error pending on this thread
    // is neither reported here nor cleared
    return attn_launch(c, out, q, k_pages, v_pages, block_table, sinks, n_heads, n_kv_heads, head_dim,
                       kv_begin, n_kv, page_tokens, scale, kv_type, scratch, sb, nullptr, 0, 0, nullptr);
}

}  // extern "C"
