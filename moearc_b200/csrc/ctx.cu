// ctx.cu — context lifecycle, memory, copies, event profiling, timers and synthetic fills.
//
// The ABI is crates/moearc-kernels/src/ffi.rs:19-59, defined for SYCL in
// kernels.cpp:734-967. Here a context is one CUDA device with one in-order stream: kernels are
// enqueued and return, and ordering between them is the stream's (kernels.cpp:806-810).
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "common.cuh"

using namespace moearc;

namespace moearc {

// Fold every completed event pair into `totals` (kernels.cpp:760-783). Called only from the
// report, after the caller's work: reading an event's time waits for it.
static void flush_events(moearc_ctx *c) {
    for (auto &pe : c->pending) {
        float ms = 0.f;
        if (cudaEventSynchronize(pe.stop) == cudaSuccess &&
            cudaEventElapsedTime(&ms, pe.start, pe.stop) == cudaSuccess) {
            const unsigned long long ns = (unsigned long long)(ms * 1e6);
            bool found = false;
            for (auto &kt : c->totals)
                if (kt.key == pe.key) {
                    kt.ns += ns;
                    kt.calls += 1;
                    found = true;
                    break;
                }
            if (!found) c->totals.push_back(kernel_time{pe.key, ns, 1});
        }
        cudaEventDestroy(pe.start);
        cudaEventDestroy(pe.stop);
    }
    c->pending.clear();
    cudaGetLastError();
}

int launch_scope::finish() {
    const cudaError_t e = cudaGetLastError();
    if (c->profiling && e0) {
        cudaEvent_t e1;
        cudaEventCreate(&e1);
        cudaEventRecord(e1, c->stream);
        char key[96];
        std::snprintf(key, sizeof(key), "%s r%lu m%u", what, rows, mats);
        c->pending.push_back(pending_event{key, e0, e1});
        if (c->pending.size() >= 16384) flush_events(c);
    }
    if (e != cudaSuccess) return ERR;
    if (c->sync_each && cudaStreamSynchronize(c->stream) != cudaSuccess) return ERR;
    return OK;
}

void *ctx_scratch(moearc_ctx *c, size_t bytes) {
    if (bytes <= c->scratch_bytes) return c->scratch;
    cudaStreamSynchronize(c->stream);
    if (c->scratch) cudaFree(c->scratch);
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    want = (want + 255) & ~size_t(255);
    if (cudaMalloc(&c->scratch, want) != cudaSuccess) {
        c->scratch = nullptr;
        c->scratch_bytes = 0;
        return nullptr;
    }
    c->scratch_bytes = want;
    return c->scratch;
}

namespace {
__global__ void k_parts_empty(uint32_t *p, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        p[i] = PART_EMPTY;
}
}  // namespace

void parts_empty(float *p, size_t n, cudaStream_t s, int sm_count) {
    if (p && n) k_parts_empty<<<sm_count, 256, 0, s>>>(reinterpret_cast<uint32_t *>(p), n);
}

}  // namespace moearc

extern "C" {

moearc_ctx *moearc_ctx_create(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return nullptr;
    }
    auto *c = new moearc_ctx();
    if (cudaGetDevice(&c->device) != cudaSuccess) {
        delete c;
        return nullptr;
    }
    cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, c->device);
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete c;
        return nullptr;
    }
    cudaEventCreate(&c->t0);
    cudaEventCreate(&c->t1);
    const char *ev = std::getenv("MOEARC_PROFILE_EVENTS");
    c->profiling = ev && ev[0] == '1';
    const char *se = std::getenv("MOEARC_SYNC_EACH");
    c->sync_each = se && se[0] == '1';
    return c;
}

void moearc_ctx_destroy(moearc_ctx *c) {
    if (!c) return;
    cudaStreamSynchronize(c->stream);
    cudaStreamSynchronize(c->copy_stream);
    for (auto &pe : c->pending) {
        cudaEventDestroy(pe.start);
        cudaEventDestroy(pe.stop);
    }
    if (c->scratch) cudaFree(c->scratch);
    if (c->t0) cudaEventDestroy(c->t0);
    if (c->t1) cudaEventDestroy(c->t1);
    cudaStreamDestroy(c->stream);
    cudaStreamDestroy(c->copy_stream);
    delete c;
}

int moearc_profile_events_enabled(moearc_ctx *c) { return (c && c->profiling) ? 1 : 0; }

int moearc_profile_events_reset(moearc_ctx *c) {
    if (!c) return ERR;
    for (auto &pe : c->pending) {
        cudaEventDestroy(pe.start);
        cudaEventDestroy(pe.stop);
    }
    c->pending.clear();
    c->totals.clear();
    return OK;
}

// One `key nanoseconds calls` line per kernel shape (kernels.cpp:838-862).
int moearc_profile_events_report(moearc_ctx *c, char *out, unsigned long cap) {
    if (!c || !out || cap == 0) return ERR;
    if (!c->profiling) {
        out[0] = '\0';
        return OK;
    }
    flush_events(c);
    unsigned long used = 0;
    for (const auto &kt : c->totals) {
        char line[160];
        const int n = std::snprintf(line, sizeof(line), "%s %llu %llu\n", kt.key.c_str(), kt.ns,
                                    kt.calls);
        if (n <= 0 || used + (unsigned long)n + 1 > cap) break;
        std::memcpy(out + used, line, (size_t)n);
        used += (unsigned long)n;
    }
    out[used] = '\0';
    return OK;
}

// Wait for everything enqueued; a fault from any kernel since the last wait surfaces here
// (kernels.cpp:866-884).
int moearc_sync(moearc_ctx *c) {
    if (!c) return ERR;
    return cudaStreamSynchronize(c->stream) == cudaSuccess ? OK : ERR;
}

int moearc_device_name(moearc_ctx *c, char *out, unsigned long cap) {
    if (!c || !out || cap == 0) return ERR;
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, c->device) != cudaSuccess) return ERR;
    std::strncpy(out, p.name, cap - 1);
    out[cap - 1] = '\0';
    return OK;
}

void *moearc_alloc_device(moearc_ctx *c, unsigned long bytes) {
    if (!c) return nullptr;
    void *p = nullptr;
    if (cudaMalloc(&p, bytes ? bytes : 1) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return p;
}

void moearc_free_device(moearc_ctx *c, void *p) {
    if (!c || !p) return;
    cudaStreamSynchronize(c->stream);
    cudaFree(p);
}

// Blocking copies wait for the stream, so they are ordered after every kernel already
// enqueued (kernels.cpp:895-903).
int moearc_copy_h2d(moearc_ctx *c, void *dst, const void *src, unsigned long bytes) {
    if (!c || !dst || !src) return ERR;
    if (!bytes) return OK;
    if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        return ERR;
    return cudaStreamSynchronize(c->stream) == cudaSuccess ? OK : ERR;
}

int moearc_copy_d2h(moearc_ctx *c, void *dst, const void *src, unsigned long bytes) {
    if (!c || !dst || !src) return ERR;
    if (!bytes) return OK;
    if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
        return ERR;
    return cudaStreamSynchronize(c->stream) == cudaSuccess ? OK : ERR;
}

// Enqueue and return (kernels.cpp:905-967): `src` must stay alive and unchanged until the
// copy has run, which the caller cannot observe except through a later wait.
int moearc_copy_h2d_async(moearc_ctx *c, void *dst, const void *src, unsigned long bytes) {
    if (!c || !dst || !src) return ERR;
    if (!bytes) return OK;
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->stream) == cudaSuccess
               ? OK
               : ERR;
}

// ---- extensions ------------------------------------------------------------------------

// Page-locked host memory, so host<->device copies run at full PCIe rate and can overlap.
void *moearc_x_host_alloc(unsigned long bytes) {
    void *p = nullptr;
    if (cudaMallocHost(&p, bytes ? bytes : 1) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return p;
}

void moearc_x_host_free(void *p) {
    if (p) cudaFreeHost(p);
}

int moearc_x_copy_d2h_async(moearc_ctx *c, void *dst, const void *src, unsigned long bytes) {
    if (!c || !dst || !src) return ERR;
    if (!bytes) return OK;
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c->stream) == cudaSuccess ? OK : ERR;
}

void *moearc_x_stream(moearc_ctx *c) { return c ? (void *)c->stream : nullptr; }

int moearc_x_sm_count(moearc_ctx *c) { return c ? c->sm_count : 0; }

int moearc_x_timer_start(moearc_ctx *c) {
    if (!c) return ERR;
    return cudaEventRecord(c->t0, c->stream) == cudaSuccess ? OK : ERR;
}

int moearc_x_timer_stop(moearc_ctx *c, float *ms) {
    if (!c || !ms) return ERR;
    if (cudaEventRecord(c->t1, c->stream) != cudaSuccess) return ERR;
    if (cudaEventSynchronize(c->t1) != cudaSuccess) return ERR;
    return cudaEventElapsedTime(ms, c->t0, c->t1) == cudaSuccess ? OK : ERR;
}

}  // extern "C"
