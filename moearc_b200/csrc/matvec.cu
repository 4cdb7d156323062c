// matvec.cu — the ABI matvecs over GGUF-layout weights (kernels.cpp:1046-1206) and the f32
// router GEMV (kernels.cpp:1116-1135).
//
// GGUF rows are runs of 17-byte (MXFP4), 18-byte (Q4_0) or 34-byte (Q8_0) blocks, so no block
// after the first is 4-byte aligned. Each lane owns one block at a time: it loads the aligned
// 32-bit words that cover it, re-aligns them to the block with one funnel shift per word
// (a shift that is the same for every word, so the window stays in registers), and decodes
// from there. The activation vector is staged once per CTA in shared memory transposed,
// xT[j][b] = x[32b + j], so the 32 lanes of a warp — 32 consecutive blocks — read 32
// consecutive words: no bank conflicts.
//
// This is the drop-in path for callers that hand over GGUF pointers; the fused MoE path
// (moe.cu) reads a re-laid bank on the tensor cores instead.
#include "common.cuh"
#include "kquant.cuh"

using namespace moearc;

namespace {

constexpr int ROWS_PER_WARP = 4;
constexpr int WARPS = 8;
constexpr int ROWS_PER_CTA = ROWS_PER_WARP * WARPS;

// Words needed to cover a BB-byte block that starts anywhere within a word.
template <int BB>
constexpr int nwords() { return (BB + 3 + 3) / 4; }

// v[i] = the four bytes at p + 4i, for i < nwords-1, read through aligned words.
template <int BB>
__device__ __forceinline__ void load_block(const uint8_t *p, const uint8_t *end, bool aligned,
                                           uint32_t (&v)[nwords<BB>()]) {
    constexpr int NW = nwords<BB>();
    uint32_t w[NW];
    const uintptr_t a = reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3);
    const int s = (int)(reinterpret_cast<uintptr_t>(p) & 3) * 8;
    if (aligned && a + 4 * NW <= reinterpret_cast<uintptr_t>(end)) {
        const uint32_t *wp = reinterpret_cast<const uint32_t *>(a);
#pragma unroll
        for (int i = 0; i < NW; ++i) w[i] = __ldg(wp + i);
    } else {
        // The matrix's last block, or an unaligned matrix: bytes, none outside the block.
#pragma unroll
        for (int i = 0; i < NW; ++i) {
            uint32_t x = 0;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const uint8_t *q = reinterpret_cast<const uint8_t *>(a) + 4 * i + t;
                if (q >= p && q < p + BB) x |= (uint32_t)__ldg(q) << (8 * t);
            }
            w[i] = x;
        }
    }
#pragma unroll
    for (int i = 0; i < NW - 1; ++i) v[i] = __funnelshift_r(w[i], w[i + 1], s);
    v[NW - 1] = __funnelshift_r(w[NW - 1], 0u, s);
}

// One block's dot product with its 32 activations, xt pointing at xT[0][b] (row stride nb).
template <unsigned T>
__device__ __forceinline__ float block_dot(const uint8_t *p, const uint8_t *end, bool aligned,
                                           const float *xt, size_t nb) {
    if constexpr (T == T_MXFP4) {
        uint32_t v[nwords<17>()];
        load_block<17>(p, end, aligned, v);
        const float d = e8m0_half(v[0] & 0xFFu);
        float lo = 0.f, hi = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t q = __funnelshift_r(v[i], v[i + 1], 8);  // qs bytes 4i..4i+3
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const uint32_t h2 = e2m1x2_to_f16x2((q >> (8 * t)) & 0xFFu);
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h2));
                const int j = 4 * i + t;
                lo = fmaf(f.x, xt[(size_t)j * nb], lo);
                hi = fmaf(f.y, xt[(size_t)(j + 16) * nb], hi);
            }
        }
        // The E2M1 values are the true ones, half the reference's doubled table entries, so
        // the block sum is doubled (exactly) before the halved scale (reference.rs:51-70).
        return (2.f * (lo + hi)) * d;
    } else if constexpr (T == T_Q4_0) {
        uint32_t v[nwords<18>()];
        load_block<18>(p, end, aligned, v);
        const float d = f16_bits_to_f32((uint16_t)(v[0] & 0xFFFFu));
        float lo = 0.f, hi = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t q = __funnelshift_r(v[i], v[i + 1], 16);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const uint32_t byte = (q >> (8 * t)) & 0xFFu;
                const int j = 4 * i + t;
                lo = fmaf((float)((int)(byte & 15u) - 8), xt[(size_t)j * nb], lo);
                hi = fmaf((float)((int)(byte >> 4) - 8), xt[(size_t)(j + 16) * nb], hi);
            }
        }
        return (lo + hi) * d;
    } else {  // Q8_0
        uint32_t v[nwords<34>()];
        load_block<34>(p, end, aligned, v);
        const float d = f16_bits_to_f32((uint16_t)(v[0] & 0xFFFFu));
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t q = __funnelshift_r(v[i], v[i + 1], 16);
#pragma unroll
            for (int t = 0; t < 4; ++t)
                acc = fmaf((float)(int8_t)((q >> (8 * t)) & 0xFFu), xt[(size_t)(4 * i + t) * nb], acc);
        }
        return acc * d;
    }
}

struct mat_table {
    const uint8_t *p[MAX_BATCHED_MATS];
};

// Grid: (ceil(n_rows / 32), n_mat). Matrix m = blockIdx.y reads x + m * x_stride.
template <unsigned T, int BB>
__global__ void __launch_bounds__(WARPS * 32)
    k_matvec_q(float *__restrict__ out, mat_table w, const float *__restrict__ x, size_t x_stride,
               size_t n_rows, size_t n_cols, bool aligned) {
    extern __shared__ float xT[];
    const size_t nb = n_cols / 32;
    const size_t ld = nb | 1;  // odd stride: the transposing writes spread over all banks
    const unsigned m = blockIdx.y;
    const float *xm = x + (size_t)m * x_stride;
    for (size_t i = threadIdx.x; i < n_cols; i += blockDim.x) {
        const size_t b = i >> 5, j = i & 31;
        xT[j * ld + b] = xm[i];
    }
    __syncthreads();
    const uint8_t *base = w.p[m];
    const size_t row_bytes = nb * BB;
    const uint8_t *end = base + n_rows * row_bytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = 0; i < ROWS_PER_WARP; ++i) {
        const size_t r = (size_t)blockIdx.x * ROWS_PER_CTA + warp * ROWS_PER_WARP + i;
        if (r >= n_rows) break;  // uniform across the warp
        const uint8_t *row = base + r * row_bytes;
        float acc = 0.f;
        for (size_t b = lane; b < nb; b += 32) acc += block_dot<T>(row + b * BB, end, aligned, xT + b, ld);
        acc = warp_sum(acc);
        if (lane == 0) out[(size_t)m * n_rows + r] = acc;
    }
}

// K-quant rows (256-element super-blocks): warp per row, each super-block spread over the warp,
// lane l expanding its elements 8l .. 8l + 7 (kquant.cuh) and folding them with x in order; a
// butterfly sums the lanes.
template <unsigned T, int BB>
__global__ void __launch_bounds__(WARPS * 32)
    k_matvec_kq(float *__restrict__ out, mat_table w, const float *__restrict__ x, size_t x_stride,
                size_t n_rows, size_t n_cols) {
    const unsigned m = blockIdx.y;
    const float *xm = x + (size_t)m * x_stride;
    const size_t nb = n_cols / 256;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = 0; i < ROWS_PER_WARP; ++i) {
        const size_t r = (size_t)blockIdx.x * ROWS_PER_CTA + warp * ROWS_PER_WARP + i;
        if (r >= n_rows) break;  // uniform across the warp
        const uint8_t *row = w.p[m] + r * nb * BB;
        float acc = 0.f;
        for (size_t b = 0; b < nb; ++b) {
            float v[8];
            kq_decode8<T>(row + b * BB, 8 * lane, v);
            const float *xb = xm + b * 256 + 8 * lane;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc = fmaf(v[e], __ldg(xb + e), acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) out[(size_t)m * n_rows + r] = acc;
    }
}

// f32 / f16 / bf16 rows: warp per row, lanes stride the columns (kernels.cpp:1027-1044).
template <unsigned T>
__global__ void __launch_bounds__(WARPS * 32)
    k_matvec_scalar(float *__restrict__ out, mat_table w, const float *__restrict__ x,
                    size_t x_stride, size_t n_rows, size_t n_cols) {
    const unsigned m = blockIdx.y;
    const float *xm = x + (size_t)m * x_stride;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = 0; i < ROWS_PER_WARP; ++i) {
        const size_t r = (size_t)blockIdx.x * ROWS_PER_CTA + warp * ROWS_PER_WARP + i;
        if (r >= n_rows) break;
        float acc = 0.f;
        for (size_t c = lane; c < n_cols; c += 32) {
            float wv;
            if constexpr (T == T_F32) wv = reinterpret_cast<const float *>(w.p[m])[r * n_cols + c];
            else if constexpr (T == T_F16) wv = f16_bits_to_f32(reinterpret_cast<const uint16_t *>(w.p[m])[r * n_cols + c]);
            else wv = bf16_bits_to_f32(reinterpret_cast<const uint16_t *>(w.p[m])[r * n_cols + c]);
            acc = fmaf(wv, xm[c], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) out[(size_t)m * n_rows + r] = acc;
    }
}

// The router GEMV in a fixed order the host can reproduce: lane l folds columns
// 4l + 128i .. +3 in ascending order with fma, then the xor butterfly 16, 8, 4, 2, 1.
__global__ void __launch_bounds__(WARPS * 32)
    k_matvec_f32(float *__restrict__ out, const float *__restrict__ w, const float *__restrict__ x,
                 size_t n_rows, size_t n_cols, bool vec) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t r = (size_t)blockIdx.x * WARPS + warp;
    if (r >= n_rows) return;
    const float *wr = w + r * n_cols;
    const size_t n4 = (n_cols + 3) / 4;
    float acc = 0.f;
    if (vec) {
        const float4 *w4 = reinterpret_cast<const float4 *>(wr);
        const float4 *x4 = reinterpret_cast<const float4 *>(x);
        for (size_t c4 = lane; c4 < n4; c4 += 32) {
            const float4 a = __ldg(w4 + c4), b = __ldg(x4 + c4);
            acc = fmaf(a.x, b.x, acc);
            acc = fmaf(a.y, b.y, acc);
            acc = fmaf(a.z, b.z, acc);
            acc = fmaf(a.w, b.w, acc);
        }
    } else {
        for (size_t c4 = lane; c4 < n4; c4 += 32)
            for (int t = 0; t < 4; ++t) {
                const size_t cc = 4 * c4 + t;
                if (cc < n_cols) acc = fmaf(wr[cc], x[cc], acc);
            }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) out[r] = acc;
}

int launch_matvec(moearc_ctx *c, unsigned t, float *out, const mat_table &tab, unsigned n_mat,
                  const float *x, size_t x_stride, size_t n_rows, size_t n_cols, const char *what) {
    launch_scope ls(c, what, n_rows, n_mat);
    const dim3 grid(cdiv(n_rows, ROWS_PER_CTA), n_mat);
    const dim3 block(WARPS * 32);
    if (block_elems(t) == 256) {
        switch (t) {
        case T_Q4_K: k_matvec_kq<T_Q4_K, 144><<<grid, block, 0, c->stream>>>(out, tab, x, x_stride, n_rows, n_cols); break;
        case T_Q5_K: k_matvec_kq<T_Q5_K, 176><<<grid, block, 0, c->stream>>>(out, tab, x, x_stride, n_rows, n_cols); break;
        default: k_matvec_kq<T_Q6_K, 210><<<grid, block, 0, c->stream>>>(out, tab, x, x_stride, n_rows, n_cols); break;
        }
    } else if (block_elems(t) == 32) {
        const size_t smem = (n_cols + 32) * sizeof(float);
        bool aligned = true;
        for (unsigned m = 0; m < n_mat; ++m) aligned &= (reinterpret_cast<uintptr_t>(tab.p[m]) & 3) == 0;
        if (smem > 48 * 1024) {
            cudaFuncSetAttribute(k_matvec_q<T_MXFP4, 17>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
            cudaFuncSetAttribute(k_matvec_q<T_Q4_0, 18>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
            cudaFuncSetAttribute(k_matvec_q<T_Q8_0, 34>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        }
        switch (t) {
        case T_MXFP4: k_matvec_q<T_MXFP4, 17><<<grid, block, smem, c->stream>>>(out, tab, x, x_stride, n_rows, n_cols, aligned); break;
        case T_Q4_0: k_matvec_q<T_Q4_0, 18><<<grid, block, smem, c->stream>>>(out, tab, x, x_stride, n_rows, n_cols, aligned); break;
        default: k_matvec_q<T_Q8_0, 34><<<grid, block, smem, c->stream>>>(out, tab, x, x_stride, n_rows, n_cols, aligned); break;
        }
    } else {
        switch (t) {
        case T_F32: k_matvec_scalar<T_F32><<<grid, block, 0, c->stream>>>(out, tab, x, x_stride, n_rows, n_cols); break;
        case T_F16: k_matvec_scalar<T_F16><<<grid, block, 0, c->stream>>>(out, tab, x, x_stride, n_rows, n_cols); break;
        default: k_matvec_scalar<T_BF16><<<grid, block, 0, c->stream>>>(out, tab, x, x_stride, n_rows, n_cols); break;
        }
    }
    return ls.finish();
}

}  // namespace

extern "C" {

// kernels.cpp:1046-1114.
int moearc_matvec_q(moearc_ctx *c, unsigned int type_id, float *out, const void *w,
                    const float *x, unsigned long n_rows, unsigned long n_cols) {
    if (!c || !out || !w || !x) return ERR;
    if (!block_bytes(type_id)) return ERR_ARG;
    if (n_cols % (unsigned long)block_elems(type_id)) return ERR_ARG;
    if ((n_cols + 32) * sizeof(float) > 227ul * 1024 && block_elems(type_id) == 32) return ERR_ARG;
    if (n_rows == 0) return OK;
    mat_table t{};
    for (int i = 0; i < MAX_BATCHED_MATS; ++i) t.p[i] = static_cast<const uint8_t *>(w);
    return launch_matvec(c, type_id, out, t, 1, x, 0, n_rows, n_cols, "mvq");
}

// kernels.cpp:1146-1206.
int moearc_matvec_q_batched(moearc_ctx *c, unsigned int type_id, float *out,
                            const void *const *w, unsigned int n_mat, const float *x,
                            unsigned long x_stride, unsigned long n_rows, unsigned long n_cols) {
    if (!c || !out || !w || !x) return ERR;
    if (n_mat == 0 || n_rows == 0) return OK;
    if (n_mat > (unsigned)MAX_BATCHED_MATS) return ERR_ARG;
    if (!block_bytes(type_id)) return ERR_ARG;
    if (n_cols % (unsigned long)block_elems(type_id)) return ERR_ARG;
    if ((n_cols + 32) * sizeof(float) > 227ul * 1024 && block_elems(type_id) == 32) return ERR_ARG;
    mat_table t{};
    for (unsigned i = 0; i < n_mat; ++i) {
        if (!w[i]) return ERR;
        t.p[i] = static_cast<const uint8_t *>(w[i]);
    }
    for (int i = (int)n_mat; i < MAX_BATCHED_MATS; ++i) t.p[i] = t.p[0];
    return launch_matvec(c, type_id, out, t, n_mat, x, x_stride, n_rows, n_cols, "mvq_batched");
}

// kernels.cpp:1116-1135, in the fixed order documented in moearc.h.
int moearc_matvec_f32(moearc_ctx *c, float *out, const float *w, const float *x,
                      unsigned long n_rows, unsigned long n_cols) {
    if (!c || !out || !w || !x) return ERR;
    if (n_rows == 0) return OK;
    const bool vec = (n_cols % 4 == 0) && ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x)) & 15) == 0;
    launch_scope ls(c, "mv_f32", n_rows, 1);
    k_matvec_f32<<<cdiv(n_rows, WARPS), WARPS * 32, 0, c->stream>>>(out, w, x, n_rows, n_cols, vec);
    return ls.finish();
}

}  // extern "C"
