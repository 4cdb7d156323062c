// dequant.cu — block expansion, embedding gather, narrowing, expert gather, synthetic fills.
//
// moearc_dequant restates kernels.cpp:1009-1026 (one work-item per element there, each
// recomputing its block's scale), for every type the reference expands (F32, F16, Q8_0, Q4_K,
// Q5_K, Q6_K, MXFP4) plus Q4_0 and BF16. Here one thread expands four consecutive elements of a block
// and writes them as one 16-byte store, so a warp writes 512 contiguous bytes: the expansion
// is bound by its output stream, which is 7.5x (MXFP4) the input.
#include <cmath>

#include "common.cuh"
#include "kquant.cuh"

using namespace moearc;

namespace {

// Four consecutive elements e0..e0+3 (e0 % 4 == 0) of the block at `b`, exactly as the
// reference twin expands them (reference.rs:194-216; Q4_0 per ggml's dequantize_row_q4_0).
template <unsigned T>
__device__ __forceinline__ float4 quad(const uint8_t *b, int e0) {
    float4 r;
    if constexpr (T == T_MXFP4) {
        const float d = e8m0_half(b[0]);
        const int j = e0 & 15;
        const int sh = (e0 >= 16) ? 4 : 0;  // high nibbles are elements 16..31
        r.x = kv_mxfp4((b[1 + j] >> sh) & 15u) * d;
        r.y = kv_mxfp4((b[2 + j] >> sh) & 15u) * d;
        r.z = kv_mxfp4((b[3 + j] >> sh) & 15u) * d;
        r.w = kv_mxfp4((b[4 + j] >> sh) & 15u) * d;
    } else if constexpr (T == T_Q4_0) {
        const float d = f16_bits_to_f32((uint16_t)(b[0] | (b[1] << 8)));
        const int j = e0 & 15;
        const int sh = (e0 >= 16) ? 4 : 0;
        r.x = (float)((int)((b[2 + j] >> sh) & 15u) - 8) * d;
        r.y = (float)((int)((b[3 + j] >> sh) & 15u) - 8) * d;
        r.z = (float)((int)((b[4 + j] >> sh) & 15u) - 8) * d;
        r.w = (float)((int)((b[5 + j] >> sh) & 15u) - 8) * d;
    } else {  // Q8_0
        const float d = f16_bits_to_f32((uint16_t)(b[0] | (b[1] << 8)));
        r.x = (float)(int8_t)b[2 + e0] * d;
        r.y = (float)(int8_t)b[3 + e0] * d;
        r.z = (float)(int8_t)b[4 + e0] * d;
        r.w = (float)(int8_t)b[5 + e0] * d;
    }
    return r;
}

__device__ __forceinline__ void store4(float *dst, size_t i, float4 v, bool vec) {
    if (vec) {
        *reinterpret_cast<float4 *>(dst + i) = v;
    } else {
        dst[i] = v.x;
        dst[i + 1] = v.y;
        dst[i + 2] = v.z;
        dst[i + 3] = v.w;
    }
}

// Block formats: `rows` rows of `nb` blocks each, row r starting at src + row_off(r).
// For a flat dequant rows = 1 and ids = nullptr; for the embedding gather each row is the
// table row of one token id.
template <unsigned T, int BB>
__global__ void k_dequant_blocks(float *__restrict__ dst, const uint8_t *__restrict__ src,
                                 const unsigned *__restrict__ ids, size_t rows, size_t nb,
                                 bool vec) {
    const size_t quads_per_row = nb * 8;
    const size_t total = rows * quads_per_row;
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < total;
         g += (size_t)gridDim.x * blockDim.x) {
        const size_t r = g / quads_per_row;
        const size_t qi = g - r * quads_per_row;
        const size_t blk = qi >> 3;
        const int e0 = (int)(qi & 7) * 4;
        const size_t row = ids ? (size_t)ids[r] : r;
        const uint8_t *b = src + (row * nb + blk) * BB;
        store4(dst, r * nb * 32 + blk * 32 + e0, quad<T>(b, e0), vec);
    }
}

// K-quant super-blocks: one thread expands eight consecutive elements (32 threads a block).
template <unsigned T, int BB>
__global__ void k_dequant_kq(float *__restrict__ dst, const uint8_t *__restrict__ src,
                             const unsigned *__restrict__ ids, size_t rows, size_t nb, bool vec) {
    const size_t per_row = nb * 32;
    const size_t total = rows * per_row;
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < total;
         g += (size_t)gridDim.x * blockDim.x) {
        const size_t r = g / per_row;
        const size_t gi = g - r * per_row;
        const size_t blk = gi >> 5;
        const int e0 = (int)(gi & 31) * 8;
        const size_t row = ids ? (size_t)ids[r] : r;
        float v[8];
        kq_decode8<T>(src + (row * nb + blk) * BB, e0, v);
        const size_t o = r * nb * 256 + blk * 256 + e0;
        store4(dst, o, make_float4(v[0], v[1], v[2], v[3]), vec);
        store4(dst, o + 4, make_float4(v[4], v[5], v[6], v[7]), vec);
    }
}

// One-element "blocks": f32, f16, bf16.
template <unsigned T>
__global__ void k_dequant_scalar(float *__restrict__ dst, const uint8_t *__restrict__ src,
                                 const unsigned *__restrict__ ids, size_t rows, size_t n) {
    const size_t total = rows * n;
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < total;
         g += (size_t)gridDim.x * blockDim.x) {
        const size_t r = g / n, i = g - r * n;
        const size_t e = (ids ? (size_t)ids[r] : r) * n + i;
        float v;
        if constexpr (T == T_F32) v = reinterpret_cast<const float *>(src)[e];
        else if constexpr (T == T_F16) v = f16_bits_to_f32(reinterpret_cast<const uint16_t *>(src)[e]);
        else v = bf16_bits_to_f32(reinterpret_cast<const uint16_t *>(src)[e]);
        dst[g] = v;
    }
}

unsigned grid_for(moearc_ctx *c, size_t work, unsigned threads) {
    size_t g = (work + threads - 1) / threads;
    const size_t cap = (size_t)c->sm_count * 32;
    return (unsigned)(g < cap ? (g ? g : 1) : cap);
}

int launch_expand(moearc_ctx *c, unsigned t, float *dst, const uint8_t *src, const unsigned *ids,
                  size_t rows, size_t n_per_row, const char *what) {
    launch_scope ls(c, what, rows, 1);
    const bool vec = (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
    const unsigned th = 256;
    if (block_elems(t) == 256) {
        const size_t nb = n_per_row / 256;
        const unsigned g = grid_for(c, rows * nb * 32, th);
        switch (t) {
        case T_Q4_K: k_dequant_kq<T_Q4_K, 144><<<g, th, 0, c->stream>>>(dst, src, ids, rows, nb, vec); break;
        case T_Q5_K: k_dequant_kq<T_Q5_K, 176><<<g, th, 0, c->stream>>>(dst, src, ids, rows, nb, vec); break;
        default: k_dequant_kq<T_Q6_K, 210><<<g, th, 0, c->stream>>>(dst, src, ids, rows, nb, vec); break;
        }
    } else if (block_elems(t) == 32) {
        const size_t nb = n_per_row / 32;
        const unsigned g = grid_for(c, rows * nb * 8, th);
        switch (t) {
        case T_MXFP4: k_dequant_blocks<T_MXFP4, 17><<<g, th, 0, c->stream>>>(dst, src, ids, rows, nb, vec); break;
        case T_Q4_0: k_dequant_blocks<T_Q4_0, 18><<<g, th, 0, c->stream>>>(dst, src, ids, rows, nb, vec); break;
        default: k_dequant_blocks<T_Q8_0, 34><<<g, th, 0, c->stream>>>(dst, src, ids, rows, nb, vec); break;
        }
    } else {
        const unsigned g = grid_for(c, rows * n_per_row, th);
        switch (t) {
        case T_F32: k_dequant_scalar<T_F32><<<g, th, 0, c->stream>>>(dst, src, ids, rows, n_per_row); break;
        case T_F16: k_dequant_scalar<T_F16><<<g, th, 0, c->stream>>>(dst, src, ids, rows, n_per_row); break;
        default: k_dequant_scalar<T_BF16><<<g, th, 0, c->stream>>>(dst, src, ids, rows, n_per_row); break;
        }
    }
    return ls.finish();
}

__global__ void k_to_f16(uint16_t *dst, const float *src, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = __half_as_ushort(__float2half_rn(src[i]));
}
__global__ void k_to_bf16(uint16_t *dst, const float *src, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = f32_to_bf16_bits(src[i]);
}

// ---- synthetic fills (SplitMix64, counter-based) -----------------------------------------

__device__ __forceinline__ uint64_t sm64_at(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ double normal_at(uint64_t seed, size_t i) {
    const uint64_t a = sm64_at(seed, 2 * (i / 2)), b = sm64_at(seed, 2 * (i / 2) + 1);
    const double u1 = ((double)(a >> 11) + 1.0) * 0x1.0p-53;
    const double u2 = (double)(b >> 11) * 0x1.0p-53;
    const double r = sqrt(-2.0 * log(u1));
    double s, co;
    sincospi(2.0 * u2, &s, &co);
    return (i & 1) ? r * s : r * co;
}

__global__ void k_synth(uint8_t *dst, size_t n, unsigned kind, uint64_t seed, float sigma, int lo,
                        int hi) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        if (kind == 0) {
            reinterpret_cast<float *>(dst)[i] = (float)(normal_at(seed, i) * (double)sigma);
        } else if (kind == 4) {
            reinterpret_cast<float *>(dst)[i] = (float)(1.0 + normal_at(seed, i) * (double)sigma);
        } else if (kind == 1) {
            reinterpret_cast<uint16_t *>(dst)[i] = f32_to_bf16_bits((float)(normal_at(seed, i) * (double)sigma));
        } else if (kind == 2) {
            uint8_t *p = dst + i * 17;
            const uint64_t r0 = sm64_at(seed, 3 * i), r1 = sm64_at(seed, 3 * i + 1), r2 = sm64_at(seed, 3 * i + 2);
            p[0] = (uint8_t)(127 + lo + (int)(r0 % (uint64_t)(hi - lo + 1)));
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                p[1 + j] = (uint8_t)(r1 >> (8 * j));
                p[9 + j] = (uint8_t)(r2 >> (8 * j));
            }
        } else {
            uint8_t *p = dst + i * 18;
            const uint64_t r0 = sm64_at(seed, 3 * i), r1 = sm64_at(seed, 3 * i + 1), r2 = sm64_at(seed, 3 * i + 2);
            const double u1 = ((double)(r0 >> 32) + 1.0) * 0x1.0p-32;
            const double u2 = (double)(r0 & 0xFFFFFFFFu) * 0x1.0p-32;
            const double z = sqrt(-2.0 * log(u1)) * cospi(2.0 * u2);
            const uint16_t d = __half_as_ushort(__float2half_rn((float)fabs(z * (double)sigma)));
            // the block's nine 16-bit words: the delta, then the nibble bytes of r1 and r2 in
            // little-endian order; a block is 18 bytes, so on an even destination every word
            // is 2-byte aligned and goes out as one store
            uint16_t w[9];
            w[0] = d;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                w[1 + j] = (uint16_t)(r1 >> (16 * j));
                w[5 + j] = (uint16_t)(r2 >> (16 * j));
            }
            if ((reinterpret_cast<uintptr_t>(p) & 1) == 0) {
#pragma unroll
                for (int j = 0; j < 9; ++j) reinterpret_cast<uint16_t *>(p)[j] = w[j];
            } else {
#pragma unroll
                for (int j = 0; j < 9; ++j) {
                    p[2 * j] = (uint8_t)w[j];
                    p[2 * j + 1] = (uint8_t)(w[j] >> 8);
                }
            }
        }
    }
}

}  // namespace

extern "C" {

// kernels.cpp:1009-1026.
int moearc_dequant(moearc_ctx *c, unsigned int type_id, float *dst, const void *src,
                   unsigned long nblocks) {
    if (!c || !dst || !src) return ERR;
    if (!block_bytes(type_id)) return ERR_ARG;
    if (nblocks == 0) return OK;
    return launch_expand(c, type_id, dst, static_cast<const uint8_t *>(src), nullptr, 1,
                         (size_t)nblocks * block_elems(type_id), "dequant");
}

// kernels.cpp:1749-1770: rows must start on a block boundary.
int moearc_embed_rows(moearc_ctx *c, unsigned int type_id, float *out, const void *table,
                      const unsigned int *token_ids, unsigned long n_tokens,
                      unsigned long n_embd) {
    if (!c || !out || !table || !token_ids) return ERR;
    if (!block_bytes(type_id)) return ERR_ARG;
    if (n_embd == 0 || n_embd % (unsigned long)block_elems(type_id)) return ERR_ARG;
    if (n_tokens == 0) return OK;
    return launch_expand(c, type_id, out, static_cast<const uint8_t *>(table), token_ids, n_tokens,
                         n_embd, "embed_rows");
}

// kernels.cpp:1727-1735: f32 -> f16, round to nearest even.
int moearc_quantize_f16(moearc_ctx *c, void *dst, const float *src, unsigned long n) {
    if (!c || !dst || !src) return ERR;
    if (n == 0) return OK;
    launch_scope ls(c, "quantize_f16", n, 1);
    k_to_f16<<<grid_for(c, n, 256), 256, 0, c->stream>>>(static_cast<uint16_t *>(dst), src, n);
    return ls.finish();
}

int moearc_x_quantize_bf16(moearc_ctx *c, void *dst, const float *src, unsigned long n) {
    if (!c || !dst || !src) return ERR;
    if (n == 0) return OK;
    launch_scope ls(c, "quantize_bf16", n, 1);
    k_to_bf16<<<grid_for(c, n, 256), 256, 0, c->stream>>>(static_cast<uint16_t *>(dst), src, n);
    return ls.finish();
}

// kernels.cpp:976-998: gather `count` pool slots into a packed buffer. The reference uploads
// the index list and launches a word copy; here each slot is one device-to-device copy on the
// stream, with the host index list read directly.
int moearc_gather_experts(moearc_ctx *c, void *dst, const void *pool, const unsigned int *idx,
                          unsigned int count, unsigned long slot_bytes) {
    if (!c || !dst || !pool || !idx) return ERR;
    for (unsigned i = 0; i < count; ++i) {
        if (cudaMemcpyAsync(static_cast<uint8_t *>(dst) + (size_t)i * slot_bytes,
                            static_cast<const uint8_t *>(pool) + (size_t)idx[i] * slot_bytes,
                            slot_bytes, cudaMemcpyDeviceToDevice, c->stream) != cudaSuccess)
            return ERR;
    }
    return OK;
}

int moearc_x_synth(moearc_ctx *c, void *dst, unsigned long n, unsigned int kind,
                   unsigned long long seed, float sigma, int lo, int hi) {
    if (!c || !dst) return ERR;
    if (kind > 4 || (kind == 2 && hi < lo)) return ERR_ARG;
    if (n == 0) return OK;
    launch_scope ls(c, "synth", n, kind);
    k_synth<<<grid_for(c, n, 256), 256, 0, c->stream>>>(static_cast<uint8_t *>(dst), n, kind, seed,
                                                        sigma, lo, hi);
    return ls.finish();
}

}  // extern "C"
