// dense.cuh — the decoder's dense bf16 projections (Q/K/V and O) as tensor-core GEMVs.
//
// The reference issues these as four matvecs plus separate RMSNorm, RoPE, KV-append and
// residual-add launches per block (crates/moearc-engine/src/moe.rs:1936-2072). Here one
// persistent kernel per projection does all of it:
//   prologue  each CTA issues its first weight copies, then builds the activation's B
//             fragments in shared memory — RMSNorm of the residual stream applied on the way
//             for Q/K/V — while those copies land;
//   body      warps stream packed 16x64 bf16 tiles with TMA bulk copies and multiply on the
//             tensor cores; the activation enters as three bf16 columns (its rounding and two
//             rounding residuals), ~24 bits of the f32 value;
//   epilogue  the last warp to finish a unit reduces the split-K partials in a fixed order
//             and either applies RoPE and writes q (f32) and K/V (bf16, into the paged cache
//             at this step's page and slot), or adds the residual.
#pragma once

#include "common.cuh"

namespace moearc {

// Packed bf16 tile: 16 rows x 64 columns = 2 KB; lane l = 4r + q holds 64 contiguous bytes,
// for each 16-column sub-block s: (row r, cols 16s+2q..+1), (row r+8, same), (row r,
// 16s+2q+8..+9), (row r+8, same) — the m16n8k16 A fragment.
constexpr int DENSE_TILE = 2048;

struct dense_rope {
    int n_q_heads, n_kv_heads, head_dim, n_rot;
    double theta_scale;
    float freq_scale, ext_factor, attn_factor, corr_lo, corr_hi;
};

struct dense_kv {
    uint16_t *k_pages, *v_pages;  // this layer's pools, bf16 [page][slot][kv_head][d]
    const unsigned *table;        // logical page -> physical page
    int page_tokens;
};

// Pack a row-major bf16 matrix [n_rows][n_cols] (n_rows % 16 == 0, n_cols % 64 == 0) into
// tiles ordered tile-row major.
int dense_pack(moearc_ctx *c, void *dst, const void *src, int n_rows, int n_cols);

struct dense_gemv;  // plan: sizes, chunking, scratch

dense_gemv *dense_create(moearc_ctx *c, int n_rows, int n_cols, int mode);
void dense_destroy(dense_gemv *g);

// mode 0 (QKV): out_q = rope(q), K/V -> cache; input = rmsnorm(h) * norm_w.
// mode 1 (residual): out = residual + W . x; input x as is.
int dense_run(dense_gemv *g, const void *w_packed, const float *in, const float *norm_w, float eps,
              float *out, const float *residual, const int *pos, const dense_rope *rope,
              const dense_kv *kv);

}  // namespace moearc
