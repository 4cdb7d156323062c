// dense.cuh — the decoder's dense bf16 projections (Q/K/V and O) as tensor-core GEMVs.
//
// The reference issues these as four matvecs plus separate RMSNorm, RoPE, KV-append and
// residual-add launches per block (crates/moearc-engine/src/moe.rs:1936-2072). Here one
// kernel per projection does all of it, one CTA per SM:
//   split     the packed tiles, in memory order, are cut into one equal contiguous range per
//             CTA and that range into one per warp, so every SM streams the same number of
//             bytes whatever the matrix shape;
//   prologue  each warp issues the bulk copies of its first tiles before waiting for the
//             previous kernel (the weights do not depend on it), so they stream while that
//             kernel finishes; after the wait the activation becomes B fragments in one pass,
//             RMSNorm of the residual stream applied on the way for Q/K/V;
//   body      warps multiply 16x64 bf16 tiles on the tensor cores; the activation enters as
//             three bf16 columns (its rounding and two rounding residuals), ~24 bits of the
//             f32 value;
//   epilogue  per-tile-row sums of the CTA's warps go to partial slots (an empty marker until
//             stored); the CTA holding a unit's first tile (a head for Q/K/V, a tile-row for O)
//             polls the unit's slots (bounded), sums them in a fixed order, empties them and
//             either applies RoPE and writes q (f32) and K/V (bf16, into the paged cache at this
//             step's page and slot), or adds the residual.
#pragma once

#include "common.cuh"

namespace moearc {

// Packed bf16 tile: 16 rows x 64 columns = 2 KB, tiles in tile-row-major order. Inside a tile,
// 16-column sub-block s holds 32 lanes x 16 bytes at 512 s + 16 l; lane l = 4r + q holds
// (row r, cols 16s+2q..+1), (row r+8, same), (row r, 16s+2q+8..+9), (row r+8, same) — the
// m16n8k16 A fragment — so a warp's 16-byte shared-memory reads of one sub-block touch every
// bank once.
constexpr int DENSE_TILE = 2048;

// NeoX RoPE of the Q and K heads: pair p of a head at position pos turns by pos * freq[p]
// (device, head_dim / 2 doubles: base^(-2p/head_dim) times the YaRN blend of the pair) and both
// outputs scale by mscale.
struct dense_rope {
    int n_q_heads, n_kv_heads, head_dim;
    const double *freq;
    double mscale;
    // QK-norm before the rotation (moe.rs:1961-1985): each q and k head RMS-normalised over its
    // head_dim values and scaled by q_norm / k_norm [head_dim] (both null: none)
    const float *q_norm = nullptr, *k_norm = nullptr;
    float norm_eps = 0.f;
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
// Reads and clears the plan's status word (0, or STATUS_WAIT_TIMEOUT when a poll gave up; then
// every partial slot is emptied again); ERR when the read fails.
int dense_status(dense_gemv *g);

// mode 0 (QKV): out_q = rope(q), K/V -> cache; input = rmsnorm(h) * norm_w.
// mode 1 (residual): out = residual + W . x; input x as is.
int dense_run(dense_gemv *g, const void *w_packed, const float *in, const float *norm_w, float eps,
              float *out, const float *residual, const int *pos, const dense_rope *rope,
              const dense_kv *kv);

}  // namespace moearc
