"""Every ABI kernel on the B200, through the C ABI, against the CPU oracle.

The shapes and fixtures follow the reference's own GPU tests (kernels_gpu.rs, forward_pass_gpu.rs):
37-row matrices that are not a multiple of a work-group, scattered page tables, a planted router
tie, bit-identity where the arithmetic order is claimed identical. Each tolerance is stated
where it is used and each test prints the error it measured.
"""
import math

import numpy as np
import pytest

import oracle as O
from moearc_b200 import BadArgument, Context

pytestmark = pytest.mark.gpu

U = 2.0 ** -24


@pytest.fixture(scope="module")
def ctx():
    c = Context()
    yield c
    c.close()


def rel_err(got, want, floor=1.0):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.max(np.abs(got - want) / np.maximum(np.abs(want), floor))) if got.size else 0.0


def report(label, err, tol):
    print(f"{label}: max error {err:.3e} (tolerance {tol:.3e})")
    assert err <= tol, f"{label}: {err} > {tol}"


def synth_blocks(t, nblocks, seed):
    rng = np.random.default_rng(seed)
    if t == O.MXFP4:
        b = rng.integers(0, 256, size=(nblocks, 17), dtype=np.uint8)
        b[:, 0] = rng.integers(100, 156, size=nblocks)  # kernels_gpu.rs / common/mod.rs:71
        return b.ravel()
    if t == O.Q4_0 or t == O.Q8_0:
        bb = O.BLOCK_BYTES[t]
        b = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
        scale = (0x1000 + rng.integers(0, 0x1800, size=nblocks)).astype(np.uint16)  # common/mod.rs:48
        b[:, 0] = scale & 0xFF
        b[:, 1] = scale >> 8
        return b.ravel()
    if t in (O.Q4_K, O.Q5_K, O.Q6_K):
        # random payload (every nibble, 6-bit scale split and high-bit position), finite f16
        # deltas: d and dmin at the front of Q4_K / Q5_K, d at the end of Q6_K (common/mod.rs:50-80)
        bb = O.BLOCK_BYTES[t]
        b = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
        for off in ((208,) if t == O.Q6_K else (0, 2)):
            scale = (0x1000 + rng.integers(0, 0x1800, size=nblocks)).astype(np.uint16)
            b[:, off] = scale & 0xFF
            b[:, off + 1] = scale >> 8
        return b.ravel()
    if t == O.F32:
        return rng.uniform(-1, 1, nblocks).astype(np.float32).view(np.uint8)
    if t == O.F16:
        return rng.uniform(-1, 1, nblocks).astype(np.float16).view(np.uint8)
    if t == O.BF16:
        return O.f32_to_bf16(rng.uniform(-1, 1, nblocks).astype(np.float32)).view(np.uint8)
    raise ValueError(t)


# ---- dequant ---------------------------------------------------------------------------------

@pytest.mark.parametrize("t", [O.MXFP4, O.Q4_0, O.Q8_0, O.Q4_K, O.Q5_K, O.Q6_K, O.F32, O.F16, O.BF16])
def test_dequant_is_bit_exact(ctx, t):
    nblocks = {1: 4099, 32: 1000, 256: 128}[O.BLOCK_ELEMS[t]]
    blocks = synth_blocks(t, nblocks, 0xC0FFEE ^ t)
    want = O.dequant(t, blocks, nblocks)
    src = ctx.upload_new(blocks)
    dst = ctx.alloc_n(np.float32, want.size)
    ctx.dequant(t, dst, src, nblocks)
    got = ctx.download(dst, np.float32, want.size)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), t


def test_dequant_from_an_unaligned_source_and_to_an_unaligned_destination(ctx):
    blocks = synth_blocks(O.MXFP4, 257, 5)
    want = O.dequant(O.MXFP4, blocks, 257)
    src = ctx.upload_new(np.concatenate([np.zeros(3, np.uint8), blocks]))
    dst = ctx.alloc_n(np.float32, want.size + 1)
    lib = ctx.lib
    rc = lib.moearc_dequant(ctx.raw, O.MXFP4, dst.ptr + 4, src.ptr + 3, 257)
    assert rc == 0
    got = ctx.download(dst, np.float32, want.size + 1)[1:]
    assert np.array_equal(got, want)


def test_synthetic_mxfp4_is_identical_on_host_and_device(ctx):
    n = 4096
    want = O.synth_mxfp4(0x5EED, n)
    dst = ctx.alloc(n * 17)
    ctx.synth(dst, n, 2, 0x5EED, 1.0, -8, -4)
    assert np.array_equal(ctx.download(dst, np.uint8, n * 17), want)


@pytest.mark.parametrize("offset", [0, 1])
def test_synthetic_q4_0_is_identical_on_host_and_device(ctx, offset):
    """The decoder's Q4_0 expert banks are generated on the device; the oracle rebuilds them on
    the host. The f16 deltas (|N(0, 0.01)| rounded to nearest even) and the nibble bytes agree
    byte for byte, at an even and at an odd destination address."""
    n = 4096
    want = O.synth_q4_0(0x5EED, n, 0.01)
    dst = ctx.alloc(n * 18 + 2)
    ctx.synth(dst.view(offset, n * 18), n, 3, 0x5EED, 0.01)
    got = ctx.download(dst.view(offset, n * 18), np.uint8, n * 18)
    assert np.array_equal(got, want), f"{int(np.sum(got != want))} bytes differ"


def test_unsupported_types_are_refused(ctx):
    b = ctx.alloc(1024)
    with pytest.raises(BadArgument):
        ctx.dequant(3, b, b, 1)  # Q4_1: expanded by neither the reference nor this library
    x, o = ctx.alloc_n(np.float32, 300), ctx.alloc_n(np.float32, 4)
    with pytest.raises(BadArgument):
        ctx.matvec_q(O.Q4_K, o, b, x, 4, 300)  # kernels_gpu.rs:183: 300 is not whole super-blocks


@pytest.mark.parametrize("t", [O.Q4_K, O.Q8_0, O.F16, O.Q6_K])
def test_embed_rows_gathers_and_expands_exactly(ctx, t):
    """forward_pass_gpu.rs:201-242: the rows of the named tokens, expanded exactly as dequant
    expands them (Q4_K is OLMoE's token_embd type), and a row width that is not whole blocks
    refused."""
    n_vocab, n_embd = 50, 512
    nb_row = n_embd // O.BLOCK_ELEMS[t]
    table = synth_blocks(t, n_vocab * nb_row, 0xE3B ^ t)
    ids = np.array([7, 0, 49, 7, 23], np.uint32)
    full = O.dequant(t, table, n_vocab * nb_row).reshape(n_vocab, n_embd)
    out = ctx.alloc_n(np.float32, ids.size * n_embd)
    dt, di = ctx.upload_new(table), ctx.upload_new(ids)
    ctx.embed_rows(t, out, dt, di, ids.size, n_embd)
    got = ctx.download(out, np.float32, ids.size * n_embd).reshape(ids.size, n_embd)
    assert np.array_equal(got.view(np.uint32), full[ids].view(np.uint32))
    if O.BLOCK_ELEMS[t] > 1:
        with pytest.raises(BadArgument):
            ctx.embed_rows(t, out, dt, di, 1, 300)


# ---- matvecs ---------------------------------------------------------------------------------

@pytest.mark.parametrize("t", [O.MXFP4, O.Q4_0, O.Q8_0, O.Q4_K, O.Q5_K, O.Q6_K, O.F32, O.F16, O.BF16])
@pytest.mark.parametrize("shape", [(37, 1024), (64, 2880), (5, 96)])
def test_matvec_q_matches_the_oracle(ctx, t, shape):
    rows, cols = shape
    if cols % O.BLOCK_ELEMS[t]:
        cols = 2048 if cols == 2880 else 512  # whole 256-element super-blocks
    nb = rows * cols // O.BLOCK_ELEMS[t]
    w = synth_blocks(t, nb, 0x0BA7 + rows)
    x = np.random.default_rng(rows).uniform(-1, 1, cols).astype(np.float32)
    want = O.matvec_q(t, w, x, rows, cols)
    dw, dx, do = ctx.upload_new(w), ctx.upload_new(x), ctx.alloc_n(np.float32, rows)
    ctx.matvec_q(t, do, dw, dx, rows, cols)
    got = ctx.download(do, np.float32, rows)
    # f32 tree against a double sum: (n/32 + log2 32) U relative to the sum of |terms|
    # (kernels_gpu.rs:7-25); reported on the north-star scale |a-b| / max(|b|, 1) <= 1e-4.
    report(f"matvec t={t} {rows}x{cols}", rel_err(got, want), 1e-4)


@pytest.mark.parametrize("t", [O.MXFP4, O.Q4_0, O.Q8_0])
def test_a_batched_matvec_is_bit_identical_to_the_calls_it_replaces(ctx, t):
    """kernels_gpu.rs:493-534: batching must not move a single bit."""
    rows, cols, mats = 37, 1024, 5
    nb = rows * cols // 32
    x = np.random.default_rng(1).uniform(-1, 1, cols).astype(np.float32)
    dx = ctx.upload_new(x)
    dws, want = [], []
    for m in range(mats):
        dw = ctx.upload_new(synth_blocks(t, nb, 100 + m))
        one = ctx.alloc_n(np.float32, rows)
        ctx.matvec_q(t, one, dw, dx, rows, cols)
        want.append(ctx.download(one, np.float32, rows))
        dws.append(dw)
    out = ctx.alloc_n(np.float32, mats * rows)
    ctx.matvec_q_batched(t, out, dws, dx, 0, rows, cols)
    got = ctx.download(out, np.float32, mats * rows)
    assert np.array_equal(got, np.concatenate(want))
    assert np.any(got != 0)


def test_a_batched_matvec_gives_each_matrix_its_own_activation_when_strided(ctx):
    rows, cols, mats = 20, 512, 4
    nb = rows * cols // 32
    xs = np.random.default_rng(2).uniform(-1, 1, mats * cols).astype(np.float32)
    ws = [synth_blocks(O.Q4_0, nb, 40 + m) for m in range(mats)]
    out = ctx.alloc_n(np.float32, mats * rows)
    ctx.matvec_q_batched(O.Q4_0, out, [ctx.upload_new(w) for w in ws], ctx.upload_new(xs), cols, rows, cols)
    got = ctx.download(out, np.float32, mats * rows).reshape(mats, rows)
    for m in range(mats):
        want = O.matvec_q(O.Q4_0, ws[m], xs[m * cols:(m + 1) * cols], rows, cols)
        report(f"strided matrix {m}", rel_err(got[m], want), 1e-4)


def test_more_matrices_than_one_launch_takes_is_refused(ctx):
    w = ctx.alloc(34)
    x = ctx.alloc_n(np.float32, 32)
    out = ctx.alloc_n(np.float32, 64)
    with pytest.raises(BadArgument):
        ctx.matvec_q_batched(O.Q8_0, out, [w] * 33, x, 0, 1, 32)
    arr = (__import__("ctypes").c_void_p * 33)(*([w.ptr] * 33))
    assert ctx.lib.moearc_matvec_q_batched(ctx.raw, O.Q8_0, out.ptr, arr, 33, x.ptr, 0, 1, 32) == -2


@pytest.mark.parametrize("shape", [(32, 2880), (128, 2880), (128, 2048), (7, 13)])
def test_router_matvec_reproduces_its_documented_order_bit_for_bit(ctx, shape):
    rows, cols = shape
    rng = np.random.default_rng(cols)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    out = ctx.alloc_n(np.float32, rows)
    ctx.matvec_f32(out, ctx.upload_new(w), ctx.upload_new(x), rows, cols)
    got = ctx.download(out, np.float32, rows)
    assert np.array_equal(got, O.matvec_f32(w, x, gpu_order=True))
    report("router matvec vs double", rel_err(got, O.matvec_f32(w, x), 1e-3), 1e-4)


# ---- router ----------------------------------------------------------------------------------

@pytest.mark.parametrize("gating", [0, 1, 2])
def test_router_planted_tie_and_weights(ctx, gating):
    """kernels_gpu.rs:406-467: 6 tokens x 128 experts, k = 8, a tie at 3 and 77."""
    from test_oracle_kat import planted_tie_logits
    logits = planted_tie_logits()
    T, E = logits.shape
    K = 8
    didx, dw = ctx.alloc_n(np.uint32, T * K), ctx.alloc_n(np.float32, T * K)
    ctx.topk_router(didx, dw, ctx.upload_new(logits), T, E, K, gating)
    idx = ctx.download(didx, np.uint32, T * K).reshape(T, K)
    w = ctx.download(dw, np.float32, T * K).reshape(T, K)
    want_idx, want_w = O.topk_router(logits, K, gating)
    assert np.array_equal(idx, want_idx)
    assert idx[0, 0] == 3 and idx[0, 1] == 77
    report(f"router weights gating={gating}", float(np.abs(w - want_w).max()), (4 + 4 + E / 32 + 5 + 1) * U)
    assert np.all(np.diff(w, axis=1) <= 1e-7)


def test_router_refuses_k_above_32(ctx):
    b = ctx.alloc(4096)
    with pytest.raises(BadArgument):
        ctx.topk_router(b, b, b, 1, 16, 64, 1)
    assert ctx.lib.moearc_topk_router(ctx.raw, b.ptr, b.ptr, b.ptr, 1, 16, 33, 1) == -2


def test_router_on_many_tokens_with_random_ties(ctx):
    rng = np.random.default_rng(9)
    logits = rng.integers(-3, 4, size=(517, 32)).astype(np.float32)  # ties everywhere
    idx = ctx.alloc_n(np.uint32, 517 * 4)
    w = ctx.alloc_n(np.float32, 517 * 4)
    ctx.topk_router(idx, w, ctx.upload_new(logits), 517, 32, 4, 2)
    want_idx, _ = O.topk_router(logits, 4, 2)
    assert np.array_equal(ctx.download(idx, np.uint32, 517 * 4).reshape(517, 4), want_idx)


# ---- elementwise -----------------------------------------------------------------------------

def test_the_moe_combine_is_bit_identical_to_a_zero_and_a_run_of_axpys(ctx):
    """kernels_gpu.rs:595-628."""
    n, mats = 2048, 8
    rng = np.random.default_rng(3)
    parts = rng.uniform(-1, 1, (mats, n)).astype(np.float32)
    weights = rng.uniform(-1, 1, mats).astype(np.float32)
    dparts, dweights = ctx.upload_new(parts), ctx.upload_new(weights)
    acc = ctx.alloc_n(np.float32, n)
    ctx.zero(acc, n)
    part1 = ctx.alloc_n(np.float32, n)
    for m in range(mats):
        ctx.upload(part1, parts[m])
        ctx.axpy(acc, part1, float(weights[m]), n)
    want = ctx.download(acc, np.float32, n)
    out = ctx.alloc_n(np.float32, n)
    ctx.moe_combine(out, dparts, dweights, mats, n)
    got = ctx.download(out, np.float32, n)
    assert np.array_equal(got, want)
    emu = np.zeros(n, np.float32)
    O.lib().or_moe_combine(O.ptr(parts), O.ptr(weights), mats, n, O.ptr(emu))
    assert np.array_equal(got, emu)


def test_swiglu_over_two_halves_matches_swiglu_over_two_buffers(ctx):
    n = 4096
    gu = np.random.default_rng(4).uniform(-1, 1, 2 * n).astype(np.float32)
    a, b = ctx.alloc_n(np.float32, n), ctx.alloc_n(np.float32, n)
    ctx.swiglu(a, ctx.upload_new(gu[:n]), ctx.upload_new(gu[n:]), n)
    ctx.swiglu_halves(b, ctx.upload_new(gu), n)
    ga, gb = ctx.download(a, np.float32, n), ctx.download(b, np.float32, n)
    assert np.array_equal(ga, gb)
    want = np.zeros(n, np.float32)
    g_half, u_half = gu[:n].copy(), gu[n:].copy()  # held: the oracle reads them by address
    O.lib().or_swiglu(O.ptr(g_half), O.ptr(u_half), n, O.ptr(want))
    report("swiglu", rel_err(ga, want, 1e-6), 8 * U)


def test_swiglu_oai_matches_the_oracle(ctx):
    n = 4096
    rng = np.random.default_rng(5)
    g = (rng.standard_normal(n) * 6).astype(np.float32)
    u = (rng.standard_normal(n) * 6).astype(np.float32)
    out = ctx.alloc_n(np.float32, n)
    ctx.swiglu_oai(out, ctx.upload_new(g), ctx.upload_new(u), n, 1.702, 7.0)
    want = np.zeros(n, np.float32)
    O.lib().or_swiglu_oai(O.ptr(g), O.ptr(u), n, 1.702, 7.0, O.ptr(want))
    report("swiglu_oai", rel_err(ctx.download(out, np.float32, n), want, 1e-6), 16 * U)


def test_add_bias_id_adds_each_matrix_its_experts_bias_row(ctx):
    """kernels.cpp:1654-1670 as moe.rs:2310-2331 uses it: out[m * n_rows + r] += bias[idx[m]
    * n_rows + r], gathered by router id, repeats and a 37-row (non-multiple) stride included;
    a single f32 add per element, so bit-exact against the oracle."""
    n_expert, n_rows = 32, 37
    idx = [5, 0, 31, 5, 17, 2]
    rng = np.random.default_rng(21)
    bias = rng.uniform(-1, 1, (n_expert, n_rows)).astype(np.float32)
    base = rng.uniform(-1, 1, (len(idx), n_rows)).astype(np.float32)
    out = ctx.upload_new(base)
    ctx.add_bias_id(out, ctx.upload_new(bias), idx, n_rows)
    got = ctx.download(out, np.float32, base.size)
    want = base.ravel().copy()
    idx_a = np.asarray(idx, np.uint32)
    O.lib().or_add_bias_id(O.ptr(want), O.ptr(bias), O.ptr(idx_a), len(idx), n_rows)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(want.reshape(len(idx), n_rows), base + bias[idx])


def test_silu_and_mul_match_the_oracle(ctx):
    """reference.rs:363-366 (silu) and 700-703 (mul) over a length that is not a multiple of a
    warp; mul is one f32 product per element (bit-exact), silu goes through expf (a few ulp)."""
    n = 4099
    rng = np.random.default_rng(22)
    x = (rng.standard_normal(n) * 8).astype(np.float32)
    y = rng.uniform(-2, 2, n).astype(np.float32)
    dx, dy = ctx.upload_new(x), ctx.upload_new(y)
    out = ctx.alloc_n(np.float32, n)
    ctx.silu(out, dx, n)
    want = np.zeros(n, np.float32)
    O.lib().or_silu(O.ptr(x), n, O.ptr(want))
    report("silu", rel_err(ctx.download(out, np.float32, n), want, 1e-6), 8 * U)
    ctx.mul(out, dx, dy, n)
    O.lib().or_mul(O.ptr(x), O.ptr(y), n, O.ptr(want))
    assert np.array_equal(ctx.download(out, np.float32, n).view(np.uint32), want.view(np.uint32))


def test_quantize_f16_rounds_like_the_twin(ctx):
    """reference.rs:647-691 (round to nearest even, NaN kept, overflow to infinity, subnormals):
    every value, including the edges, gives the twin's f16 bits."""
    edge = np.array([0.0, -0.0, 65504.0, 65520.0, -65520.0, 1e9, 2.0 ** -24, 2.0 ** -25,
                     3 * 2.0 ** -26, 2.0 ** -14, 2.0 ** -14 - 2.0 ** -25, 1.0 + 2.0 ** -11,
                     1.0 + 3 * 2.0 ** -11, np.inf, -np.inf, np.nan], np.float32)
    rng = np.random.default_rng(23)
    x = np.concatenate([edge, (rng.standard_normal(5000) * 10.0 ** rng.uniform(-8, 5, 5000)).astype(np.float32)])
    n = x.size
    dst = ctx.alloc_n(np.uint16, n)
    ctx.quantize_f16(dst, ctx.upload_new(x), n)
    got = ctx.download(dst, np.uint16, n)
    want = np.array([O.lib().or_f32_to_f16(float(v)) for v in x], np.uint16)
    nan = np.isnan(x)
    assert np.array_equal(got[~nan], want[~nan])
    assert np.all((got[nan] & 0x7C00) == 0x7C00) and np.all((got[nan] & 0x03FF) != 0)


def test_rmsnorm_and_softmax_match_the_oracle(ctx):
    rng = np.random.default_rng(6)
    rows, cols = 3, 2880
    x = rng.standard_normal(rows * cols).astype(np.float32)
    wt = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    out = ctx.alloc_n(np.float32, rows * cols)
    ctx.rmsnorm(out, ctx.upload_new(x), ctx.upload_new(wt), rows, cols, 1e-5)
    want = np.zeros(rows * cols, np.float32)
    O.lib().or_rmsnorm(O.ptr(x), O.ptr(wt), rows, cols, 1e-5, O.ptr(want))
    report("rmsnorm", rel_err(ctx.download(out, np.float32, rows * cols), want), (cols / 256 + 16) * U)
    s = rng.standard_normal(5 * 200).astype(np.float32) * 4
    mask = np.zeros(5 * 200, np.float32)
    mask[3::7] = -np.inf
    sm = ctx.alloc_n(np.float32, 1000)
    ctx.softmax(sm, ctx.upload_new(s), ctx.upload_new(mask), 5, 200, 0.5)
    want = np.zeros(1000, np.float32)
    O.lib().or_softmax_ext(O.ptr(s), O.ptr(mask), 5, 200, 0.5, O.ptr(want))
    report("softmax", float(np.abs(ctx.download(sm, np.float32, 1000) - want).max()), 32 * U)


@pytest.mark.parametrize("neox", [True, False])
def test_rope_matches_the_closed_form_oracle(ctx, neox):
    T, H, D = 3, 8, 64
    rng = np.random.default_rng(7)
    src = rng.standard_normal(T * H * D).astype(np.float32)
    pos = np.array([0, 17, 8191], np.int32)
    args = (T, H, D, D, 150000.0, 1 / 32, 1.0, 1.0, 8.0, 17.0)
    out = ctx.alloc_n(np.float32, src.size)
    ctx.rope_ext(out, ctx.upload_new(src), ctx.upload_new(pos), *args, neox=neox)
    want = np.zeros(src.size, np.float32)
    O.lib().or_rope_ext(O.ptr(src), O.ptr(pos), *args, 1 if neox else 0, O.ptr(want))
    report("rope (YaRN)", float(np.abs(ctx.download(out, np.float32, src.size) - want).max()), 4 * U * 8)
    # and in place
    buf = ctx.upload_new(src)
    ctx.rope_ext(buf, buf, ctx.upload_new(pos), *args, neox=neox)
    report("rope in place", float(np.abs(ctx.download(buf, np.float32, src.size) - want).max()), 4 * U * 8)


# ---- KV cache and attention -------------------------------------------------------------------

@pytest.mark.parametrize("kv", [O.F32, O.F16, O.BF16])
def test_kv_append_writes_exactly_the_slot_it_was_given(ctx, kv):
    H, D, PT, PAGES = 3, 16, 4, 5
    dt = np.float32 if kv == O.F32 else np.uint16
    pool = PAGES * PT * H * D
    fill = np.full(pool, 0x3F80 if kv != O.F32 else -7.5, dt)
    kp, vp = ctx.upload_new(fill), ctx.upload_new(fill)
    k = np.random.default_rng(8).uniform(-1, 1, H * D).astype(np.float32)
    v = -k
    ctx.kv_append(kp, vp, ctx.upload_new(k), ctx.upload_new(v), 3, 2, H, D, PT, kv)
    want_k, want_v = fill.copy(), fill.copy()
    assert O.lib().or_kv_append(O.ptr(want_k), O.ptr(want_v), O.ptr(k), O.ptr(v), 3, 2, H, D, PT, kv) == 0
    assert np.array_equal(ctx.download(kp, dt, pool), want_k)
    assert np.array_equal(ctx.download(vp, dt, pool), want_v)


def fill_cache(ctx, table, n_kv, n_kv_heads, hd, pt, pages, kv, seed):
    """forward_pass_gpu.rs:383-428: per key, K then V from one stream, written by kv_append
    on the device and by the oracle on the host."""
    rng = O.SplitMix64(seed)
    dt = np.float32 if kv == O.F32 else np.uint16
    pool = pages * pt * n_kv_heads * hd
    kh, vh = np.zeros(pool, dt), np.zeros(pool, dt)
    dk, dv = ctx.upload_new(kh), ctx.upload_new(vh)
    row = n_kv_heads * hd
    dkt, dvt = ctx.alloc_n(np.float32, row), ctx.alloc_n(np.float32, row)
    ks = np.array([rng.unit() for _ in range(n_kv * 2 * row)], np.float32).reshape(n_kv, 2, row)
    for j in range(n_kv):
        k, v = ks[j, 0].copy(), ks[j, 1].copy()
        page, slot = int(table[j // pt]), j % pt
        ctx.upload(dkt, k)
        ctx.upload(dvt, v)
        ctx.kv_append(dk, dv, dkt, dvt, page, slot, n_kv_heads, hd, pt, kv)
        O.lib().or_kv_append(O.ptr(kh), O.ptr(vh), O.ptr(k), O.ptr(v), page, slot, n_kv_heads, hd, pt, kv)
    return dk, dv, kh, vh, rng


def run_attn(ctx, q, dk, dv, table, sinks, H, KVH, D, begin, n_kv, pt, scale, kv):
    out = ctx.alloc_n(np.float32, H * D)
    ctx.attn_decode_ext(out, ctx.upload_new(q), dk, dv, ctx.upload_new(np.asarray(table, np.uint32)),
                        None if sinks is None else ctx.upload_new(sinks), H, KVH, D, begin, n_kv, pt,
                        scale, kv)
    return ctx.download(out, np.float32, H * D)


def oracle_attn(q, kh, vh, table, sinks, H, KVH, D, begin, n_kv, pt, scale, kv):
    out = np.zeros(H * D, np.float32)
    t = np.asarray(table, np.uint32)
    rc = O.lib().or_attn_decode(O.ptr(q), O.ptr(kh), O.ptr(vh), O.ptr(t), O.ptr(sinks), H, KVH, D, begin,
                                n_kv, pt, scale, kv, O.ptr(out))
    assert rc == 0
    return out


@pytest.mark.parametrize("kv", [O.F32, O.F16, O.BF16])
def test_paged_attention_across_scattered_pages(ctx, kv):
    """forward_pass_gpu.rs:500-592: 16 heads x 128, 37 keys over pages [11, 2, 15, 7, 0]."""
    H, KVH, D, PT, PAGES, N = 16, 16, 128, 8, 16, 37
    table = [11, 2, 15, 7, 0]
    dk, dv, kh, vh, rng = fill_cache(ctx, table, N, KVH, D, PT, PAGES, kv, 0xA77E ^ kv)
    q = rng.vec_unit(H * D)
    scale = 1 / math.sqrt(D)
    got = run_attn(ctx, q, dk, dv, table, None, H, KVH, D, 0, N, PT, scale, kv)
    want = oracle_attn(q, kh, vh, table, None, H, KVH, D, 0, N, PT, scale, kv)
    tol = 8.0 * ((D / 32 + 5) * U + N * U + 8 * U) if kv == O.F32 else 1e-4
    report(f"attn kv={kv}", float(np.abs(got - want).max()), tol)


@pytest.mark.parametrize("kv", [O.F32, O.BF16])
def test_paged_attention_grouped_query_heads(ctx, kv):
    H, KVH, D, PT, PAGES, N = 8, 2, 64, 4, 6, 10
    table = [5, 1, 3]
    dk, dv, kh, vh, rng = fill_cache(ctx, table, N, KVH, D, PT, PAGES, kv, 0x6A11)
    q = rng.vec_unit(H * D)
    got = run_attn(ctx, q, dk, dv, table, None, H, KVH, D, 0, N, PT, 0.125, kv)
    want = oracle_attn(q, kh, vh, table, None, H, KVH, D, 0, N, PT, 0.125, kv)
    report(f"attn GQA 8/2 kv={kv}", float(np.abs(got - want).max()), 1e-4)
    assert not np.array_equal(got[:D], got[D:2 * D])


def test_attention_with_a_single_cached_key_returns_that_value_exactly(ctx):
    H, D, PT = 4, 32, 4
    dk, dv, kh, vh, rng = fill_cache(ctx, [1], 1, H, D, PT, 2, O.F32, 0x01E1)
    q = rng.vec_unit(H * D)
    got = run_attn(ctx, q, dk, dv, [1], None, H, H, D, 0, 1, PT, 0.125, O.F32)
    base = O.lib().or_kv_index(1, 0, 0, 0, H, D, PT)
    assert np.allclose(got, vh[base:base + H * D], rtol=1e-6, atol=0)


@pytest.mark.parametrize("kv", [O.F32, O.BF16])
def test_a_windowed_span_attends_to_the_last_keys_and_only_those(ctx, kv):
    H, KVH, D, PT, PAGES, N, WIN = 8, 2, 64, 4, 8, 21, 6
    table = [7, 0, 4, 2, 6, 1]
    dk, dv, kh, vh, rng = fill_cache(ctx, table, N, KVH, D, PT, PAGES, kv, 0x5A11)
    q = rng.vec_unit(H * D)
    got = run_attn(ctx, q, dk, dv, table, None, H, KVH, D, N - WIN, N, PT, 0.125, kv)
    want = oracle_attn(q, kh, vh, table, None, H, KVH, D, N - WIN, N, PT, 0.125, kv)
    report("attn window", float(np.abs(got - want).max()), 1e-4)
    full = run_attn(ctx, q, dk, dv, table, None, H, KVH, D, 0, N, PT, 0.125, kv)
    assert float(np.abs(got - full).max()) > 1e-3
    one = run_attn(ctx, q, dk, dv, table, None, H, KVH, D, N - 1, N, PT, 0.125, kv)
    vals = vh if kv == O.F32 else O.bf16_to_f32(vh)
    for h in range(H):
        base = O.lib().or_kv_index(table[(N - 1) // PT], (N - 1) % PT, h // 4, 0, KVH, D, PT)
        assert np.allclose(one[h * D:(h + 1) * D], vals[base:base + D], rtol=2 ** -15, atol=0)


def test_attention_refusals(ctx):
    b = ctx.alloc(1 << 16)
    bt = ctx.alloc_n(np.uint32, 4)
    with pytest.raises(BadArgument):
        ctx.attn_decode_ext(b, b, b, b, bt, None, 4, 4, 8, 4, 4, 4, 1.0, O.F32)
    with pytest.raises(BadArgument):
        ctx.attn_decode(b, b, b, b, bt, 6, 4, 8, 4, 4, 1.0, O.F32)
    lib = ctx.lib
    assert lib.moearc_attn_decode(ctx.raw, b.ptr, b.ptr, b.ptr, b.ptr, bt.ptr, None, 4, 4, 8, 4, 4, 4, 1.0, 0) == -2
    assert lib.moearc_attn_decode(ctx.raw, b.ptr, b.ptr, b.ptr, b.ptr, bt.ptr, None, 6, 4, 8, 0, 4, 4, 1.0, 0) == -2


@pytest.mark.parametrize("geom", [(64, 8, 64, 1000, 0), (64, 8, 64, 300, 172), (32, 4, 128, 777, 0)])
def test_split_k_attention_at_model_geometry_with_sinks(ctx, geom):
    """gpt-oss (64 q / 8 kv heads of 64, one windowed span) and Qwen3 (32/4 of 128), bf16 cache,
    many splits, page 32, scattered pages, per-head sinks."""
    H, KVH, D, N, begin = geom
    PT = 32
    pages = (N + PT - 1) // PT
    table = np.random.default_rng(N).permutation(pages + 3)[:pages].astype(np.uint32)
    rng = np.random.default_rng(D + N)
    kf = (rng.standard_normal(((pages + 3) * PT, KVH * D)) * 0.5).astype(np.float32)
    vf = rng.standard_normal(((pages + 3) * PT, KVH * D)).astype(np.float32)
    kh, vh = O.f32_to_bf16(kf).ravel(), O.f32_to_bf16(vf).ravel()
    q = (rng.standard_normal(H * D) * 0.5).astype(np.float32)
    sinks = rng.standard_normal(H).astype(np.float32)
    dk, dv = ctx.upload_new(kh), ctx.upload_new(vh)
    scale = 1 / math.sqrt(D)
    got = run_attn(ctx, q, dk, dv, table, sinks, H, KVH, D, begin, N, PT, scale, O.BF16)
    want = oracle_attn(q, kh, vh, table, sinks, H, KVH, D, begin, N, PT, scale, O.BF16)
    report(f"split-K attention {geom}", rel_err(got, want), 1e-4)


def test_tensor_core_peaks_of_the_block_scaled_kinds(ctx):
    """The library's own tcgen05 loop times each MMA kind: every rate is finite and positive, and
    the block-scaled kinds run at least as fast as bf16 (fp8 about twice, fp4 about four times on
    B200)."""
    rates = {k: ctx.mma_peak(k) for k in ("bf16", "mxf8", "mxf4", "mxf8_e2m1")}
    print("tensor-core peaks, TFLOP/s:", {k: round(v, 1) for k, v in rates.items()})
    assert all(np.isfinite(v) and v > 0 for v in rates.values())
    assert rates["mxf8"] >= 1.5 * rates["bf16"] and rates["mxf4"] >= 1.5 * rates["mxf8"]
