"""The CPU oracle against the reference's own known answers, and against hand-computed blocks.

The reference's CPU twin (reference.rs) cannot be run here — it is Rust and there is no
toolchain — so the oracle is pinned to the values the reference's own tests assert, extracted
from their source text into tests/golden/reference_kats.json by tests/golden/make_golden.py,
and to blocks worked out by hand from the format definitions for the formats the reference
never tested (MXFP4, Q4_0, bf16).
"""
import json
import math
import os
import struct

import numpy as np
import pytest

import oracle as O

KATS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))["kats"]


def f32_bits(v: float) -> int:
    return struct.unpack("<I", struct.pack("<f", v))[0]


# ---- scalar formats --------------------------------------------------------------------------

def test_f16_kats_from_reference_rs():
    lib = O.lib()
    assert len(KATS["f16_to_f32"]) >= 10
    for kat in KATS["f16_to_f32"]:
        got = lib.or_f16_to_f32(kat["bits"])
        if kat["value"] == "infinite":
            assert math.isinf(got), kat
        elif kat["value"] == "nan":
            assert math.isnan(got), kat
        else:
            assert got == kat["value"], kat
    # the signed zero: reference.rs:883 asserts -0.0
    assert f32_bits(lib.or_f16_to_f32(0x8000)) == 0x80000000


def test_f16_round_trip_every_bit_pattern():
    """forward_pass_gpu.rs:75: narrowing undoes widening on all 65536 patterns, NaNs aside."""
    lib = O.lib()
    n = 0
    for h in range(65536):
        v = lib.or_f16_to_f32(h)
        if math.isnan(v):
            assert math.isnan(lib.or_f16_to_f32(lib.or_f32_to_f16(v)))
            continue
        assert lib.or_f32_to_f16(v) == h, hex(h)
        n += 1
    assert n == 65536 - 2046


def test_f16_narrowing_rounds_to_nearest_even():
    lib = O.lib()
    # 1 + 2^-11 is exactly half way between 1.0 and the next half: ties to even -> 1.0
    assert lib.or_f32_to_f16(1.0 + 2.0 ** -11) == 0x3C00
    # 1 + 3*2^-11 ties between 0x3C01 and 0x3C02 -> even 0x3C02
    assert lib.or_f32_to_f16(1.0 + 3 * 2.0 ** -11) == 0x3C02
    assert lib.or_f32_to_f16(70000.0) == 0x7C00          # overflow to infinity
    assert lib.or_f32_to_f16(2.0 ** -25) == 0x0000        # exact tie at half the smallest subnormal
    assert lib.or_f32_to_f16(2.0 ** -25 * 1.5) == 0x0001  # rounds up to the smallest subnormal
    assert lib.or_f32_to_f16(65519.0) == 0x7BFF           # below the rounding boundary
    assert lib.or_f32_to_f16(65520.0) == 0x7C00           # at it


def test_bf16_rounding_and_nan():
    lib = O.lib()
    assert lib.or_f32_to_bf16(1.0) == 0x3F80
    assert lib.or_bf16_to_f32(0x3F80) == 1.0
    one_and_tie = struct.unpack("<f", struct.pack("<I", 0x3F808000))[0]
    assert lib.or_f32_to_bf16(one_and_tie) == 0x3F80      # tie to even (down)
    odd_tie = struct.unpack("<f", struct.pack("<I", 0x3F818000))[0]
    assert lib.or_f32_to_bf16(odd_tie) == 0x3F82          # tie to even (up)
    assert lib.or_f32_to_bf16(float("inf")) == 0x7F80
    nan = struct.unpack("<f", struct.pack("<I", 0x7F800001))[0]
    assert (lib.or_f32_to_bf16(nan) & 0x7FFF) > 0x7F80    # a NaN stays a NaN
    # vectorised twin used by the tests agrees with the C one
    xs = O.synth_normal_f32(5, 4096, 3.0)
    want = np.array([lib.or_f32_to_bf16(float(v)) for v in xs], np.uint16)
    assert np.array_equal(O.f32_to_bf16(xs), want)


def test_e8m0_half_including_the_subnormal_arm():
    lib = O.lib()
    assert lib.or_e8m0_half(128) == 1.0
    assert lib.or_e8m0_half(127) == 0.5
    assert lib.or_e8m0_half(2) == 2.0 ** -126
    assert lib.or_e8m0_half(1) == 2.0 ** -127            # subnormal
    assert lib.or_e8m0_half(0) == 2.0 ** -128            # subnormal
    assert lib.or_e8m0_half(255) == 2.0 ** 127


# ---- block formats ---------------------------------------------------------------------------

def test_block_sizes_match_the_reference():
    lib = O.lib()
    bb = KATS["block_bytes"]
    assert lib.or_block_bytes(O.Q8_0) == bb["Q80"]["bytes"] == 34
    assert lib.or_block_bytes(O.MXFP4) == 17            # reference.rs:86-87
    assert lib.or_block_bytes(O.Q4_0) == 18             # crates/moearc-model/src/quant.rs:54
    assert lib.or_block_elems(O.MXFP4) == lib.or_block_elems(O.Q4_0) == 32
    # reference.rs:896-905: the K-quant super-blocks ggml asserts, 256 elements each
    QK_K = 256
    assert lib.or_block_bytes(O.Q4_K) == 2 + 2 + 12 + QK_K // 2 == 144
    assert lib.or_block_bytes(O.Q5_K) == 2 + 2 + 12 + QK_K // 8 + QK_K // 2 == 176
    assert lib.or_block_bytes(O.Q6_K) == 2 + QK_K // 16 + 3 * QK_K // 4 == 210
    assert lib.or_block_elems(O.Q4_K) == lib.or_block_elems(O.Q5_K) == lib.or_block_elems(O.Q6_K) == QK_K


def test_mxfp4_block_by_hand():
    # scale byte 127 -> d = 2^(127-128) = 0.5, so each element is the true E2M1 value.
    qs = [(j & 0xF) | ((15 - j) << 4) for j in range(16)]
    blk = np.array([127] + qs, np.uint8)
    e2m1 = [0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6]
    want = np.zeros(32, np.float32)
    for j in range(16):
        want[j] = e2m1[j]             # low nibble -> element j
        want[j + 16] = e2m1[15 - j]   # high nibble -> element j + 16 (split halves)
    got = O.dequant(O.MXFP4, blk, 1)
    assert np.array_equal(got, want)
    # a larger scale multiplies exactly
    blk[0] = 130  # d = 4
    assert np.array_equal(O.dequant(O.MXFP4, blk, 1), want * 8)


def test_q4_0_block_by_hand():
    d = 0.125  # exact in f16: 0x3000
    qs = [(j & 0xF) | (((j + 3) & 0xF) << 4) for j in range(16)]
    blk = np.array([0x00, 0x30] + qs, np.uint8)
    want = np.zeros(32, np.float32)
    for j in range(16):
        want[j] = ((j & 0xF) - 8) * d
        want[j + 16] = (((j + 3) & 0xF) - 8) * d
    assert np.array_equal(O.dequant(O.Q4_0, blk, 1), want)


def test_a_zero_scale_block_dequantises_to_zero():
    """reference.rs:907-920 for the formats with an f16 delta (Q6_K keeps its at the end,
    Q4_K / Q5_K keep d and dmin at the front): a block at a wrong offset would not collapse."""
    for t in (O.Q8_0, O.Q4_0, O.Q4_K, O.Q5_K, O.Q6_K):
        blk = np.full(O.BLOCK_BYTES[t], 0xAB, np.uint8)
        if t == O.Q6_K:
            blk[208:210] = 0
        elif t in (O.Q4_K, O.Q5_K):
            blk[0:4] = 0
        else:
            blk[0:2] = 0
        assert np.all(O.dequant(t, blk, 1) == 0.0), t


def _scale_min_bytes(pairs):
    """The 12 packed bytes that give sub-block j the (6-bit scale, 6-bit min) pairs[j]: the
    inverse of ggml's get_scale_min_k4."""
    q = [0] * 12
    for j, (sc, m) in enumerate(pairs):
        if j < 4:
            q[j] |= sc & 63
            q[j + 4] |= m & 63
        else:
            q[j + 4] |= (sc & 15) | ((m & 15) << 4)
            q[j - 4] |= (sc >> 4) << 6
            q[j] |= (m >> 4) << 6
    return q


def test_q4_k_and_q5_k_blocks_by_hand():
    """Element 64r + 32h + l of a Q4_K super-block is (d * scale) * q - (dmin * min) of
    sub-block 2r + h, q the low (h = 0) or high (h = 1) nibble of byte l of run r (reference.rs:
    218-243); Q5_K adds 16 where bit 2r + h of high-plane byte l is set (reference.rs:245-276).
    Scales 4-7 exercise the split six-bit encoding."""
    pairs = [(1, 0), (2, 1), (3, 2), (63, 63), (17, 33), (40, 5), (9, 62), (32, 16)]
    d, dmin = 0.5, 0.25  # f16 0x3800, 0x3400
    qs = np.array([(l % 16) | (((l * 7) % 16) << 4) for l in range(32)] * 4, np.uint8)
    for r in range(4):
        qs[32 * r:32 * r + 32] = np.roll(qs[32 * r:32 * r + 32], r)
    qh = np.array([(l * 37) & 0xFF for l in range(32)], np.uint8)
    head = np.array([0x00, 0x38, 0x00, 0x34] + _scale_min_bytes(pairs), np.uint8)
    for t in (O.Q4_K, O.Q5_K):
        blk = np.concatenate([head, qh, qs]) if t == O.Q5_K else np.concatenate([head, qs])
        want = np.zeros(256, np.float32)
        for r in range(4):
            for h in range(2):
                sc, m = pairs[2 * r + h]
                for l in range(32):
                    byte = int(qs[32 * r + l])
                    q = (byte >> 4) if h else (byte & 15)
                    if t == O.Q5_K and (int(qh[l]) >> (2 * r + h)) & 1:
                        q += 16
                    want[64 * r + 32 * h + l] = np.float32(np.float32(d * sc) * np.float32(q)) - np.float32(dmin * m)
        assert np.array_equal(O.dequant(t, blk, 1), want), t


def test_q6_k_block_by_hand():
    """Element 128n + 32k + l of a Q6_K super-block: low four bits from byte l (+32 for odd k)
    of half n's low bytes (high nibble for k >= 2), two high bits from bits 2k, 2k+1 of half n's
    high byte l, minus 32, times d times int8 scale 2k + l/16 of the half (reference.rs:278-300)."""
    rng = np.random.default_rng(6)
    blk = rng.integers(0, 256, 210, dtype=np.uint8)
    blk[208:210] = [0x00, 0x30]  # d = 0.125
    want = np.zeros(256, np.float32)
    for n in range(2):
        ql, qh, sc = blk[64 * n:64 * n + 64], blk[128 + 32 * n:160 + 32 * n], blk[192 + 8 * n:200 + 8 * n].view(np.int8)
        for k in range(4):
            for l in range(32):
                lo = int(ql[l + 32 * (k & 1)])
                q = ((lo >> 4) if k >= 2 else (lo & 15)) | (((int(qh[l]) >> (2 * k)) & 3) << 4)
                want[128 * n + 32 * k + l] = np.float32(0.125 * int(sc[2 * k + l // 16])) * np.float32(q - 32)
    assert np.array_equal(O.dequant(O.Q6_K, blk, 1), want)


def test_synthetic_mxfp4_matches_the_spec():
    blocks = O.synth_mxfp4(1234, 4096).reshape(4096, 17)
    assert blocks[:, 0].min() == 119 and blocks[:, 0].max() == 123  # e in [-8, -4]
    nib = np.concatenate([blocks[:, 1:] & 0xF, blocks[:, 1:] >> 4]).ravel()
    counts = np.bincount(nib, minlength=16)
    assert counts.min() > 0.9 * counts.mean()  # all 16 codes, near uniform


def test_synthetic_q4_0_scales_are_half_normal():
    blocks = O.synth_q4_0(77, 20000, 0.01).reshape(20000, 18)
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    assert d.min() >= 0
    assert abs(d.mean() - 0.01 * math.sqrt(2 / math.pi)) < 3e-4


# ---- matvec ----------------------------------------------------------------------------------

def test_matvec_q_is_dequant_then_double_dot():
    rng = np.random.default_rng(0)
    w = O.synth_mxfp4(9, 37 * 8)  # 37 rows x 256 cols
    x = rng.standard_normal(256).astype(np.float32)
    got = O.matvec_q(O.MXFP4, w, x, 37, 256)
    full = O.dequant(O.MXFP4, w, 37 * 8).reshape(37, 256).astype(np.float64)
    want = (full @ x.astype(np.float64)).astype(np.float32)
    assert np.array_equal(got, want)


def test_gpu_order_matvec_is_close_to_the_double_one():
    rng = np.random.default_rng(1)
    w = rng.standard_normal((32, 2880)).astype(np.float32) * 0.02
    x = rng.standard_normal(2880).astype(np.float32)
    a = O.matvec_f32(w, x, gpu_order=True)
    b = O.matvec_f32(w, x, gpu_order=False)
    scale = np.abs(w).astype(np.float64) @ np.abs(x).astype(np.float64)
    assert np.all(np.abs(a - b) <= (2880 / 32 + 5) * 2.0 ** -24 * scale)


# ---- router ----------------------------------------------------------------------------------

GATING = {"Softmax": 0, "SoftmaxNormalised": 1, "SoftmaxAfterTopK": 2}


def test_router_small_kat():
    """reference.rs:922-930: the two 4.0s tie-break by index, weights sum to one."""
    kat = KATS["router_small"]
    logits = np.array(kat["logits"], np.float32).reshape(1, -1)
    idx, w = O.topk_router(logits, kat["k"], GATING[kat["gating"]])
    assert idx[0].tolist() == kat["idx"]
    assert abs(float(w.sum()) - 1.0) < 1e-6
    assert w[0, 0] > w[0, 1]


def planted_tie_logits() -> np.ndarray:
    kat = KATS["router_planted_tie"]
    rng = O.SplitMix64(kat["seed"])
    logits = np.array([np.float32(rng.unit()) * np.float32(kat["unit_scale"])
                       for _ in range(kat["tokens"] * kat["experts"])], np.float32)
    for i, v in kat["ties"]:
        logits[i] = v
    return logits.reshape(kat["tokens"], kat["experts"])


@pytest.mark.parametrize("gating", [0, 1, 2])
def test_router_planted_tie(gating):
    """kernels_gpu.rs:406-467 on the oracle: the lower id wins the tie, weights descend."""
    kat = KATS["router_planted_tie"]
    logits = planted_tie_logits()
    idx, w = O.topk_router(logits, kat["k"], gating)
    assert idx[0, 0] == kat["expect_first"][0] and idx[0, 1] == kat["expect_first"][1]
    assert np.all(np.diff(w, axis=1) <= 1e-7)
    if gating != 0:
        assert np.all(np.abs(w.sum(axis=1) - 1.0) < 1e-5)
    # selection is by logit: the chosen set is exactly the k largest
    for t in range(kat["tokens"]):
        assert set(idx[t].tolist()) == set(np.argsort(-logits[t], kind="stable")[: kat["k"]].tolist())


def test_gating_after_topk_is_a_softmax_of_the_selected_logits():
    logits = np.array([[1.0, 3.0, 2.0, -1.0, 0.5]], np.float32)
    idx, w = O.topk_router(logits, 2, 2)
    sel = logits[0, idx[0]].astype(np.float64)
    e = np.exp(sel - sel.max())
    assert np.allclose(w[0], e / e.sum(), rtol=1e-6)


# ---- activations, combine ---------------------------------------------------------------------

def test_swiglu_oai_clamps_as_written():
    lib = O.lib()
    g = np.array([10.0, -10.0, 0.0, 1.0], np.float32)
    u = np.array([-10.0, 10.0, 0.0, 0.0], np.float32)
    out = np.zeros(4, np.float32)
    lib.or_swiglu_oai(O.ptr(g), O.ptr(u), 4, 1.702, 7.0, O.ptr(out))
    sig = lambda v: 1 / (1 + math.exp(-v))
    assert out[0] == pytest.approx(7 * sig(1.702 * 7) * (-6), rel=1e-6)   # gate clamped above
    assert out[1] == pytest.approx(-10 * sig(-17.02) * 8, rel=1e-5)     # gate not clamped below
    assert out[2] == 0.0
    assert out[3] == pytest.approx(sig(1.702), rel=1e-6)                 # up of 0 passes the gate


def test_moe_combine_is_the_fused_axpy_chain():
    rng = np.random.default_rng(2)
    parts = rng.standard_normal((8, 2048)).astype(np.float32)
    w = rng.standard_normal(8).astype(np.float32)
    out = np.zeros(2048, np.float32)
    O.lib().or_moe_combine(O.ptr(parts), O.ptr(w), 8, 2048, O.ptr(out))
    acc = np.zeros(2048, np.float64)
    for m in range(8):
        acc += np.float64(w[m]) * parts[m]
    assert np.allclose(out, acc, atol=1e-5)


# ---- attention -------------------------------------------------------------------------------

def _cache(case_seed, n_kv, n_kv_heads, head_dim, page_tokens, n_pages, table, kv_type):
    """Fill a pool the way forward_pass_gpu.rs:383-428 does: per key, K then V from one stream."""
    rng = O.SplitMix64(case_seed)
    esz = 4 if kv_type == O.F32 else 2
    pool = n_pages * page_tokens * n_kv_heads * head_dim
    dt = np.float32 if kv_type == O.F32 else np.uint16
    kp = np.zeros(pool, dt)
    vp = np.zeros(pool, dt)
    row = n_kv_heads * head_dim
    for j in range(n_kv):
        k = rng.vec_unit(row)
        v = rng.vec_unit(row)
        rc = O.lib().or_kv_append(O.ptr(kp), O.ptr(vp), O.ptr(k), O.ptr(v), table[j // page_tokens],
                                  j % page_tokens, n_kv_heads, head_dim, page_tokens, kv_type)
        assert rc == 0
    return kp, vp, rng


def test_single_key_attention_returns_v_exactly():
    """forward_pass_gpu.rs:676: softmax over one score is 1, so the output is V."""
    table = np.array([1], np.uint32)
    kp, vp, rng = _cache(0x01E1, 1, 4, 32, 4, 2, table, O.F32)
    q = rng.vec_unit(4 * 32)
    out = np.zeros(4 * 32, np.float32)
    rc = O.lib().or_attn_decode(O.ptr(q), O.ptr(kp), O.ptr(vp), O.ptr(table), None, 4, 4, 32, 0, 1,
                                4, 0.125, O.F32, O.ptr(out))
    assert rc == 0
    base = O.lib().or_kv_index(1, 0, 0, 0, 4, 32, 4)
    assert np.array_equal(out, vp[base:base + 128])


def test_attention_sink_drains_mass():
    table = np.array([0, 1], np.uint32)
    kp, vp, rng = _cache(7, 5, 2, 16, 4, 2, table, O.F32)
    q = rng.vec_unit(4 * 16)
    a = np.zeros(64, np.float32)
    b = np.zeros(64, np.float32)
    sinks = np.full(4, 50.0, np.float32)  # a sink far above every score takes all the mass
    O.lib().or_attn_decode(O.ptr(q), O.ptr(kp), O.ptr(vp), O.ptr(table), None, 4, 2, 16, 0, 5, 4,
                           0.25, O.F32, O.ptr(a))
    O.lib().or_attn_decode(O.ptr(q), O.ptr(kp), O.ptr(vp), O.ptr(table), O.ptr(sinks), 4, 2, 16, 0,
                           5, 4, 0.25, O.F32, O.ptr(b))
    assert np.abs(a).max() > 0.05 and np.abs(b).max() < 1e-15


def test_attention_refusals():
    """forward_pass_gpu.rs:874/890: an empty span and n_heads % n_kv_heads != 0 are refused."""
    z = np.zeros(4096, np.float32)
    t = np.zeros(4, np.uint32)
    o = np.zeros(64, np.float32)
    L = O.lib()
    assert L.or_attn_decode(O.ptr(z), O.ptr(z), O.ptr(z), O.ptr(t), None, 4, 4, 8, 4, 4, 4, 1.0, 0,
                            O.ptr(o)) == -2
    assert L.or_attn_decode(O.ptr(z), O.ptr(z), O.ptr(z), O.ptr(t), None, 6, 4, 8, 0, 4, 4, 1.0, 0,
                            O.ptr(o)) == -2


def test_kv_append_writes_only_its_slot():
    n_h, d, pt, pages = 3, 16, 4, 5
    pool = pages * pt * n_h * d
    kp = np.full(pool, -7.5, np.float32)
    vp = np.full(pool, -7.5, np.float32)
    k = np.arange(n_h * d, dtype=np.float32)
    v = -k
    assert O.lib().or_kv_append(O.ptr(kp), O.ptr(vp), O.ptr(k), O.ptr(v), 3, 2, n_h, d, pt, 0) == 0
    base = O.lib().or_kv_index(3, 2, 0, 0, n_h, d, pt)
    assert np.array_equal(kp[base:base + n_h * d], k)
    assert kp[base - 1] == -7.5 and kp[base + n_h * d] == -7.5
    assert np.count_nonzero(kp != -7.5) == n_h * d  # nothing outside the slot moved


def test_window_of_one_key_is_that_value():
    table = np.array([7, 0, 4, 2, 6, 1], np.uint32)
    kp, vp, rng = _cache(0x5A11, 21, 2, 64, 4, 8, table, O.F32)
    q = rng.vec_unit(8 * 64)
    out = np.zeros(8 * 64, np.float32)
    assert O.lib().or_attn_decode(O.ptr(q), O.ptr(kp), O.ptr(vp), O.ptr(table), None, 8, 2, 64,
                                  20, 21, 4, 0.125, 0, O.ptr(out)) == 0
    for h in range(8):
        base = O.lib().or_kv_index(int(table[20 // 4]), 20 % 4, h // 4, 0, 2, 64, 4)
        assert np.array_equal(out[h * 64:(h + 1) * 64], vp[base:base + 64])


# ---- the MoE FFN of one token -----------------------------------------------------------------

def test_moe_ffn_token_composes_the_block():
    H, I, E, k = 64, 96, 8, 2
    cfg = O.MoeCfg(H, I, E, k, 2, 1, 1.702, 7.0, O.MXFP4, 0)
    rng = np.random.default_rng(3)
    x = rng.standard_normal(H).astype(np.float32)
    rw = (rng.standard_normal((E, H)) * 0.5).astype(np.float32)
    gate = O.synth_mxfp4(11, E * I * H // 32)
    up = O.synth_mxfp4(12, E * I * H // 32)
    down = O.synth_mxfp4(13, E * H * I // 32)
    out = np.zeros(H, np.float32)
    idx = np.zeros(k, np.uint32)
    w = np.zeros(k, np.float32)
    rc = O.lib().or_moe_ffn_token(cfg, O.ptr(x), O.ptr(rw), None, O.ptr(gate), O.ptr(up), O.ptr(down),
                                  None, None, None, O.ptr(out), O.ptr(idx), O.ptr(w))
    assert rc == 0
    # recompute by hand from dequantised banks
    logits = rw.astype(np.float64) @ x.astype(np.float64)
    assert idx.tolist() == np.argsort(-logits.astype(np.float32), kind="stable")[:k].tolist()
    G = O.dequant(O.MXFP4, gate, E * I * H // 32).reshape(E, I, H).astype(np.float64)
    U = O.dequant(O.MXFP4, up, E * I * H // 32).reshape(E, I, H).astype(np.float64)
    D = O.dequant(O.MXFP4, down, E * H * I // 32).reshape(E, H, I).astype(np.float64)
    acc = np.zeros(H)
    for m, e in enumerate(idx):
        g = np.minimum(G[e] @ x, 7.0)
        u = np.clip(U[e] @ x, -7.0, 7.0)
        a = g / (1 + np.exp(-1.702 * g)) * (u + 1)
        acc += w[m] * (D[e] @ a)
    assert np.allclose(out, acc, rtol=1e-4, atol=1e-5)
