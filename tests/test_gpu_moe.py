"""The fused MoE decode path on the B200 against the oracle's MoE block.

configs[0] of the benchmark description at full size: hidden 2880, 32 experts, top-4,
intermediate 2880, MXFP4 experts (nibbles uniform, e8m0 exponent in [-8, -4]), router weights
f32 N(0, 0.02), 16 tokens of N(0, 1) activations. Routing is checked bit-exact: the device
router GEMV folds in a fixed, documented order and the oracle reproduces that order
(or_matvec_f32_gpu_order), so both select from identical logits. Outputs are checked at the
f32 check-mode bound, max |a - b| / max(|b|, 1) <= 1e-4.
"""
import numpy as np
import pytest

import oracle as O
from moearc_b200 import Context
from moearc_b200.moe import MoeLayer

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = Context()
    yield c
    c.close()


def rel_err(got, want):
    return float(np.max(np.abs(got.astype(np.float64) - want) / np.maximum(np.abs(want), 1.0)))


def make_layer(ctx, H, I, E, k, gating, act, wtype, T, seed):
    nb_gate = E * I * H // 32
    nb_down = E * H * I // 32
    if wtype == O.MXFP4:
        gate, up, down = (O.synth_mxfp4(seed + i, n) for i, n in enumerate((nb_gate, nb_gate, nb_down)))
    else:
        gate, up, down = (O.synth_q4_0(seed + i, n, 0.01) for i, n in enumerate((nb_gate, nb_gate, nb_down)))
    router = O.synth_normal_f32(seed + 7, E * H, 0.02)
    layer = MoeLayer(ctx, H, I, E, k, gating, act, wtype, max_tokens=T)
    layer.pack(ctx.upload_new(gate), ctx.upload_new(up), ctx.upload_new(down))
    return layer, (gate, up, down, router)


def oracle_token(H, I, E, k, gating, act, wtype, host, x):
    gate, up, down, router = host
    cfg = O.MoeCfg(H, I, E, k, gating, act, 1.702, 7.0, wtype, 1)
    out = np.zeros(H, np.float32)
    idx = np.zeros(k, np.uint32)
    w = np.zeros(k, np.float32)
    rc = O.lib().or_moe_ffn_token(cfg, O.ptr(x), O.ptr(router), None, O.ptr(gate), O.ptr(up), O.ptr(down),
                                  None, None, None, O.ptr(out), O.ptr(idx), O.ptr(w))
    assert rc == 0
    return out, idx, w


@pytest.mark.parametrize("act", [0, 1])
def test_config0_moe_layer_matches_the_oracle(ctx, act):
    H = I = 2880
    E, k, T, gating = 32, 4, 16, 2
    layer, host = make_layer(ctx, H, I, E, k, gating, act, O.MXFP4, T, 0x5EED0)
    x = O.synth_normal_f32(0x5EED9, T * H, 1.0)
    dx = ctx.upload_new(x)
    out = ctx.alloc_n(np.float32, T * H)
    layer.forward(dx, T, ctx.upload_new(host[3]), out)
    got = ctx.download(out, np.float32, T * H).reshape(T, H)
    assert layer.status() == 0
    idx = layer.buffer(0, np.uint32, T * k).reshape(T, k)
    wts = layer.buffer(1, np.float32, T * k).reshape(T, k)
    logits = layer.buffer(3, np.float32, T * E).reshape(T, E)
    worst = 0.0
    for t in range(T):
        xt = x[t * H:(t + 1) * H].copy()
        assert np.array_equal(logits[t], O.matvec_f32(host[3].reshape(E, H), xt, gpu_order=True))
        if t % 4 == 0:  # the oracle's MoE block on a quarter of the tokens keeps this bounded
            want, widx, ww = oracle_token(H, I, E, k, gating, act, O.MXFP4, host, xt)
            assert np.array_equal(idx[t], widx), (t, idx[t], widx)
            assert np.allclose(wts[t], ww, rtol=1e-6, atol=1e-7)
            worst = max(worst, rel_err(got[t], want))
    print(f"config0 act={act}: max rel err {worst:.3e} over 4 tokens (bound 1e-4)")
    assert worst <= 1e-4


def test_batch_invariance_and_the_residual(ctx):
    """A token's output does not depend on which other tokens share the call, and the
    residual lands on top of the MoE output."""
    H = I = 2880
    E, k, gating = 32, 4, 2
    layer, host = make_layer(ctx, H, I, E, k, gating, 1, O.MXFP4, 16, 0xBA7C4)
    rw = ctx.upload_new(host[3])
    x = O.synth_normal_f32(0xBA7C5, 16 * H, 1.0)
    res = O.synth_normal_f32(0xBA7C6, 16 * H, 1.0)
    out16 = ctx.alloc_n(np.float32, 16 * H)
    layer.forward(ctx.upload_new(x), 16, rw, out16)
    all16 = ctx.download(out16, np.float32, 16 * H)
    for t in (0, 5, 15):
        o1 = ctx.alloc_n(np.float32, H)
        layer.forward(ctx.upload_new(x[t * H:(t + 1) * H].copy()), 1, rw, o1)
        assert np.array_equal(ctx.download(o1, np.float32, H), all16[t * H:(t + 1) * H])
    outr = ctx.alloc_n(np.float32, 16 * H)
    layer.forward(ctx.upload_new(x), 16, rw, outr, residual=ctx.upload_new(res))
    assert np.array_equal(ctx.download(outr, np.float32, 16 * H), (res + all16).astype(np.float32))


def test_activation_buffer_matches_the_oracle(ctx):
    """The intermediate SwiGLU-OAI activations of one token, column by column."""
    H = I = 2880
    E, k = 32, 4
    layer, (gate, up, down, router) = make_layer(ctx, H, I, E, k, 2, 1, O.MXFP4, 1, 0xAC7)
    x = O.synth_normal_f32(0xAC8, H, 1.0)
    out = ctx.alloc_n(np.float32, H)
    layer.forward(ctx.upload_new(x), 1, ctx.upload_new(router), out)
    idx = layer.buffer(0, np.uint32, k)
    act = layer.buffer(2, np.float32, k * I).reshape(k, I)
    gb = I * H // 32 * 17
    for col, e in enumerate(sorted(idx.tolist())):  # columns: experts ascending
        g = O.matvec_q(O.MXFP4, gate[e * gb:(e + 1) * gb], x, I, H)
        u = O.matvec_q(O.MXFP4, up[e * gb:(e + 1) * gb], x, I, H)
        want = np.zeros(I, np.float32)
        O.lib().or_swiglu_oai(O.ptr(g), O.ptr(u), I, 1.702, 7.0, O.ptr(want))
        err = rel_err(act[col], want)
        print(f"expert {e}: activation max rel err {err:.3e}")
        assert err <= 1e-4


def test_qwen3_shaped_q4_0_layer(ctx):
    """Hidden 2048, 128 experts, top-8, intermediate 768, Q4_0 (f16 deltas |N(0, 0.01)|),
    renormalised softmax gating, SwiGLU, 4 tokens."""
    H, I, E, k, T = 2048, 768, 128, 8, 4
    layer, host = make_layer(ctx, H, I, E, k, 1, 0, O.Q4_0, T, 0x0E3)
    x = O.synth_normal_f32(0x0E4, T * H, 1.0)
    out = ctx.alloc_n(np.float32, T * H)
    layer.forward(ctx.upload_new(x), T, ctx.upload_new(host[3]), out)
    got = ctx.download(out, np.float32, T * H).reshape(T, H)
    idx = layer.buffer(0, np.uint32, T * k).reshape(T, k)
    worst = 0.0
    for t in range(T):
        want, widx, _ = oracle_token(H, I, E, k, 1, 0, O.Q4_0, host, x[t * H:(t + 1) * H].copy())
        assert np.array_equal(idx[t], widx)
        worst = max(worst, rel_err(got[t], want))
    print(f"qwen3 Q4_0: max rel err {worst:.3e} (bound 1e-4)")
    assert worst <= 1e-4


@pytest.mark.parametrize("wtype", [O.MXFP4, O.Q4_0])
def test_decode_path_is_batch_invariant_and_matches_the_oracle(ctx, wtype):
    """Up to 32 (token, expert) columns take the decode path (per-CTA routing tables, pieces
    of fixed k-extent): a token's output is bit-identical whether it is decoded alone or among
    eight, every token matches the oracle, and the residual lands on top."""
    H, I, E, k, T = 2880, 1024, 64, 4, 8
    layer, host = make_layer(ctx, H, I, E, k, 0, 1, wtype, T, 0xDEC0DE)
    rw = ctx.upload_new(host[3])
    x = O.synth_normal_f32(0xDEC1, T * H, 1.0)
    res = O.synth_normal_f32(0xDEC2, T * H, 1.0)
    out = ctx.alloc_n(np.float32, T * H)
    layer.forward(ctx.upload_new(x), T, rw, out, residual=ctx.upload_new(res))
    got = ctx.download(out, np.float32, T * H).reshape(T, H)
    assert layer.status() == 0
    idx = layer.buffer(0, np.uint32, T * k).reshape(T, k)
    worst = 0.0
    for t in range(T):
        xt = x[t * H:(t + 1) * H].copy()
        o1 = ctx.alloc_n(np.float32, H)
        layer.forward(ctx.upload_new(xt), 1, rw, o1, residual=ctx.upload_new(res[t * H:(t + 1) * H].copy()))
        assert np.array_equal(ctx.download(o1, np.float32, H), got[t]), t
        want, widx, _ = oracle_token(H, I, E, k, 0, 1, wtype, host, xt)
        assert np.array_equal(idx[t], widx)
        worst = max(worst, rel_err(got[t] - res[t * H:(t + 1) * H], want))
    print(f"decode path wtype={wtype}: max rel err {worst:.3e} over {T} tokens (bound 1e-4)")
    assert worst <= 1e-4


@pytest.mark.parametrize("env", ["MOEARC_MOE_FUSED_GD", "MOEARC_FUSED_MOE"])
def test_opt_in_single_launch_paths_give_the_same_bits(ctx, env, monkeypatch):
    """The opt-in launches of the decode path (gate-up and down in one PDL-chained launch; route,
    gate-up and down in one cooperative launch) run the same pieces in the same order, so their
    outputs equal the default kernels' bit for bit, for one token and for eight."""
    H, I, E, k, T = 2880, 1024, 64, 4, 8
    base, host = make_layer(ctx, H, I, E, k, 2, 1, O.MXFP4, T, 0xF05E)
    monkeypatch.setenv(env, "1")
    alt, _ = make_layer(ctx, H, I, E, k, 2, 1, O.MXFP4, T, 0xF05E)
    rw = ctx.upload_new(host[3])
    for n in (1, T):
        x = ctx.upload_new(O.synth_normal_f32(0xF05F + n, n * H, 1.0))
        res = ctx.upload_new(O.synth_normal_f32(0xF060 + n, n * H, 1.0))
        a, b = ctx.alloc_n(np.float32, n * H), ctx.alloc_n(np.float32, n * H)
        base.forward(x, n, rw, a, residual=res)
        alt.forward(x, n, rw, b, residual=res)
        ga, gb = ctx.download(a, np.float32, n * H), ctx.download(b, np.float32, n * H)
        assert base.status() == 0 and alt.status() == 0
        assert np.array_equal(ga.view(np.uint32), gb.view(np.uint32)), (env, n)


@pytest.mark.parametrize("wtype", [O.MXFP4, O.Q4_0])
def test_host_packer_writes_the_device_packers_bytes(ctx, wtype):
    """moearc_x_moe_pack_host (the host expert pool's layout source) against moearc_x_moe_pack."""
    import ctypes as C

    H, I, E = 2880, 2880, 3
    layer, (gate, up, down, _) = make_layer(ctx, H, I, E, 2, 1, 1, wtype, 1, 0x9AC0 + wtype)
    dev_gu = np.empty(E * layer.gu_bytes, np.uint8)
    dev_dn = np.empty(E * layer.dn_bytes, np.uint8)
    ctx._finish(ctx.lib.moearc_copy_d2h(ctx.raw, dev_gu.ctypes.data, layer.gateup.ptr, dev_gu.nbytes), "d2h")
    ctx._finish(ctx.lib.moearc_copy_d2h(ctx.raw, dev_dn.ctypes.data, layer.down.ptr, dev_dn.nbytes), "d2h")
    host_gu, host_dn = np.zeros_like(dev_gu), np.zeros_like(dev_dn)
    rc = ctx.lib.moearc_x_moe_pack_host(C.byref(layer.desc), gate.ctypes.data, up.ctypes.data, down.ctypes.data,
                                        E, host_gu.ctypes.data, host_dn.ctypes.data)
    assert rc == 0
    assert np.array_equal(host_gu, dev_gu) and np.array_equal(host_dn, dev_dn)
    layer.close()


@pytest.mark.parametrize("T", [1, 16])  # the decode kernels (one token) and the row kernels (64 columns)
def test_expert_biases_match_the_oracle(ctx, T):
    """gpt-oss's per-expert biases (moe.rs:2310-2331: gate/up after the matvecs, before the
    activation; 2362-2372: down inside the router weighting) fused into the decode kernels,
    against the oracle's MoE block with the same biases, at the f32 check bound."""
    H, I, E, k = 2880, 1024, 32, 4
    layer, host = make_layer(ctx, H, I, E, k, 2, 1, O.MXFP4, T, 0xB1A5)
    gu_b = O.synth_normal_f32(0xB1A6, 2 * E * I, 0.5)
    dn_b = O.synth_normal_f32(0xB1A7, E * H, 0.5)
    layer.set_bias(ctx.upload_new(gu_b), ctx.upload_new(dn_b))
    gate, up, down, router = host
    x = np.stack([O.synth_normal_f32(0xB1A8 + t, H, 1.0) for t in range(T)])
    xd, rd, od = ctx.upload_new(x), ctx.upload_new(router), ctx.alloc(4 * T * H)
    layer.forward(xd, T, rd, od)
    got = ctx.download(od, np.float32, T * H).reshape(T, H)
    cfg = O.MoeCfg(H, I, E, k, 2, 1, 1.702, 7.0, O.MXFP4, 1)
    worst = 0.0
    for t in range(T):
        want = np.zeros(H, np.float32)
        rc = O.lib().or_moe_ffn_token(cfg, O.ptr(x[t]), O.ptr(router), None, O.ptr(gate), O.ptr(up), O.ptr(down),
                                      O.ptr(gu_b[:E * I]), O.ptr(gu_b[E * I:]), O.ptr(dn_b), O.ptr(want), None, None)
        assert rc == 0
        worst = max(worst, rel_err(got[t], want))
    print(f"expert biases T={T}: max rel err {worst:.3e}")
    assert worst <= 1e-4
    layer.set_bias(None, None)
    layer.forward(xd, T, rd, od)
    nob = ctx.download(od, np.float32, T * H).reshape(T, H)
    assert not np.allclose(nob, got)  # the biases were applied, and are cleared
    assert layer.status() == 0
    layer.close()
