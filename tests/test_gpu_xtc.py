"""The batch-1 decode experts on the block-scaled FP4 tensor cores (xtc.cu) against the oracle.

The tc layout is checked byte for byte against a numpy restatement of its definition
(moearc_b200/csrc/xtc.cuh), the forward pass against the oracle's MoE block
(or_moe_ffn_token, crates/moearc-engine/src/moe.rs:2074-2427) at the f32 check-mode bound the
fragment path is held to, max |a - b| / max(|b|, 1) <= 1e-4, with routing bit-exact, and against
the fragment path on the same banks.
"""
import numpy as np
import pytest

import oracle as O
from moearc_b200 import Context
from moearc_b200.moe import MoeLayer

pytestmark = pytest.mark.gpu

KPAIR, KPAIR_HALF, ABLK = 8704, 4608, 4096


@pytest.fixture(scope="module")
def ctx():
    c = Context()
    yield c
    c.close()


def rel_err(got, want):
    return float(np.max(np.abs(got.astype(np.float64) - want) / np.maximum(np.abs(want), 1.0)))


def tile_bytes(K):
    ks = K // 64
    return (ks // 2) * KPAIR + (ks % 2) * KPAIR_HALF


def pack_tc_np(src_rows, K, n_tiles, rows_of):
    """One expert's bank in the tc layout: src_rows(r) -> the 17-byte MXFP4 blocks of row r
    ([K / 32, 17] uint8) or None past the matrix; rows_of(t, m) -> the source row of tile row m."""
    ks_n, tb = K // 64, tile_bytes(K)
    nkp = (ks_n + 1) // 2
    out = np.zeros(n_tiles * tb, np.uint8)
    q = np.arange(16)
    for t in range(n_tiles):
        base = t * tb
        for m in range(128):
            blocks = src_rows(rows_of(t, m))
            if blocks is None:
                continue
            for ks in range(ks_n):
                kp = ks // 2
                half_kp = kp == nkp - 1 and ks_n % 2 == 1
                for h in range(2):
                    blk = blocks[2 * ks + h]
                    qs = blk[1:17]
                    el = np.concatenate([qs & 15, qs >> 4])  # element i of the block
                    byte = (el[2 * q] | (el[2 * q + 1] << 4)).astype(np.uint8)
                    a = base + kp * KPAIR + (ks % 2) * ABLK + 32 * m + 16 * (h ^ ((m >> 2) & 1))
                    out[a:a + 16] = byte
                    sf = base + kp * KPAIR + (ABLK if half_kp else 2 * ABLK)
                    out[sf + (m % 32) * 16 + (m // 32) * 4 + 2 * (ks % 2) + h] = blk[0]
    return out


def make(ctx, H, I, E, k, gating, act, seed, T=1):
    nb = E * I * H // 32
    gate, up, down = (O.synth_mxfp4(seed + i, nb) for i in range(3))
    router = O.synth_normal_f32(seed + 7, E * H, 0.02)
    layer = MoeLayer(ctx, H, I, E, k, gating, act, O.MXFP4, max_tokens=T)
    g, u, d = ctx.upload_new(gate), ctx.upload_new(up), ctx.upload_new(down)
    layer.pack(g, u, d)
    assert layer.has_tc()
    layer.pack_tc(g, u, d)
    return layer, (gate, up, down, router)


def oracle(H, I, E, k, gating, act, host, x, biases=(None, None, None)):
    gate, up, down, router = host
    cfg = O.MoeCfg(H, I, E, k, gating, act, 1.702, 7.0, O.MXFP4, 1)
    out = np.zeros(H, np.float32)
    idx = np.zeros(k, np.uint32)
    w = np.zeros(k, np.float32)
    bg, bu, bd = (None if b is None else O.ptr(b) for b in biases)
    rc = O.lib().or_moe_ffn_token(cfg, O.ptr(x), O.ptr(router), None, O.ptr(gate), O.ptr(up), O.ptr(down),
                                  bg, bu, bd, O.ptr(out), O.ptr(idx), O.ptr(w))
    assert rc == 0
    return out, idx, w


@pytest.mark.parametrize("H,I", [(320, 192), (256, 448)])  # odd / even k-steps both ways; a 64-row last down tile
def test_tc_packer_writes_the_layout(ctx, H, I):
    E = 3
    layer, (gate, up, down, _) = make(ctx, H, I, E, 2, 2, 1, 0x7C00 + H)
    g = gate.reshape(E, I, H // 32, 17)
    u = up.reshape(E, I, H // 32, 17)
    d = down.reshape(E, H, I // 32, 17)
    gu_stride, dn_stride = (I // 64) * tile_bytes(H), ((H + 127) // 128) * tile_bytes(I)
    dev_gu = ctx.download(layer.gateup_tc, np.uint8, E * gu_stride)
    dev_dn = ctx.download(layer.down_tc, np.uint8, E * dn_stride)
    for e in range(E):
        want_gu = pack_tc_np(lambda r: r[0][e, r[1]] if r[0] is not None else None, H, I // 64,
                             lambda t, m: (g if m < 64 else u, 64 * t + (m & 63)))
        want_dn = pack_tc_np(lambda r: d[e, r] if r < H else None, I, (H + 127) // 128, lambda t, m: 128 * t + m)
        assert np.array_equal(dev_gu[e * gu_stride:(e + 1) * gu_stride], want_gu), e
        assert np.array_equal(dev_dn[e * dn_stride:(e + 1) * dn_stride], want_dn), e
    layer.close()


@pytest.mark.parametrize("H,I,E,k,gating,act", [
    (2880, 2880, 128, 4, 2, 1),   # configs[2] gpt-oss-120b
    (2880, 2880, 32, 4, 2, 0),    # configs[1] gpt-oss-20b experts, SwiGLU
    (2880, 1024, 64, 4, 0, 1),    # split tiles, 16 gate-up tiles per expert
    (320, 192, 8, 2, 1, 1),       # odd k-steps, a 64-row last down tile, more CTAs than units
    (640, 448, 16, 8, 2, 0),      # k = 8
])
def test_tc_forward_matches_the_oracle(ctx, H, I, E, k, gating, act):
    layer, host = make(ctx, H, I, E, k, gating, act, 0x7C10 + H + E)
    rw = ctx.upload_new(host[3])
    worst = worst_frag = 0.0
    for s in range(4):
        x = O.synth_normal_f32(0x7C20 + s, H, 1.0)
        res = O.synth_normal_f32(0x7C30 + s, H, 1.0)
        xd, rd = ctx.upload_new(x), ctx.upload_new(res)
        o_tc, o_fr = ctx.alloc_n(np.float32, H), ctx.alloc_n(np.float32, H)
        layer.forward_tc(xd, rw, o_tc, residual=rd)
        got = ctx.download(o_tc, np.float32, H)
        idx = layer.buffer(0, np.uint32, k)
        act_tc = layer.buffer(2, np.float32, k * I)
        assert layer.status() == 0
        layer.forward(xd, 1, rw, o_fr, residual=rd)
        frag = ctx.download(o_fr, np.float32, H)
        act_fr = layer.buffer(2, np.float32, k * I)
        want, widx, _ = oracle(H, I, E, k, gating, act, host, x)
        assert np.array_equal(idx, widx)
        worst = max(worst, rel_err(got - res, want))
        worst_frag = max(worst_frag, rel_err(got, frag))
        # the activation columns (experts ascending) agree with the fragment path's
        assert rel_err(act_tc, act_fr.astype(np.float64)) <= 1e-4
        # the same call again gives the same bits
        layer.forward_tc(xd, rw, o_tc, residual=rd)
        assert np.array_equal(ctx.download(o_tc, np.float32, H).view(np.uint32), got.view(np.uint32))
    print(f"tc path H={H} I={I} E={E} k={k}: max rel err {worst:.3e} against the oracle, "
          f"{worst_frag:.3e} against the fragment path (bound 1e-4)")
    assert worst <= 1e-4 and worst_frag <= 1e-4
    layer.close()


def test_tc_expert_biases_match_the_oracle(ctx):
    H, I, E, k = 2880, 1024, 32, 4
    layer, host = make(ctx, H, I, E, k, 2, 1, 0x7CB1)
    gu_b = O.synth_normal_f32(0x7CB2, 2 * E * I, 0.5)
    dn_b = O.synth_normal_f32(0x7CB3, E * H, 0.5)
    layer.set_bias(ctx.upload_new(gu_b), ctx.upload_new(dn_b))
    rw = ctx.upload_new(host[3])
    worst = 0.0
    for s in range(3):
        x = O.synth_normal_f32(0x7CB4 + s, H, 1.0)
        o = ctx.alloc_n(np.float32, H)
        layer.forward_tc(ctx.upload_new(x), rw, o)
        want, _, _ = oracle(H, I, E, k, 2, 1, host, x, (gu_b[:E * I], gu_b[E * I:], dn_b))
        worst = max(worst, rel_err(ctx.download(o, np.float32, H), want))
    assert layer.status() == 0
    print(f"tc path with expert biases: max rel err {worst:.3e}")
    assert worst <= 1e-4
    layer.close()


def test_tc_wait_that_runs_out_raises_the_status_and_the_layer_recovers(ctx):
    """A wait made to run out (set_wait's phantom) sets the status bit and leaves the context
    usable: the next call without it matches the oracle again."""
    H, I, E, k = 2880, 1024, 32, 4
    layer, host = make(ctx, H, I, E, k, 2, 1, 0x7CF0)
    rw = ctx.upload_new(host[3])
    x = O.synth_normal_f32(0x7CF1, H, 1.0)
    xd, o = ctx.upload_new(x), ctx.alloc_n(np.float32, H)
    layer.ctx._finish(ctx.lib.moearc_x_moe_set_wait(layer.h, 2_000_000, 1), "set_wait")
    layer.forward_tc(xd, rw, o)
    assert layer.status() & 1
    layer.ctx._finish(ctx.lib.moearc_x_moe_set_wait(layer.h, 0, 0), "set_wait")
    layer.forward_tc(xd, rw, o)
    want, _, _ = oracle(H, I, E, k, 2, 1, host, x)
    assert layer.status() == 0
    assert rel_err(ctx.download(o, np.float32, H), want) <= 1e-4
    layer.close()


def test_tc_forward_refuses_more_than_one_token(ctx):
    H, I, E, k = 320, 192, 8, 2
    layer, host = make(ctx, H, I, E, k, 2, 1, 0x7CA0, T=4)
    rw = ctx.upload_new(host[3])
    x, o = ctx.alloc_n(np.float32, 2 * H), ctx.alloc_n(np.float32, 2 * H)
    rc = ctx.lib.moearc_x_moe_forward_tc(layer.h, x.ptr, 2, rw.ptr, None, layer.gateup_tc.ptr, layer.down_tc.ptr,
                                         None, o.ptr)
    assert rc == -2
    layer.close()
