"""The MoE prefill path (tcgen05 grouped GEMMs) on the B200 against the oracle's MoE block.

Inputs are bf16 activations (configs[3] of the benchmark description: activations bf16 N(0,1)),
given to the oracle as their exact f32 values. Routing is checked bit-exact (the prefill router
folds in the decode router's fixed order, which the oracle reproduces). Outputs are checked the
way the reference's own tests bound a kernel (assert_close with a tolerance scaled by the
output's largest magnitude, crates/moearc-kernels/tests/common/mod.rs:106-116, used as
`k * U * max_abs(&want)` in kernels_gpu.rs:250-255), at the bf16-activation bound 1e-2:
max |a - b| <= 1e-2 * max |b|. The SwiGLU outputs are rounded to bf16 once before the down GEMM
(an absolute error near 1e-3 of a typical output) and Q4_0 weights are rounded to bf16.
The expanded MXFP4 weights are checked bit-exact against the oracle's dequantisation.
"""
import numpy as np
import pytest

import oracle as O
from moearc_b200 import Context
from moearc_b200.moe import MoeLayer, MoePrefill

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = Context()
    yield c
    c.close()


def bf16_err(got, want):
    """max |got - want| / max |want| (the bound is 1e-2)."""
    want = want.astype(np.float64)
    return float(np.max(np.abs(got.astype(np.float64) - want)) / max(float(np.max(np.abs(want))), 1e-30))


def build(ctx, H, I, E, k, gating, act, wtype, T, seed):
    nb = E * I * H // 32
    if wtype == O.MXFP4:
        gate, up, down = (O.synth_mxfp4(seed + i, nb) for i in range(3))
    else:
        gate, up, down = (O.synth_q4_0(seed + i, nb, 0.01) for i in range(3))
    router = O.synth_normal_f32(seed + 7, E * H, 0.02)
    packer = MoeLayer(ctx, H, I, E, k, gating, act, wtype, max_tokens=1)
    packer.pack(ctx.upload_new(gate), ctx.upload_new(up), ctx.upload_new(down))
    pf = MoePrefill(ctx, H, I, E, k, gating, act, wtype, max_tokens=T)
    pf.load(packer.gateup, packer.down)
    return pf, packer, (gate, up, down, router)


def oracle_token(H, I, E, k, gating, act, wtype, host, x):
    gate, up, down, router = host
    cfg = O.MoeCfg(H, I, E, k, gating, act, 1.702, 7.0, wtype, 1)
    out = np.zeros(H, np.float32)
    idx = np.zeros(k, np.uint32)
    w = np.zeros(k, np.float32)
    assert O.lib().or_moe_ffn_token(cfg, O.ptr(x), O.ptr(router), None, O.ptr(gate), O.ptr(up), O.ptr(down),
                                    None, None, None, O.ptr(out), O.ptr(idx), O.ptr(w)) == 0
    return out, idx, w


@pytest.mark.parametrize("shape", [
    # configs[0]/[3] expert shape (gpt-oss: softmax over the selected logits, SwiGLU-OAI), MXFP4
    dict(H=2880, I=2880, E=32, k=4, gating=2, act=1, wtype=O.MXFP4, T=40),
    # configs[4] expert shape (Qwen3-MoE: softmax then renormalise, SiLU), Q4_0
    dict(H=2048, I=768, E=128, k=8, gating=1, act=0, wtype=O.Q4_0, T=40),
])
def test_prefill_matches_the_oracle(ctx, shape):
    H, I, E, k, T = shape["H"], shape["I"], shape["E"], shape["k"], shape["T"]
    pf, packer, host = build(ctx, H, I, E, k, shape["gating"], shape["act"], shape["wtype"], T, 0x9F11)
    xb = O.synth_normal_bf16(0x9F12, T * H, 1.0)
    res = O.synth_normal_f32(0x9F13, T * H, 1.0)
    out = ctx.alloc_n(np.float32, T * H)
    pf.forward(ctx.upload_new(xb), T, ctx.upload_new(host[3]), out, residual=ctx.upload_new(res))
    got = ctx.download(out, np.float32, T * H).reshape(T, H) - res.reshape(T, H)
    assert pf.status() == 0
    idx = pf.buffer(0, np.uint32, T * k).reshape(T, k)
    cnt = pf.buffer(3, np.int32, E)
    assert int(cnt.sum()) == T * k
    assert np.array_equal(np.bincount(idx.ravel(), minlength=E), cnt)
    x32 = O.bf16_to_f32(xb).reshape(T, H)
    want = np.zeros((T, H), np.float32)
    for t in range(T):
        want[t], widx, _ = oracle_token(H, I, E, k, shape["gating"], shape["act"], shape["wtype"], host,
                                        np.ascontiguousarray(x32[t]))
        assert np.array_equal(idx[t], widx), t
    worst = bf16_err(got, want)
    print(f"prefill {shape}: max rel err {worst:.3e} over {T} tokens (bound 1e-2)")
    assert worst <= 1e-2
    pf.close()
    packer.close()


def test_expanded_mxfp4_weights_are_exact(ctx):
    """The bf16 expansion of the packed banks equals the oracle's dequantisation bit for bit
    (E2M1 x 2^(e-127) is representable in bf16)."""
    H, I, E, k = 2880, 2880, 4, 2
    pf, packer, host = build(ctx, H, I, E, k, 2, 1, O.MXFP4, 8, 0x9F21)
    gu = pf.buffer(4, np.uint16, E * 2 * I * H).reshape(E, 2, I, H)
    dn = pf.buffer(5, np.uint16, E * H * I).reshape(E, H, I)
    for e in (0, E - 1):
        for which, bank, mat in ((0, host[0], gu[e, 0]), (1, host[1], gu[e, 1]), (2, host[2], dn[e])):
            nb = I * H // 32
            want = O.dequant(O.MXFP4, bank[e * nb * 17:(e + 1) * nb * 17], nb)
            assert np.array_equal(O.bf16_to_f32(mat.ravel()), want), (e, which)
    pf.close()
    packer.close()


def test_skewed_routing_many_tokens_against_torch(ctx):
    """A Zipf-like skew (a few experts take most tokens, some none) over 3000 tokens: counts,
    segment handling and the grouped GEMMs against a plain fp32 torch reference built from the
    expanded weights and the kernel's own routing."""
    torch = pytest.importorskip("torch")
    H, I, E, k, T = 1024, 512, 64, 4, 3000
    pf, packer, host = build(ctx, H, I, E, k, 2, 1, O.MXFP4, T, 0x9F31)
    router = host[3].reshape(E, H).copy()
    boost = np.zeros(E, np.float32)
    boost[:6] = [3.0, 2.5, 2.0, 1.5, 1.0, 0.5]
    boost[40:] = -4.0  # experts 40.. rarely or never chosen
    xb = O.synth_normal_bf16(0x9F32, T * H, 1.0)
    x32 = O.bf16_to_f32(xb).reshape(T, H)
    rb = ctx.upload_new(boost)
    out = ctx.alloc_n(np.float32, T * H)
    pf.forward(ctx.upload_new(xb), T, ctx.upload_new(router.ravel()), out, router_b=rb)
    got = ctx.download(out, np.float32, T * H).reshape(T, H)
    assert pf.status() == 0
    idx = pf.buffer(0, np.uint32, T * k).reshape(T, k).astype(np.int64)
    wts = pf.buffer(1, np.float32, T * k).reshape(T, k)
    cnt = pf.buffer(3, np.int32, E)
    assert cnt.max() > 3 * T * k // E and (cnt == 0).any()
    # routing of a sample of tokens against the oracle's router
    logits = pf.buffer(2, np.float32, T * E).reshape(T, E)
    for t in range(0, T, 97):
        want = O.matvec_f32(router, np.ascontiguousarray(x32[t]), gpu_order=True) + boost
        assert np.array_equal(logits[t], want), t
        widx, _ = O.topk_router(want.reshape(1, E), k, 2)
        assert np.array_equal(idx[t], widx[0]), t
    dev = torch.device("cuda")
    gu = torch.from_numpy(O.bf16_to_f32(pf.buffer(4, np.uint16, E * 2 * I * H)).reshape(E, 2, I, H)).to(dev)
    dn = torch.from_numpy(O.bf16_to_f32(pf.buffer(5, np.uint16, E * H * I)).reshape(E, H, I)).to(dev)
    xt = torch.from_numpy(x32).to(dev)
    ref = torch.zeros(T, H, dtype=torch.float32, device=dev)
    it, wt = torch.from_numpy(idx).to(dev), torch.from_numpy(wts).to(dev)
    for m in range(k):
        for e in torch.unique(it[:, m]).tolist():
            sel = (it[:, m] == e).nonzero().squeeze(1)
            g = xt[sel] @ gu[e, 0].T
            u = xt[sel] @ gu[e, 1].T
            gx = torch.clamp(g, max=7.0)
            uy = torch.clamp(u, -7.0, 7.0)
            a = gx / (1 + torch.exp(-1.702 * gx)) * (uy + 1)
            ref[sel] = torch.addcmul(ref[sel], wt[sel, m:m + 1], a @ dn[e].T)
    err = bf16_err(got, ref.cpu().numpy())
    print(f"skewed prefill: counts max {cnt.max()} min {cnt.min()}, max rel err vs torch {err:.3e}")
    assert err <= 1e-2
    pf.close()
    packer.close()


@pytest.mark.parametrize("world,placement", [(2, "contiguous"), (4, "interleaved"), (4, "balanced"),
                                             (4, "balanced-4bit")])
def test_expert_parallel_split_gives_the_same_bits(ctx, world, placement):
    """Expert parallelism emulated on one GPU: each virtual rank routes its own tokens, owns a
    contiguous expert range (moearc_x_prefill_load_range), receives the rows of its experts from
    every rank as (source, expert) segments and returns the result rows; the combine on each rank
    then gives the single-GPU block's output bit for bit (a row's arithmetic does not depend on
    where its segment sits)."""
    torch = pytest.importorskip("torch")
    from moearc_b200.ep import balanced, interleaved, plan, positions

    H, I, E, k, T = 1024, 512, 32, 4, 600
    four = placement.endswith("4bit")
    whole, packer, host = build(ctx, H, I, E, k, 2, 1, O.MXFP4, T, 0x9F41)
    if four:
        whole.load4(packer.gateup, packer.down)
    xb = O.synth_normal_bf16(0x9F42, T * H, 1.0)
    rw = ctx.upload_new(host[3])
    ref = ctx.alloc_n(np.float32, T * H)
    whole.forward(ctx.upload_new(xb), T, rw, ref)
    want = ctx.download(ref, np.float32, T * H).reshape(T, H)
    Tr = T // world
    nl = E // world
    if placement == "contiguous":
        lists = [list(range(r * nl, (r + 1) * nl)) for r in range(world)]
    elif placement == "interleaved":
        lists = interleaved(E, world)
    else:
        lists = balanced(whole.buffer(3, np.int32, E), world)  # the whole batch's popularity
    pos = positions(lists)
    ranks = []
    for r in range(world):
        pf = MoePrefill(ctx, H, I, E, k, 2, 1, O.MXFP4, max_tokens=Tr)
        pf.set_order(pos)
        if placement == "contiguous":
            pf.load_range(packer.gateup, packer.down, r * nl, nl)
        elif four:
            pf.load4(packer.gateup, packer.down, lists[r])
        else:
            pf.load_list(packer.gateup, packer.down, lists[r])
        x = ctx.upload_new(xb[r * Tr * H:(r + 1) * Tr * H])
        pf.route(x, Tr, rw)
        ranks.append((pf, x, pf.buffer(3, np.int32, E)))
    counts_all = np.stack([c for _, _, c in ranks])
    plans = [plan(counts_all, r, world) for r in range(world)]
    # the rows travel as opaque 16-bit words (bf16, or f16 in the 4-bit form)
    xps = [pf.buffer(6, np.uint16, Tr * k * H).reshape(Tr * k, H) for pf, _, _ in ranks]
    send_off = [np.concatenate([[0], np.cumsum(p["send"])]) for p in plans]
    ys = []
    for r, (pf, _, _) in enumerate(ranks):
        rows = np.concatenate([xps[s][send_off[s][r]:send_off[s][r + 1]] for s in range(world)])
        n = rows.shape[0]
        assert n == plans[r]["n_recv"]
        rows_dev = ctx.upload_new(rows.ravel())
        act = ctx.alloc_n(np.uint16, max(n, 1) * I)
        y = ctx.alloc_n(np.float32, max(n, 1) * H)
        pf.experts(rows_dev.ptr, n, plans[r]["seg_counts"], plans[r]["seg_expert"], act.ptr, y.ptr)
        ys.append(ctx.download(y, np.float32, n * H).reshape(n, H))
    recv_off = [np.concatenate([[0], np.cumsum(p["recv"])]) for p in plans]
    for s, (pf, _, _) in enumerate(ranks):
        back = np.concatenate([ys[r][recv_off[r][s]:recv_off[r][s + 1]] for r in range(world)])
        out = ctx.alloc_n(np.float32, Tr * H)
        back_dev = ctx.upload_new(back)  # held: the buffer must outlive the enqueued combine
        pf.combine(back_dev.ptr, Tr, out.ptr)
        got = ctx.download(out, np.float32, Tr * H).reshape(Tr, H)
        assert np.array_equal(got.view(np.uint32), want[s * Tr:(s + 1) * Tr].view(np.uint32)), (world, s)
        assert pf.status() == 0
        pf.close()
    whole.close()
    packer.close()


@pytest.mark.parametrize("wtype", [O.MXFP4, O.Q4_0])
@pytest.mark.parametrize("shape", [(2880, 2880, 700), (1024, 512, 64)])
def test_4bit_weights_match_the_oracle(ctx, wtype, shape):
    """The 4-bit weight form (chunks bulk-copied and expanded to f16 in shared memory by decoder
    warps; f16 activations) against the bf16 form and the oracle, over a skewed routing that
    leaves some experts empty and others with several row tiles: within the bf16-activation
    bound 1e-2 of max |out| (the 4-bit form rounds less: f16 keeps 11 bits). 700 tokens run the
    128-row tiles; 64 tokens (at most 16 rows per expert on average) the decode-sized 32-row tiles
    with the stage's MMAs split between two issuing threads."""
    H, I, T = shape
    E, k = 16, 4
    tile = 128 if T * k > 16 * E else 32
    pf, packer, host = build(ctx, H, I, E, k, 2, 1, wtype, T, 0x9F51)
    bias = np.zeros(E, np.float32)
    bias[:3] = [2.0, 1.5, 1.0]
    bias[12:] = -5.0
    xb = ctx.upload_new(O.synth_normal_bf16(0x9F52, T * H, 1.0))
    rw, rb = ctx.upload_new(host[3]), ctx.upload_new(bias)
    res = ctx.upload_new(O.synth_normal_f32(0x9F53, T * H, 1.0))
    a, b = ctx.alloc_n(np.float32, T * H), ctx.alloc_n(np.float32, T * H)
    pf.forward(xb, T, rw, a, router_b=rb, residual=res)
    pf.load4(packer.gateup, packer.down)
    pf.forward(xb, T, rw, b, router_b=rb, residual=res)
    ga, gb = ctx.download(a, np.float32, T * H), ctx.download(b, np.float32, T * H)
    assert pf.status() == 0
    cnt = pf.buffer(3, np.int32, E)
    assert cnt.max() > tile and (cnt == 0).any()
    res_h = O.synth_normal_f32(0x9F53, T * H, 1.0)
    ga, gb = (ga - res_h).reshape(T, H), (gb - res_h).reshape(T, H)
    assert bf16_err(gb, ga) <= 1e-2
    x32 = O.bf16_to_f32(O.synth_normal_bf16(0x9F52, T * H, 1.0)).reshape(T, H)
    host_b = (host[0], host[1], host[2], host[3])
    want = np.zeros((16, H), np.float32)
    rows = list(range(0, T, T // 16))[:16]
    for i, t in enumerate(rows):
        # the oracle block with the same router bias
        cfg = O.MoeCfg(H, I, E, k, 2, 1, 1.702, 7.0, wtype, 1)
        out = np.zeros(H, np.float32)
        idx = np.zeros(k, np.uint32)
        w = np.zeros(k, np.float32)
        assert O.lib().or_moe_ffn_token(cfg, O.ptr(np.ascontiguousarray(x32[t])), O.ptr(host_b[3]), O.ptr(bias),
                                        O.ptr(host_b[0]), O.ptr(host_b[1]), O.ptr(host_b[2]), None, None, None,
                                        O.ptr(out), O.ptr(idx), O.ptr(w)) == 0
        want[i] = out
    err = bf16_err(gb[rows], want)
    print(f"4-bit prefill wtype={wtype} T={T} ({tile}-row tiles): vs oracle {err:.3e}, vs bf16 form {bf16_err(gb, ga):.3e}")
    assert err <= 1e-2
    pf.close()
    packer.close()


@pytest.mark.parametrize("world", [2, 4])
def test_peer_memory_exchange_gives_the_same_bits(ctx, world):
    """The exchange fused into the kernels (moearc_x_prefill_route_begin / _route_dispatch /
    _experts_to): each virtual rank's scatter stores its rows straight into the owners' receive
    buffers and each owner's down GEMM stores the results straight into the sources' y buffers.
    Here the 'peer' buffers are other virtual ranks' buffers on the same GPU, so the addressing of
    both legs is checked against the single-GPU block, bit for bit, with a balanced placement."""
    import ctypes as C

    from moearc_b200.ep import balanced, peer_plan, positions

    H, I, E, k, T = 1024, 512, 32, 4, 600
    whole, packer, host = build(ctx, H, I, E, k, 2, 1, O.MXFP4, T, 0x9F61)
    xb = O.synth_normal_bf16(0x9F62, T * H, 1.0)
    rw = ctx.upload_new(host[3])
    ref = ctx.alloc_n(np.float32, T * H)
    whole.forward(ctx.upload_new(xb), T, rw, ref)
    want = ctx.download(ref, np.float32, T * H).reshape(T, H)
    Tr, nl = T // world, E // world
    lists = balanced(whole.buffer(3, np.int32, E), world)
    pos = positions(lists)
    lib = ctx.lib
    ranks = []
    for r in range(world):
        pf = MoePrefill(ctx, H, I, E, k, 2, 1, O.MXFP4, max_tokens=Tr)
        pf.set_order(pos)
        pf.load_list(packer.gateup, packer.down, lists[r])
        x = ctx.upload_new(xb[r * Tr * H:(r + 1) * Tr * H])
        recv = ctx.alloc(T * k * H * 2)
        yb = ctx.alloc(Tr * k * H * 4)
        act = ctx.alloc(T * k * I * 2)
        ctx._finish(lib.moearc_x_prefill_route_begin(pf.h, x.ptr, Tr, rw.ptr, None), "route_begin")
        ranks.append(dict(pf=pf, x=x, recv=recv, yb=yb, act=act, counts=pf.buffer(3, np.int32, E)))
    counts_all = np.stack([d["counts"] for d in ranks])
    plans = [peer_plan(counts_all, r, world) for r in range(world)]
    dst = (C.c_void_p * world)(*[d["recv"].ptr for d in ranks])
    for r, d in enumerate(ranks):
        base = np.ascontiguousarray(plans[r]["dst_base"], np.int32)
        ctx._finish(lib.moearc_x_prefill_route_dispatch(d["pf"].h, dst, base.ctypes.data, world, nl), "dispatch")
    for r, d in enumerate(ranks):
        pl = plans[r]
        seg_dst = (C.c_void_p * len(pl["seg_row"]))(
            *[ranks[i // nl]["yb"].ptr + int(row) * H * 4 for i, row in enumerate(pl["seg_row"])])
        sc = np.ascontiguousarray(pl["seg_counts"], np.int32)
        se = np.ascontiguousarray(pl["seg_expert"], np.int32)
        ctx._finish(lib.moearc_x_prefill_experts_to(d["pf"].h, d["recv"].ptr, pl["n_recv"], sc.ctypes.data,
                                                    se.ctypes.data, len(sc), d["act"].ptr, seg_dst), "experts_to")
    for s, d in enumerate(ranks):
        out = ctx.alloc_n(np.float32, Tr * H)
        d["pf"].combine(d["yb"].ptr, Tr, out.ptr)
        got = ctx.download(out, np.float32, Tr * H).reshape(Tr, H)
        assert np.array_equal(got.view(np.uint32), want[s * Tr:(s + 1) * Tr].view(np.uint32)), (world, s)
        assert d["pf"].status() == 0
        d["pf"].close()
    whole.close()
    packer.close()


@pytest.mark.parametrize("four_bit", [False, True])
def test_expert_biases_in_the_gemm_epilogues_match_the_oracle(ctx, four_bit):
    """gpt-oss's per-expert biases (moe.rs:2310-2331 before the activation, 2362-2372 inside the
    weighting) added in the gate-up and down GEMM epilogues, bf16 and 4-bit weight forms, against
    the oracle's MoE block with the same biases at the bf16 bound."""
    H, I, E, k, T = 2880, 2880, 32, 4, 40
    pf, packer, host = build(ctx, H, I, E, k, 2, 1, O.MXFP4, T, 0x9F21)
    if four_bit:
        pf.load4(packer.gateup, packer.down)
    gu_b = O.synth_normal_f32(0x9F22, 2 * E * I, 0.5)
    dn_b = O.synth_normal_f32(0x9F23, E * H, 0.5)
    pf.set_bias(ctx.upload_new(gu_b), ctx.upload_new(dn_b))
    xb = O.synth_normal_bf16(0x9F24, T * H, 1.0)
    out = ctx.alloc_n(np.float32, T * H)
    pf.forward(ctx.upload_new(xb), T, ctx.upload_new(host[3]), out)
    got = ctx.download(out, np.float32, T * H).reshape(T, H)
    assert pf.status() == 0
    gate, up, down, router = host
    cfg = O.MoeCfg(H, I, E, k, 2, 1, 1.702, 7.0, O.MXFP4, 1)
    x32 = O.bf16_to_f32(xb).reshape(T, H)
    want = np.zeros((T, H), np.float32)
    for t in range(T):
        xt = np.ascontiguousarray(x32[t])
        assert O.lib().or_moe_ffn_token(cfg, O.ptr(xt), O.ptr(router), None, O.ptr(gate), O.ptr(up), O.ptr(down),
                                        O.ptr(gu_b[:E * I]), O.ptr(gu_b[E * I:]), O.ptr(dn_b), O.ptr(want[t]),
                                        None, None) == 0
    worst = bf16_err(got, want)
    print(f"prefill expert biases four_bit={four_bit}: max rel err {worst:.3e} over {T} tokens (bound 1e-2)")
    assert worst <= 1e-2
    pf.close()
    packer.close()


def test_mxfp8_mode_matches_the_quantisation_aware_oracle(ctx):
    """The MXFP8 perf mode (block-scaled FP8 GEMMs, tcgen05.mma kind::mxf8f6f4; MXFP4 weights exact
    as E4M3, activations quantised to MXFP8 per 32) at the gpt-oss expert shape: routing
    bit-exact; against the oracle that applies the same declared quantisation within 5e-3 of the
    output's scale; against the exact oracle the error of the quantisation itself, printed (and
    held under 5e-2)."""
    H, I, E, k, T = 2880, 2880, 32, 4, 40
    pf, packer, host = build(ctx, H, I, E, k, 2, 1, O.MXFP4, T, 0x9F31)
    pf.load8(packer.gateup, packer.down)
    xb = O.synth_normal_bf16(0x9F32, T * H, 1.0)
    out = ctx.alloc_n(np.float32, T * H)
    pf.forward(ctx.upload_new(xb), T, ctx.upload_new(host[3]), out)
    got = ctx.download(out, np.float32, T * H).reshape(T, H)
    assert pf.status() == 0
    idx = pf.buffer(0, np.uint32, T * k).reshape(T, k)
    gate, up, down, router = host
    cfg = O.MoeCfg(H, I, E, k, 2, 1, 1.702, 7.0, O.MXFP4, 1)
    x32 = O.bf16_to_f32(xb).reshape(T, H)
    want_q, want = np.zeros((T, H), np.float32), np.zeros((T, H), np.float32)
    for t in range(T):
        xt = np.ascontiguousarray(x32[t])
        widx = np.zeros(k, np.uint32)
        assert O.lib().or_moe_ffn_token_mx8(cfg, O.ptr(xt), O.ptr(router), None, O.ptr(gate), O.ptr(up), O.ptr(down),
                                            None, None, None, O.ptr(want_q[t]), O.ptr(widx), None) == 0
        assert np.array_equal(idx[t], widx), t
        want[t], _, _ = oracle_token(H, I, E, k, 2, 1, O.MXFP4, host, xt)
    err_q, err = bf16_err(got, want_q), bf16_err(got, want)
    print(f"prefill MXFP8: {T} tokens, max rel err {err_q:.3e} against the quantisation-aware oracle, "
          f"{err:.3e} against the exact oracle")
    assert err_q <= 5e-3 and err <= 5e-2
    pf.close()
    packer.close()


def test_mxfp8_mode_refuses_q4_0_experts(ctx):
    H, I, E, k = 2048, 768, 16, 4
    pf, packer, host = build(ctx, H, I, E, k, 1, 0, O.Q4_0, 8, 0x9F41)
    from moearc_b200.kernels import BadArgument
    with pytest.raises(BadArgument):
        pf.load8(packer.gateup, packer.down)
    pf.close()
    packer.close()
