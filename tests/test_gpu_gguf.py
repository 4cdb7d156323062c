"""A MoE block loaded from a GGUF file (moearc_b200.gguf.load_moe_block: the stacked expert
banks and the router go to the device straight from the file's mapping) decodes as the
oracle's MoE block does on the same bytes, for MXFP4 and Q4_0 experts, and the device copies
equal the file's bytes. The file is written by the test (tests/gguf_writer.py) in the layout of
llama.cpp's GGUF writer for gpt-oss (blk.N.ffn_{gate,up,down}_exps.weight,
blk.N.ffn_gate_inp.weight; dims fastest-varying first)."""
import numpy as np
import pytest

import gguf_writer as W
import oracle as O
from moearc_b200 import Context
from moearc_b200.gguf import GgufFile, load_moe_block
from moearc_b200.moe import MoeLayer

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = Context()
    yield c
    c.close()


@pytest.mark.parametrize("wtype", [O.MXFP4, O.Q4_0])
def test_moe_block_from_a_gguf_file_matches_the_oracle(ctx, tmp_path, wtype):
    H, I, E, k, T = 512, 256, 8, 2, 3
    nb_gate, nb_down = E * I * H // 32, E * H * I // 32
    if wtype == O.MXFP4:
        gate, up, down = (O.synth_mxfp4(0x6600 + i, n) for i, n in enumerate((nb_gate, nb_gate, nb_down)))
    else:
        gate, up, down = (O.synth_q4_0(0x6600 + i, n, 0.01) for i, n in enumerate((nb_gate, nb_gate, nb_down)))
    router = O.synth_normal_f32(0x6607, E * H, 0.02)
    w = W.GgufWriter()
    w.add("general.architecture", W.STRING, "gpt-oss")
    w.add("gpt-oss.expert_count", W.U32, E)
    w.add("gpt-oss.expert_used_count", W.U32, k)
    w.add_tensor("blk.0.ffn_gate_inp.weight", (H, E), 0, router.tobytes())
    w.add_tensor("blk.0.ffn_gate_exps.weight", (H, I, E), wtype, gate.tobytes())
    w.add_tensor("blk.0.ffn_up_exps.weight", (H, I, E), wtype, up.tobytes())
    w.add_tensor("blk.0.ffn_down_exps.weight", (I, H, E), wtype, down.tobytes())
    path = str(tmp_path / "block.gguf")
    w.write(path)

    with GgufFile(path) as g:
        bank = load_moe_block(ctx, g, 0)
        assert (bank.n_embd, bank.n_ff, bank.n_expert, bank.wtype) == (H, I, E, wtype)
        assert g.u64("gpt-oss.expert_used_count") == k
    # the device copies are the file's bytes
    for dev, host in ((bank.gate, gate), (bank.up, up), (bank.down, down), (bank.router, router)):
        got = ctx.download(dev, np.uint8, host.nbytes)
        assert np.array_equal(got, host.view(np.uint8).reshape(-1))

    layer = MoeLayer(ctx, H, I, E, k, 2, 1, wtype, max_tokens=T)
    layer.pack(bank.gate, bank.up, bank.down)
    x = O.synth_normal_f32(0x6610, T * H, 1.0)
    out = ctx.alloc_n(np.float32, T * H)
    layer.forward(ctx.upload_new(x), T, bank.router, out)
    got = ctx.download(out, np.float32, T * H).reshape(T, H)
    assert layer.status() == 0
    cfg = O.MoeCfg(H, I, E, k, 2, 1, 1.702, 7.0, wtype, 1)
    worst = 0.0
    for t in range(T):
        want = np.zeros(H, np.float32)
        widx = np.zeros(k, np.uint32)
        xt = x[t * H:(t + 1) * H].copy()
        assert O.lib().or_moe_ffn_token(cfg, O.ptr(xt), O.ptr(router), None, O.ptr(gate), O.ptr(up),
                                        O.ptr(down), None, None, None, O.ptr(want), O.ptr(widx), None) == 0
        worst = max(worst, float(np.max(np.abs(got[t].astype(np.float64) - want) / np.maximum(np.abs(want), 1.0))))
    print(f"GGUF-loaded MoE block wtype={wtype}: max rel err {worst:.3e} over {T} tokens (bound 1e-4)")
    assert worst <= 1e-4
    layer.close()
