"""One rank of tests/test_gpu_ep_nccl.py: the prefill MoE block over NCCL through the C ABI
(moearc_x_ep_*) against the single-GPU block on the same tokens. argv: rank world id_hex out_json.
The parent sets CUDA_VISIBLE_DEVICES so that device 0 is this rank's GPU."""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

import oracle as O  # noqa: E402
from moearc_b200 import Context  # noqa: E402
from moearc_b200.ep import NcclExpertParallelPrefill, balanced  # noqa: E402
from moearc_b200.moe import MoeLayer, MoePrefill  # noqa: E402


def main() -> None:
    rank, world, id_hex, out_path = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4]
    placement = sys.argv[5] if len(sys.argv) > 5 else "interleaved"
    H, I, E, k, T = 1024, 512, 32, 4, 600 * world
    Tr = T // world
    ctx = Context()
    nb = E * I * H // 32
    gate, up, down = (O.synth_mxfp4(0xE9C0 + i, nb) for i in range(3))
    router = O.synth_normal_f32(0xE9C7, E * H, 0.02)
    packer = MoeLayer(ctx, H, I, E, k, 2, 1, O.MXFP4, max_tokens=1)
    packer.pack(ctx.upload_new(gate), ctx.upload_new(up), ctx.upload_new(down))
    rw = ctx.upload_new(router)
    xb = O.synth_normal_bf16(0xE9C8, T * H, 1.0)
    x = ctx.upload_new(xb[rank * Tr * H:(rank + 1) * Tr * H].copy())
    res = ctx.upload_new(O.synth_normal_f32(0xE9C9 + rank, Tr * H, 1.0))
    whole = MoePrefill(ctx, H, I, E, k, 2, 1, O.MXFP4, max_tokens=T)
    whole.load(packer.gateup, packer.down)
    ref = ctx.alloc_n(np.float32, Tr * H)
    whole.forward(x, Tr, rw, ref, residual=res)
    want = ctx.download(ref, np.float32, Tr * H)
    lists = None
    if placement == "balanced":
        # every rank places by the whole batch's popularity (the same on every rank)
        whole.forward(ctx.upload_new(xb), T, rw, ctx.alloc_n(np.float32, T * H))
        lists = balanced(whole.buffer(3, np.int32, E), world)
    ep = NcclExpertParallelPrefill(ctx, rank, world, H, I, E, k, 2, 1, O.MXFP4, max_tokens=Tr, max_rows=T * k,
                                   unique_id=bytes.fromhex(id_hex))
    ep.load(packer.gateup, packer.down, lists)
    out = ctx.alloc_n(np.float32, Tr * H)
    results = []
    for rep in range(3):  # the exchange repeated on the same buffers gives the same bits
        n = ep.forward(x, Tr, rw, out.ptr, residual_ptr=res.ptr)
        got = ctx.download(out, np.float32, Tr * H)
        results.append({"equal": bool(np.array_equal(got.view(np.uint32), want.view(np.uint32))),
                        "max_abs": float(np.max(np.abs(got - want))), "received": int(n)})
    counts = ep.counts_all()
    status = ep.pf.status()
    ep.close()
    with open(out_path, "w") as f:
        json.dump({"rank": rank, "results": results, "status": status, "rows": int(counts.sum()),
                   "expected_rows": T * k}, f)


if __name__ == "__main__":
    main()
