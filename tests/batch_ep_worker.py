"""One rank of tests/test_gpu_batch_ep.py: the batched decoder with its experts split over the
ranks (moearc_x_batch_decoder_create_ep, NCCL inside the step graph) against the single-GPU
batched decoder of all ranks' streams, run in the same process. argv: rank world id_hex out_json.
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
from moearc_b200.decoder import BatchDecoder, DecoderConfig  # noqa: E402
from moearc_b200.ep import nccl_comm, nccl_comm_destroy  # noqa: E402


def main() -> None:
    rank, world, id_hex, out_path = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4]
    # Q4_0 experts with QK-norm (the qwen3moe form), eight experts split over the ranks
    kw = dict(n_layer=2, n_embd=256, n_head=8, n_head_kv=2, head_dim=64, n_expert=8, n_expert_used=2, n_ff=128,
              expert_type=O.Q4_0, n_swa=0, has_sinks=0, n_ctx=96, seed=0xBA7C, has_qk_norm=1, expert_layout=0)
    Bl = 3
    ctx = Context()
    comm = nccl_comm(ctx, rank, world, bytes.fromhex(id_hex))
    ep = BatchDecoder(ctx, DecoderConfig(**kw), Bl, ep=(comm, rank, world))
    whole = BatchDecoder(ctx, DecoderConfig(**kw), Bl * world)
    ep.set_pos(0)
    whole.set_pos(0)
    results = []
    for pos in range(40):  # past a page boundary
        x = np.stack([O.synth_normal_f32(0x3000 + 97 * b + pos, kw["n_embd"], 1.0) for b in range(Bl * world)])
        ep.set_input(x[rank * Bl:(rank + 1) * Bl])
        ep.step()
        whole.set_input(x)
        whole.step()
        got, want = ep.output(), whole.output()[rank * Bl:(rank + 1) * Bl]
        route_eq = all(np.array_equal(ep.routing(l), whole.routing(l)[rank * Bl:(rank + 1) * Bl])
                       for l in range(kw["n_layer"]))
        results.append({"pos": pos, "equal": bool(np.array_equal(got.view(np.uint32), want.view(np.uint32))),
                        "max_abs": float(np.max(np.abs(got - want))), "route_equal": bool(route_eq)})
    status = [ep.status(), whole.status()]
    ep.close()
    whole.close()
    nccl_comm_destroy(ctx, comm)
    ctx.close()
    with open(out_path, "w") as f:
        json.dump({"rank": rank, "results": results, "status": status}, f)


if __name__ == "__main__":
    main()
