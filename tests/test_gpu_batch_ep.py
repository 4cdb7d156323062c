"""The batched decoder with expert parallelism (moearc_x_batch_decoder_create_ep) on 2 GPUs: one
process per GPU (tests/batch_ep_worker.py), each rank decoding its own three streams with half of
the experts, the rows all-gathered and the results returned over NCCL inside each rank's step
graph — every rank's outputs and routing bit-identical, over 40 steps, to the single-GPU batched
decoder of all six streams (the same kernels on the same rows; the exchange only moves them).
Skipped on a box with fewer than two GPUs."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _gpus() -> int:
    try:
        out = subprocess.run(["nvidia-smi", "-L"], capture_output=True, text=True, timeout=60).stdout
        return sum(1 for l in out.splitlines() if l.startswith("GPU "))
    except (OSError, subprocess.SubprocessError):
        return 0


def test_expert_parallel_batched_decode_gives_the_single_gpu_bits(tmp_path):
    world = 2
    if _gpus() < world:
        pytest.skip("needs two GPUs")
    from moearc_b200 import _lib
    from moearc_b200.ep import nccl_unique_id

    uid = nccl_unique_id(_lib.load()).hex()
    procs = []
    for r in range(world):
        env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(r), NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "batch_ep_worker.py"), str(r), str(world),
                                       uid, str(tmp_path / f"r{r}.json")], env=env, start_new_session=True))
    try:
        codes = [p.wait(timeout=600) for p in procs]
    finally:
        for p in procs:
            if p.poll() is None:
                os.killpg(p.pid, 9)
    assert codes == [0] * world, codes
    for r in range(world):
        d = json.load(open(tmp_path / f"r{r}.json"))
        assert d["status"] == [0, 0]
        for res in d["results"]:
            assert res["route_equal"] and res["equal"], (r, res)
