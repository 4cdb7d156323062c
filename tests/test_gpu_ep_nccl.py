"""Expert parallelism through the C ABI over NCCL (moearc_x_ep_*) on 2 GPUs: one process per
GPU (tests/ep_nccl_worker.py), the experts split over the ranks, each rank's tokens routed,
exchanged, computed and returned through the library's NCCL calls — the output of every rank
bit-identical to the single-GPU block on its tokens, over three repeated exchanges. Skipped on a
box with fewer than two GPUs."""
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


@pytest.mark.parametrize("placement", ["interleaved", "balanced"])
def test_expert_parallel_block_over_nccl_gives_the_single_gpu_bits(tmp_path, placement):
    world = 2
    if _gpus() < world:
        pytest.skip("needs two GPUs")
    from moearc_b200 import _lib
    from moearc_b200.ep import nccl_unique_id

    uid = nccl_unique_id(_lib.load()).hex()
    procs = []
    for r in range(world):
        env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(r), NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "ep_nccl_worker.py"), str(r), str(world),
                                       uid, str(tmp_path / f"r{r}.json"), placement], env=env,
                                      start_new_session=True))
    try:
        codes = [p.wait(timeout=600) for p in procs]
    finally:
        for p in procs:
            if p.poll() is None:
                os.killpg(p.pid, 9)
    assert codes == [0] * world, codes
    rows = 0
    for r in range(world):
        d = json.load(open(tmp_path / f"r{r}.json"))
        assert d["status"] == 0
        for res in d["results"]:
            assert res["equal"], (r, res)
        assert len({res["received"] for res in d["results"]}) == 1
        rows += d["results"][0]["received"]
        assert d["rows"] == d["expected_rows"]
    assert rows == d["expected_rows"]  # every (token, choice) row computed once, on its expert's rank
