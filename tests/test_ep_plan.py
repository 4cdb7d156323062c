"""Expert-parallel exchange plan (moearc_b200.ep.plan), host logic only: the splits every rank
computes from the gathered per-expert counts agree pairwise (what a sends to b is what b
receives from a), the received segments cover the received rows, and the same holds when the
counts travel between two gloo ranks on the CPU."""
import multiprocessing as mp
import os

import numpy as np
import pytest

from moearc_b200.ep import balanced, interleaved, plan, positions


def test_plans_agree_pairwise():
    rng = np.random.default_rng(3)
    for world in (1, 2, 4, 8):
        E = 16 * world
        counts = rng.integers(0, 50, size=(world, E))
        counts[:, rng.integers(0, E, size=3)] = 0  # empty experts
        plans = [plan(counts, r, world) for r in range(world)]
        for a in range(world):
            assert sum(plans[a]["send"]) == counts[a].sum()
            assert plans[a]["n_recv"] == int(plans[a]["seg_counts"].sum())
            assert len(plans[a]["seg_counts"]) == world * (E // world)
            for b in range(world):
                assert plans[a]["send"][b] == plans[b]["recv"][a]
            # segments: source-major, each source's block in expert order
            nl = E // world
            assert np.array_equal(plans[a]["seg_expert"], np.tile(np.arange(nl), world))


def test_placements_are_owner_major_permutations():
    rng = np.random.default_rng(5)
    for world in (2, 4, 8):
        E = 16 * world
        counts = np.floor(1e4 * (1.0 + np.arange(E)) ** -1.1).astype(int)[rng.permutation(E)]
        for lists in (interleaved(E, world), balanced(counts, world)):
            assert sorted(e for l in lists for e in l) == list(range(E))
            assert all(len(l) == E // world for l in lists)
            pos = positions(lists)
            assert sorted(pos) == list(range(E))
            for r, l in enumerate(lists):
                assert all(r * (E // world) <= pos[e] < (r + 1) * (E // world) for e in l)
        # balanced is no worse than interleaved on a Zipf-like load
        load = lambda lists: max(sum(counts[e] for e in l) for l in lists)
        assert load(balanced(counts, world)) <= load(interleaved(E, world))


def test_plan_rejects_uneven_split():
    with pytest.raises(ValueError):
        plan(np.zeros((3, 8)), 0, 3)


def _rank(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(100 + rank)
    mine = torch.from_numpy(rng.integers(0, 30, size=32).astype(np.int64))
    got = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(got, mine)
    counts_all = torch.stack(got).numpy()
    p = plan(counts_all, rank, world)
    sends = [torch.empty(world, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(sends, torch.tensor(p["send"], dtype=torch.int64))
    ok = all(int(sends[s][rank]) == p["recv"][s] for s in range(world))
    dist.destroy_process_group()
    q.put((rank, ok, p["n_recv"], int(counts_all[:, rank * 16:(rank + 1) * 16].sum())))


def test_plan_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 2000
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    for rank, ok, n_recv, want in res:
        assert ok and n_recv == want, rank


def test_peer_plan_offsets():
    """The peer-memory offsets: a source's rows start in every receiver after all lower sources'
    rows, and each received segment's results go to the rows its source's route step used."""
    from moearc_b200.ep import peer_plan

    rng = np.random.default_rng(9)
    world, E = 4, 32
    nl = E // world
    counts = rng.integers(0, 20, size=(world, E))
    plans = [peer_plan(counts, r, world) for r in range(world)]
    for r in range(world):
        recv_starts = np.concatenate([[0], np.cumsum(plans[r]["recv"])])[:-1]
        for s in range(world):
            assert plans[s]["dst_base"][r] == recv_starts[s]
        for i, row in enumerate(plans[r]["seg_row"]):
            s, j = divmod(i, nl)
            assert row == counts[s, :r * nl + j].sum()
