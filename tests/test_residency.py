"""Routing-trace replay (moearc_b200.residency): the trace reader's refusals, the policies'
defining cases (crates/moearc-engine/src/residency.rs:1085-1215, cache.rs:268-380), the device
plan's slot rule, and the reference's published hit rates for its captured gpt-oss-120b
decode traces reproduced exactly (bench/policy-sweep.md:142-182). CPU only."""
from __future__ import annotations

import json
import os
import random

import numpy as np
import pytest

from moearc_b200.residency import SimError, Trace, TraceError, main, simulate

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
HEADER = '{"format":"moearc-trace-v1","phase":"decode","n_layer":2}'
MIB = 1 << 20


def trace_of(*steps):
    return Trace([list(s) for s in steps])


@pytest.fixture(scope="module")
def captured():
    z = np.load(os.path.join(GOLDEN, "traces_gptoss120b.npz"))
    return {n: Trace.from_pairs(z[n], str(z[f"{n}_header"])) for n in ("prose", "code", "reasoning")}


@pytest.fixture(scope="module")
def published():
    with open(os.path.join(GOLDEN, "policy_sweep_gptoss120b.json")) as f:
        return json.load(f)


# ---- reading ---------------------------------------------------------------------------------

def test_a_capture_round_trips_with_its_header_verbatim():
    text = "\n".join([HEADER, '{"step":0,"e":[0,7,1,3,1,9]}', "", '{"step":1,"pos":5,"e":[0,7,1,3,0,2]}'])
    t = Trace.from_text(text)
    assert t.header == HEADER
    assert t.steps == [[(0, 7), (1, 3), (1, 9)], [(0, 7), (1, 3), (0, 2)]]
    assert (t.demands(), t.working_set(), t.peak_step_demand()) == (6, 4, 3)
    r = simulate(t, 8, "lru", MIB)
    assert (r.demands, r.compulsory_misses, r.hits) == (6, 4, 2)


@pytest.mark.parametrize("line, why", [
    ('{"step":0,"e":[0,1,2]}', "odd number"),
    ('{"step":0}', 'no "e"'),
    ('{"step":0,"e":[0,1', "unterminated"),
    ('{"step":0,"e":[0,-1]}', "non-negative"),
    ('{"step":0,"e":[0,65536]}', "below 65536"),
    ('{"step":0,"e":[0,x]}', "non-negative"),
])
def test_a_malformed_step_is_refused_with_its_line(line, why):
    with pytest.raises(TraceError) as ei:
        Trace.from_text("\n".join([HEADER, '{"step":0,"e":[0,1]}', line]))
    assert "line 3" in str(ei.value) and why in str(ei.value)


def test_a_file_that_is_not_a_trace_is_refused_by_its_header():
    with pytest.raises(TraceError, match="empty"):
        Trace.from_text("\n\n")
    with pytest.raises(TraceError, match="not a moearc-trace-v1"):
        Trace.from_text('{"format":"other"}\n{"e":[0,1]}')
    with pytest.raises(TraceError, match="no step lines"):
        Trace.from_text(HEADER + "\n")


def test_an_empty_step_is_a_step():
    t = Trace.from_text(HEADER + '\n{"e":[]}\n{"e":[0,1]}')
    assert t.steps == [[], [(0, 1)]]


# ---- the shared pool (lru, optimal) and the static split ------------------------------------

def test_everything_resident_means_only_compulsory_misses():
    t = trace_of([(0, 0), (0, 1)], [(0, 0), (0, 1)], [(0, 1), (0, 0)])
    r = simulate(t, 8, "lru", MIB)
    assert (r.demands, r.misses, r.compulsory_misses, r.avoidable_misses) == (6, 2, 2, 0)
    assert r.bytes_fetched == 2 * MIB


def test_lru_evicts_the_least_recently_used():
    t = trace_of([(0, 0)], [(0, 1)], [(0, 2)], [(0, 0)])
    r = simulate(t, 2, "lru", MIB)
    assert (r.misses, r.compulsory_misses, r.avoidable_misses) == (4, 3, 1)


def test_an_expert_needed_this_step_is_never_evicted_for_another():
    # capacity 2; step 2 needs a and c: a is the LRU but pinned, so b goes
    t = trace_of([(0, 0)], [(0, 1)], [(0, 2), (0, 0)], [(0, 0)])
    r = simulate(t, 2, "lru")
    assert r.misses == 3 and r.hits == 2


def _random_trace(seed, steps=60, layers=3, experts=12, k=2):
    rng = random.Random(seed)
    return Trace([[(l, e) for l in range(layers) for e in rng.sample(range(experts), k)] for _ in range(steps)])


@pytest.mark.parametrize("seed", [1, 7, 42, 1234])
def test_optimal_is_never_worse_than_lru(seed):
    t = _random_trace(seed)
    for cap in (6, 9, 14, 20):
        assert simulate(t, cap, "optimal").hits >= simulate(t, cap, "lru").hits


def test_optimal_beats_lru_on_a_trace_designed_to_fool_recency():
    # a cyclic scan one larger than the cache: LRU misses every time, Belady keeps most
    t = trace_of(*([[(0, e)] for e in range(4)] * 6))
    assert simulate(t, 3, "lru").hits == 0
    assert simulate(t, 3, "optimal").hits > 0


def test_capacity_below_a_single_step_is_refused_rather_than_thrashing():
    t = trace_of([(0, 0), (0, 1), (0, 2)])
    for p in ("lru", "optimal"):
        with pytest.raises(SimError, match="unservable"):
            simulate(t, 2, p)
    with pytest.raises(SimError):
        simulate(t, 0, "lru")


def test_a_static_split_may_not_exceed_the_shared_capacity():
    t = trace_of([(0, 0), (0, 1), (1, 0)], [(0, 2), (1, 1)])
    assert t.widest_static_split(3) == 1
    r = simulate(t, 3, "static")
    assert (r.hits, r.misses, r.compulsory_misses) == (3, 2, 0)
    with pytest.raises(SimError, match="needs 5 slots"):
        simulate(t, 3, "static", resident_layers=2)


def test_lru2_keeps_an_expert_used_twice_over_one_used_once():
    # capacity 2: a is used twice, then b once; c's miss evicts b (one reference) not a
    t = trace_of([(0, 0)], [(0, 0)], [(0, 1)], [(0, 2)], [(0, 0)])
    assert simulate(t, 2, "lru").hits == 1          # LRU evicts a, the least recent
    assert simulate(t, 2, "lru2").hits == 2


def test_slru_lets_a_once_used_expert_leave_before_a_reused_one():
    # capacity 2, one protected slot: a is promoted by its second use, b and c pass through
    t = trace_of([(0, 0)], [(0, 0)], [(0, 1)], [(0, 2)], [(0, 0)])
    assert simulate(t, 2, "slru", protected_pct=50).hits == 2


def test_transfer_time_converts_bytes_into_seconds():
    t = trace_of([(0, 0)], [(0, 1)])
    r = simulate(t, 1, "lru", 10 * MIB)
    assert r.transfer_seconds(10 * MIB) == pytest.approx(2.0)
    assert r.transfer_seconds(0) == float("inf")


# ---- the device plan: per-block slots, step stamps -------------------------------------------

def test_block_cold_cache_loads_each_expert_once():
    t = trace_of([(0, 3), (0, 1), (1, 1)], [(0, 1), (0, 3), (1, 1)])
    r = simulate(t, 2, "block", MIB)
    assert (r.misses, r.compulsory_misses, r.hits, r.bytes_fetched) == (3, 3, 3, 3 * MIB)
    assert r.per_layer_misses == [2, 1]
    assert r.capacity == 4


def test_block_every_slot_is_used_before_anything_is_evicted():
    t = trace_of(*[[(0, e)] for e in range(4)], *[[(0, e)] for e in range(4)])
    r = simulate(t, 4, "block")
    assert (r.misses, r.hits) == (4, 4)


def test_block_evicts_the_oldest_step_and_the_lowest_slot_on_a_tie():
    # 2 slots; step 0 fills slots 0, 1 with experts 1, 2 (same stamp); expert 3 takes slot 0
    # (the tie's lowest index), so expert 2 still hits at step 2 and expert 1 misses at step 3
    t = trace_of([(0, 2), (0, 1)], [(0, 3)], [(0, 2)], [(0, 1)])
    r = simulate(t, 2, "block")
    assert (r.hits, r.misses) == (1, 4)
    # a touch refreshes the stamp: after 1 is used again, 2 is the one that leaves
    t = trace_of([(0, 1), (0, 2)], [(0, 1)], [(0, 3)], [(0, 1)], [(0, 2)])
    r = simulate(t, 2, "block")
    assert (r.hits, r.misses) == (2, 4)


def test_block_never_evicts_an_expert_the_step_holds():
    # 2 slots: step 1 needs 1 (resident, oldest) and 3: 2 leaves, not 1
    t = trace_of([(0, 1)], [(0, 2)], [(0, 3), (0, 1)], [(0, 1)])
    r = simulate(t, 2, "block")
    assert (r.hits, r.misses) == (2, 3)


def test_block_takes_one_capacity_per_block_and_refuses_a_step_larger_than_it():
    t = trace_of([(0, 0), (0, 1), (1, 0)])
    assert simulate(t, [2, 1], "block").capacity == 3
    with pytest.raises(SimError, match="block 0 needs 2"):
        simulate(t, [1, 1], "block")
    with pytest.raises(SimError):
        simulate(t, [2], "block")
    with pytest.raises(SimError):
        simulate(t, 0, "block")


def test_a_repeat_within_a_step_is_one_fetch_then_a_hit():
    t = trace_of([(0, 5), (0, 5)])
    for p, cap in (("lru", 2), ("block", 1)):
        r = simulate(t, cap, p)
        assert (r.misses, r.hits) == (1, 1), p


# ---- the reference's captured traces and published numbers -----------------------------------

def test_captured_traces_have_the_shape_the_reference_published(captured, published):
    for name, t in captured.items():
        want = published["shape"][name]
        assert '"format":"moearc-trace-v1"' in t.header and '"n_expert_used":4' in t.header
        assert len(t.steps) == want["steps"] == 512
        assert t.peak_step_demand() == 144 and t.n_layers() == 36
        assert t.working_set() == want["working_set"], name
        assert round(100 * t.step_reuse(), 1) == want["step_reuse_pct"], name
        assert round(100 * t.top_share(0.1, round_up=False), 1) == want["top10_pct"], name


def test_replays_reproduce_the_published_hit_rates(captured, published):
    """static / lru / slru80 / lru-2 / belady at nine capacities on three traces, to the
    published 0.1 %."""
    got, want = [], []
    for name, t in captured.items():
        for row in published["sweeps"][name]:
            for ours, theirs in (("static", "static"), ("lru", "lru"), ("slru", "slru80"), ("lru2", "lru-2"),
                                 ("optimal", "belady")):
                got.append((name, row["slots"], ours, round(100 * simulate(t, row["slots"], ours).hit_rate, 1)))
                want.append((name, row["slots"], ours, row[theirs]))
    assert got == want


def test_per_block_slots_cost_little_against_one_shared_pool(captured):
    """The device's partitioned cache against a shared LRU pool of the same total size: within
    two points at every size tried, on every trace."""
    for name, t in captured.items():
        for per in (6, 16, 32):
            b = simulate(t, per, "block").hit_rate
            p = simulate(t, per * 36, "lru").hit_rate
            assert abs(b - p) < 0.02, (name, per, b, p)


def test_the_command_line_prints_a_table(tmp_path, capsys):
    f = tmp_path / "t.ndjson"
    f.write_text("\n".join([HEADER] + ['{"e":[0,%d,1,%d]}' % (i % 3, i % 2) for i in range(8)]) + "\n")
    main([str(f), "--capacity", "4", "--per-block", "2", "--expert-mib", "1"])
    out = capsys.readouterr().out
    assert "working set 5" in out and "lru" in out and "2/block" in out


def test_the_bench_steers_each_offloaded_block_to_the_trace(captured):
    """bench.py --trace: the router of each steered block has one nonzero column holding
    positive, distinct values at exactly that step's experts, ffn_norm[0] is set to 1 once, and
    the fetch prediction is the block replay of the steps applied."""
    import bench

    class FakeDecoder:
        class cfg:
            n_expert, n_embd, n_expert_used = 128, 64, 4

        def __init__(self):
            self.t = {}

        def tensor(self, which, layer, dtype):
            return np.full(self.cfg.n_embd, -0.5, np.float32)

        def set_tensor(self, which, layer, data):
            self.t[(which, layer)] = np.array(data)

    dec = FakeDecoder()
    route = bench.TraceRoute(dec, "code", 3)
    assert all(dec.t[(1, l)][0] == 1.0 and dec.t[(1, l)][1] == -0.5 for l in range(3))
    steps = [[[e for l2, e in s if l2 == l] for l in range(3)] for s in captured["code"].steps[:5]]
    for s in steps:
        route.apply()
        for l in range(3):
            w = dec.t[(3, l)]
            assert not w[:, 1:].any()
            col = w[:, 0]
            assert sorted(np.flatnonzero(col)) == sorted(s[l]) and np.all(col[s[l]] > 0)
            assert len(set(col[s[l]])) == len(s[l])
    t = Trace([[(l, e) for l in range(3) for e in s[l]] for s in steps])
    assert route.replay_fetches(8, 5) == simulate(t, 8, "block").misses
    assert route.replay_fetches(8, 0) == 0


def test_the_bench_reads_a_trace_file_and_refuses_one_that_does_not_fit(tmp_path):
    import bench

    class FakeDecoder:
        class cfg:
            n_expert, n_embd, n_expert_used = 8, 16, 2

        def tensor(self, which, layer, dtype):
            return np.zeros(self.cfg.n_embd, np.float32)

        def set_tensor(self, which, layer, data):
            pass

    f = tmp_path / "t.ndjson"
    f.write_text(HEADER + '\n{"e":[0,1,0,2,1,3,1,4]}\n{"e":[0,1,0,5,1,3,1,7]}\n')
    route = bench.TraceRoute(FakeDecoder(), str(f), 2)
    assert route.steps == [[[1, 2], [3, 4]], [[1, 5], [3, 7]]]
    f.write_text(HEADER + '\n{"e":[0,1,0,9,1,3,1,4]}\n')
    with pytest.raises(SystemExit, match="not 2 distinct of 8"):
        bench.TraceRoute(FakeDecoder(), str(f), 2)
