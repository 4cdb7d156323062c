"""Offline replay of captured expert-routing traces: what an HBM residency cache of a given size
would have hit, before any device time is spent on it.

The host-side sizing tool for the decoder's residency cache of offloaded blocks
(`moearc_x_decoder_cfg.n_cache`). It reads the reference's trace format (moearc-trace-v1,
crates/moearc-engine/src/residency.rs:163-219) and replays it through

- ``lru``: one pool of `capacity` slots shared by every block, least recently used evicted,
  never an expert the current step needs (residency.rs:415-509, `Policy::Lru` at 935);
- ``optimal``: Belady's furthest-next-use victim over the same pool, the bound no online policy
  reaches (residency.rs:937-941, next-use index 970-1000);
- ``static``: the first `resident_layers` blocks wholly resident, every other activation a
  fetch, charged no compulsory misses (residency.rs:433-456; `widest_static_split` 87-99);
- ``lru2`` and ``slru``: the two online candidates the reference found to beat LRU on every
  content type, LRU-2 and segmented LRU with `protected_pct` of the pool protected
  (residency.rs:942-956, 746-812), over the same shared pool;
- ``block``: the policy the device runs (`k_xplan` in csrc/moe.cu): each block owns its own
  `n_cache` slots; per step a block's distinct experts, ascending, keep their slots if resident,
  and each miss takes the slot with the oldest step stamp no expert of that step holds (an empty
  slot first, the lowest slot index on a tie). `capacity` may be one count for every block or a
  list, one per block.

Nothing here touches the device; the decode path never calls it.

    t = Trace.from_file("gptoss120b-code.decode.ndjson")
    simulate(t, 600, "lru").hit_rate
    simulate(t, 16, "block").hit_rate          # 16 slots in each of the 36 blocks
"""
from __future__ import annotations

import argparse
import heapq
import math
from collections import OrderedDict
from dataclasses import dataclass, field

import numpy as np

FORMAT = "moearc-trace-v1"
_EXPERTS_KEY = '"e":['


class TraceError(ValueError):
    """A capture file that is not a readable moearc-trace-v1 trace. A malformed step is refused,
    never skipped: a trace that silently lost steps would understate every miss count."""


@dataclass
class Trace:
    """Per step, the (layer, expert) activations in the order the router named them."""
    steps: list[list[tuple[int, int]]]
    header: str = ""

    # ---- reading -------------------------------------------------------------------------
    @classmethod
    def from_text(cls, text: str) -> "Trace":
        """Parse a capture held in memory (residency.rs:178-219): line 1 (after blank lines) a
        header naming the format, then one step per non-blank line, of which only the flat
        ``"e":[layer, expert, ...]`` array is read."""
        lines = [(i + 1, ln) for i, ln in enumerate(text.splitlines()) if ln.strip()]
        if not lines:
            raise TraceError("trace file is empty: no header line")
        header = lines[0][1]
        if f'"format":"{FORMAT}"' not in header:
            raise TraceError(f"not a {FORMAT} file; first line begins: {header[:60]}")
        steps = []
        for lineno, ln in lines[1:]:
            at = ln.find(_EXPERTS_KEY)
            if at < 0:
                raise TraceError(f'malformed step on line {lineno}: no "e":[...] field')
            rest = ln[at + len(_EXPERTS_KEY):]
            end = rest.find("]")
            if end < 0:
                raise TraceError(f'malformed step on line {lineno}: unterminated "e" array')
            body = rest[:end].strip()
            flat = []
            for tok in (body.split(",") if body else []):
                tok = tok.strip()
                if not tok.isdigit() or int(tok) > 0xFFFF:
                    raise TraceError(f"malformed step on line {lineno}: expected a non-negative "
                                     "integer below 65536")
                flat.append(int(tok))
            if len(flat) % 2:
                raise TraceError(f"malformed step on line {lineno}: odd number of integers; "
                                 "expected layer,expert pairs")
            steps.append(list(zip(flat[0::2], flat[1::2])))
        if not steps:
            raise TraceError("trace file has a header but no step lines")
        return cls(steps, header)

    @classmethod
    def from_file(cls, path: str) -> "Trace":
        with open(path, encoding="utf-8") as f:
            return cls.from_text(f.read())

    @classmethod
    def from_pairs(cls, pairs: np.ndarray, header: str = "") -> "Trace":
        """From an integer array [steps, pairs, 2] of (layer, expert)."""
        a = np.asarray(pairs)
        if a.ndim != 3 or a.shape[2] != 2:
            raise ValueError(f"pairs must be [steps, n, 2], got {a.shape}")
        return cls([[(int(l), int(e)) for l, e in s] for s in a], header)

    # ---- shape ---------------------------------------------------------------------------
    def demands(self) -> int:
        return sum(len(s) for s in self.steps)

    def working_set(self) -> int:
        return len({x for s in self.steps for x in s})

    def peak_step_demand(self) -> int:
        return max((len(s) for s in self.steps), default=0)

    def n_layers(self) -> int:
        return 1 + max((l for s in self.steps for l, _ in s), default=-1)

    def distinct_per_layer(self) -> list[int]:
        seen = [set() for _ in range(self.n_layers())]
        for s in self.steps:
            for l, e in s:
                seen[l].add(e)
        return [len(x) for x in seen]

    def experts_in_layers_below(self, layer: int) -> int:
        return len({x for s in self.steps for x in s if x[0] < layer})

    def top_share(self, frac: float, round_up: bool = True) -> float:
        """Share of all activations taken by the busiest frac x touched experts, that count
        rounded up (examples/trace_report.rs:64-69) or down (the trace table of
        bench/policy-sweep.md:48-52 counts this way)."""
        counts: dict[tuple[int, int], int] = {}
        for s in self.steps:
            for x in s:
                counts[x] = counts.get(x, 0) + 1
        c = sorted(counts.values(), reverse=True)
        k = math.ceil(len(c) * frac) if round_up else int(len(c) * frac)
        return sum(c[:k]) / max(1, self.demands())

    def step_reuse(self) -> float:
        """Share of activations whose expert the immediately preceding step also used."""
        hit = den = 0
        for prev, cur in zip(self.steps, self.steps[1:]):
            p = set(prev)
            den += len(cur)
            hit += sum(x in p for x in cur)
        return hit / max(1, den)

    def widest_static_split(self, capacity: int) -> int:
        """The most blocks, from block 0, whose touched experts fit in `capacity` slots."""
        best = 0
        for l in range(1, self.n_layers() + 1):
            if self.experts_in_layers_below(l) > capacity:
                break
            best = l
        return best


@dataclass
class Residency:
    policy: str
    capacity: int                 # total slots
    steps: int = 0
    demands: int = 0
    hits: int = 0
    misses: int = 0
    compulsory_misses: int = 0
    bytes_fetched: int = 0
    per_layer_misses: list[int] = field(default_factory=list)

    @property
    def hit_rate(self) -> float:
        return self.hits / self.demands if self.demands else 0.0

    @property
    def avoidable_misses(self) -> int:
        return max(0, self.misses - self.compulsory_misses)

    def transfer_seconds(self, bytes_per_second: float) -> float:
        return self.bytes_fetched / bytes_per_second if bytes_per_second > 0 else math.inf


class SimError(ValueError):
    """A replay that cannot run: no slots, fewer slots than one step needs, or a static split
    larger than the budget it is compared at."""


def _count(r: Residency, layer: int, hit: bool, first: bool, per_expert_bytes: int) -> None:
    r.demands += 1
    if hit:
        r.hits += 1
        return
    r.misses += 1
    r.bytes_fetched += per_expert_bytes
    r.per_layer_misses[layer] += 1
    if first:
        r.compulsory_misses += 1


def _pool(trace: Trace, capacity: int, belady: bool, per_expert_bytes: int) -> Residency:
    """One shared pool, per-reference recency (or furthest next use), the step's experts pinned."""
    r = Residency("optimal" if belady else "lru", capacity, len(trace.steps),
                  per_layer_misses=[0] * trace.n_layers())
    seen: set = set()
    lru: OrderedDict = OrderedDict()     # resident experts, least recently used first
    if belady:
        occ: dict = {}
        for i, s in enumerate(trace.steps):
            for x in s:
                v = occ.setdefault(x, [])
                if not v or v[-1] != i:
                    v.append(i)
        ptr: dict = {}                   # index into occ[x] of the step being served
        heap: list = []                  # (-next use, -arrival, expert, version)
        version: dict = {}               # expert -> its live heap entry's serial
        arrival: dict = {}
        tick = serial = 0
    for i, s in enumerate(trace.steps):
        pinned = set(s)
        for x in s:
            first = x not in seen
            seen.add(x)
            if belady:
                while occ[x][ptr.get(x, 0)] < i:
                    ptr[x] = ptr.get(x, 0) + 1
                j = ptr.get(x, 0)
                nxt = occ[x][j + 1] if j + 1 < len(occ[x]) else math.inf
            if x in lru:
                lru.move_to_end(x)
                _count(r, x[0], True, False, per_expert_bytes)
            else:
                _count(r, x[0], False, first, per_expert_bytes)
                if len(lru) >= capacity:
                    if belady:
                        held = []
                        while True:
                            ent = heapq.heappop(heap)
                            v = ent[2]
                            if version.get(v) != ent[3]:
                                continue
                            if v in pinned:
                                held.append(ent)
                                continue
                            break
                        for ent in held:
                            heapq.heappush(heap, ent)
                        del lru[v]
                        version.pop(v)
                    else:
                        v = next(y for y in lru if y not in pinned)
                        del lru[v]
                lru[x] = True
                if belady:
                    tick += 1
                    arrival[x] = tick
            if belady:
                # the victim rule's key: the first step after this one that uses x, which stays
                # fixed until x is used again; ties leave the most recent arrival first
                serial += 1
                version[x] = serial
                heapq.heappush(heap, (-nxt, -arrival[x], x, version[x]))
    return r


def _lru2(trace: Trace, capacity: int, per_expert_bytes: int) -> Residency:
    """LRU-2 over one shared pool (residency.rs:942-956): the victim is the unpinned resident
    expert with the oldest reference before its last one (0 for an expert referenced once), the
    last reference breaking ties; reference history survives eviction."""
    r = Residency("lru2", capacity, len(trace.steps), per_layer_misses=[0] * trace.n_layers())
    seen: set = set()
    last: dict = {}
    prev: dict = {}
    resident: set = set()
    heap: list = []                  # ((prev, last), expert) per reference; stale ones skipped
    clock = 0
    for s in trace.steps:
        pinned = set(s)
        for x in s:
            clock += 1
            prev[x] = last.get(x, 0)
            last[x] = clock
            first = x not in seen
            seen.add(x)
            if x in resident:
                _count(r, x[0], True, False, per_expert_bytes)
            else:
                _count(r, x[0], False, first, per_expert_bytes)
                if len(resident) >= capacity:
                    held = []
                    while True:
                        key, v = heapq.heappop(heap)
                        if v not in resident or key != (prev[v], last[v]):
                            continue
                        if v in pinned:
                            held.append((key, v))
                            continue
                        break
                    for ent in held:
                        heapq.heappush(heap, ent)
                    resident.discard(v)
                resident.add(x)
            heapq.heappush(heap, ((prev[x], last[x]), x))
    return r


def _slru(trace: Trace, capacity: int, protected_pct: int, per_expert_bytes: int) -> Residency:
    """Segmented LRU over one shared pool (residency.rs:746-812): a miss enters probation, a hit
    there promotes to protected, protected's overflow is demoted to probation's recent end, and
    the victim is probation's least recent unpinned expert, else protected's."""
    r = Residency(f"slru{protected_pct}", capacity, len(trace.steps), per_layer_misses=[0] * trace.n_layers())
    protected_cap = capacity * min(protected_pct, 100) // 100
    seen: set = set()
    probation: OrderedDict = OrderedDict()   # least recently stamped first
    protected: OrderedDict = OrderedDict()

    def oldest(seg, pinned):
        return next((y for y in seg if y not in pinned), None)

    for s in trace.steps:
        pinned = set(s)
        for x in s:
            first = x not in seen
            seen.add(x)
            if x in probation or x in protected:
                _count(r, x[0], True, False, per_expert_bytes)
                if x in probation:
                    del probation[x]
                    protected[x] = True
                    while len(protected) > protected_cap:
                        v = oldest(protected, pinned)
                        if v is None:
                            break
                        del protected[v]
                        probation[v] = True
                else:
                    protected.move_to_end(x)
                continue
            _count(r, x[0], False, first, per_expert_bytes)
            if len(probation) + len(protected) >= capacity:
                v = oldest(probation, pinned)
                if v is not None:
                    del probation[v]
                else:
                    del protected[oldest(protected, pinned)]
            probation[x] = True
    return r


def _static(trace: Trace, capacity: int, resident_layers: int | None, per_expert_bytes: int) -> Residency:
    if resident_layers is None:
        resident_layers = trace.widest_static_split(capacity)
    needs = trace.experts_in_layers_below(resident_layers)
    if needs > capacity:
        raise SimError(f"a static split of the first {resident_layers} layers needs {needs} slots "
                       f"but capacity is {capacity}")
    r = Residency(f"static({resident_layers})", capacity, len(trace.steps),
                  per_layer_misses=[0] * trace.n_layers())
    for s in trace.steps:
        for l, _ in s:
            _count(r, l, l < resident_layers, False, per_expert_bytes)
    return r


def _block(trace: Trace, n_cache, per_expert_bytes: int) -> Residency:
    """The device plan (k_xplan) replayed: per-block slots with step stamps."""
    L = trace.n_layers()
    caps = [int(n_cache)] * L if np.isscalar(n_cache) else [int(c) for c in n_cache]
    if len(caps) < L:
        raise SimError(f"{len(caps)} per-block capacities for a trace of {L} blocks")
    r = Residency("block", sum(caps[:L]), len(trace.steps), per_layer_misses=[0] * L)
    empty = np.iinfo(np.int64).min
    stamp = [np.full(c, empty, np.int64) for c in caps]
    owner = [np.full(c, -1, np.int64) for c in caps]
    slot_of = [dict() for _ in range(L)]
    seen: set = set()
    for i, s in enumerate(trace.steps):
        per: dict = {}
        for l, e in s:
            per.setdefault(l, []).append(e)
        for l, es in per.items():
            distinct = sorted(set(es))
            if len(distinct) > caps[l]:
                raise SimError(f"block {l} needs {len(distinct)} experts in step {i} but has "
                               f"{caps[l]} slots")
            resident = {e for e in distinct if e in slot_of[l]}
            used = np.zeros(caps[l], bool)
            for e in resident:
                used[slot_of[l][e]] = True
                stamp[l][slot_of[l][e]] = i
            for e in distinct:
                if e in resident:
                    continue
                v = int(np.argmin(np.where(used, np.iinfo(np.int64).max, stamp[l])))
                if owner[l][v] >= 0:
                    del slot_of[l][int(owner[l][v])]
                owner[l][v] = e
                slot_of[l][e] = v
                stamp[l][v] = i
                used[v] = True
            # per activation: a hit when resident before the plan, or a repeat within the step
            fetched: set = set()
            for e in es:
                x = (l, e)
                first = x not in seen
                seen.add(x)
                hit = e in resident or e in fetched
                fetched.add(e)
                _count(r, l, hit, first and not hit, per_expert_bytes)
    return r


POLICIES = ("lru", "optimal", "static", "block", "lru2", "slru")


def simulate(trace: Trace, capacity, policy: str = "lru", per_expert_bytes: int = 0,
             resident_layers: int | None = None, protected_pct: int = 80) -> Residency:
    """Replay `trace` at `capacity` slots under `policy` (see the module docstring). For
    ``block`` the capacity is slots per block (an int, or one per block); for the others the
    total. ``static`` takes the widest split that fits unless `resident_layers` is given."""
    if policy == "block":
        caps = [capacity] if np.isscalar(capacity) else list(capacity)
        if not caps or min(caps) <= 0:
            raise SimError("capacity must be at least one expert per block")
        return _block(trace, capacity, per_expert_bytes)
    capacity = int(capacity)
    if capacity <= 0:
        raise SimError("capacity must be at least one expert")
    if policy == "static":
        return _static(trace, capacity, resident_layers, per_expert_bytes)
    if policy not in POLICIES:
        raise ValueError(f"unknown policy {policy!r}; one of {POLICIES}")
    if capacity < trace.peak_step_demand():  # activations, repeats included (residency.rs:423)
        raise SimError(f"capacity {capacity} cannot hold the {trace.peak_step_demand()} experts one "
                       "step activates: unservable at this capacity under any policy")
    if policy == "lru2":
        return _lru2(trace, capacity, per_expert_bytes)
    if policy == "slru":
        return _slru(trace, capacity, protected_pct, per_expert_bytes)
    return _pool(trace, capacity, policy == "optimal", per_expert_bytes)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="Replay a moearc-trace-v1 routing trace through "
                                             "residency policies and print hit rates.")
    ap.add_argument("trace")
    ap.add_argument("--capacity", type=int, nargs="+", default=[600],
                    help="total slots for lru / optimal / static")
    ap.add_argument("--per-block", type=int, nargs="*", default=[],
                    help="slots per block for the device policy")
    ap.add_argument("--expert-mib", type=float, default=0.0, help="bytes per expert, for traffic")
    args = ap.parse_args(argv)
    t = Trace.from_file(args.trace)
    b = int(args.expert_mib * 2**20)
    print(f"{args.trace}: {len(t.steps)} steps, {t.demands()} activations, working set "
          f"{t.working_set()}, top 10% {100 * t.top_share(0.1):.1f}%, step reuse "
          f"{100 * t.step_reuse():.1f}%")
    for c in args.capacity:
        row = [simulate(t, c, p, b) for p in ("static", "lru", "lru2", "slru", "optimal")]
        print(f"  {c:6d} slots  " + "  ".join(f"{x.policy} {100 * x.hit_rate:5.1f}%" for x in row))
    for c in args.per_block:
        x = simulate(t, c, "block", b)
        print(f"  {c:4d}/block ({x.capacity} slots)  block {100 * x.hit_rate:5.1f}%"
              + (f"  {x.bytes_fetched / len(t.steps) / 2**20:.0f} MiB/step" if b else ""))


if __name__ == "__main__":
    main()
