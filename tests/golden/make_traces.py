"""Pack the reference's captured gpt-oss-120b decode routing traces, and the hit rates it
published for them, into fixtures the residency tests read.

Run in a container that has the MoEArc checkout; the files it writes are committed and the tests
read them, never the reference tree.

    python tests/golden/make_traces.py /path/to/MoEArc

- traces_gptoss120b.npz: per trace (prose, code, reasoning; bench/traces/gptoss120b-*.decode.ndjson)
  the step activations as uint8 [steps, 144, 2] (layer, expert) in file order, and the header
  line verbatim. Every step of these captures names exactly 36 blocks x 4 experts; the script
  refuses a file that does not, rather than pad it.
- policy_sweep_gptoss120b.json: the trace shape table and the static / lru / slru80 / lru-2 /
  belady columns of the capacity sweeps in bench/policy-sweep.md, each entry with the line it
  came from.
"""
from __future__ import annotations

import json
import os
import re
import sys

import numpy as np

NAMES = ("prose", "code", "reasoning")
HERE = os.path.dirname(os.path.abspath(__file__))


def pack_trace(path: str) -> tuple[np.ndarray, str]:
    lines = [ln for ln in open(path, encoding="utf-8").read().splitlines() if ln.strip()]
    header = lines[0]
    steps = []
    for ln in lines[1:]:
        flat = json.loads(ln)["e"]
        if len(flat) != 288:
            raise SystemExit(f"{path}: a step with {len(flat) // 2} activations, not 144")
        steps.append(np.array(flat, np.int64).reshape(144, 2))
    a = np.stack(steps)
    if a.min() < 0 or a.max() > 255:
        raise SystemExit(f"{path}: ids outside uint8")
    return a.astype(np.uint8), header


def sweep_tables(md_path: str) -> dict:
    lines = open(md_path, encoding="utf-8").read().splitlines()
    shape, sweeps = {}, {}
    current = None
    for i, ln in enumerate(lines, 1):
        m = re.match(r"\| gptoss120b-(\w+) \| (\d+) \| (\d+) / (\d+) \| [\d.]+% \| ([\d.]+)% \| ([\d.]+)% \|", ln)
        if m:
            shape[m.group(1)] = {"steps": int(m.group(2)), "working_set": int(m.group(3)),
                                 "total_experts": int(m.group(4)), "top10_pct": float(m.group(5)),
                                 "step_reuse_pct": float(m.group(6)),
                                 "at": f"bench/policy-sweep.md:{i}"}
            continue
        m = re.match(r"### gptoss120b-(\w+) \(working set (\d+)\)", ln)
        if m:
            current = m.group(1)
            sweeps[current] = []
            continue
        if current and ln.startswith("| slots"):
            cols = [c.strip().strip("*") for c in ln.strip("|").split("|")]
            continue
        if current and ln.startswith("|") and not ln.startswith("|---"):
            cells = [c.strip().strip("*") for c in ln.strip("|").split("|")]
            try:
                slots = int(cells[0])
            except ValueError:
                continue
            row = {"slots": slots}
            for name in ("static", "lru", "slru80", "lru-2", "belady"):
                row[name] = float(cells[cols.index(name)])
            row["at"] = f"bench/policy-sweep.md:{i}"
            sweeps[current].append(row)
        elif current and not ln.strip() and sweeps[current]:
            current = None
    return {"source": "chrisdesrochers/MoEArc", "shape": shape, "sweeps": sweeps}


def main(ref_root: str) -> None:
    arrays = {}
    for n in NAMES:
        a, header = pack_trace(os.path.join(ref_root, f"bench/traces/gptoss120b-{n}.decode.ndjson"))
        arrays[n] = a
        arrays[f"{n}_header"] = np.array(header)
    np.savez_compressed(os.path.join(HERE, "traces_gptoss120b.npz"), **arrays)
    tables = sweep_tables(os.path.join(ref_root, "bench/policy-sweep.md"))
    for n in NAMES:
        if n not in tables["shape"] or len(tables["sweeps"].get(n, [])) != 9:
            raise SystemExit(f"policy-sweep.md: table for {n} not found whole")
    with open(os.path.join(HERE, "policy_sweep_gptoss120b.json"), "w") as f:
        json.dump(tables, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(f"usage: python {sys.argv[0]} /path/to/MoEArc")
    main(sys.argv[1])
