"""Extract the reference's own known-answer tests for this path into reference_kats.json.

Run in a container that has the MoEArc checkout (the reference is Rust and cannot be compiled
here, so its test files are read as text). The JSON it writes is committed; the tests read the
JSON, never the reference tree, so they run the same on a machine without it.

    python tests/golden/make_golden.py /path/to/MoEArc

Every entry records the file and line it came from.
"""
from __future__ import annotations

import json
import os
import re
import sys


def _eval_f32_expr(expr: str) -> float:
    """Evaluate the few float spellings the reference's asserts use, without eval()."""
    expr = expr.strip()
    total = 0.0
    terms = re.findall(r"(^|[+-])(2f32\.powi\((-?\d+)\)|-?\d+(?:\.\d+)?)", expr.replace(" ", ""))
    for op, tok, pw in terms:
        v = 2.0 ** int(pw) if pw else float(tok)
        total = total - v if op == "-" else total + v
    return total


def extract(ref_root: str) -> dict:
    out: dict = {"source": "chrisdesrochers/MoEArc", "kats": {}}
    rr = os.path.join(ref_root, "crates/moearc-kernels/src/reference.rs")
    lines = open(rr).read().splitlines()

    f16 = []
    for i, ln in enumerate(lines, 1):
        m = re.search(r"assert_eq!\(f16_to_f32\(0x([0-9A-Fa-f]{4})\),\s*(.+?)\);", ln)
        if m:
            f16.append({"bits": int(m.group(1), 16), "value": _eval_f32_expr(m.group(2)),
                        "at": f"crates/moearc-kernels/src/reference.rs:{i}"})
        m = re.search(r"assert!\(f16_to_f32\(0x([0-9A-Fa-f]{4})\)\.is_(infinite|nan)\(\)\);", ln)
        if m:
            f16.append({"bits": int(m.group(1), 16), "value": m.group(2),
                        "at": f"crates/moearc-kernels/src/reference.rs:{i}"})
    out["kats"]["f16_to_f32"] = f16

    sizes = {}
    for i, ln in enumerate(lines, 1):
        m = re.search(r"assert_eq!\(QuantType::(\w+)\.block_bytes\(\),\s*(\d+)\);", ln)
        if m:
            sizes[m.group(1)] = {"bytes": int(m.group(2)),
                                 "at": f"crates/moearc-kernels/src/reference.rs:{i}"}
    out["kats"]["block_bytes"] = sizes

    # reference.rs: the router tie KAT
    txt = "\n".join(lines)
    m = re.search(r"let logits = vec!\[([^\]]+)\];\s*\n\s*let \(idx, w\) = topk_router\(&logits, "
                  r"(\d+), (\d+), (\d+), Gating::(\w+)\);\s*\n\s*assert_eq!\(idx, vec!\[([^\]]+)\]",
                  txt)
    if m:
        at = txt[: m.start()].count("\n") + 1
        out["kats"]["router_small"] = {
            "logits": [float(v) for v in m.group(1).split(",")],
            "n_tokens": int(m.group(2)), "n_expert": int(m.group(3)), "k": int(m.group(4)),
            "gating": m.group(5), "idx": [int(v) for v in m.group(6).split(",")],
            "at": f"crates/moearc-kernels/src/reference.rs:{at}"}

    # kernels_gpu.rs: the planted tie across all three gatings
    kg = os.path.join(ref_root, "crates/moearc-kernels/tests/kernels_gpu.rs")
    ktxt = open(kg).read()
    m = re.search(r"const TOKENS: usize = (\d+);\s*const EXPERTS: usize = (\d+);\s*"
                  r"const K: usize = (\d+);\s*let mut rng = Rng::new\((0x[0-9A-Fa-f_]+)\);\s*"
                  r"let mut logits: Vec<f32> = \(0\.\.TOKENS \* EXPERTS\)\.map\(\|_\| rng\.unit\(\) "
                  r"\* ([\d.]+)\)\.collect\(\);", ktxt)
    ties = re.findall(r"logits\[(\d+)\] = ([\d.]+);", ktxt)
    if m:
        at = ktxt[: m.start()].count("\n") + 1
        out["kats"]["router_planted_tie"] = {
            "tokens": int(m.group(1)), "experts": int(m.group(2)), "k": int(m.group(3)),
            "seed": int(m.group(4).replace("_", ""), 16), "unit_scale": float(m.group(5)),
            "ties": [[int(a), float(b)] for a, b in ties[:2]],
            "expect_first": [int(ties[0][0]), int(ties[1][0])],
            "at": f"crates/moearc-kernels/tests/kernels_gpu.rs:{at}"}
    m = re.search(r"let tol = \(4\.0 \+ 4\.0 \+ EXPERTS as f64 / 32\.0 \+ 5\.0 \+ 1\.0\) \* U;", ktxt)
    if m:
        out["kats"]["router_planted_tie"]["weight_tol_ulps"] = "(4+4+E/32+5+1) * 2^-24"

    # forward_pass_gpu.rs: attention geometry of the scattered-page, GQA and window tests
    fp = os.path.join(ref_root, "crates/moearc-kernels/tests/forward_pass_gpu.rs")
    ftxt = open(fp).read()
    cases = []
    for mm in re.finditer(r"fn (\w+)\(\) \{(.*?)\n\}", ftxt, re.S):
        body = mm.group(2)
        if "attn_decode" not in body:
            continue
        consts = dict(re.findall(r"const (\w+): usize = ([^;]+);", body))
        bt = re.search(r"let block_table: Vec<u32> = vec!\[([^\]]+)\];", body)
        seed = re.search(r"Rng::new\((0x[0-9A-Fa-f_]+)", body)
        if not bt:
            continue
        at = ftxt[: mm.start()].count("\n") + 1
        cases.append({"test": mm.group(1), "consts": consts,
                      "block_table": [int(v) for v in bt.group(1).split(",")],
                      "seed": int(seed.group(1).replace("_", ""), 16) if seed else None,
                      "at": f"crates/moearc-kernels/tests/forward_pass_gpu.rs:{at}"})
    out["kats"]["attention_cases"] = cases
    return out


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the MoEArc source tree>")
    ref = sys.argv[1]
    data = extract(ref)
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kats.json")
    with open(dst, "w") as f:
        json.dump(data, f, indent=1, sort_keys=True)
    print(f"wrote {dst}")


if __name__ == "__main__":
    main()
