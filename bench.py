"""Benchmark: MoE decode tok/s at gpt-oss-120b shape (configs[2], experts resident in HBM).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--depth D] [--config 120b|20b]
    python bench.py --impl reference ...   # the reference's CPU path, timed on the host cores
    python bench.py --offload 30 ...       # configs[2] mode (b): experts of blocks 0-29 in
                                           # pinned host memory, fetched over PCIe every step
    python bench.py --offload 30 --cache 32 [--trace code]
                                           # with 32 HBM slots per offloaded block keeping
                                           # fetched experts; routed as a captured trace

A step is one batch-1 decode token through the whole synthetic decoder (36 blocks: RMSNorm,
Q/K/V, RoPE, paged-KV append, attention with sinks over a full or 128-key window, O
projection, and the fused MoE FFN with 128 MXFP4 experts, top-4). Weights are random (seeded)
and generated on the device; inputs are synthetic. The weights (≈63 GB) are far larger than
the 126 MB L2, so consecutive steps never hit in L2 for them; no flush is needed.

value     tokens/s with the input already on the device, timed with CUDA events over K steps
e2e       the same through the public API with host buffers: per step the input embedding is
          copied from pinned host memory and the output read back, wall-clock timed
roofline  the MoE expert kernel (the path's dominant kernel: gate-up, SwiGLU, down and the
          combine in one launch): algorithmic bytes per launch (4 experts x 3 matrices x 2880 x
          2880 MXFP4 = 52.88 MB) over its average device time, against the measured HBM copy
          bandwidth in MEASURED_PEAKS.json
          (with --offload: the PCIe bytes of the offloaded blocks' routed experts per step over the
          step time, against a pinned host-to-device copy measured in the same run)
Multi-GPU: batch-1 decode does not shard; with N GPUs each rank runs an independent replica
(weak scaling) and `value` sums their tokens/s, timed as the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# One process per GPU: pin this rank's device before anything initialises CUDA (the rank's entry
# of an existing device list, or the device numbered by the local rank).
if "LOCAL_RANK" in os.environ:
    _lr = int(os.environ["LOCAL_RANK"])
    _vis = [d for d in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if d.strip()]
    if len(_vis) > 1:
        os.environ["CUDA_VISIBLE_DEVICES"] = _vis[_lr % len(_vis)]
    elif not _vis:
        os.environ["CUDA_VISIBLE_DEVICES"] = str(_lr)

METRIC = "MoE decode tok/s at gpt-oss-120b shape; expert-GEMM HBM GB/s vs 8 TB/s"
UNIT = "tok/s"


def expert_traffic(fused: bool, tc: bool = False) -> float | None:
    """DRAM read + write bytes of one launch of the roofline kernel, from the committed ncu
    capture summaries (profiles/decode_expert_kernels_tc_gpt_oss_120b.md for the tensor-core gate-up;
    profiles/moe_and_dense_kernels_gpt_oss_120b_1layer.md: the fused gate-up +
    down row, the gate-up row of the fragment kernels, or the tensor-core gate-up row); None if
    absent."""
    import re
    p = os.path.join(ROOT, "profiles", "decode_expert_kernels_tc_gpt_oss_120b.md" if tc and not fused
                     else "moe_and_dense_kernels_gpt_oss_120b_1layer.md")
    if not os.path.exists(p):
        return None
    row = "| `k_moe_fused<39,false>`" if fused else ("| `k_xtc<0>`" if tc else "| `k_xexpert<39,0>`")
    for line in open(p):
        if line.startswith(row):
            m = re.search(r"\| ([\d.]+) MB / ([\d.]+) MB \|", line)
            if m:
                return (float(m.group(1)) + float(m.group(2))) * 1e6
    return None


def load_peaks() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---- clocks during the timed region --------------------------------------------------------

class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.path = tempfile.mktemp(prefix="clocks_", suffix=".csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9 or (vis.isdigit() and parts[0] != vis):
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---- the CPU baseline (the reference's CPU path, restated) ---------------------------------

def cpu_decode_sample(cfg, layers: int = 2, budget_s: float = 12.0, threads: int = 0) -> dict:
    """Time the restated CPU decode path (host_experts.rs's pinned pool for the experts, the
    same-style threaded matvec for the dense projections, reference.rs attention) on `layers`
    blocks of the configuration, and extrapolate to the whole model: tokens/s =
    1 / (n_layer x seconds per block-token)."""
    import ctypes as C

    import numpy as np

    import oracle as O

    H, Dq, Dkv = cfg.n_embd, cfg.n_head * cfg.head_dim, cfg.n_head_kv * cfg.head_dim
    nb = cfg.n_expert * cfg.n_ff * H // 32
    keep, arr = [], []
    t0 = time.time()
    for l in range(layers):
        t = {
            "attn_norm": np.ones(H, np.float32), "ffn_norm": np.ones(H, np.float32),
            "wq": O.synth_normal_bf16(100 + l, Dq * H, 0.02), "wk": O.synth_normal_bf16(200 + l, Dkv * H, 0.02),
            "wv": O.synth_normal_bf16(300 + l, Dkv * H, 0.02), "wo": O.synth_normal_bf16(400 + l, H * Dq, 0.02),
            "sinks": np.zeros(cfg.n_head, np.float32),
            "router": O.synth_normal_f32(500 + l, cfg.n_expert * H, 0.02),
            "gate": O.synth_mxfp4(600 + l, nb), "up": O.synth_mxfp4(700 + l, nb), "down": O.synth_mxfp4(800 + l, nb),
        }
        pool = 4096 * Dkv
        t["k"] = np.zeros(pool, np.uint16)
        t["v"] = np.zeros(pool, np.uint16)
        t["table"] = np.arange(4096 // 32, dtype=np.uint32)
        keep.append(t)
        arr.append(O.CdLayer(*[O.ptr(t[n]) for n in ("attn_norm", "ffn_norm", "wq", "wk", "wv", "wo", "sinks",
                                                     "router", "gate", "up", "down", "k", "v", "table")]))
    gen_s = time.time() - t0
    layers_arr = (O.CdLayer * layers)(*arr)
    c = O.CdCfg(layers, H, cfg.n_head, cfg.n_head_kv, cfg.head_dim, cfg.n_expert, cfg.n_ff, cfg.n_expert_used,
                cfg.gating, cfg.act, O.MXFP4, O.BF16, cfg.alpha, cfg.limit, cfg.rms_eps, cfg.n_swa,
                cfg.swa_pattern, 32, cfg.rope_base, cfg.rope_freq_scale, cfg.rope_ext_factor,
                cfg.rope_attn_factor, cfg.rope_corr_lo, cfg.rope_corr_hi)
    pool = O.lib().hx_create(threads)
    n_threads = O.lib().hx_threads(pool)
    h = O.synth_normal_f32(9, H, 1.0)
    # warm: touch every weight once
    O.lib().cd_layers(C.byref(c), layers_arr, 0, layers, O.ptr(h), 0, pool, None)
    tokens, t0 = 0, time.time()
    while True:
        h = O.synth_normal_f32(10 + tokens, H, 1.0)
        rc = O.lib().cd_layers(C.byref(c), layers_arr, 0, layers, O.ptr(h), tokens + 1, pool, None)
        assert rc == 0, rc
        tokens += 1
        el = time.time() - t0
        if (el > budget_s and tokens >= 3) or tokens >= 4000:
            break
    O.lib().hx_destroy(pool)
    per_block_token = el / (tokens * layers)
    tps = 1.0 / (per_block_token * cfg.n_layer)
    load = os.getloadavg()[0] if hasattr(os, "getloadavg") else None
    return {"value": tps, "unit": UNIT, "cores": n_threads, "kind": "port",
            "sample": f"{tokens} tokens x {layers} of {cfg.n_layer} blocks ({el:.1f} s; weights generated in "
                      f"{gen_s:.1f} s), extrapolated to {cfg.n_layer} blocks; restated host_experts.rs pool, "
                      f"{n_threads} threads, nproc {os.cpu_count()}, load {load}"}


# ---- the GPU run ----------------------------------------------------------------------------

def pcie_h2d_gbs(ctx, nbytes: int = 256 << 20, reps: int = 5) -> float:
    """Pinned host-to-device copy bandwidth (one copy engine, CUDA events): the PCIe peak the
    offload roofline is quoted against (the BULK method of the reference's stream_bench)."""
    lib = ctx.lib
    hb = lib.moearc_x_host_alloc(nbytes)
    db = lib.moearc_alloc_device(ctx.raw, nbytes)
    assert hb and db, "pcie probe: allocation failed"
    lib.moearc_copy_h2d_async(ctx.raw, db, hb, nbytes)
    ctx.sync()
    ctx.timer_start()
    for _ in range(reps):
        lib.moearc_copy_h2d_async(ctx.raw, db, hb, nbytes)
    ms = ctx.timer_stop()
    lib.moearc_free_device(ctx.raw, db)
    lib.moearc_x_host_free(hb)
    return nbytes * reps / (ms / 1000.0) / 1e9


class TraceRoute:
    """Routes blocks 0 .. n-1 of a decoder as a captured gpt-oss-120b decode trace routed them
    (the reference's bench/traces/gptoss120b-*.decode.ndjson, packed under tests/golden): before
    each step every such block's router gets one nonzero column, 0, with positive, distinct
    values at that step's experts, and ffn_norm[0] = 1; the step inputs keep activation 0 large
    and positive, so those experts win the top-k and every other logit is exactly 0."""

    def __init__(self, dec, name: str, n: int):
        import numpy as np

        if os.path.exists(name):  # any moearc-trace-v1 capture
            from moearc_b200.residency import Trace

            pairs = Trace.from_file(name).steps
        else:
            pairs = np.load(os.path.join(ROOT, "tests", "golden", "traces_gptoss120b.npz"))[name]
        self.steps = [[[int(e) for l2, e in s if l2 == l] for l in range(n)] for s in pairs]
        k, E = dec.cfg.n_expert_used, dec.cfg.n_expert
        for i, s in enumerate(self.steps):
            for l, es in enumerate(s):
                if len(es) != k or len(set(es)) != k or max(es) >= E:
                    raise SystemExit(f"{name}: step {i} routes block {l} to {es}, not {k} distinct of {E} experts")
        self.dec, self.n, self.i, self.history = dec, n, 0, []
        self.w = np.zeros((dec.cfg.n_expert, dec.cfg.n_embd), np.float32)
        for l in range(n):
            norm = dec.tensor(1, l, np.float32)
            norm[0] = 1.0
            dec.set_tensor(1, l, norm)

    def apply(self) -> None:
        """Set the routers for the next step (blocking copies, outside any timed region)."""
        s = self.steps[self.i % len(self.steps)]
        for l, es in enumerate(s):
            self.w[:, 0] = 0.0
            for r, e in enumerate(es):
                self.w[e, 0] = 2.0 - 0.25 * r
            self.dec.set_tensor(3, l, self.w)
        self.history.append(s)
        self.i += 1

    def replay_fetches(self, n_cache: int, upto: int) -> int:
        """Experts the device cache must have fetched over the first `upto` steps (the host
        replay of its slot rule)."""
        from moearc_b200.residency import Trace, simulate

        t = Trace([[(l, e) for l, es in enumerate(s) for e in es] for s in self.history[:upto]])
        return simulate(t, n_cache, "block").misses if upto else 0


def gpu_run(args, cfg, rank: int, world: int, dist) -> dict:
    import ctypes as C

    import numpy as np

    from moearc_b200 import Context
    from moearc_b200.decoder import Decoder

    ctx = Context()
    cfg.n_ctx = args.depth + args.warmup + 3 * args.steps + 64
    t0 = time.time()
    dec = Decoder(ctx, cfg)
    ctx.sync()
    build_s = time.time() - t0
    if args.depth:
        dec.fill_kv(args.depth)
    else:
        dec.set_pos(0)
    if args.host:
        kind, _, val = args.host.partition(":")
        if kind == "fraction":
            dec.host_experts("fraction", fraction=float(val), threads=args.host_threads)
        else:
            dec.host_experts("over", over=int(val), threads=args.host_threads)
    lib = ctx.lib
    H = cfg.n_embd
    host_in = lib.moearc_x_host_alloc(4 * H)
    host_out = lib.moearc_x_host_alloc(4 * H)
    C.memmove(host_in, np.random.default_rng(rank).standard_normal(H).astype(np.float32).ctypes.data, 4 * H)
    lib.moearc_copy_h2d(ctx.raw, dec.in_ptr, host_in, 4 * H)
    # with a residency cache the routing must change from step to step as it does when decoding
    # text: each step takes the next of 64 distinct N(0, 1) inputs from pinned host memory
    n_pool = 64 if cfg.n_cache else 0
    pool = lib.moearc_x_host_alloc(4 * H * max(n_pool, 1))
    if n_pool:
        xs = np.random.default_rng(100 + rank).standard_normal((n_pool, H)).astype(np.float32)
        if args.trace:
            xs[:, 0] = 1000.0  # keeps the steered routers' one column decisive
        C.memmove(pool, xs.ctypes.data, 4 * H * n_pool)
    route = TraceRoute(dec, args.trace, cfg.n_offload) if args.trace else None

    def next_input(i):
        if route:
            route.apply()
        if n_pool:
            lib.moearc_copy_h2d_async(ctx.raw, dec.in_ptr, pool + 4 * H * (i % n_pool), 4 * H)

    for i in range(args.warmup):
        next_input(i)
        dec.step()
    ctx.sync()

    # per-kernel device times (one un-graphed step; events between launches)
    ms = (C.c_float * 8)()
    cnt = (C.c_int * 8)()
    ctx._finish(lib.moearc_x_decoder_profile(dec.h, ms, cnt, 8), "profile")
    kernel_ms = {k: ms[i] for i, k in enumerate(["qkv", "attention", "o_proj", "moe_route", "moe_gate_up",
                                                  "moe_down", "final_norm", "expert_fetch"])}
    launches_per_step = sum(cnt[i] for i in range(8))
    if route:
        route.history.append(route.history[-1])  # the profiled step repeated the last routing

    sampler = ClockSampler() if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.5)
    if dist:
        dist.barrier()
    ctx.sync()
    fetched0 = dec.fetched()
    host0 = dec.host_stats() if args.host else None
    h0 = len(route.history) if route else 0
    if route:
        # the routers are set between steps, so each step is timed on its own
        ms_total = 0.0
        for i in range(args.steps):
            route.apply()
            lib.moearc_copy_h2d_async(ctx.raw, dec.in_ptr, pool + 4 * H * (i % n_pool), 4 * H)
            ctx.timer_start()
            dec.step()
            ms_total += ctx.timer_stop()
    else:
        ctx.timer_start()
        for i in range(args.steps):
            next_input(i)
            dec.step()
        ms_total = ctx.timer_stop()
    fetched = dec.fetched() - fetched0
    host = None
    if args.host:
        h1 = dec.host_stats()
        host = {k: (h1[k] - host0[k]) / args.steps for k in h1}
    replay = (route.replay_fetches(cfg.n_cache, len(route.history)) - route.replay_fetches(cfg.n_cache, h0)
              if route else None)

    # end to end through the public API: host input in, host output out, every step, one call
    # a step (moearc_x_decoder_step_host: the copies and the step as one graph launch)
    ctx.sync()
    xs_host = (np.ctypeslib.as_array(C.cast(pool, C.POINTER(C.c_float)), (n_pool, H)) if n_pool else
               np.ctypeslib.as_array(C.cast(host_in, C.POINTER(C.c_float)), (1, H)))
    y_host = np.empty(H, np.float32)
    # warm-up: the first call pins its staging rows and captures the graph with the copies
    for i in range(min(args.warmup, 3)):
        dec.step_host(xs_host[i % len(xs_host)], y_host)
    e2e_s = 0.0
    t1 = time.perf_counter()
    for i in range(args.steps):
        if route:
            route.apply()
            t1 = time.perf_counter()
        dec.step_host(xs_host[i % len(xs_host)], y_host)
        if route:
            e2e_s += time.perf_counter() - t1
    if not route:
        e2e_s = time.perf_counter() - t1
    # the same with the input copy, the step and the output copy as three enqueues and a wait
    e2e_calls_s = 0.0
    t1 = time.perf_counter()
    for i in range(args.steps):
        if route:
            route.apply()
            t1 = time.perf_counter()
        lib.moearc_copy_h2d_async(ctx.raw, dec.in_ptr, pool + 4 * H * (i % n_pool) if n_pool else host_in, 4 * H)
        dec.step()
        lib.moearc_x_copy_d2h_async(ctx.raw, host_out, dec.out_ptr, 4 * H)
        ctx.sync()
        if route:
            e2e_calls_s += time.perf_counter() - t1
    if not route:
        e2e_calls_s = time.perf_counter() - t1
    clocks = sampler.stop() if sampler else None
    pcie = pcie_h2d_gbs(ctx) if cfg.n_offload else None

    # the expert kernels timed from inside graphed steps: every CTA stamps its start, the end of
    # its dependency wait and its end; per block, the latest end minus the earliest wait-over
    in_graph = None
    if not cfg.n_offload:
        dec.kernel_spans(True)
        gu, dn = [], []
        for i in range(4):
            next_input(i)
            dec.step()
            ctx.sync()
            if i:  # the first step captured the graph again
                g, d_ = dec.expert_kernel_ms()
                gu.append(g)
                dn.append(d_)
        dec.kernel_spans(False)
        in_graph = {"gate_up": statistics.mean(gu), "down": statistics.mean(dn), "steps": len(gu)}

    # the same decoder with the whole step as one persistent kernel (opt-in path), for comparison
    step_kernel = None
    if not args.no_step_kernel and dec.has_step_kernel():
        dec.use_step_kernel(True)
        for i in range(3):
            next_input(i)
            dec.step()
        ctx.sync()
        n_sk = min(args.steps, 20)
        ctx.timer_start()
        for i in range(n_sk):
            next_input(i)
            dec.step()
        sk_ms = ctx.timer_stop() / n_sk
        # per phase: latest CTA end minus earliest CTA start, averaged over the blocks
        words = dec.trace_words()
        buf = ctx.alloc(8 * words)
        dec.set_trace(buf)
        dec.step()
        ctx.sync()
        tr = np.empty(words, np.uint64)
        ctx._finish(lib.moearc_copy_d2h(ctx.raw, tr.ctypes.data, buf.ptr, 8 * words), "trace")
        dec.set_trace(None)
        buf.free()
        n_cta = words // (cfg.n_layer * 6 * 4)
        t = tr.astype(np.int64).reshape(cfg.n_layer, 6, 4, n_cta)
        span = (t[:, :, 3, :].max(axis=2) - t[:, :, 0, :].min(axis=2)) / 1e3
        names = ["qkv", "attention", "o_proj", "route", "gate_up", "down"]
        step_kernel = {"ms_per_step": sk_ms, "tok_s": 1000.0 / sk_ms, "steps": n_sk,
                       "status": dec.status(),
                       "phase_span_us_per_block": {n: float(span[:, j].mean()) for j, n in enumerate(names)}}
        dec.use_step_kernel(False)
    out = np.ctypeslib.as_array(C.cast(host_out, C.POINTER(C.c_float)), (H,)).copy()
    assert np.all(np.isfinite(out)), "non-finite decoder output"
    lib.moearc_x_host_free(host_in)
    lib.moearc_x_host_free(host_out)
    lib.moearc_x_host_free(pool)
    dec.close()
    ctx.close()
    return {"ms_total": ms_total, "e2e_s": e2e_s, "e2e_calls_s": e2e_calls_s, "kernel_ms": kernel_ms,
            "counts": [cnt[i] for i in range(8)], "launches_per_step": launches_per_step, "clocks": clocks, "build_s": build_s, "pcie_gbs": pcie,
            "fetched_per_step": fetched / args.steps, "replay_fetches": replay, "fetched": fetched,
            "in_graph": in_graph, "step_kernel": step_kernel, "host": host}


# ---- MoE prefill on the tensor cores, one GPU -------------------------------------

def prefill_bench(args) -> dict:
    """One gpt-oss-120b-shaped MoE block (128 MXFP4 experts, top-4, 2880 x 2880) over 8 x 4096
    tokens of bf16 N(0,1) activations, Zipf(1.1) expert popularity (the router bias is log p_e,
    p_e ~ rank(e)^-1.1 over a seeded permutation; the router GEMV adds the per-token noise).
    A step = one moearc_x_prefill_forward (route, scatter, two tcgen05 grouped GEMMs, combine)."""
    import ctypes as C

    import numpy as np

    from moearc_b200 import Context
    from moearc_b200.moe import MoeLayer, MoePrefill

    ctx = Context()
    lib = ctx.lib
    H = I = 2880
    E, k, T = args.experts, 4, args.tokens
    nb = E * I * H // 32
    banks = [ctx.alloc(nb * 17) for _ in range(3)]
    for i, b in enumerate(banks):
        ctx._finish(lib.moearc_x_synth(ctx.raw, b.ptr, nb, 2, 0x9F00 + i, 0.0, -8, -4), "synth")
    router = ctx.alloc(E * H * 4)
    ctx._finish(lib.moearc_x_synth(ctx.raw, router.ptr, E * H, 0, 0x9F07, 0.02, 0, 0), "synth")
    rank = np.random.default_rng(0x21FF).permutation(E) + 1
    p = rank.astype(np.float64) ** -1.1
    bias = ctx.upload_new(np.log(p / p.sum()).astype(np.float32))
    packer = MoeLayer(ctx, H, I, E, k, 2, 1, 39, max_tokens=1)
    packer.pack(*banks)
    for b in banks:
        b.free()
    pf = MoePrefill(ctx, H, I, E, k, 2, 1, 39, max_tokens=T)
    x = ctx.alloc(T * H * 2)
    ctx._finish(lib.moearc_x_synth(ctx.raw, x.ptr, T * H, 1, 0x9F08, 1.0, 0, 0), "synth")
    out = ctx.alloc(T * H * 4)
    ctx.sync()
    ctx.timer_start()
    if args.weights == "4bit":
        pf.load4(packer.gateup, packer.down)
    elif args.weights == "fp8":
        pf.load8(packer.gateup, packer.down)
    else:
        pf.load(packer.gateup, packer.down)
    load_ms = ctx.timer_stop()
    for _ in range(args.warmup):
        pf.forward(x, T, router, out, router_b=bias)
    ms = (C.c_float * 7)()
    ctx._finish(lib.moearc_x_prefill_profile(pf.h, x.ptr, T, router.ptr, bias.ptr, None, out.ptr, ms, 7), "profile")
    kernel_ms = dict(zip(["route_logits", "topk", "scan", "scatter", "gemm_gate_up", "gemm_down", "combine"],
                         [ms[i] for i in range(7)]))
    sampler = ClockSampler()
    sampler.start()
    time.sleep(0.3)
    ctx.sync()
    ctx.timer_start()
    for _ in range(args.steps):
        pf.forward(x, T, router, out, router_b=bias)
    ms_total = ctx.timer_stop()
    # end to end: the activations from pinned host memory in, the output back, every step
    hin, hout = lib.moearc_x_host_alloc(T * H * 2), lib.moearc_x_host_alloc(T * H * 4)
    ctx._finish(lib.moearc_copy_d2h(ctx.raw, hin, x.ptr, T * H * 2), "d2h")
    ctx.sync()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        lib.moearc_copy_h2d_async(ctx.raw, x.ptr, hin, T * H * 2)
        pf.forward(x, T, router, out, router_b=bias)
        lib.moearc_x_copy_d2h_async(ctx.raw, hout, out.ptr, T * H * 4)
        ctx.sync()
    e2e_s = time.perf_counter() - t0
    clocks = sampler.stop()
    res = np.ctypeslib.as_array(C.cast(hout, C.POINTER(C.c_float)), (T * H,))
    assert np.all(np.isfinite(res[: 1 << 20])), "non-finite prefill output"
    lib.moearc_x_host_free(hin)
    lib.moearc_x_host_free(hout)
    cnt = pf.buffer(3, np.int32, E)
    assert pf.status() == 0
    pf.close()
    packer.close()
    ctx.close()
    return {"ms_step": ms_total / args.steps, "e2e_s": e2e_s, "kernel_ms": kernel_ms, "load_ms": load_ms,
            "counts": cnt, "clocks": clocks, "T": T, "H": H, "I": I, "E": E, "k": k}


def prefill_ep_bench(args, rank: int, world: int, own_group: bool = True) -> dict:
    """configs[3] with the experts split over `world` GPUs (16 per GPU at 8): each rank holds
    tokens / world tokens, routes them, dispatches rows to the experts' owners and combines the
    returned rows (moearc_b200.ep over NCCL). Per step the device time is taken on every rank
    (events on the library stream around whole steps, which wait for their collectives) and the
    maximum over ranks is reported."""
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    from moearc_b200 import Context
    from moearc_b200.ep import ExpertParallelPrefill, NcclExpertParallelPrefill, PeerExpertParallelPrefill, nccl_unique_id
    from moearc_b200.moe import MoeLayer

    if own_group:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    torch.cuda.set_device(0)
    ctx = Context()
    lib = ctx.lib
    H = I = 2880
    E, k = args.experts, 4
    T = args.tokens // world
    nb = E * I * H // 32
    banks = [ctx.alloc(nb * 17) for _ in range(3)]
    for i, b in enumerate(banks):
        ctx._finish(lib.moearc_x_synth(ctx.raw, b.ptr, nb, 2, 0x9F00 + i, 0.0, -8, -4), "synth")
    router = ctx.alloc(E * H * 4)
    ctx._finish(lib.moearc_x_synth(ctx.raw, router.ptr, E * H, 0, 0x9F07, 0.02, 0, 0), "synth")
    rank_e = np.random.default_rng(0x21FF).permutation(E) + 1
    pz = rank_e.astype(np.float64) ** -1.1
    bias = ctx.upload_new(np.log(pz / pz.sum()).astype(np.float32))
    packer = MoeLayer(ctx, H, I, E, k, 2, 1, 39, max_tokens=1)
    packer.pack(*banks)
    for b in banks:
        b.free()
    if args.exchange == "nccl-c":
        # the library's own NCCL communicator (moearc_x_ep_*): rank 0's unique id reaches the
        # others over the process group
        uid = [nccl_unique_id(lib) if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ep = NcclExpertParallelPrefill(ctx, rank, world, H, I, E, k, 2, 1, 39, max_tokens=T,
                                       max_rows=args.tokens * k, unique_id=uid[0])
    else:
        cls = PeerExpertParallelPrefill if args.exchange == "peer" else ExpertParallelPrefill
        ep = cls(ctx, None, H, I, E, k, 2, 1, 39, max_tokens=T, max_rows=args.tokens * k)
    ep.load(packer.gateup, packer.down)
    x = ctx.alloc(T * H * 2)
    ctx._finish(lib.moearc_x_synth(ctx.raw, x.ptr, T * H, 1, 0x9F08 + rank, 1.0, 0, 0), "synth")
    out = ctx.alloc(T * H * 4)
    ep.forward(x, T, router, out.ptr, router_b=bias)
    ep.rebalance()  # place the experts by the popularity one step saw (every rank agrees)
    for _ in range(args.warmup):
        ep.forward(x, T, router, out.ptr, router_b=bias)
    ctx.sync()
    dist.barrier()
    ctx.timer_start()
    recv = []
    for _ in range(args.steps):
        pl = ep.forward(x, T, router, out.ptr, router_b=bias)
        recv.append(pl if isinstance(pl, int) else pl["n_recv"])
    ms = ctx.timer_stop()
    t = torch.tensor([ms, float(max(recv))], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.barrier()
    ep.close()
    packer.close()
    if own_group:
        dist.destroy_process_group()
    ctx.close()
    return {"ms_step": float(t[0]) / args.steps, "max_rows": int(t[1]), "T": T * world, "H": H, "I": I, "E": E,
            "k": k, "rows_total": args.tokens * k}


def prefill_main(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        rank = int(os.environ.get("RANK", "0"))
        r = prefill_ep_bench(args, rank, world)
        if rank != 0:
            return
        T, H, I, k = r["T"], r["H"], r["I"], r["k"]
        flops = 6.0 * T * k * H * I
        line = {
            "metric": "MoE prefill TFLOP/s, one gpt-oss-120b-shaped MoE block, experts split over the GPUs (configs[3])",
            "value": flops / (r["ms_step"] / 1000.0) / 1e12, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms_step"], "tokens_per_s": T / (r["ms_step"] / 1000.0),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16 operands, f32 accumulate", "data": "synthetic (as the 1-GPU prefill line)",
            "config": {"workload": f"configs[3] MoE block: {T} tokens, {r['E']} experts top-4, {r['E'] // world} per GPU, "
                                   + ("rows stored into the owners' buffers by the route scatter and results back by "
                                      "the down GEMM epilogue over NVLink peer memory" if args.exchange == "peer" else
                                      "count all-gather, dispatch and return by NCCL inside the library's C ABI "
                                      "(moearc_x_ep_forward; no torch in the forward)" if args.exchange == "nccl-c" else
                                      "dispatch and combine by NCCL all-to-all")
                                   + "; experts placed by the popularity of one warm-up step", "max_rows_on_a_rank": r["max_rows"], "rows_total": r["rows_total"],
                       "parallelism": f"ep{world}"},
        }
        print(json.dumps(line))
        return
    r = prefill_bench(args)
    T, H, I, k = r["T"], r["H"], r["I"], r["k"]
    flops = 6.0 * T * k * H * I  # gate and up (2 x 2 H I) and down (2 H I) per (token, expert)
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))
    peak_kind = "measured bf16 (MEASURED_PEAKS.json)" if peaks else "fallback"
    if args.weights == "fp8":
        # the block-scaled FP8 MMA's peak, measured in this run by the library's own tcgen05 loop
        from moearc_b200 import Context
        pc = Context()
        peak = pc.mma_peak("mxf8")
        pc.close()
        peak_kind = "measured in this run: kind::mxf8f6f4 E4M3 tcgen05 loop (moearc_x_mma_peak)"
    gu_ms = r["kernel_ms"]["gemm_gate_up"]
    gu_tflops = 4.0 * T * k * H * I / (gu_ms / 1000.0) / 1e12
    value = flops / (r["ms_step"] / 1000.0) / 1e12
    cnt = r["counts"]
    line = {
        "metric": "MoE prefill TFLOP/s, one gpt-oss-120b-shaped MoE block (configs[3] shape, 1 GPU)",
        "value": value, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["ms_step"], "tokens_per_s": T / (r["ms_step"] / 1000.0), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": ("bf16 operands, f32 accumulate (MXFP4 weights staged at 4 bits, expanded in shared memory)"
                                                           if args.weights == "4bit" else
                                                           "MXFP8 (E4M3 x E4M3, E8M0 per 32) operands, f32 accumulate: the perf mode"
                                                           if args.weights == "fp8" else
                                                           "bf16 operands, f32 accumulate (MXFP4 weights expanded to bf16)"),
        "data": "synthetic (seeded MXFP4 experts, bf16 N(0,1) activations, Zipf(1.1) router bias)",
        "config": {"workload": f"configs[3] MoE block: {T} tokens (8 x 4096 at full size), {r['E']} experts top-4, 2880 x 2880",
                   "tokens": T, "expert_load_max": int(cnt.max()), "expert_load_mean": float(cnt.mean()),
                   "l2": "operands (1.5 GB activations, 6.4 GB bf16 weights) far exceed the 126 MB L2"},
        "roofline": {"bound": "tensor", "kernel": ("gate-up grouped GEMM (tcgen05 kind::mxf8f6f4.block_scale, SwiGLU + "
                                                   "MXFP8 quantisation epilogue)" if args.weights == "fp8" else
                                                   "gate-up grouped GEMM (tcgen05 kind::f16, SwiGLU epilogue)"),
                     "achieved": gu_tflops, "peak": peak, "unit": "TFLOP/s", "frac": gu_tflops / peak,
                     "peak_kind": peak_kind, "traffic": None},
        "kernel_ms": r["kernel_ms"], "weight_load_ms": r["load_ms"], "weights": args.weights,
        "e2e": {"value": flops * args.steps / r["e2e_s"] / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 4},
        "gpu_launches": 7 * args.steps, "clocks": r["clocks"],
    }
    print(json.dumps(line))


# ---- batched decode, 64 streams ---------------------------------------------------

def batch_main(args) -> None:
    """a Qwen3-MoE-shaped decoder (48 blocks, hidden 2048, 32 q / 4 kv heads of 128,
    128 Q4_0 experts top-8, I 768) decoding one token for each of `--batch` streams per step at
    depth `--depth` (default 4096; every stream's KV filled with synthetic bf16)."""
    import ctypes as C

    import numpy as np

    from moearc_b200 import Context
    from moearc_b200.decoder import BatchDecoder, DecoderConfig

    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as tdist

        # the process group only hands out the NCCL unique id and takes the max over ranks; the
        # step's exchanges run on the library's own communicator inside its graph
        tdist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
        dist = tdist
    ctx = Context()
    lib = ctx.lib
    B = args.batch
    if B % world:
        raise SystemExit("qwen3: --batch must split evenly over the GPUs")
    Bl = B // world  # this rank's streams
    depth = args.depth or 4096
    cfg = DecoderConfig.qwen3_moe()
    weights = args.weights or "4bit"
    if weights not in ("4bit", "bf16"):
        raise SystemExit("qwen3: --weights 4bit or bf16")
    cfg.expert_layout = 0 if weights == "4bit" else 1
    if args.layers:
        cfg.n_layer = args.layers
    cfg.n_ctx = depth + args.warmup + 2 * args.steps + 64
    t0 = time.time()
    comm = None
    if world > 1:
        from moearc_b200.ep import nccl_comm, nccl_unique_id

        uid = [nccl_unique_id(lib) if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = nccl_comm(ctx, rank, world, uid[0])
        bd = BatchDecoder(ctx, cfg, Bl, ep=(comm, rank, world))
    else:
        bd = BatchDecoder(ctx, cfg, B)
    bd.set_pos(depth, fill=True)
    ctx.sync()
    build_s = time.time() - t0
    H = cfg.n_embd
    nb = 4 * Bl * H  # this rank's input and output bytes per step
    host_in = lib.moearc_x_host_alloc(nb)
    host_out = lib.moearc_x_host_alloc(nb)
    C.memmove(host_in, np.random.default_rng(4 + rank).standard_normal(Bl * H).astype(np.float32).ctypes.data, nb)
    lib.moearc_copy_h2d(ctx.raw, bd.in_ptr, host_in, nb)
    for _ in range(args.warmup):
        bd.step()
    ctx.sync()
    sampler = ClockSampler() if rank == 0 else None
    if sampler:
        sampler.start()
    time.sleep(0.3)
    if dist:
        dist.barrier()
    ctx.sync()
    ctx.timer_start()
    for _ in range(args.steps):
        bd.step()
    ms_total = ctx.timer_stop()
    ctx.sync()
    if dist:
        dist.barrier()
    t1 = time.perf_counter()
    for _ in range(args.steps):
        lib.moearc_copy_h2d_async(ctx.raw, bd.in_ptr, host_in, nb)
        bd.step()
        lib.moearc_x_copy_d2h_async(ctx.raw, host_out, bd.out_ptr, nb)
        ctx.sync()
    e2e_s = time.perf_counter() - t1
    clocks = sampler.stop() if sampler else None
    out = np.ctypeslib.as_array(C.cast(host_out, C.POINTER(C.c_float)), (Bl * H,)).copy()
    assert np.all(np.isfinite(out)), "non-finite batch decoder output"
    assert bd.status() == 0, "a bounded wait gave up"
    lib.moearc_x_host_free(host_in)
    lib.moearc_x_host_free(host_out)
    bd.close()
    if comm:
        from moearc_b200.ep import nccl_comm_destroy

        nccl_comm_destroy(ctx, comm)
    ctx.close()
    ms_total, e2e_s = slowest_rank(ms_total, e2e_s, dist)
    if dist:
        dist.destroy_process_group()
    if rank != 0:
        return
    ms_step = ms_total / args.steps
    E, k, I = cfg.n_expert, cfg.n_expert_used, cfg.n_ff
    Dq, Dkv = cfg.n_head * cfg.head_dim, cfg.n_head_kv * cfg.head_dim
    distinct = E * (1.0 - (1.0 - k / E) ** B)  # expected experts a step touches per block
    dense_b = (H * (Dq + 2 * Dkv) + H * Dq) * 2
    expert_q4 = distinct * 3 * I * H * 18 / 32
    kv_b = B * (depth + 1) * Dkv * 2 * 2
    step_b = cfg.n_layer * (world * (dense_b + E * H * 4) + expert_q4 + kv_b)  # dense and router on every GPU
    peak, peak_kind = load_peaks()
    achieved = step_b / (ms_step / 1000.0) / 1e9
    where = "1 GPU" if world == 1 else f"expert-parallel over {world} GPUs, {Bl} streams each"
    line = {
        "metric": f"batched decode tok/s (all streams), Qwen3-MoE shape, {B} streams at depth {depth} (configs[4], {where})",
        "value": B / (ms_step / 1000.0), "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak" if world == 1 else "strong",
        "vs_baseline": None,
        "dtype": ("f16 expert operands (Q4_0 read at 4 bits, expanded in shared memory), bf16 attention operands, "
                  "f32 accumulate" if weights == "4bit" else
                  "bf16 operands (Q4_0 experts expanded to bf16 at load), f32 accumulate"),
        "weights": weights,
        "data": "synthetic (seeded weights of the configs[4] architecture, synthetic KV at the depth)",
        "config": {"workload": f"configs[4] Qwen3-MoE shape, {cfg.n_layer} blocks, {B} streams, depth {depth}",
                   "batch": B, "depth": depth, "l2": "weights and KV (~100 GB) far exceed the 126 MB L2",
                   "parallelism": "1 GPU" if world == 1 else
                   f"ep{world}: experts split over the GPUs, attention and projections per GPU on its own "
                   f"streams, rows all-gathered and results returned over NCCL inside each GPU's step graph"},
        "roofline": {"bound": "hbm", "kernel": "whole step (algorithmic bytes: bf16 dense weights, 4-bit experts, KV span)"
                     + ("" if world == 1 else f"; {world} GPUs: the dense weights read on each, the peak {world} x"),
                     "achieved": achieved, "peak": peak * world, "unit": "GB/s", "frac": achieved / (peak * world),
                     "peak_kind": peak_kind, "traffic": None, "bytes_per_step": step_b},
        "e2e": {"value": B * args.steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4 * B * H,
                "d2h_bytes_per_step": 4 * B * H},
        "gpu_launches": None, "clocks": clocks, "build_s": build_s,
    }
    print(json.dumps(line))


def shard_sample(args, rank: int, world: int) -> dict | None:
    """A short sample of the path that does shard over GPUs: configs[3]'s MoE prefill block with
    the experts split over the `world` ranks (at 1, the same block on one GPU), so the scaling run
    measures expert parallelism beside the decode replicas. Every rank runs it (the same
    collectives in the same order); rank 0 gets the numbers."""
    import copy

    a = copy.copy(args)
    a.steps, a.warmup, a.tokens, a.experts = 5, 3, 8 * 4096, 128
    a.weights = "bf16"
    if world > 1:
        r = prefill_ep_bench(a, rank, world, own_group=False)
        label = f"ep{world}, rows exchanged over " + ("NVLink peer memory" if a.exchange == "peer" else
                                                     "NCCL inside the C ABI" if a.exchange == "nccl-c" else "NCCL all-to-all")
    else:
        r = prefill_bench(a)
        label = "1 GPU"
    flops = 6.0 * r["T"] * r["k"] * r["H"] * r["I"]
    return {"metric": "MoE prefill TFLOP/s, configs[3] block (32768 tokens, 128 experts top-4, 2880 x 2880)",
            "value": flops / (r["ms_step"] / 1000.0) / 1e12, "unit": "TFLOP/s", "ms_per_step": r["ms_step"],
            "steps": a.steps, "warmup": a.warmup, "parallelism": label, "scaling": "strong"}


def slowest_rank(ms_total: float, e2e_s: float, dist) -> tuple[float, float]:
    """The timed region's device time and the end-to-end wall time, each the maximum over the
    ranks (every rank calls this, the same collectives in the same order)."""
    if not dist:
        return ms_total, e2e_s
    import torch

    t = torch.tensor([ms_total, e2e_s], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.barrier()
    return float(t[0]), float(t[1])


def replica_throughput(world: int, steps: int, ms_total: float, e2e_s: float) -> tuple[float, float]:
    """Whole-job tokens per second of `world` independent replicas that each decoded `steps`
    tokens, over the slowest rank's device time and end-to-end time."""
    return world * steps / (ms_total / 1000.0), world * steps / e2e_s


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--depth", type=int, default=0)
    ap.add_argument("--config", default="120b", choices=["120b", "20b", "prefill", "qwen3"])
    ap.add_argument("--batch", type=int, default=64, help="qwen3: concurrent streams (configs[4]: 64)")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl", "nccl-c"],
                    help="prefill on several GPUs: rows exchanged by the kernels over peer memory, or NCCL all-to-all")
    ap.add_argument("--weights", default=None, choices=["4bit", "bf16", "fp8"],
                    help="prefill (default bf16): expert weights staged at 4 bits (expanded in shared memory), "
                         "expanded to bf16, or the MXFP8 perf mode (E4M3 weights and MXFP8 activations on the "
                         "block-scaled FP8 MMA); qwen3 (default 4bit): 4bit or bf16")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--layers", type=int, default=0,
                    help="blocks to build (default: the configuration's); a smaller model for profiling")
    ap.add_argument("--tokens", type=int, default=8 * 4096, help="prefill: tokens per step (configs[3]: 8 x 4096)")
    ap.add_argument("--experts", type=int, default=128, help="prefill: experts (configs[3]: 128)")
    ap.add_argument("--offload", type=int, default=0,
                    help="blocks whose experts stay in pinned host memory (configs[2] mode (b): 30)")
    ap.add_argument("--cache", type=int, default=0,
                    help="with --offload: device slots per offloaded block that keep fetched experts (0: none)")
    ap.add_argument("--trace", default=None,
                    help="with --offload and --cache on the 120b shape: route the offloaded blocks as the "
                         "captured gpt-oss-120b decode trace prose, code or reasoning did, or as a "
                         "moearc-trace-v1 file")
    ap.add_argument("--host", default=None,
                    help="with --offload: part of the offloaded blocks' experts on host threads beside the GPU, "
                         "'fraction:F' (the first ceil(misses x F) of each block's misses) or 'over:N' (the misses "
                         "beyond the first N)")
    ap.add_argument("--host-threads", type=int, default=0, help="host pool threads (0: the online cores - 1)")
    ap.add_argument("--no-step-kernel", action="store_true",
                    help="skip the comparison run of the persistent step kernel")
    ap.add_argument("--layout", default="tc", choices=["tc", "fragment"],
                    help="120b/20b: resident experts in the tensor-core layout (block-scaled FP4 MMA) or the "
                         "fragment layout (mma.sync kernels; the persistent step kernel needs it)")
    ap.add_argument("--no-ep", action="store_true",
                    help="skip the expert-parallel prefill sample (configs[3] over the N GPUs)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.weights is None and args.config != "qwen3":
        args.weights = "bf16"
    if args.config == "prefill":
        prefill_main(args)
        return
    if args.config == "qwen3":
        batch_main(args)  # every rank: expert parallelism over the GPUs when launched on several
        return

    from moearc_b200.decoder import DecoderConfig

    cfg = DecoderConfig.gpt_oss_120b() if args.config == "120b" else DecoderConfig.gpt_oss_20b()
    cfg.expert_layout = 0 if args.layout == "tc" else 1
    if args.layers:
        cfg.n_layer = args.layers
    cfg.n_offload = min(args.offload, cfg.n_layer)
    cfg.n_cache = args.cache if cfg.n_offload else 0
    residency = ("experts resident in HBM" if not cfg.n_offload else
                 f"mode (b): experts of blocks 0-{cfg.n_offload - 1} in pinned host memory, the routed ones "
                 f"fetched over PCIe every step" if not cfg.n_cache else
                 f"mode (b) with a residency cache: experts of blocks 0-{cfg.n_offload - 1} in pinned host memory, "
                 f"{cfg.n_cache} device slots per block keep fetched experts (least recently used evicted), "
                 + (f"the offloaded blocks routed as the captured gpt-oss-120b {args.trace} decode trace"
                    if args.trace else "a new N(0,1) input every step"))
    if args.host and not cfg.n_offload:
        raise SystemExit("--host needs --offload")
    if args.host:
        residency += f"; host experts {args.host} of each offloaded block's misses on the host cores beside the GPU"
    if args.trace and not (cfg.n_cache and args.config == "120b" and cfg.n_offload <= 36):
        raise SystemExit("--trace needs --config 120b, --offload and --cache")
    workload = (f"configs[{2 if args.config == '120b' else 1}] gpt-oss-{args.config} shape, batch-1 decode, "
                f"depth {args.depth}, {residency}")
    config = {"workload": workload, "n_layer": cfg.n_layer, "n_embd": cfg.n_embd, "n_expert": cfg.n_expert,
              "top_k": cfg.n_expert_used, "n_ff": cfg.n_ff, "expert_type": "MXFP4", "kv": "bf16, pages of 32",
              "attention": "64 q / 8 kv heads x 64, sinks, alternating full / 128-key window",
              "depth": args.depth, "batch": 1, "offloaded_blocks": cfg.n_offload,
              "l2": "weights (~63 GB) far exceed the 126 MB L2; no flush",
              "expert_layout": ("tensor-core (block-scaled FP4 MMA)" if cfg.expert_layout == 0 and cfg.n_offload < cfg.n_layer
                                else "fragment (mma.sync)")}

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        cpu = cpu_decode_sample(cfg, budget_s=12.0)
        # Our arm at N GPUs runs N independent replicas and sums their tokens/s; the reference arm
        # is the same sum of N replicas of the reference's CPU path, each timed as one replica on
        # this host's cores (the reference has no multi-GPU decode).
        value = cpu["value"] * world
        line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 / cpu["value"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": config, "replicas": world, "per_replica_value": cpu["value"],
                "note": "value = replicas x one replica's tokens/s, as our arm sums its N replicas",
                "steps_note": ("steps and warmup echo the command line: this arm ran no K steps but one "
                               "bounded sample (cpu_baseline.sample), extrapolated to the whole model; "
                               "ms_per_step is derived from that sample"),
                "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu["cores"], "kind": "port",
                                 "sample": cpu["sample"]},
                "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as tdist

        # CPU tensors (the replicas' timing) over gloo, CUDA tensors (the expert-parallel
        # sample) over NCCL
        tdist.init_process_group("cpu:gloo,cuda:nccl", timeout=datetime.timedelta(seconds=300))
        dist = tdist
    r = gpu_run(args, cfg, rank, world, dist)
    ms_total, e2e_s = slowest_rank(r["ms_total"], r["e2e_s"], dist)
    _, e2e_calls_s = slowest_rank(r["ms_total"], r["e2e_calls_s"], dist)
    ep = None if args.no_ep else shard_sample(args, rank, world)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    ms_step = ms_total / args.steps
    value, e2e = replica_throughput(world, args.steps, ms_total, e2e_s)

    peak, peak_kind = load_peaks()
    H, I, k = cfg.n_embd, cfg.n_ff, cfg.n_expert_used
    fused = r["counts"][5] == 0  # gate-up and down in one launch (the opt-in fused decode path)
    tc_layout = cfg.expert_layout == 0 and cfg.n_offload < cfg.n_layer
    gu_bytes = k * (3 if fused else 2) * I * H // 32 * 17
    n_gu = max(1, r["counts"][4])
    gu_ms_serial = r["kernel_ms"]["moe_gate_up"] / n_gu
    # the launch time inside the timed graph (CTA timestamps), else the serialised profile's
    ig = r["in_graph"]
    gu_ms = ig["gate_up"] / cfg.n_layer if ig and not fused else gu_ms_serial
    achieved = gu_bytes / (gu_ms / 1000.0) / 1e9
    # the whole step's algorithmic bytes: dense bf16 projections, routers, the 4 chosen experts'
    # three matrices, the KV span each block reads
    Dq, Dkv = cfg.n_head * cfg.head_dim, cfg.n_head_kv * cfg.head_dim
    dense_b = (H * (Dq + 2 * Dkv) + H * Dq) * 2
    expert_b = 3 * k * I * H // 32 * 17
    router_b = cfg.n_expert * H * 4
    kv_b = 0
    for l in range(cfg.n_layer):
        span = args.depth + 1
        if cfg.n_swa and (l % cfg.swa_pattern) < cfg.swa_pattern - 1:
            span = min(span, cfg.n_swa)
        kv_b += span * Dkv * 2 * 2
    step_bytes = cfg.n_layer * (dense_b + expert_b + router_b) + kv_b
    step_gbs = step_bytes / (ms_step / 1000.0) / 1e9

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random weights, N(0,1) inputs)",
        "config": config,
        "roofline": {"bound": "hbm",
                     "kernel": ("moe gate-up + SwiGLU + down + combine, one launch (k_moe_fused, MXFP4, tensor cores)"
                                if fused else
                                "moe gate-up, MXFP4 on the block-scaled FP4 tensor cores (k_xtc<0>, tcgen05.mma "
                                "kind::mxf4, 12 E2M1 digits of the activation)" if tc_layout else
                                "moe gate-up grouped GEMV (MXFP4, mma.sync fragments, k_xexpert<39,0>)"),
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind, "traffic": expert_traffic(fused, tc_layout),
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, profiles/",
                     "bytes_per_launch": gu_bytes, "avg_launch_ms": gu_ms,
                     "avg_launch_ms_source": ("in the timed graph: latest CTA end minus earliest end of a CTA's "
                                              "dependency wait (%globaltimer), mean over blocks and steps"
                                              if ig and not fused else "serialised profile (events between launches)"),
                     "avg_launch_ms_serialised": gu_ms_serial,
                     "frac_of_8tbs": achieved / 8000.0},
        "step_hbm": {"algorithmic_bytes": step_bytes, "achieved_gbs": step_gbs, "frac": step_gbs / peak,
                     "frac_of_8tbs": step_gbs / 8000.0},
        "kernel_ms_per_step_serialised": r["kernel_ms"],
        "expert_kernels_in_graph_ms_per_step": ig,
        "step_kernel": r["step_kernel"],
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": 4 * H, "d2h_bytes_per_step": 4 * H,
                "api": "moearc_x_decoder_step_host (host row in, host row out, one call a step)",
                "three_calls_value": replica_throughput(world, args.steps, ms_total, e2e_calls_s)[1]},
        "gpu_launches": r["launches_per_step"] * args.steps,
        "clocks": r["clocks"],
        "build_s": r["build_s"],
    }
    if cfg.n_offload:
        # mode (b) is bound by PCIe: the offloaded blocks' routed experts cross it every step
        # (with a cache, only the misses: the experts counted as fetched)
        pcie_b = cfg.n_offload * expert_b
        if r["host"] and not cfg.n_cache:
            # the experts the host computes do not cross PCIe
            pcie_b = (cfg.n_offload * k - r["host"]["experts"]) * expert_b / k
        if cfg.n_cache:
            pcie_b = r["fetched_per_step"] * expert_b / cfg.n_expert_used
            line["cache"] = {"slots_per_block": cfg.n_cache, "experts_fetched_per_step": r["fetched_per_step"],
                             "hit_rate": 1.0 - r["fetched_per_step"] / (cfg.n_offload * cfg.n_expert_used)}
            if args.trace:
                # the fetch count the host replay of the slot rule predicts for the same steps
                line["cache"].update(trace=args.trace, fetched=r["fetched"], replay_fetches=r["replay_fetches"],
                                     matches_replay=r["fetched"] == r["replay_fetches"])
        pcie_gbs = pcie_b / (ms_step / 1000.0) / 1e9
        line["roofline_hbm_gate_up"] = line["roofline"]
        line["roofline"] = {"bound": "pcie", "kernel": "expert fetch of the offloaded blocks (whole step)",
                            "achieved": pcie_gbs, "peak": r["pcie_gbs"], "unit": "GB/s",
                            "frac": pcie_gbs / r["pcie_gbs"], "peak_kind": "measured in this run (pinned H2D copy)",
                            "traffic": None, "bytes_per_step": pcie_b}
    if r["host"]:
        h = r["host"]
        line["host_experts"] = {"policy": args.host, "experts_per_step": h["experts"], "jobs_per_step": h["jobs"],
                                "pool_busy_ms_per_step": h["busy_ns"] / 1e6,
                                "sync_wait_ms_per_step": h["wait_ns"] / 1e6}
    if ep:
        line["ep_prefill"] = ep
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_decode_sample(cfg, budget_s=12.0)
    print(json.dumps(line))


if __name__ == "__main__":
    main()
