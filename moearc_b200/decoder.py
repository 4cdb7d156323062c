"""The synthetic decoder (include/moearc.h, moearc_x_decoder_*), host side.

``Decoder`` builds a gpt-oss- or Qwen3-MoE-shaped model with seeded random weights on the
device and decodes one token per ``step()``: the per-block sequence of
crates/moearc-engine/src/moe.rs:1862-2443 (Model::decode), captured once as a CUDA graph.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, fields

import numpy as np

from . import _lib
from .kernels import BadArgument, Context, Failed

MXFP4, Q4_0 = 39, 2


@dataclass
class DecoderConfig:
    n_layer: int
    n_embd: int
    n_head: int
    n_head_kv: int
    head_dim: int
    n_expert: int
    n_expert_used: int
    n_ff: int
    expert_type: int = MXFP4
    gating: int = 2
    act: int = 1
    alpha: float = 1.702
    limit: float = 7.0
    n_swa: int = 128
    swa_pattern: int = 2
    rope_base: float = 150000.0
    rope_freq_scale: float = 1.0
    rope_ext_factor: float = 0.0
    rope_attn_factor: float = 1.0
    rope_corr_lo: float = 0.0
    rope_corr_hi: float = 0.0
    rms_eps: float = 1e-5
    has_sinks: int = 1
    n_ctx: int = 4096
    seed: int = 0x5EED
    # blocks 0 .. n_offload-1 keep their experts in pinned host memory, fetched over PCIe each
    # step (the -ncmoe mirror, moe.rs:1179-1299); 0 = all resident
    n_offload: int = 0
    # device slots per offloaded block that keep fetched experts across steps (the reference's
    # ExpertCache); 0 = pure streaming, else n_expert_used <= n_cache <= n_expert
    n_cache: int = 0
    # QK-norm per head before RoPE (moe.rs:1961-1985; qwen3moe has it, gpt-oss not)
    has_qk_norm: int = 0
    # rows of the output head (logits after the final norm, moe.rs:2434-2437); 0 = none
    n_vocab: int = 0
    # resident blocks' expert banks: 0 = the tensor-core layout run on the block-scaled FP4
    # tensor cores where the shape has one (MXFP4), 1 = the fragment layout (the persistent step
    # kernel needs it)
    expert_layout: int = 0

    def yarn(self, factor: float, n_ctx_orig: int, beta_fast: float = 32.0, beta_slow: float = 1.0):
        """YaRN parameters the way reference.rs:572-591 derives them (RopeScaling::yarn)."""
        n_dims = self.head_dim

        def corr(beta):
            return n_dims * math.log(n_ctx_orig / (beta * 2 * math.pi)) / (2 * math.log(self.rope_base))

        self.rope_freq_scale = 1.0 / factor
        self.rope_ext_factor = 1.0
        self.rope_attn_factor = 1.0
        self.rope_corr_lo = max(0.0, math.floor(corr(beta_fast)))
        self.rope_corr_hi = min(n_dims - 1.0, math.ceil(corr(beta_slow)))
        return self

    def to_c(self) -> _lib.DecoderCfg:
        return _lib.DecoderCfg(*[getattr(self, f.name) for f in fields(self)])

    # ---- the BASELINE configurations ---------------------------------------------------------
    @staticmethod
    def gpt_oss_20b(**kw) -> "DecoderConfig":
        """24 layers, hidden 2880, 64 q / 8 kv heads of 64, 32 experts top-4, I 2880."""
        c = DecoderConfig(**{**dict(n_layer=24, n_embd=2880, n_head=64, n_head_kv=8, head_dim=64, n_expert=32,
                                    n_expert_used=4, n_ff=2880), **kw})
        return c.yarn(32.0, 4096)

    @staticmethod
    def gpt_oss_120b(**kw) -> "DecoderConfig":
        """as configs[1] with 36 layers and 128 experts."""
        c = DecoderConfig(**{**dict(n_layer=36, n_embd=2880, n_head=64, n_head_kv=8, head_dim=64, n_expert=128,
                                    n_expert_used=4, n_ff=2880), **kw})
        return c.yarn(32.0, 4096)

    @staticmethod
    def qwen3_moe(**kw) -> "DecoderConfig":
        """48 layers, hidden 2048, 32 q / 4 kv heads of 128, 128 experts top-8,
        I 768, Q4_0 experts, renormalised softmax gating, SwiGLU, QK-norm, no window, no sinks."""
        kw.setdefault("expert_type", Q4_0)
        kw.setdefault("gating", 1)
        kw.setdefault("act", 0)
        kw.setdefault("n_swa", 0)
        kw.setdefault("has_sinks", 0)
        kw.setdefault("rope_base", 1000000.0)
        kw.setdefault("rms_eps", 1e-6)
        kw.setdefault("has_qk_norm", 1)
        return DecoderConfig(**{**dict(n_layer=48, n_embd=2048, n_head=32, n_head_kv=4, head_dim=128, n_expert=128,
                                       n_expert_used=8, n_ff=768), **kw})


class Decoder:
    def __init__(self, ctx: Context, cfg: DecoderConfig):
        self.ctx, self.cfg = ctx, cfg
        self._c = cfg.to_c()
        self.h = ctx.lib.moearc_x_decoder_create(ctx.raw, C.byref(self._c))
        if not self.h:
            raise BadArgument("moearc_x_decoder_create refused the configuration or ran out of memory")
        self.in_ptr = ctx.lib.moearc_x_decoder_input(self.h)
        self.out_ptr = ctx.lib.moearc_x_decoder_output(self.h)

    def close(self) -> None:
        if self.h:
            self.ctx.lib.moearc_x_decoder_destroy(self.h)
            self.h = None

    @property
    def pos(self) -> int:
        return self.ctx.lib.moearc_x_decoder_pos(self.h)

    def fill_kv(self, depth: int, seed: int = 0xC0DE) -> None:
        self.ctx._finish(self.ctx.lib.moearc_x_decoder_fill_kv(self.h, depth, seed), "fill_kv")

    def set_pos(self, pos: int) -> None:
        self.ctx._finish(self.ctx.lib.moearc_x_decoder_set_pos(self.h, pos), "set_pos")

    def use_graph(self, on: bool) -> None:
        self.ctx._finish(self.ctx.lib.moearc_x_decoder_use_graph(self.h, 1 if on else 0), "use_graph")

    def has_step_kernel(self) -> bool:
        """True when this shape can run the step as one persistent kernel."""
        return self.ctx.lib.moearc_x_decoder_has_step_kernel(self.h) == 1

    def uses_step_kernel(self) -> bool:
        """True when steps run as one persistent kernel, False for the per-block kernel chain."""
        return self.ctx.lib.moearc_x_decoder_uses_step_kernel(self.h) == 1

    def use_step_kernel(self, on: bool) -> None:
        self.ctx._finish(self.ctx.lib.moearc_x_decoder_use_step_kernel(self.h, 1 if on else 0), "use_step_kernel")

    def set_wait(self, limit_ns: int = 0, phantom: int = 0) -> None:
        """The decode kernels' wait limits (0: default) and phantom=1 to make them run out (testing)."""
        self.ctx._finish(self.ctx.lib.moearc_x_decoder_set_wait(self.h, limit_ns, phantom), "set_wait")

    def trace_words(self) -> int:
        return self.ctx.lib.moearc_x_decoder_trace_words(self.h)

    def set_trace(self, buf) -> None:
        """Phase timestamps into a device buffer of trace_words() u64 (None: off)."""
        self.ctx._finish(self.ctx.lib.moearc_x_decoder_set_trace(self.h, buf.ptr if buf is not None else None),
                         "set_trace")

    def routing(self, layer: int) -> tuple[np.ndarray, np.ndarray]:
        """Block `layer`'s expert ids and gating weights of the last step (persistent kernel)."""
        return self.tensor(12, layer, np.uint32), self.tensor(13, layer, np.float32)

    HOST_POLICIES = {"off": 0, "fraction": 1, "over": 2}

    def host_experts(self, policy: str = "fraction", fraction: float = 0.5, over: int = 0,
                     threads: int = 0) -> None:
        """Compute part of the offloaded blocks' experts on host threads beside the device:
        "fraction" takes the first ceil(misses x fraction) of a block's misses (router order),
        "over" the misses beyond the first `over`, "off" none (the reference's HostPolicy)."""
        self.ctx._finish(self.ctx.lib.moearc_x_decoder_host_experts(self.h, self.HOST_POLICIES[policy], fraction,
                                                                    over, threads), "host_experts")

    def host_wait(self, limit_ns: int = 0, hold: bool = False) -> None:
        """The fold's wait limit for the host's answer (0: 2 s); hold=True makes the host thread
        ignore new jobs, so the wait runs out (testing)."""
        self.ctx._finish(self.ctx.lib.moearc_x_decoder_host_wait(self.h, limit_ns, 1 if hold else 0), "host_wait")

    def host_stats(self) -> dict:
        """The host pool's counters: jobs, experts, busy and wait nanoseconds."""
        st = (C.c_ulonglong * 4)()
        self.ctx._finish(self.ctx.lib.moearc_x_decoder_host_stats(self.h, st), "host_stats")
        return {"jobs": st[0], "experts": st[1], "busy_ns": st[2], "wait_ns": st[3]}

    def kernel_spans(self, on: bool) -> None:
        """Per-CTA timestamps of the kernel chain's expert kernels in every following step."""
        self.ctx._finish(self.ctx.lib.moearc_x_decoder_kernel_spans(self.h, 1 if on else 0), "kernel_spans")

    def expert_kernel_ms(self) -> tuple[float, float]:
        """The last step's gate-up and down expert kernels, each timed from inside the step (a
        graph replay included) as the latest CTA end minus the earliest moment a CTA's
        dependency wait was over, summed over the blocks: (gate-up ms, down ms)."""
        tot = [0.0, 0.0]
        for layer in range(self.cfg.n_layer):
            s = self.tensor(14, layer, np.uint64).reshape(2, -1, 3).astype(np.int64)
            for k in range(2):
                live = s[k, :, 1] > 0  # records of CTAs the kernel launched
                ends, waits = s[k, live, 2], s[k, live, 1]
                tot[k] += (ends.max() - waits.min()) / 1e6
        return tot[0], tot[1]

    def fetched(self) -> int:
        """Experts the offloaded blocks' residency caches fetched over PCIe since create."""
        return self.ctx.lib.moearc_x_decoder_fetched(self.h)

    def status(self) -> int:
        """Reads and clears the kernels' device status words: 0, or nonzero when a bounded
        wait gave up (the steps since the last read are then invalid)."""
        st = self.ctx.lib.moearc_x_decoder_status(self.h)
        if st < 0:
            self.ctx._finish(st, "status")
        return st

    def step(self) -> None:
        """Enqueue one decode step (the caller synchronises when it needs the output)."""
        self.ctx._finish(self.ctx.lib.moearc_x_decoder_step(self.h), "decoder step")

    def step_host(self, x: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        """Decode one token from a host row to a host row in one call: the input copy, the step
        and the output copy run as one graph launch, and the call returns when the output has
        arrived (moearc_x_decoder_step_host)."""
        x = np.ascontiguousarray(x, np.float32)
        assert x.size == self.cfg.n_embd
        if out is None:
            out = np.empty(self.cfg.n_embd, np.float32)
        assert out.dtype == np.float32 and out.size == self.cfg.n_embd and out.flags.c_contiguous
        self.ctx._finish(self.ctx.lib.moearc_x_decoder_step_host(self.h, x.ctypes.data, out.ctypes.data),
                         "decoder step (host buffers)")
        return out

    def set_input(self, x: np.ndarray) -> None:
        x = np.ascontiguousarray(x, np.float32)
        assert x.size == self.cfg.n_embd
        self.ctx._finish(self.ctx.lib.moearc_copy_h2d(self.ctx.raw, self.in_ptr, x.ctypes.data, x.nbytes), "input")

    def logits(self) -> np.ndarray:
        """The last step's output-head logits (n_vocab floats; the configuration must have a head)."""
        p = self.ctx.lib.moearc_x_decoder_logits(self.h)
        if not p:
            raise BadArgument("the decoder has no output head (n_vocab = 0)")
        out = np.empty(self.cfg.n_vocab, np.float32)
        self.ctx._finish(self.ctx.lib.moearc_copy_d2h(self.ctx.raw, out.ctypes.data, p, out.nbytes), "logits")
        return out

    def output(self) -> np.ndarray:
        out = np.empty(self.cfg.n_embd, np.float32)
        self.ctx._finish(self.ctx.lib.moearc_copy_d2h(self.ctx.raw, out.ctypes.data, self.out_ptr, out.nbytes), "output")
        return out

    def tensor(self, which: int, layer: int, dtype) -> np.ndarray:
        n = C.c_ulong()
        p = self.ctx.lib.moearc_x_decoder_tensor(self.h, which, layer, C.byref(n))
        if not p and n.value:
            raise Failed("no such tensor")
        out = np.empty(n.value // np.dtype(dtype).itemsize, dtype)
        if n.value:
            self.ctx._finish(self.ctx.lib.moearc_copy_d2h(self.ctx.raw, out.ctypes.data, p, n.value), "tensor")
        return out

    def read(self, which: int, layer: int, offset: int, n: int, dtype) -> np.ndarray:
        """n elements of one block's tensor (the `tensor` numbering) from element `offset`."""
        size = C.c_ulong()
        p = self.ctx.lib.moearc_x_decoder_tensor(self.h, which, layer, C.byref(size))
        item = np.dtype(dtype).itemsize
        if not p or (offset + n) * item > size.value:
            raise BadArgument(f"elements [{offset}, {offset + n}) of tensor {which} of block {layer}")
        out = np.empty(n, dtype)
        self.ctx._finish(self.ctx.lib.moearc_copy_d2h(self.ctx.raw, out.ctypes.data, p + offset * item, n * item),
                         "tensor read")
        return out

    def set_tensor(self, which: int, layer: int, data: np.ndarray) -> None:
        """Overwrite one block's tensor (the `tensor` numbering) with `data`, which must have its
        exact size; ordered before the next step on the context stream."""
        n = C.c_ulong()
        p = self.ctx.lib.moearc_x_decoder_tensor(self.h, which, layer, C.byref(n))
        data = np.ascontiguousarray(data)
        if not p or data.nbytes != n.value:
            raise BadArgument(f"tensor {which} of block {layer} holds {n.value} bytes, not {data.nbytes}")
        self.ctx._finish(self.ctx.lib.moearc_copy_h2d(self.ctx.raw, p, data.ctypes.data, data.nbytes), "tensor")

    def seed(self, kind: int, layer: int) -> int:
        return self.ctx.lib.moearc_x_decoder_seed(self.h, kind, layer, self.cfg.seed)


class BatchDecoder:
    """n_batch independent sequences decoding one token each per step (moearc_x_batch_decoder_*):
    the batched serving case (configs[4]: 64 streams of a Qwen3-MoE-shaped model)."""

    def __init__(self, ctx: Context, cfg: DecoderConfig, n_batch: int, ep: tuple | None = None):
        """ep = (comm, rank, n_ranks): expert parallelism over an NCCL communicator (a handle from
        moearc_b200.ep.nccl_comm); n_batch is then this rank's streams."""
        self.ctx, self.cfg, self.n_batch = ctx, cfg, n_batch
        self._c = cfg.to_c()
        if ep is None:
            self.h = ctx.lib.moearc_x_batch_decoder_create(ctx.raw, C.byref(self._c), n_batch)
        else:
            comm, rank, world = ep
            self.h = ctx.lib.moearc_x_batch_decoder_create_ep(ctx.raw, C.byref(self._c), n_batch, comm, rank, world)
        if not self.h:
            raise BadArgument("moearc_x_batch_decoder_create refused the configuration or ran out of memory")
        self.in_ptr = ctx.lib.moearc_x_batch_decoder_input(self.h)
        self.out_ptr = ctx.lib.moearc_x_batch_decoder_output(self.h)

    def close(self) -> None:
        if self.h:
            self.ctx.lib.moearc_x_batch_decoder_destroy(self.h)
            self.h = None

    def set_pos(self, pos: int, fill: bool = False, seed: int = 0xC0DE) -> None:
        self.ctx._finish(self.ctx.lib.moearc_x_batch_decoder_set_pos(self.h, pos, 1 if fill else 0, seed), "set_pos")

    def step(self) -> None:
        self.ctx._finish(self.ctx.lib.moearc_x_batch_decoder_step(self.h), "batch decoder step")

    def set_input(self, x: np.ndarray) -> None:
        x = np.ascontiguousarray(x, np.float32)
        assert x.size == self.n_batch * self.cfg.n_embd
        self.ctx._finish(self.ctx.lib.moearc_copy_h2d(self.ctx.raw, self.in_ptr, x.ctypes.data, x.nbytes), "input")

    def output(self) -> np.ndarray:
        out = np.empty((self.n_batch, self.cfg.n_embd), np.float32)
        self.ctx._finish(self.ctx.lib.moearc_copy_d2h(self.ctx.raw, out.ctypes.data, self.out_ptr, out.nbytes), "output")
        return out

    def routing(self, layer: int) -> np.ndarray:
        """Block `layer`'s expert choice of the last step, [n_batch][k] in router order."""
        p = self.ctx.lib.moearc_x_batch_decoder_routing(self.h, layer)
        if not p:
            raise BadArgument(f"no block {layer}")
        out = np.empty((self.n_batch, self.cfg.n_expert_used), np.uint32)
        self.ctx._finish(self.ctx.lib.moearc_copy_d2h(self.ctx.raw, out.ctypes.data, p, out.nbytes), "routing")
        return out

    def status(self) -> int:
        st = self.ctx.lib.moearc_x_batch_decoder_status(self.h)
        if st < 0:
            raise Failed("reading the batch decoder status")
        return st


def unpack_dense(packed: np.ndarray, n_rows: int, n_cols: int) -> np.ndarray:
    """Invert the packed bf16 tile layout (dense.cuh) back to a row-major [n_rows][n_cols] bf16
    matrix: tile (tr, tk) = 16 rows x 64 cols; inside it, for each 16-column sub-block s, lane
    l = 4r + q holds four u32: (row r, cols 16s+2q..+1), (row r+8, same), (row r,
    16s+2q+8..+9), (row r+8, same)."""
    ntr, nkt = n_rows // 16, n_cols // 64
    p = packed.view(np.uint16).reshape(ntr, nkt, 4, 8, 4, 4, 2)  # tr, tk, s, r, q, reg, half
    w = np.empty((ntr, 16, nkt, 64), np.uint16)
    offs = ((0, 0), (8, 0), (0, 8), (8, 8))  # (row, col) offset of register reg
    for r in range(8):
        for q in range(4):
            for s in range(4):
                for reg, (ro, co) in enumerate(offs):
                    for half in range(2):
                        w[:, r + ro, :, 16 * s + 2 * q + co + half] = p[:, :, s, r, q, reg, half]
    return w.reshape(n_rows, n_cols)


def pack_dense(w: np.ndarray) -> np.ndarray:
    """The packed bf16 tile layout, built on the host (the inverse of unpack_dense)."""
    n_rows, n_cols = w.shape
    ntr, nkt = n_rows // 16, n_cols // 64
    v = w.reshape(ntr, 16, nkt, 64)
    p = np.empty((ntr, nkt, 4, 8, 4, 4, 2), np.uint16)
    offs = ((0, 0), (8, 0), (0, 8), (8, 8))
    for r in range(8):
        for q in range(4):
            for s in range(4):
                for reg, (ro, co) in enumerate(offs):
                    for half in range(2):
                        p[:, :, s, r, q, reg, half] = v[:, r + ro, :, 16 * s + 2 * q + co + half]
    return p.ravel()
