"""The fused MoE decode path (include/moearc.h, moearc_x_moe_*), host side.

``MoeLayer`` owns the device state of one MoE FFN shape and the packed expert banks of one
layer; ``forward`` runs route -> gate/up + activation -> down + combine (+ residual) on the
device with no host round trip, the sequence of crates/moearc-engine/src/moe.rs:2074-2427.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from .kernels import BadArgument, Context, DeviceBuffer, Failed


class MoeLayer:
    def __init__(self, ctx: Context, n_embd: int, n_ff: int, n_expert: int, k: int, gating: int,
                 act: int, wtype: int, max_tokens: int = 1, alpha: float = 1.702, limit: float = 7.0):
        self.ctx = ctx
        self.desc = _lib.MoeDesc(n_embd, n_ff, n_expert, k, gating, act, alpha, limit, wtype, max_tokens)
        self.h = ctx.lib.moearc_x_moe_create(ctx.raw, C.byref(self.desc))
        if not self.h:
            raise BadArgument("moearc_x_moe_create refused the shape")
        self.gu_bytes = ctx.lib.moearc_x_moe_packed_bytes(C.byref(self.desc), 0)
        self.dn_bytes = ctx.lib.moearc_x_moe_packed_bytes(C.byref(self.desc), 1)
        self.gateup: DeviceBuffer | None = None
        self.down: DeviceBuffer | None = None

    def close(self) -> None:
        if self.h:
            self.ctx.lib.moearc_x_moe_destroy(self.h)
            self.h = None

    def pack(self, gate: DeviceBuffer, up: DeviceBuffer, down: DeviceBuffer) -> None:
        """Repack GGUF-layout banks (device) into this layer's packed banks."""
        E = self.desc.n_expert
        self.gateup = self.ctx.alloc(E * self.gu_bytes)
        self.down = self.ctx.alloc(E * self.dn_bytes)
        rc = self.ctx.lib.moearc_x_moe_pack(self.h, gate.ptr, up.ptr, down.ptr, E, self.gateup.ptr,
                                            self.down.ptr)
        self.ctx._finish(rc, "moe_pack")

    def set_bias(self, gate_up_bias: DeviceBuffer | None, down_bias: DeviceBuffer | None) -> None:
        """Per-expert biases for the following forward calls: gate_up_bias f32 [2E][I] (gate of
        expert e at row e, up at E + e), down_bias f32 [E][H]; None: none."""
        E, H, I = self.desc.n_expert, self.desc.n_embd, self.desc.n_ff
        if gate_up_bias is not None:
            gate_up_bias.require("gate/up bias", 4 * 2 * E * I)
        if down_bias is not None:
            down_bias.require("down bias", 4 * E * H)
        rc = self.ctx.lib.moearc_x_moe_set_bias(self.h, gate_up_bias.ptr if gate_up_bias is not None else None,
                                                down_bias.ptr if down_bias is not None else None)
        self.ctx._finish(rc, "moe_set_bias")
        self._bias = (gate_up_bias, down_bias)  # the library keeps the pointers: keep the buffers alive

    def forward(self, x: DeviceBuffer, n_tokens: int, router_w: DeviceBuffer, out: DeviceBuffer,
                router_b: DeviceBuffer | None = None, residual: DeviceBuffer | None = None) -> None:
        H = self.desc.n_embd
        x.require("moe input", 4 * n_tokens * H)
        out.require("moe output", 4 * n_tokens * H)
        router_w.require("router weights", 4 * self.desc.n_expert * H)
        rc = self.ctx.lib.moearc_x_moe_forward(self.h, x.ptr, n_tokens, router_w.ptr,
                                               None if router_b is None else router_b.ptr,
                                               self.gateup.ptr, self.down.ptr,
                                               None if residual is None else residual.ptr, out.ptr)
        self.ctx._finish(rc, "moe_forward")

    def has_tc(self) -> bool:
        """Whether one-token calls can run on the block-scaled FP4 tensor cores (xtc.cu)."""
        return bool(self.ctx.lib.moearc_x_moe_has_tc(self.h))

    def pack_tc(self, gate: DeviceBuffer, up: DeviceBuffer, down: DeviceBuffer) -> None:
        """Repack GGUF-layout MXFP4 banks (device) into the tensor-core layout for forward_tc."""
        if not self.has_tc():
            raise BadArgument("this layer has no tensor-core path")
        E = self.desc.n_expert
        self.gateup_tc = self.ctx.alloc(self.ctx.lib.moearc_x_moe_tc_bytes(C.byref(self.desc), 0))
        self.down_tc = self.ctx.alloc(self.ctx.lib.moearc_x_moe_tc_bytes(C.byref(self.desc), 1))
        rc = self.ctx.lib.moearc_x_moe_pack_tc(self.h, gate.ptr, up.ptr, down.ptr, E, self.gateup_tc.ptr,
                                               self.down_tc.ptr)
        self.ctx._finish(rc, "moe_pack_tc")

    def forward_tc(self, x: DeviceBuffer, router_w: DeviceBuffer, out: DeviceBuffer,
                   router_b: DeviceBuffer | None = None, residual: DeviceBuffer | None = None) -> None:
        """forward for one token on the tensor-core layout banks of pack_tc."""
        H = self.desc.n_embd
        x.require("moe input", 4 * H)
        out.require("moe output", 4 * H)
        router_w.require("router weights", 4 * self.desc.n_expert * H)
        rc = self.ctx.lib.moearc_x_moe_forward_tc(self.h, x.ptr, 1, router_w.ptr,
                                                  None if router_b is None else router_b.ptr,
                                                  self.gateup_tc.ptr, self.down_tc.ptr,
                                                  None if residual is None else residual.ptr, out.ptr)
        self.ctx._finish(rc, "moe_forward_tc")

    def status(self) -> int:
        st = self.ctx.lib.moearc_x_moe_status(self.h)
        if st < 0:
            raise Failed("reading the MoE status word")
        return st

    def buffer(self, which: int, dtype, n: int) -> np.ndarray:
        p = self.ctx.lib.moearc_x_moe_buffer(self.h, which)
        out = np.empty(n, dtype)
        self.ctx._finish(self.ctx.lib.moearc_copy_d2h(self.ctx.raw, out.ctypes.data, p, out.nbytes), "download")
        return out


class MoePrefill:
    """The MoE block for many tokens per call on the tcgen05 tensor cores
    (``moearc_x_prefill_*``): bf16 activations in, f32 out, routing bit-exact with the decode
    path's router."""

    def __init__(self, ctx: Context, n_embd: int, n_ff: int, n_expert: int, k: int, gating: int,
                 act: int, wtype: int, max_tokens: int, alpha: float = 1.702, limit: float = 7.0):
        self.ctx = ctx
        self.desc = _lib.MoeDesc(n_embd, n_ff, n_expert, k, gating, act, alpha, limit, wtype, max_tokens)
        self.h = ctx.lib.moearc_x_prefill_create(ctx.raw, C.byref(self.desc))
        if not self.h:
            raise BadArgument("moearc_x_prefill_create refused the shape")

    def close(self) -> None:
        if self.h:
            self.ctx.lib.moearc_x_prefill_destroy(self.h)
            self.h = None

    def load8(self, gateup: DeviceBuffer, down: DeviceBuffer) -> None:
        """The MXFP8 perf mode: E4M3 weights (exact for MXFP4) and MXFP8 activations on the
        block-scaled FP8 tensor cores."""
        self.ctx._finish(self.ctx.lib.moearc_x_prefill_load8(self.h, gateup.ptr, down.ptr), "prefill_load8")

    def set_bias(self, gate_up_bias: DeviceBuffer | None, down_bias: DeviceBuffer | None) -> None:
        """Per-expert biases (indexed by weight block) for the following forward calls."""
        rc = self.ctx.lib.moearc_x_prefill_set_bias(self.h, gate_up_bias.ptr if gate_up_bias is not None else None,
                                                    down_bias.ptr if down_bias is not None else None)
        self.ctx._finish(rc, "prefill_set_bias")
        self._bias = (gate_up_bias, down_bias)  # the library keeps the pointers

    def load(self, gateup: DeviceBuffer, down: DeviceBuffer) -> None:
        """Expand packed banks (MoeLayer.pack's output) into the bf16 weights the GEMMs read."""
        self.ctx._finish(self.ctx.lib.moearc_x_prefill_load(self.h, gateup.ptr, down.ptr), "prefill_load")

    def forward(self, x_bf16: DeviceBuffer, n_tokens: int, router_w: DeviceBuffer, out: DeviceBuffer,
                router_b: DeviceBuffer | None = None, residual: DeviceBuffer | None = None) -> None:
        H = self.desc.n_embd
        x_bf16.require("prefill input", 2 * n_tokens * H)
        out.require("prefill output", 4 * n_tokens * H)
        router_w.require("router weights", 4 * self.desc.n_expert * H)
        rc = self.ctx.lib.moearc_x_prefill_forward(self.h, x_bf16.ptr, n_tokens, router_w.ptr,
                                                   None if router_b is None else router_b.ptr,
                                                   None if residual is None else residual.ptr, out.ptr)
        self.ctx._finish(rc, "prefill_forward")

    def status(self) -> int:
        st = self.ctx.lib.moearc_x_prefill_status(self.h)
        if st < 0:
            raise Failed("reading the prefill status word")
        return st

    def buffer(self, which: int, dtype, n: int) -> np.ndarray:
        p = self.ctx.lib.moearc_x_prefill_buffer(self.h, which)
        out = np.empty(n, dtype)
        self.ctx._finish(self.ctx.lib.moearc_copy_d2h(self.ctx.raw, out.ctypes.data, p, out.nbytes), "download")
        return out


def _prefill_split_methods():
    """The expert-parallel parts of MoePrefill (route / experts / combine, ranged load)."""

    def load_range(self, gateup: DeviceBuffer, down: DeviceBuffer, e_first: int, n: int) -> None:
        self.ctx._finish(self.ctx.lib.moearc_x_prefill_load_range(self.h, gateup.ptr, down.ptr, e_first, n),
                         "prefill_load_range")

    def route(self, x_bf16, n_tokens: int, router_w: DeviceBuffer, router_b: DeviceBuffer | None = None) -> None:
        ptr = x_bf16 if isinstance(x_bf16, int) else x_bf16.ptr
        rc = self.ctx.lib.moearc_x_prefill_route(self.h, ptr, n_tokens, router_w.ptr,
                                                 None if router_b is None else router_b.ptr)
        self.ctx._finish(rc, "prefill_route")

    def experts(self, rows_ptr: int, n_rows: int, seg_counts: np.ndarray, seg_expert: np.ndarray,
                act_ptr: int, y_ptr: int) -> None:
        sc = np.ascontiguousarray(seg_counts, np.int32)
        se = np.ascontiguousarray(seg_expert, np.int32)
        rc = self.ctx.lib.moearc_x_prefill_experts(self.h, rows_ptr, n_rows, sc.ctypes.data, se.ctypes.data,
                                                   len(sc), act_ptr, y_ptr)
        self.ctx._finish(rc, "prefill_experts")

    def combine(self, y_ptr: int, n_tokens: int, out_ptr: int, residual_ptr: int | None = None) -> None:
        rc = self.ctx.lib.moearc_x_prefill_combine(self.h, y_ptr, n_tokens, residual_ptr, out_ptr)
        self.ctx._finish(rc, "prefill_combine")

    def buffer_ptr(self, which: int) -> int:
        return self.ctx.lib.moearc_x_prefill_buffer(self.h, which)

    def load_list(self, gateup: DeviceBuffer, down: DeviceBuffer, experts) -> None:
        ids = np.ascontiguousarray(experts, np.int32)
        self.ctx._finish(self.ctx.lib.moearc_x_prefill_load_list(self.h, gateup.ptr, down.ptr, ids.ctypes.data,
                                                                 len(ids)), "prefill_load_list")

    def set_order(self, pos) -> None:
        pos = np.ascontiguousarray(pos, np.int32)
        self.ctx._finish(self.ctx.lib.moearc_x_prefill_set_order(self.h, pos.ctypes.data), "prefill_set_order")

    def load4(self, gateup: DeviceBuffer, down: DeviceBuffer, experts=None) -> None:
        """The 4-bit form (all experts, or experts[i] -> slot i); same results as the bf16 form."""
        if experts is None:
            rc = self.ctx.lib.moearc_x_prefill_load4(self.h, gateup.ptr, down.ptr)
        else:
            ids = np.ascontiguousarray(experts, np.int32)
            rc = self.ctx.lib.moearc_x_prefill_load4_list(self.h, gateup.ptr, down.ptr, ids.ctypes.data, len(ids))
        self.ctx._finish(rc, "prefill_load4")

    for f in (load_range, route, experts, combine, buffer_ptr, load_list, set_order, load4):
        setattr(MoePrefill, f.__name__, f)


_prefill_split_methods()
