"""The host-side mirror of the reference's safe wrapper (crates/moearc-kernels/src/lib.rs).

``Context`` and ``DeviceBuffer`` have the reference's method names, argument meaning and error
behaviour: buffer sizes are checked here before a launch (lib.rs:149-155 — a kernel that
overruns an allocation corrupts its neighbour and reports success), a -2 from the library is
``BadArgument``, any other failure is ``Failed``, and a failing call drains the stream before
it raises so no buffer is freed under a running kernel (lib.rs:198-215). Every method calls
the CUDA library through its C ABI; nothing here computes.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _lib

F32, F16, Q4_0, Q8_0, BF16, MXFP4 = 0, 1, 2, 8, 30, 39
Q4_K, Q5_K, Q6_K = 12, 13, 14
BLOCK_BYTES = {F32: 4, F16: 2, BF16: 2, Q4_0: 18, Q8_0: 34, MXFP4: 17, Q4_K: 144, Q5_K: 176, Q6_K: 210}
BLOCK_ELEMS = {F32: 1, F16: 1, BF16: 1, Q4_0: 32, Q8_0: 32, MXFP4: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}
KV_ELEM_BYTES = {F32: 4, F16: 2, BF16: 2}
MAX_BATCHED_MATS = 32
MAX_TOPK = 32


class KernelError(Exception):
    """Why a device operation failed (lib.rs:71-89)."""


class NoDevice(KernelError):
    pass


class OutOfMemory(KernelError):
    pass


class Failed(KernelError):
    pass


class BufferTooSmall(KernelError):
    def __init__(self, what: str, need: int, have: int):
        super().__init__(f"the {what} buffer holds {have} bytes but the requested shape needs {need}")
        self.what, self.need, self.have = what, need, have


class BadArgument(KernelError):
    pass


class DeviceBuffer:
    """An owned device allocation (lib.rs:128-155)."""

    def __init__(self, ctx: "Context", ptr: int, nbytes: int, owned: bool = True):
        self.ctx, self.ptr, self.nbytes, self.owned = ctx, ptr, nbytes, owned

    def __len__(self) -> int:
        return self.nbytes

    def view(self, offset: int, nbytes: int) -> "DeviceBuffer":
        """A non-owning window [offset, offset + nbytes) of this allocation."""
        if offset < 0 or offset + nbytes > self.nbytes:
            raise BufferTooSmall("view", offset + nbytes, self.nbytes)
        return DeviceBuffer(self.ctx, self.ptr + offset, nbytes, owned=False)

    def free(self) -> None:
        if self.ptr and self.owned:
            self.ctx.lib.moearc_free_device(self.ctx.raw, self.ptr)
        self.ptr = 0

    def __del__(self):
        try:
            if self.ptr and self.ctx.raw:
                self.free()
        except Exception:
            pass

    def require(self, what: str, need: int) -> None:
        if self.nbytes < need:
            raise BufferTooSmall(what, need, self.nbytes)


def _p(b: DeviceBuffer | None) -> int | None:
    return None if b is None else b.ptr


class Context:
    """One device and one in-order stream (lib.rs:64-69, 188-196)."""

    def __init__(self):
        self.lib = _lib.load()
        self.raw = self.lib.moearc_ctx_create()
        if not self.raw:
            raise NoDevice("no usable CUDA device")
        self.sync_each = os.environ.get("MOEARC_SYNC_EACH") == "1"

    def close(self) -> None:
        if self.raw:
            self.lib.moearc_ctx_destroy(self.raw)
            self.raw = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # ---- plumbing --------------------------------------------------------------------------

    def _finish(self, rc: int, what: str) -> None:
        if rc != 0:
            self.lib.moearc_sync(self.raw)  # drain before reporting (lib.rs:198-215)
            if rc == -2:
                raise BadArgument(f"{what} was rejected by the kernel")
            raise Failed(f"{what} failed on the device")
        if self.sync_each:
            self.sync()

    def sync(self) -> None:
        if self.lib.moearc_sync(self.raw) != 0:
            raise Failed("stream synchronisation")

    def device_name(self) -> str:
        buf = C.create_string_buffer(256)
        if self.lib.moearc_device_name(self.raw, buf, 256) != 0:
            raise Failed("querying the device name")
        return buf.value.decode()

    def sm_count(self) -> int:
        return self.lib.moearc_x_sm_count(self.raw)

    def alloc(self, nbytes: int) -> DeviceBuffer:
        ptr = self.lib.moearc_alloc_device(self.raw, nbytes)
        if not ptr:
            raise OutOfMemory(f"device allocation of {nbytes} bytes failed")
        return DeviceBuffer(self, ptr, nbytes)

    def alloc_n(self, dtype, n: int) -> DeviceBuffer:
        return self.alloc(np.dtype(dtype).itemsize * n)

    def upload(self, buf: DeviceBuffer, data: np.ndarray) -> None:
        data = np.ascontiguousarray(data)
        buf.require("upload destination", data.nbytes)
        self._finish(self.lib.moearc_copy_h2d(self.raw, buf.ptr, data.ctypes.data, data.nbytes), "upload")

    upload_slice = upload

    def upload_new(self, data: np.ndarray) -> DeviceBuffer:
        data = np.ascontiguousarray(data)
        b = self.alloc(max(data.nbytes, 1))
        self.upload(b, data)
        return b

    def download(self, buf: DeviceBuffer, dtype, n: int) -> np.ndarray:
        out = np.empty(n, dtype)
        buf.require("download source", out.nbytes)
        self._finish(self.lib.moearc_copy_d2h(self.raw, out.ctypes.data, buf.ptr, out.nbytes), "download")
        return out

    def download_slice(self, out: np.ndarray, buf: DeviceBuffer) -> None:
        assert out.flags["C_CONTIGUOUS"]
        buf.require("download source", out.nbytes)
        self._finish(self.lib.moearc_copy_d2h(self.raw, out.ctypes.data, buf.ptr, out.nbytes), "download")

    def zero(self, buf: DeviceBuffer, n: int) -> None:
        buf.require("zero destination", 4 * n)
        self._finish(self.lib.moearc_zero(self.raw, buf.ptr, n), "zero")

    # ---- kernels (lib.rs:426-1242) -----------------------------------------------------------

    def dequant(self, ty: int, dst: DeviceBuffer, src: DeviceBuffer, nblocks: int) -> None:
        if ty in BLOCK_BYTES:
            src.require("dequant source", nblocks * BLOCK_BYTES[ty])
            dst.require("dequant destination", 4 * nblocks * BLOCK_ELEMS[ty])
        self._finish(self.lib.moearc_dequant(self.raw, ty, dst.ptr, src.ptr, nblocks), "dequant")

    def matvec_q(self, ty: int, out: DeviceBuffer, w: DeviceBuffer, x: DeviceBuffer, n_rows: int,
                 n_cols: int) -> None:
        if ty in BLOCK_BYTES and n_cols % BLOCK_ELEMS[ty] == 0:
            w.require("matvec weights", n_rows * n_cols // BLOCK_ELEMS[ty] * BLOCK_BYTES[ty])
        x.require("matvec input", 4 * n_cols)
        out.require("matvec output", 4 * n_rows)
        self._finish(self.lib.moearc_matvec_q(self.raw, ty, out.ptr, w.ptr, x.ptr, n_rows, n_cols), "matvec_q")

    def matvec_q_batched(self, ty: int, out: DeviceBuffer, ws: list[DeviceBuffer], x: DeviceBuffer,
                         x_stride: int, n_rows: int, n_cols: int) -> None:
        n = len(ws)
        if n > MAX_BATCHED_MATS:
            raise BadArgument(f"{n} matrices in one batched matvec")
        if ty in BLOCK_BYTES and n_cols % BLOCK_ELEMS[ty] == 0:
            for w in ws:
                w.require("batched matvec weights", n_rows * n_cols // BLOCK_ELEMS[ty] * BLOCK_BYTES[ty])
        x.require("batched matvec input", 4 * ((n - 1) * x_stride + n_cols) if n else 0)
        out.require("batched matvec output", 4 * n * n_rows)
        arr = (C.c_void_p * max(n, 1))(*[w.ptr for w in ws])
        self._finish(self.lib.moearc_matvec_q_batched(self.raw, ty, out.ptr, arr, n, x.ptr, x_stride,
                                                      n_rows, n_cols), "matvec_q_batched")

    def moe_combine(self, out: DeviceBuffer, parts: DeviceBuffer, weights: DeviceBuffer, n_mat: int,
                    n: int) -> None:
        parts.require("combine parts", 4 * n_mat * n)
        weights.require("combine weights", 4 * n_mat)
        out.require("combine output", 4 * n)
        self._finish(self.lib.moearc_moe_combine(self.raw, out.ptr, parts.ptr, weights.ptr, n_mat, n), "moe_combine")

    def matvec_f32(self, out: DeviceBuffer, w: DeviceBuffer, x: DeviceBuffer, n_rows: int, n_cols: int) -> None:
        w.require("matvec weights", 4 * n_rows * n_cols)
        x.require("matvec input", 4 * n_cols)
        out.require("matvec output", 4 * n_rows)
        self._finish(self.lib.moearc_matvec_f32(self.raw, out.ptr, w.ptr, x.ptr, n_rows, n_cols), "matvec_f32")

    def rmsnorm(self, out: DeviceBuffer, x: DeviceBuffer, weight: DeviceBuffer | None, n_rows: int,
                n_cols: int, eps: float) -> None:
        x.require("rmsnorm input", 4 * n_rows * n_cols)
        out.require("rmsnorm output", 4 * n_rows * n_cols)
        if weight is not None:
            weight.require("rmsnorm weight", 4 * n_cols)
        self._finish(self.lib.moearc_rmsnorm(self.raw, out.ptr, x.ptr, _p(weight), n_rows, n_cols, eps), "rmsnorm")

    def silu(self, out: DeviceBuffer, x: DeviceBuffer, n: int) -> None:
        self._finish(self.lib.moearc_silu(self.raw, out.ptr, x.ptr, n), "silu")

    def swiglu(self, out: DeviceBuffer, gate: DeviceBuffer, up: DeviceBuffer, n: int) -> None:
        for b, w in ((out, "swiglu output"), (gate, "swiglu gate"), (up, "swiglu up")):
            b.require(w, 4 * n)
        self._finish(self.lib.moearc_swiglu(self.raw, out.ptr, gate.ptr, up.ptr, n), "swiglu")

    def swiglu_halves(self, out: DeviceBuffer, gu: DeviceBuffer, n: int) -> None:
        gu.require("swiglu input", 8 * n)
        out.require("swiglu output", 4 * n)
        self._finish(self.lib.moearc_swiglu_halves(self.raw, out.ptr, gu.ptr, n), "swiglu_halves")

    def swiglu_oai(self, out, gate, up, n: int, alpha: float, limit: float) -> None:
        self._finish(self.lib.moearc_swiglu_oai(self.raw, out.ptr, gate.ptr, up.ptr, n, alpha, limit), "swiglu_oai")

    def swiglu_oai_halves(self, out, gu, n: int, alpha: float, limit: float) -> None:
        gu.require("swiglu input", 8 * n)
        self._finish(self.lib.moearc_swiglu_oai_halves(self.raw, out.ptr, gu.ptr, n, alpha, limit), "swiglu_oai_halves")

    def add_bias_id(self, out: DeviceBuffer, bias: DeviceBuffer, idx: list[int], n_rows: int) -> None:
        n = len(idx)
        if n > MAX_BATCHED_MATS:
            raise BadArgument("more bias rows than one launch takes")
        arr = (C.c_uint * max(n, 1))(*idx)
        out.require("bias output", 4 * n * n_rows)
        self._finish(self.lib.moearc_add_bias_id(self.raw, out.ptr, bias.ptr, arr, n, n_rows), "add_bias_id")

    def softmax(self, out, x, mask, n_rows: int, n_cols: int, scale: float) -> None:
        self._finish(self.lib.moearc_softmax(self.raw, out.ptr, x.ptr, _p(mask), n_rows, n_cols, scale), "softmax")

    def add(self, out, a, b, n: int) -> None:
        self._finish(self.lib.moearc_add(self.raw, out.ptr, a.ptr, b.ptr, n), "add")

    def mul(self, out, a, b, n: int) -> None:
        self._finish(self.lib.moearc_mul(self.raw, out.ptr, a.ptr, b.ptr, n), "mul")

    def axpy(self, out, x, alpha: float, n: int) -> None:
        self._finish(self.lib.moearc_axpy(self.raw, out.ptr, x.ptr, alpha, n), "axpy")

    def quantize_f16(self, dst, src, n: int) -> None:
        dst.require("f16 destination", 2 * n)
        self._finish(self.lib.moearc_quantize_f16(self.raw, dst.ptr, src.ptr, n), "quantize_f16")

    def quantize_bf16(self, dst, src, n: int) -> None:
        dst.require("bf16 destination", 2 * n)
        self._finish(self.lib.moearc_x_quantize_bf16(self.raw, dst.ptr, src.ptr, n), "quantize_bf16")

    def embed_rows(self, ty: int, out, table, token_ids, n_tokens: int, n_embd: int) -> None:
        out.require("embedding output", 4 * n_tokens * n_embd)
        self._finish(self.lib.moearc_embed_rows(self.raw, ty, out.ptr, table.ptr, token_ids.ptr, n_tokens,
                                                n_embd), "embed_rows")

    def kv_append(self, k_pages, v_pages, k, v, page_id: int, slot: int, n_kv_heads: int,
                  head_dim: int, page_tokens: int, kv_type: int) -> None:
        if kv_type in KV_ELEM_BYTES and page_tokens:
            need = ((page_id * page_tokens + slot + 1) * n_kv_heads * head_dim) * KV_ELEM_BYTES[kv_type]
            k_pages.require("K pool", need)
            v_pages.require("V pool", need)
        self._finish(self.lib.moearc_kv_append(self.raw, k_pages.ptr, v_pages.ptr, k.ptr, v.ptr, page_id,
                                               slot, n_kv_heads, head_dim, page_tokens, kv_type), "kv_append")

    def attn_decode_ext(self, out, q, k_pages, v_pages, block_table, sinks, n_heads: int,
                        n_kv_heads: int, head_dim: int, kv_begin: int, n_kv: int, page_tokens: int,
                        scale: float, kv_type: int) -> None:
        # lib.rs:1188-1242 refuses these shapes before touching the device.
        if n_kv_heads == 0 or n_heads % n_kv_heads:
            raise BadArgument("n_heads is not a multiple of n_kv_heads")
        if page_tokens == 0:
            raise BadArgument("page_tokens is zero")
        if kv_begin >= n_kv:
            raise BadArgument("an empty key span")
        out.require("attention output", 4 * n_heads * head_dim)
        q.require("attention query", 4 * n_heads * head_dim)
        block_table.require("block table", 4 * ((n_kv + page_tokens - 1) // page_tokens))
        self._finish(self.lib.moearc_attn_decode(self.raw, out.ptr, q.ptr, k_pages.ptr, v_pages.ptr,
                                                 block_table.ptr, _p(sinks), n_heads, n_kv_heads, head_dim,
                                                 kv_begin, n_kv, page_tokens, scale, kv_type), "attn_decode")

    def attn_decode(self, out, q, k_pages, v_pages, block_table, n_heads, n_kv_heads, head_dim, n_kv,
                    page_tokens, scale, kv_type) -> None:
        self.attn_decode_ext(out, q, k_pages, v_pages, block_table, None, n_heads, n_kv_heads, head_dim,
                             0, n_kv, page_tokens, scale, kv_type)

    def rope_ext(self, dst, src, pos, n_tokens: int, n_heads: int, head_dim: int, n_dims: int,
                 freq_base: float, freq_scale: float = 1.0, ext_factor: float = 0.0,
                 attn_factor: float = 1.0, corr_lo: float = 0.0, corr_hi: float = 0.0,
                 neox: bool = True) -> None:
        self._finish(self.lib.moearc_rope(self.raw, dst.ptr, src.ptr, pos.ptr, n_tokens, n_heads, head_dim,
                                          n_dims, freq_base, freq_scale, ext_factor, attn_factor, corr_lo,
                                          corr_hi, 1 if neox else 0), "rope")

    def topk_router(self, idx, weights, logits, n_tokens: int, n_expert: int, k: int, gating: int) -> None:
        if k > MAX_TOPK:
            raise BadArgument(f"k = {k} above the router's ceiling")
        idx.require("router indices", 4 * n_tokens * k)
        weights.require("router weights", 4 * n_tokens * k)
        logits.require("router logits", 4 * n_tokens * n_expert)
        self._finish(self.lib.moearc_topk_router(self.raw, idx.ptr, weights.ptr, logits.ptr, n_tokens,
                                                 n_expert, k, gating), "topk_router")

    def synth(self, dst: DeviceBuffer, n: int, kind: int, seed: int, sigma: float = 1.0, lo: int = -8,
              hi: int = -4) -> None:
        self._finish(self.lib.moearc_x_synth(self.raw, dst.ptr, n, kind, seed, sigma, lo, hi), "synth")

    MMA_KINDS = {"bf16": 0, "mxf8": 1, "mxf4": 2, "mxf8_e2m1": 3}

    def mma_peak(self, kind: str, iters: int = 32768) -> float:
        """Dense TFLOP/s of one tensor-core MMA kind on this device, from the library's own
        tcgen05 loop: "bf16" (kind::f16), "mxf8" (E4M3 x E4M3), "mxf4" (E2M1 x E2M1),
        "mxf8_e2m1" (E4M3 x E2M1), the block-scaled kinds with E8M0 scales per 32."""
        v = C.c_double()
        self._finish(self.lib.moearc_x_mma_peak(self.raw, self.MMA_KINDS[kind], iters, C.byref(v)), "mma_peak")
        return v.value

    def timer_start(self) -> None:
        self._finish(self.lib.moearc_x_timer_start(self.raw), "timer")

    def timer_stop(self) -> float:
        ms = C.c_float()
        self._finish(self.lib.moearc_x_timer_stop(self.raw, C.byref(ms)), "timer")
        return ms.value

    def profile_report(self) -> str:
        buf = C.create_string_buffer(1 << 16)
        self._finish(self.lib.moearc_profile_events_report(self.raw, buf, 1 << 16), "profile report")
        return buf.value.decode()
