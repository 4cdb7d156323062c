"""CPU oracle for the MoE decode hot path — TEST INFRASTRUCTURE ONLY.

A ctypes binding to ``liboracle.so`` (built from the C sources beside this file by its
Makefile): the restatement of MoEArc's CPU twin (``crates/moearc-kernels/src/reference.rs``),
the restated CPU expert path (``crates/moearc-engine/src/host_experts.rs``) and the CPU decode
step. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs import this
package, and only as the checker or as the timed CPU baseline. The shipped library
(``moearc_b200``) never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, F16, Q4_0, Q8_0, BF16, MXFP4 = 0, 1, 2, 8, 30, 39
Q4_K, Q5_K, Q6_K = 12, 13, 14
GATING_SOFTMAX, GATING_SOFTMAX_NORM, GATING_SOFTMAX_AFTER_TOPK = 0, 1, 2

_lib = None


def build() -> str:
    """Compile liboracle.so with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
SZ = C.c_size_t
U = C.c_uint
F = C.c_float


class MoeCfg(C.Structure):
    _fields_ = [("n_embd", SZ), ("n_ff", SZ), ("n_expert", SZ), ("k", U), ("gating", U),
                ("act", U), ("alpha", F), ("limit", F), ("wtype", U), ("router_gpu_order", C.c_int)]


class CdCfg(C.Structure):
    _fields_ = [("n_layer", SZ), ("n_embd", SZ), ("n_head", SZ), ("n_head_kv", SZ),
                ("head_dim", SZ), ("n_expert", SZ), ("n_ff", SZ), ("k", U), ("gating", U),
                ("act", U), ("wtype", U), ("kv_type", U), ("alpha", F), ("limit", F), ("eps", F),
                ("n_swa", SZ), ("swa_pattern", SZ), ("page_tokens", SZ), ("rope_base", F),
                ("freq_scale", F), ("ext_factor", F), ("attn_factor", F), ("corr_lo", F),
                ("corr_hi", F), ("qk_norm", U)]


class CdLayer(C.Structure):
    _fields_ = [("attn_norm", P), ("ffn_norm", P), ("wq", P), ("wk", P), ("wv", P), ("wo", P),
                ("sinks", P), ("router", P), ("gate", P), ("up", P), ("down", P),
                ("k_pages", P), ("v_pages", P), ("table", P), ("q_norm", P), ("k_norm", P)]


def _declare(l: C.CDLL) -> None:
    sig = {
        "or_f16_to_f32": (F, [C.c_uint16]),
        "or_f32_to_f16": (C.c_uint16, [F]),
        "or_bf16_to_f32": (F, [C.c_uint16]),
        "or_f32_to_bf16": (C.c_uint16, [F]),
        "or_e8m0_half": (F, [C.c_uint8]),
        "or_block_bytes": (C.c_int, [U]),
        "or_block_elems": (C.c_int, [U]),
        "or_dequant": (C.c_int, [U, P, SZ, P]),
        "or_matvec_q": (C.c_int, [U, P, P, SZ, SZ, P]),
        "or_matvec_f32": (None, [P, P, SZ, SZ, P]),
        "or_matvec_f32_gpu_order": (None, [P, P, SZ, SZ, P]),
        "or_rmsnorm": (None, [P, P, SZ, SZ, F, P]),
        "or_silu": (None, [P, SZ, P]),
        "or_swiglu": (None, [P, P, SZ, P]),
        "or_swiglu_oai": (None, [P, P, SZ, F, F, P]),
        "or_softmax_ext": (None, [P, P, SZ, SZ, F, P]),
        "or_add": (None, [P, P, SZ, P]),
        "or_mul": (None, [P, P, SZ, P]),
        "or_axpy": (None, [P, P, F, SZ]),
        "or_moe_combine": (None, [P, P, U, SZ, P]),
        "or_add_bias_id": (None, [P, P, P, U, SZ]),
        "or_embed_rows": (C.c_int, [U, P, P, SZ, SZ, P]),
        "or_rope": (None, [P, P, SZ, SZ, SZ, SZ, F, C.c_int, P]),
        "or_rope_ext": (None, [P, P, SZ, SZ, SZ, SZ, F, F, F, F, F, F, C.c_int, P]),
        "or_topk_router": (C.c_int, [P, SZ, SZ, U, U, P, P]),
        "or_kv_index": (SZ, [C.c_uint32, C.c_uint32, SZ, SZ, SZ, SZ, SZ]),
        "or_kv_store": (F, [F, U]),
        "or_kv_append": (C.c_int, [P, P, P, P, C.c_uint32, C.c_uint32, SZ, SZ, SZ, U]),
        "or_attn_decode": (C.c_int, [P, P, P, P, P, SZ, SZ, SZ, SZ, SZ, SZ, F, U, P]),
        "or_moe_ffn_token": (C.c_int, [C.POINTER(MoeCfg), P, P, P, P, P, P, P, P, P, P, P, P]),
        "or_moe_ffn_token_mx8": (C.c_int, [C.POINTER(MoeCfg), P, P, P, P, P, P, P, P, P, P, P, P]),
        "or_mx8_quantize": (None, [P, SZ, P]),
        "or_synth_mxfp4": (None, [C.c_uint64, SZ, C.c_int, C.c_int, P]),
        "or_synth_q4_0": (None, [C.c_uint64, SZ, C.c_double, P]),
        "or_synth_normal_f32": (None, [C.c_uint64, SZ, C.c_double, P]),
        "or_synth_normal_bf16": (None, [C.c_uint64, SZ, C.c_double, P]),
        "hx_default_threads": (C.c_int, []),
        "hx_create": (P, [C.c_int]),
        "hx_destroy": (None, [P]),
        "hx_threads": (C.c_int, [P]),
        "hx_ffn": (C.c_int, [P, U, SZ, SZ, U, P, P, P, P, P, C.c_int, F, F, P]),
        "hx_matvec": (C.c_int, [P, U, P, P, SZ, SZ, P]),
        "cd_step": (C.c_int, [C.POINTER(CdCfg), P, P, P, SZ, P, P, P]),
        "cd_step_margins": (C.c_int, [C.POINTER(CdCfg), P, P, P, SZ, P, P, P]),
        "cd_layers": (C.c_int, [C.POINTER(CdCfg), P, SZ, SZ, P, SZ, P, P]),
        "cd_logits": (C.c_int, [C.POINTER(CdCfg), P, SZ, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(l, name)
        fn.restype = res
        fn.argtypes = args


def ptr(a: np.ndarray | None) -> int | None:
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ---- numpy conveniences -------------------------------------------------------------------

BLOCK_BYTES = {F32: 4, F16: 2, BF16: 2, Q4_0: 18, Q8_0: 34, MXFP4: 17, Q4_K: 144, Q5_K: 176, Q6_K: 210}
BLOCK_ELEMS = {F32: 1, F16: 1, BF16: 1, Q4_0: 32, Q8_0: 32, MXFP4: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}


def row_bytes(t: int, n_cols: int) -> int:
    return n_cols // BLOCK_ELEMS[t] * BLOCK_BYTES[t]


def dequant(t: int, src: np.ndarray, nblocks: int) -> np.ndarray:
    out = np.zeros(nblocks * BLOCK_ELEMS[t], np.float32)
    rc = lib().or_dequant(t, ptr(src), nblocks, ptr(out))
    assert rc == 0, rc
    return out


def matvec_q(t: int, w: np.ndarray, x: np.ndarray, n_rows: int, n_cols: int) -> np.ndarray:
    out = np.zeros(n_rows, np.float32)
    rc = lib().or_matvec_q(t, ptr(w), ptr(np.ascontiguousarray(x, np.float32)), n_rows, n_cols,
                           ptr(out))
    assert rc == 0, rc
    return out


def matvec_f32(w: np.ndarray, x: np.ndarray, gpu_order: bool = False) -> np.ndarray:
    n_rows, n_cols = w.shape
    out = np.zeros(n_rows, np.float32)
    fn = lib().or_matvec_f32_gpu_order if gpu_order else lib().or_matvec_f32
    fn(ptr(np.ascontiguousarray(w, np.float32)), ptr(np.ascontiguousarray(x, np.float32)),
       n_rows, n_cols, ptr(out))
    return out


def topk_router(logits: np.ndarray, k: int, gating: int):
    logits = np.ascontiguousarray(logits, np.float32)
    n_tokens, n_expert = logits.shape
    idx = np.zeros((n_tokens, k), np.uint32)
    w = np.zeros((n_tokens, k), np.float32)
    rc = lib().or_topk_router(ptr(logits), n_tokens, n_expert, k, gating, ptr(idx), ptr(w))
    assert rc == 0, rc
    return idx, w


def synth_mxfp4(seed: int, nblocks: int, e_lo: int = -8, e_hi: int = -4) -> np.ndarray:
    out = np.zeros(nblocks * 17, np.uint8)
    lib().or_synth_mxfp4(seed, nblocks, e_lo, e_hi, ptr(out))
    return out


def synth_q4_0(seed: int, nblocks: int, sigma: float = 0.01) -> np.ndarray:
    out = np.zeros(nblocks * 18, np.uint8)
    lib().or_synth_q4_0(seed, nblocks, sigma, ptr(out))
    return out


def synth_normal_f32(seed: int, n: int, sigma: float = 1.0) -> np.ndarray:
    out = np.zeros(n, np.float32)
    lib().or_synth_normal_f32(seed, n, sigma, ptr(out))
    return out


def synth_normal_bf16(seed: int, n: int, sigma: float = 1.0) -> np.ndarray:
    out = np.zeros(n, np.uint16)
    lib().or_synth_normal_bf16(seed, n, sigma, ptr(out))
    return out


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """RNE, NaN kept quiet — the same rule as or_f32_to_bf16, vectorised."""
    b = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    nan = ((b & 0x7F800000) == 0x7F800000) & ((b & 0x7FFFFF) != 0)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((b[nan] >> 16) | 0x40).astype(np.uint16)
    return r


class SplitMix64:
    """SplitMix64 (tests/common/mod.rs:11-38 in the reference): a seeded, replayable stream."""

    def __init__(self, seed: int):
        self.s = seed & 0xFFFFFFFFFFFFFFFF

    def next_u64(self) -> int:
        M = 0xFFFFFFFFFFFFFFFF
        self.s = (self.s + 0x9E3779B97F4A7C15) & M
        z = self.s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        return z ^ (z >> 31)

    def next_u32(self) -> int:
        return self.next_u64() & 0xFFFFFFFF

    def unit(self) -> float:
        """Uniform in [-1, 1), as f32 (tests/common/mod.rs:31-33)."""
        return float(np.float32(np.float32(self.next_u32()) / np.float32(4294967296.0)) * 2 - 1)

    def vec_unit(self, n: int) -> np.ndarray:
        return np.array([self.unit() for _ in range(n)], np.float32)
