"""The C-ABI library, checked without a GPU: it loads, exports every symbol include/*.h
declares, and refuses null contexts with the reference's return codes instead of crashing."""
import ctypes as C
import glob
import os
import re
import subprocess

import pytest

from moearc_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols() -> set[str]:
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        names |= set(re.findall(r"^\s*(?:[\w\*\s]+?)\b(moearc_\w+)\s*\(", open(h).read(), re.M))
    return names


def test_every_declared_symbol_is_exported_and_bound():
    lib = _lib.load()
    names = header_symbols()
    assert len(names) >= 40
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T (moearc_\w+)", out))
    assert names <= exported, names - exported
    assert names == set(_lib.SIGNATURES), names ^ set(_lib.SIGNATURES)
    for n in names:
        assert getattr(lib, n) is not None


def test_the_reference_abi_is_all_there():
    """Every function of crates/moearc-kernels/src/ffi.rs:19-263, by name."""
    ffi = ["ctx_create", "ctx_destroy", "profile_events_enabled", "profile_events_reset",
           "profile_events_report", "sync", "zero", "device_name", "alloc_device", "free_device",
           "copy_h2d", "copy_h2d_async", "copy_d2h", "gather_experts", "dequant", "matvec_q",
           "matvec_q_batched", "moe_combine", "matvec_f32", "rmsnorm", "silu", "swiglu",
           "swiglu_halves", "swiglu_oai", "swiglu_oai_halves", "add_bias_id", "softmax", "add",
           "mul", "axpy", "quantize_f16", "embed_rows", "kv_append", "attn_decode", "rope",
           "topk_router"]
    names = header_symbols()
    for f in ffi:
        assert "moearc_" + f in names, f


def test_null_context_is_refused_not_dereferenced():
    lib = _lib.load()
    assert lib.moearc_sync(None) == -1
    assert lib.moearc_dequant(None, 39, None, None, 1) == -1
    assert lib.moearc_topk_router(None, None, None, None, 1, 8, 2, 0) == -1
    assert lib.moearc_alloc_device(None, 16) is None
    assert lib.moearc_profile_events_enabled(None) == 0
    lib.moearc_ctx_destroy(None)  # a no-op, like the reference's delete of null


def test_context_without_a_device_is_null_not_a_crash():
    import torch  # noqa: F401  (only to ask whether a device exists)
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    lib = _lib.load()
    assert not lib.moearc_ctx_create()


def test_the_library_has_no_cpu_fallback_symbols():
    """The shipped library links neither the oracle nor the restated CPU path."""
    out = subprocess.run(["nm", "-D", _lib.LIB_PATH], capture_output=True, text=True, check=True).stdout
    assert "or_matvec" not in out and "hx_ffn" not in out and "cd_step" not in out
