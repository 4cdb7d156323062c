"""The host expert pool (moearc_x_host_*): expert FFNs on the CPU cores, read from the packed banks.

No GPU: the pool is host code, checked against the oracle's restatement of the reference's CPU
expert path (hx_ffn, host_experts.rs:624-761) on the GGUF-layout banks the packed ones come from.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

import oracle as O
from moearc_b200 import _lib

H, I, E = 256, 192, 6


def _desc(wtype: int, act: int) -> _lib.MoeDesc:
    return _lib.MoeDesc(H, I, E, 4, 1, act, 1.702, 7.0, wtype, 1)


def _banks(wtype: int, seed: int):
    """GGUF-layout gate, up, down of E experts (each expert contiguous)."""
    nb = E * H * I // 32
    if wtype == O.MXFP4:
        g, u, d = (O.synth_mxfp4(seed + i, nb, -6, -3) for i in range(3))
    else:
        g, u, d = (O.synth_q4_0(seed + i, nb, 0.02) for i in range(3))
    return g, u, d


def _packed(wtype: int, act: int, g, u, d):
    lib = _lib.load()
    desc = _desc(wtype, act)
    gu = np.zeros(2 * g.size, np.uint8)
    dn = np.zeros(d.size, np.uint8)
    rc = lib.moearc_x_moe_pack_host(C.byref(desc), g.ctypes.data, u.ctypes.data, d.ctypes.data, E,
                                    gu.ctypes.data, dn.ctypes.data)
    assert rc == 0
    return desc, gu, dn


def _oracle_ffn(wtype, act, g, u, d, ids, wts, x):
    ol = O.lib()
    mat = H * I // 32 * O.BLOCK_BYTES[wtype]
    n = len(ids)
    arr = C.c_void_p * max(n, 1)
    gp = arr(*[g.ctypes.data + int(e) * mat for e in ids])
    up = arr(*[u.ctypes.data + int(e) * mat for e in ids])
    dp = arr(*[d.ctypes.data + int(e) * mat for e in ids])
    pool = ol.hx_create(2)
    out = np.zeros(H, np.float32)
    w = np.ascontiguousarray(wts, np.float32)
    rc = ol.hx_ffn(pool, wtype, H, I, n, gp, up, dp, w.ctypes.data, x.ctypes.data, act, 1.702, 7.0,
                   out.ctypes.data)
    ol.hx_destroy(pool)
    assert rc == 0
    return out


def _pool_ffn(pool, desc, gu, dn, ids, wts, x):
    lib = _lib.load()
    ids = np.ascontiguousarray(ids, np.uint32)
    wts = np.ascontiguousarray(wts, np.float32)
    out = np.full(H, np.nan, np.float32)
    rc = lib.moearc_x_host_ffn(pool, C.byref(desc), gu.ctypes.data, dn.ctypes.data, ids.ctypes.data,
                               wts.ctypes.data, len(ids), x.ctypes.data, out.ctypes.data)
    assert rc == 0
    return out


@pytest.fixture(params=["avx2", "scalar"])
def isa(request, monkeypatch):
    if request.param == "scalar":
        monkeypatch.setenv("MOEARC_HOST_SCALAR", "1")
    else:
        monkeypatch.delenv("MOEARC_HOST_SCALAR", raising=False)
    return request.param


@pytest.mark.parametrize("wtype,act", [(O.MXFP4, 1), (O.MXFP4, 0), (O.Q4_0, 0), (O.Q4_0, 1)])
def test_pool_matches_the_restated_reference_cpu_path(isa, wtype, act):
    """Router-weighted sum over 1..4 experts, packed banks on the pool against GGUF rows on the
    restated HostExecutor: the portable kernel (the reference's f32 arithmetic) within f32
    reordering, 1e-5 of the output's scale; the AVX2 kernel (input in int16 per 16 elements)
    within the f32 check bound, 1e-4."""
    lib = _lib.load()
    g, u, d = _banks(wtype, 0x4057 + wtype)
    desc, gu, dn = _packed(wtype, act, g, u, d)
    pool = lib.moearc_x_host_pool_create(3)
    assert pool and lib.moearc_x_host_pool_threads(pool) == 3
    rng = np.random.default_rng(7)
    try:
        for n in (1, 2, 4):
            ids = rng.choice(E, n, replace=False).astype(np.uint32)
            wts = rng.random(n).astype(np.float32)
            x = rng.standard_normal(H).astype(np.float32)
            got = _pool_ffn(pool, desc, gu, dn, ids, wts, x)
            want = _oracle_ffn(wtype, act, g, u, d, ids, wts, x)
            scale = max(1e-30, float(np.abs(want).max()))
            err = float(np.abs(got - want).max()) / scale
            assert err < (1e-4 if isa == "avx2" else 1e-5), (isa, wtype, act, n, err)
    finally:
        lib.moearc_x_host_pool_destroy(pool)


def test_results_do_not_depend_on_the_thread_count():
    """Every unit is computed by one thread in a fixed order and the fold is fixed: 1, 2 and 7
    threads give the same bits."""
    lib = _lib.load()
    g, u, d = _banks(O.MXFP4, 0x77)
    desc, gu, dn = _packed(O.MXFP4, 1, g, u, d)
    rng = np.random.default_rng(3)
    ids, wts = np.array([5, 0, 3, 2], np.uint32), rng.random(4).astype(np.float32)
    x = rng.standard_normal(H).astype(np.float32)
    outs = []
    for nt in (1, 2, 7):
        pool = lib.moearc_x_host_pool_create(nt)
        outs.append(_pool_ffn(pool, desc, gu, dn, ids, wts, x))
        outs.append(_pool_ffn(pool, desc, gu, dn, ids, wts, x))  # the pool reused
        lib.moearc_x_host_pool_destroy(pool)
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])


def test_no_experts_is_zero_and_stats_count_jobs_and_experts():
    lib = _lib.load()
    g, u, d = _banks(O.Q4_0, 0x99)
    desc, gu, dn = _packed(O.Q4_0, 0, g, u, d)
    pool = lib.moearc_x_host_pool_create(2)
    x = np.ones(H, np.float32)
    out = _pool_ffn(pool, desc, gu, dn, np.zeros(0, np.uint32), np.zeros(0, np.float32), x)
    assert np.array_equal(out, np.zeros(H, np.float32))
    _pool_ffn(pool, desc, gu, dn, np.array([1, 4, 2], np.uint32), np.ones(3, np.float32), x)
    st = (C.c_ulonglong * 4)()
    lib.moearc_x_host_stats(pool, st)
    assert st[0] == 2 and st[1] == 3 and st[2] > 0
    lib.moearc_x_host_pool_destroy(pool)


def test_submit_and_sync_are_paired_and_bad_shapes_are_refused():
    lib = _lib.load()
    g, u, d = _banks(O.MXFP4, 0x31)
    desc, gu, dn = _packed(O.MXFP4, 0, g, u, d)
    pool = lib.moearc_x_host_pool_create(2)
    x = np.ones(H, np.float32)
    ids, w = np.array([0], np.uint32), np.ones(1, np.float32)
    out = np.zeros(H, np.float32)
    assert lib.moearc_x_host_sync(pool, out.ctypes.data) == -1  # nothing pending
    assert lib.moearc_x_host_submit(pool, C.byref(desc), gu.ctypes.data, dn.ctypes.data, ids.ctypes.data,
                                    w.ctypes.data, 1, x.ctypes.data) == 0
    # a second job before the first is synced
    assert lib.moearc_x_host_submit(pool, C.byref(desc), gu.ctypes.data, dn.ctypes.data, ids.ctypes.data,
                                    w.ctypes.data, 1, x.ctypes.data) == -1
    assert lib.moearc_x_host_sync(pool, out.ctypes.data) == 0
    assert np.all(np.isfinite(out)) and np.abs(out).max() > 0
    many = np.zeros(33, np.uint32)
    assert lib.moearc_x_host_submit(pool, C.byref(desc), gu.ctypes.data, dn.ctypes.data, many.ctypes.data,
                                    np.ones(33, np.float32).ctypes.data, 33, x.ctypes.data) == -2
    bad = _lib.MoeDesc(100, I, E, 4, 1, 0, 1.702, 7.0, O.MXFP4, 1)  # n_embd not a multiple of 64
    assert lib.moearc_x_host_submit(pool, C.byref(bad), gu.ctypes.data, dn.ctypes.data, ids.ctypes.data,
                                    w.ctypes.data, 1, x.ctypes.data) == -2
    lib.moearc_x_host_pool_destroy(pool)


def test_default_thread_count_follows_the_environment(monkeypatch):
    """host_experts.rs:451-456: MOEARC_HOST_THREADS, else the online cores less one."""
    lib = _lib.load()
    monkeypatch.setenv("MOEARC_HOST_THREADS", "3")
    p = lib.moearc_x_host_pool_create(0)
    assert lib.moearc_x_host_pool_threads(p) == 3
    lib.moearc_x_host_pool_destroy(p)
    monkeypatch.delenv("MOEARC_HOST_THREADS")
    p = lib.moearc_x_host_pool_create(0)
    assert lib.moearc_x_host_pool_threads(p) == max(1, (os.cpu_count() or 2) - 1)
    lib.moearc_x_host_pool_destroy(p)
