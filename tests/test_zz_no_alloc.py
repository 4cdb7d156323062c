"""moearc_x_attn_decode_static — decode attention whose split-K partials sit in a fixed device
array — against moearc_attn_decode, both called through the C ABI on the same inputs.

The two entry points run the same kernels in the same order and differ only in where the
partials live, so their outputs must agree; the tolerance below allows last-bit noise only.
Each case calls the fixed-array entry point twice in a row (and a different problem in
between), so stale partials from an earlier call would show up as a mismatch.
"""
import numpy as np
import pytest

from moearc_b200 import Context, _lib

pytestmark = pytest.mark.gpu

F32, F16, BF16 = 0, 1, 30
LIMIT = 2 << 20  # MOEARC_X_ATTN_STATIC_SCRATCH_BYTES in include/moearc.h
TOL = 1e-6


@pytest.fixture(scope="module")
def ctx():
    c = Context()
    yield c
    c.close()


def splits(sm_count, n_kv_heads, n_heads, span, mma):
    """The split count the library picks for a key span (attention.cu, attn_splits)."""
    units = n_kv_heads if mma else n_heads
    want = (2 * sm_count + units - 1) // units
    kps = max(64, ((-(-span // want) + 63) // 64) * 64)
    return -(-span // kps)


def make_case(ctx, H, KVH, D, n_kv, PT, kv, seed, sinks=False):
    rng = np.random.default_rng(seed)
    pages = -(-n_kv // PT) + 3
    table = rng.permutation(pages).astype(np.uint32)
    pool = pages * PT * KVH * D
    if kv == F32:
        kh = rng.standard_normal(pool, np.float32)
        vh = rng.standard_normal(pool, np.float32)
    else:
        def half(a):
            if kv == F16:
                return a.astype(np.float16).view(np.uint16)
            return (a.view(np.uint32) + 0x7FFF + ((a.view(np.uint32) >> 16) & 1) >> 16).astype(np.uint16)
        kh = half(rng.standard_normal(pool, np.float32))
        vh = half(rng.standard_normal(pool, np.float32))
    q = rng.standard_normal(H * D, np.float32)
    s = rng.standard_normal(H, np.float32) if sinks else None
    return {
        "q": ctx.upload_new(q), "k": ctx.upload_new(kh), "v": ctx.upload_new(vh),
        "t": ctx.upload_new(table), "s": None if s is None else ctx.upload_new(s),
        "H": H, "KVH": KVH, "D": D, "n_kv": n_kv, "PT": PT, "kv": kv, "scale": 1.0 / np.sqrt(D),
    }


def call(ctx, fn, c, out, begin):
    lib = _lib.load()
    f = getattr(lib, fn)
    return f(ctx.raw, out.ptr, c["q"].ptr, c["k"].ptr, c["v"].ptr, c["t"].ptr,
             None if c["s"] is None else c["s"].ptr, c["H"], c["KVH"], c["D"], begin, c["n_kv"], c["PT"],
             c["scale"], c["kv"])


def run(ctx, fn, c, begin):
    out = ctx.alloc_n(np.float32, c["H"] * c["D"])
    assert call(ctx, fn, c, out, begin) == 0
    ctx.sync()
    return ctx.download(out, np.float32, c["H"] * c["D"])


def rel(a, b):
    return float(np.max(np.abs(a.astype(np.float64) - b) / np.maximum(np.abs(b), 1.0)))


CASES = [
    # (H, KVH, D, n_kv, PT, kv, sinks, window) — tensor-core path, generic path, sliding window
    (64, 8, 64, 4096, 32, BF16, True, 0),
    (64, 8, 128, 3000, 32, F16, False, 0),
    (4, 4, 96, 2000, 16, F32, True, 0),
    (64, 8, 64, 5000, 32, BF16, True, 128),
]


@pytest.mark.parametrize("H,KVH,D,n_kv,PT,kv,sinks,window", CASES)
def test_static_partials_match_scratch_partials(ctx, H, KVH, D, n_kv, PT, kv, sinks, window):
    c = make_case(ctx, H, KVH, D, n_kv, PT, kv, seed=H * 7919 + n_kv, sinks=sinks)
    other = make_case(ctx, 16, 2, 64, 1500, 32, BF16, seed=5)
    begin = n_kv - window if window else 0
    mma = kv != F32 and H // KVH <= 8 and D in (64, 128)
    n_splits = splits(ctx.sm_count(), KVH, H, n_kv - begin, mma)
    assert n_splits > 1, "the case must exercise the split-K partials"
    want = run(ctx, "moearc_attn_decode", c, begin)
    first = run(ctx, "moearc_x_attn_decode_static", c, begin)
    run(ctx, "moearc_x_attn_decode_static", other, 0)
    second = run(ctx, "moearc_x_attn_decode_static", c, begin)
    e1, e2 = rel(first, want), rel(second, want)
    print(f"H={H} KVH={KVH} D={D} span={n_kv - begin} splits={n_splits}: rel err {e1:.2e}, {e2:.2e}")
    assert e1 <= TOL and e2 <= TOL


def test_partials_above_the_fixed_size_are_refused(ctx):
    """2048 heads of 128 over 256 KV heads split twice need 2.03 MiB of partials (on 148 SMs):
    the call returns -2 and enqueues nothing. The buffers are full size, so the launch would
    stay in bounds even if the size check were missing."""
    H, KVH, D, n_kv, PT = 2048, 256, 128, 256, 32
    n_splits = splits(ctx.sm_count(), KVH, H, n_kv, True)
    need = H * n_splits * (D + 2) * 4
    if need <= LIMIT:
        pytest.skip(f"this device's split count ({n_splits}) keeps the partials within the limit")
    c = make_case(ctx, H, KVH, D, n_kv, PT, BF16, seed=11)
    sentinel = np.full(H * D, 3.25, np.float32)
    out = ctx.upload_new(sentinel)
    assert call(ctx, "moearc_x_attn_decode_static", c, out, 0) == -2
    ctx.sync()
    assert np.array_equal(ctx.download(out, np.float32, H * D), sentinel)


def test_calls_leave_the_free_device_memory_unchanged(ctx):
    """What the entry point is for: no call takes device memory. After one warm-up call (which
    loads the kernels' code and looks the array's address up), twenty more calls over spans
    that split differently leave the device's free memory exactly where it was; the scratch
    path would have grown its buffer (a cudaMalloc) on its first split call."""
    torch = pytest.importorskip("torch")
    c = make_case(ctx, 64, 8, 64, 6000, 32, BF16, seed=17, sinks=True)
    out = ctx.alloc_n(np.float32, 64 * 64)
    assert call(ctx, "moearc_x_attn_decode_static", c, out, 0) == 0
    ctx.sync()
    free0, _ = torch.cuda.mem_get_info(0)
    for i in range(20):
        assert call(ctx, "moearc_x_attn_decode_static", c, out, (i * 997) % 5000) == 0
    ctx.sync()
    free1, _ = torch.cuda.mem_get_info(0)
    print(f"free device memory before / after 20 calls: {free0} / {free1} bytes")
    assert free1 == free0
