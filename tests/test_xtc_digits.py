"""The E2M1 digit form of an activation (moearc_b200/csrc/xtc.cuh, tc_write_digits), restated in
numpy: each 32-element block is split into 12 E2M1 x E8M0 digits, the first under the scale that
puts the block's largest magnitude in (3, 6], each next under a scale four times smaller; no digit
saturates, every remainder is exact, and the digits sum to the block within 2^-23 of its largest
magnitude. No GPU: this checks the arithmetic the tensor-core decode path relies on."""
import numpy as np

E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def e2m1_exp(amax):
    """X with amax / 2^X in (3, 6], at least -126."""
    if amax <= 0:
        return -126
    m, e = np.frexp(np.float32(amax))  # amax = m 2^e, m in [0.5, 1)
    s, e = 2 * float(m), int(e) - 1     # amax = s 2^e, s in [1, 2)
    return max(-126, e - 2 + (1 if s > 1.5 else 0))


def e2m1_round(v):
    """Nearest E2M1 value, ties to the even code."""
    a = np.abs(v)
    if a < 2:
        q = np.rint(a * 2) / 2
    elif a < 4:
        q = np.rint(a)
    else:
        q = 2 * np.rint(a / 2)
    return np.float32(np.copysign(q, v) if q else 0.0)


def digits(block, n=12):
    r = block.astype(np.float32).copy()
    out = []
    X = e2m1_exp(float(np.max(np.abs(r))))
    for _ in range(n):
        down, up = np.float32(2.0 ** -X), np.float32(2.0 ** X)
        v = (r * down).astype(np.float32)
        assert np.all(np.abs(v) <= 6.0)  # the schedule never saturates
        q = np.array([e2m1_round(x) for x in v], np.float32)
        assert np.all(np.isin(np.abs(q), E2M1))
        d = (q * up).astype(np.float32)
        nr = (r - d).astype(np.float32)
        # the remainder is exact: the digit plus it gives back the value bit for bit
        assert np.array_equal((d.astype(np.float64) + nr.astype(np.float64)), r.astype(np.float64))
        assert float(np.max(np.abs(nr))) <= 2.0 ** X  # at most one E2M1 spacing at the top
        out.append((q, X))
        r = nr
        X = max(-126, X - 2)
    return out, r


def test_digits_sum_to_the_block_within_the_bound():
    rng = np.random.default_rng(0x7C)
    for scale in (1.0, 1e-3, 37.0, 1e6):
        for _ in range(20):
            x = (rng.standard_normal(32) * scale).astype(np.float32)
            x[rng.integers(0, 32, 3)] *= np.float32(1e-4)  # small elements beside large ones
            ds, rem = digits(x)
            total = sum(q.astype(np.float64) * 2.0 ** X for q, X in ds)
            amax = float(np.max(np.abs(x)))
            assert np.max(np.abs(total - x)) <= amax * 2.0 ** -23
            assert np.array_equal(total + rem, x.astype(np.float64))


def test_zero_and_tiny_blocks():
    ds, rem = digits(np.zeros(32, np.float32))
    assert all(not q.any() for q, _ in ds) and not rem.any()
    x = np.full(32, np.float32(1e-30))
    ds, rem = digits(x)
    total = sum(q.astype(np.float64) * 2.0 ** X for q, X in ds)
    assert np.max(np.abs(total - x)) <= 1e-30 * 2.0 ** -23


def test_ties_round_to_the_even_code():
    assert e2m1_round(0.25) == 0.0 and e2m1_round(0.75) == 1.0 and e2m1_round(1.25) == 1.0
    assert e2m1_round(1.75) == 2.0 and e2m1_round(2.5) == 2.0 and e2m1_round(3.5) == 4.0 and e2m1_round(5.0) == 4.0
    assert e2m1_round(-5.5) == -6.0 and e2m1_round(-0.2) == 0.0
