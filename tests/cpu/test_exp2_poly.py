"""The FMA-pipe exp2 of the tcgen05 attention softmax (``ex2_fma`` in ``ops/csrc/exp2_fma.cuh``),
emulated step by step in float32: round-down add against 1.5 * 2^23 for the floor, a degree-3
polynomial for 2^f, the integer added to the exponent field.  Its relative error against exact
2^x stays below the minimax bound of the fit (8.6e-5), far below the 2^-9 half-ulp of the bf16
probabilities it produces, over the whole input range the softmax uses (scores minus a running
max that may lag by up to 2^8)."""

import numpy as np

C1, C2, C3 = np.float32(0.6951168179512024), np.float32(0.22764486074447632), np.float32(0.07706713676452637)
SHIFT = np.float32(12582912.0)


def _add_round_down(x: np.ndarray, y: np.float32) -> np.ndarray:
    """float32 x + y rounded toward -inf (the kernel's add.rm.f32), exact via float64."""
    exact = x.astype(np.float64) + np.float64(y)
    near = exact.astype(np.float32)
    return np.where(near.astype(np.float64) > exact, np.nextafter(near, np.float32(-np.inf)), near)


def ex2_fma(x: np.ndarray) -> np.ndarray:
    x = np.maximum(x.astype(np.float32), np.float32(-127.0))
    j = _add_round_down(x, SHIFT)
    f = (x - (j - SHIFT)).astype(np.float32)
    poly = np.float32(1.0) + f * (C1 + f * (C2 + f * C3))  # float32 Horner (fused in the kernel)
    n = j.view(np.int32) - SHIFT.view(np.int32)
    return (poly.astype(np.float32).view(np.int32) + (n << 23)).view(np.float32)


def test_floor_and_fraction_are_exact():
    x = np.linspace(-126.0, 8.0, 200001, dtype=np.float32)
    j = _add_round_down(np.maximum(x, np.float32(-127)), SHIFT)
    n = j.view(np.int32) - SHIFT.view(np.int32)
    assert np.array_equal(n, np.floor(x).astype(np.int32))
    f = x - (j - SHIFT)
    assert np.all((f >= 0) & (f < 1))


def test_relative_error_below_the_minimax_bound():
    rng = np.random.default_rng(0)
    x = np.concatenate([np.linspace(-125.0, 8.0, 400001), rng.uniform(-30, 8, 200000),
                        np.arange(-125, 9, dtype=np.float64)]).astype(np.float32)
    got = ex2_fma(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got - want) / want
    assert rel.max() < 9e-5, rel.max()
    assert rel.max() < 2.0 ** -9 / 20


def test_masked_scores_give_exact_zero():
    x = np.array([-np.inf, -127.0, -1e30], dtype=np.float32)
    assert np.array_equal(ex2_fma(x), np.zeros(3, dtype=np.float32))


def test_step_at_integer_boundaries_within_the_bound():
    """The fit has p(0) = 1 and p(1) = 1.99983: the step at each integer stays within the bound."""
    for n in range(-20, 8):
        below = ex2_fma(np.array([np.nextafter(np.float32(n), np.float32(-np.inf))], dtype=np.float32))[0]
        at = ex2_fma(np.array([n], dtype=np.float32))[0]
        assert abs(float(at) - float(below)) / float(at) < 1e-4
