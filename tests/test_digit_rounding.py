"""The Ozaki digit kernels round with the add-and-subtract of 1.5 * 2^(52 - 7s)
(trnblas_b200/csrc/ozaki_split.cuh, `oz_digit_loop` and the digit kernel)
instead of the reference's rint recurrence d = rint(v), v = 128 (v - d)
(trnblas/ozaki.py:123-219). This checks, on the CPU, that the two give the
same digits for every slice count, including exact ties at every digit
level, signed zeros and subnormals: numpy's float64 + and - are the same
IEEE round-to-nearest-even operations as the kernels' __dadd_rn / __dsub_rn.
The GPU tests compare the kernels' digits with the oracle's bit for bit on
real operands; ties deep in the recurrence are what random operands rarely
reach."""

from __future__ import annotations

import numpy as np
import pytest


def rint_digits(v: np.ndarray, slices: int) -> np.ndarray:
    out = []
    for s in range(slices):
        if s:
            v = v * 128.0
        d = np.rint(v)
        if s + 1 < slices:
            v = v - d
        out.append(d.astype(np.int64))
    return np.stack(out)


def add_subtract_digits(u: np.ndarray, slices: int) -> np.ndarray:
    out = []
    for s in range(slices):
        m = np.float64(1.5) * np.float64(2.0) ** (52 - 7 * s)
        t = u + m
        lo = t.view(np.int64) & 0xFFFFFFFF  # the kernel's __double2loint
        out.append(np.where(lo >= 2**31, lo - 2**32, lo))
        u = u - (t - m)
    return np.stack(out)


def _values(rng):
    v = rng.standard_normal(400_000) * np.exp2(rng.integers(-70, 6, 400_000).astype(float))
    parts = [np.clip(v, -63.999, 63.999)]
    for s in range(12):  # exact halves at digit level s
        lim = min(64 * 128**s, 2**52)
        k = rng.integers(-lim, lim, 4000).astype(float)
        parts.append((k + 0.5) / 128.0**s)
    parts.append(np.array([0.0, -0.0, 0.5, -0.5, 1.5, -1.5, 2.5, 63.5, -63.5, 5e-324, -5e-324, 2.0**-1030]))
    v = np.concatenate(parts)
    return v[np.abs(v) < 64]


@pytest.mark.parametrize("slices", [1, 3, 5, 8, 12])
def test_add_subtract_rounding_equals_rint_recurrence(slices):
    v = _values(np.random.default_rng(slices))
    a, b = rint_digits(v.copy(), slices), add_subtract_digits(v.copy(), slices)
    assert np.array_equal(a, b)
    assert np.abs(b).max() <= 64
