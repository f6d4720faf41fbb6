"""Element-wise tolerance for bf16 results against a float64 oracle.

One bf16 step is 2^-8 of the value (relative 3.9e-3), so a result computed
in float32 and rounded once is within 2^-9 of the oracle.  The bar used by
the GPU tests is the north-star's ``rel <= 2e-2`` PER ELEMENT wherever the
oracle's magnitude is at least ``floor``; below the floor (values that
cancel to near zero, where a relative bound means nothing) the absolute
error must stay under ``rel * floor``.  Tests state their floor: by default
1e-2 of the largest magnitude (a hundredfold below the output scale).
"""
from __future__ import annotations

import numpy as np


def assert_bf16_close(got, want, rel: float = 2e-2, floor: float | None = None, what: str = ""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    if floor is None:
        floor = 1e-2 * float(np.max(np.abs(want))) if want.size else 0.0
    err = np.abs(got - want)
    bound = rel * np.maximum(np.abs(want), floor)
    bad = ~(err <= bound)
    if bad.any():
        i = np.unravel_index(np.argmax(np.where(bad, err / np.maximum(bound, 1e-300), 0)), want.shape)
        raise AssertionError(f"{what}: {int(bad.sum())} of {want.size} elements beyond rel {rel} (floor {floor:.3g}); "
                             f"worst at {i}: got {got[i]!r}, want {want[i]!r}")
