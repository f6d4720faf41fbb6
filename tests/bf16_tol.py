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


def rms_floor(want, k: float = 0.5) -> float:
    """The floor for a perturbed op's bf16 output: `k` times the RMS of the
    oracle's output.  Its low-rank term passes through bf16 operands (u =
    bf16(s x A), the noise s n) whose rounding errs by ~2^-9 of the TERMS'
    size, not of each output element's, so an element that cancels to near
    zero keeps an absolute error of that order: ~1e-3 of the RMS typically,
    ~5e-3 at the extremes of a large output, inside rel * floor = 1e-2 RMS."""
    want = np.asarray(want, np.float64)
    return k * float(np.sqrt(np.mean(want * want))) if want.size else 0.0


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


def assert_perturbation_close(got, want, base, rel: float = 0.05, what: str = ""):
    """The perturbation itself, not only the dominant unperturbed term: the
    deltas got - base and want - base (base = the unperturbed output, float64)
    agree within `rel` of the largest delta plus one bf16 step (2^-8) of the
    output scale, the rounding of the output itself."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    base = np.asarray(base, np.float64)
    d_got, d_want = got - base, want - base
    bound = rel * float(np.max(np.abs(d_want))) + 2.0 ** -8 * float(np.max(np.abs(want)))
    err = float(np.max(np.abs(d_got - d_want))) if want.size else 0.0
    assert err <= bound, f"{what}: perturbation off by {err:.3g} > {bound:.3g}"
