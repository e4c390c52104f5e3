"""Tolerances of the GPU parity tests, in one place, and a record of the errors they saw.

The bounds follow the stated contract: pointwise bit-exact; reductions and norms within
1e-5 relative of an fp64 result; matmul and attention within 1e-4 relative of fp64.

* :func:`elementwise` -- ``|got - ref| <= rel * |ref|`` for every element. Used for the row
  normalisations (RMSNorm, softmax, L2), whose outputs are products and quotients of the input
  (no cancellation), so every element, small or large, is held to the relative bound. An
  optional absolute floor ``rel * floor * max|ref|`` applies only to elements with
  ``|ref| < floor * max|ref|`` (RMSNorm and L2 outputs of inputs at or next to zero).
* :func:`sums` -- ``|got - ref| <= rel * sum|x|`` per output, for sums (the scalar sum and
  mean, row sums). The relative condition number of a sum is ``sum|x| / |sum x|``: an f32
  summation's error scales with ``sum|x|`` whatever the order of the additions, so a bound on
  ``|sum x|`` alone would fail on any row whose terms cancel. Where no cancellation happens
  (``|sum x|`` close to ``sum|x|``) it is the plain relative bound.
* :func:`rowscaled` -- ``|got - ref| <= rel * |ref| + rel * max_row|ref|``, the maximum taken
  over the output's last axis (one matmul row, one attention query row): the normwise bound of
  a contraction, whose entries are sums of products with cancellation (K = 4096 terms). It is
  tighter than scaling by the whole tensor's maximum.

Each check records its largest errors under a label; ``conftest.py`` prints the table at the
end of the run.
"""

from __future__ import annotations

import numpy as np

# label -> {"bound": str, "max_rel_elem": float, "max_err_over_bound": float}
RECORD: dict = {}


def _record(label, bound, got, ref, err, allowed):
    if label is None:
        return
    ref = np.asarray(ref, np.float64)
    with np.errstate(divide="ignore", invalid="ignore"):
        rel_elem = np.where(ref != 0, err / np.abs(ref), np.where(err == 0, 0.0, np.inf))
        ratio = np.where(allowed > 0, err / allowed, np.where(err == 0, 0.0, np.inf))
    prev = RECORD.get(label)
    cur = {"bound": bound, "max_rel_elem": float(np.max(rel_elem)) if rel_elem.size else 0.0,
           "max_err_over_bound": float(np.max(ratio)) if ratio.size else 0.0}
    if prev is not None:
        cur = {"bound": bound, "max_rel_elem": max(prev["max_rel_elem"], cur["max_rel_elem"]),
               "max_err_over_bound": max(prev["max_err_over_bound"],
                                         cur["max_err_over_bound"])}
    RECORD[label] = cur


def _prep(got, ref):
    ref = np.asarray(ref, dtype=np.float64)
    got = np.asarray(got, dtype=np.float64).reshape(ref.shape)
    return got, ref


def elementwise(got, ref, rel, *, floor=None, label=None):
    """(ok, max elementwise relative error): ``|got - ref| <= rel * |ref|`` everywhere, plus
    ``rel * floor * max|ref|`` where ``|ref| < floor * max|ref|`` when ``floor`` is given."""
    got, ref = _prep(got, ref)
    err = np.abs(got - ref)
    allowed = rel * np.abs(ref)
    if floor is not None and ref.size:
        scale = float(np.max(np.abs(ref)))
        small = np.abs(ref) < floor * scale
        allowed = np.where(small, allowed + rel * floor * scale, allowed)
    ok = bool(np.all(err <= allowed)) and bool(np.all(np.isfinite(got)))
    _record(label, f"elementwise {rel:g}" + (f" (floor {floor:g} of max)" if floor else ""),
            got, ref, err, allowed)
    with np.errstate(divide="ignore", invalid="ignore"):
        worst = float(np.max(np.where(ref != 0, err / np.abs(ref), err))) if ref.size else 0.0
    return ok, worst


def sums(got, ref, abs_sum, rel, *, label=None):
    """(ok, max error / sum|x|): ``|got - ref| <= rel * abs_sum`` with ``abs_sum`` the fp64
    sum of the absolute terms for each output (same shape as ``ref``)."""
    got, ref = _prep(got, ref)
    abs_sum = np.asarray(abs_sum, np.float64).reshape(ref.shape)
    err = np.abs(got - ref)
    allowed = rel * abs_sum
    ok = bool(np.all(err <= allowed)) and bool(np.all(np.isfinite(got)))
    _record(label, f"{rel:g} * sum|x|", got, ref, err, allowed)
    with np.errstate(divide="ignore", invalid="ignore"):
        worst = float(np.max(np.where(abs_sum > 0, err / abs_sum, err))) if ref.size else 0.0
    return ok, worst


def rowscaled(got, ref, rel, *, label=None):
    """(ok, max error / row max): ``|got - ref| <= rel * |ref| + rel * max_row|ref|``."""
    got, ref = _prep(got, ref)
    err = np.abs(got - ref)
    rowmax = np.max(np.abs(ref), axis=-1, keepdims=True) if ref.ndim else np.abs(ref)
    allowed = rel * np.abs(ref) + rel * rowmax
    ok = bool(np.all(err <= allowed)) and bool(np.all(np.isfinite(got)))
    _record(label, f"{rel:g} * (|ref| + row max|ref|)", got, ref, err, allowed)
    with np.errstate(divide="ignore", invalid="ignore"):
        worst = float(np.max(np.where(rowmax > 0, err / rowmax, err))) if ref.size else 0.0
    return ok, worst


def report_lines():
    if not RECORD:
        return []
    w = max(len(k) for k in RECORD)
    lines = [f"{'check'.ljust(w)}  {'bound':<34} {'max rel (elem)':>14} {'max err/bound':>13}"]
    for k in sorted(RECORD):
        r = RECORD[k]
        lines.append(f"{k.ljust(w)}  {r['bound']:<34} {r['max_rel_elem']:>14.3e} "
                     f"{r['max_err_over_bound']:>13.3e}")
    return lines
