"""Fit the adaptive fetch selector's critical-density model to comm_test measurements.

The selector (src/comm_man.h:396-405, ``dsp_comm_select``) fetches a tile row by row when
its needed-row density is below

    threshold(k) = 1 / (a * k^u + b / k),   k = min(dims, c)

and whole otherwise. The reference fits (a, b, c, u) per tier with scipy's ``curve_fit``
on this piecewise function from p0 = (1, 1, 100, 1), to the mean over several buffer sizes
of the critical densities its comm_test microbenchmark prints (tools/fit_comm_model.py:
64-116). This module does the same fit on measurements of this engine's fetch paths
(``python -m distspmm_b200.comm_test ... --json out.json``):

    python -m distspmm_b200.fit_comm_model out_400k.json out_1000k.json ...

prints the fitted constants; the B200 preset of ``dsp_comm_model_preset`` holds the
result of one such fit.
"""
from __future__ import annotations

import argparse
import json
import sys

import numpy as np


def piecewise(x, a, b, c, u):
    """threshold(k) for every k in x (floats); constant beyond k = c."""
    x = np.asarray(x, dtype=np.float64)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        kc = np.where(x < c, x, c)
        return 1.0 / (a * kc ** u + b / kc)


def fit(dims, thresholds, p0=(1.0, 1.0, 100.0, 1.0)):
    """(a, b, c, u) by least squares (scipy curve_fit, Levenberg-Marquardt)."""
    from scipy.optimize import curve_fit
    x = np.asarray(dims, dtype=np.float64)
    y = np.asarray(thresholds, dtype=np.float64)

    def f(xx, a, b, c, u):  # np.piecewise form of the reference: branch on x < c
        with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
            return np.piecewise(xx, [xx < c, xx >= c],
                                [lambda v: 1 / (a * v ** u + b / v), lambda v: 1 / (a * c ** u + b / c)])

    params, _ = curve_fit(f, x, y, p0=list(p0), maxfev=10000)
    return tuple(float(p) for p in params)


def mean_thresholds(runs):
    """Average the per-dims critical densities of several comm_test runs (same dims)."""
    dims = runs[0]["dims"]
    for r in runs:
        if r["dims"] != dims:
            raise ValueError("comm_test runs with different dims lists")
    return dims, np.mean([r["threshold"] for r in runs], axis=0)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("runs", nargs="+", help="comm_test --json outputs (one per buffer size)")
    a = ap.parse_args(argv)
    runs = [json.load(open(p)) for p in a.runs]
    dims, y = mean_thresholds(runs)
    pa, pb, pc, pu = fit(dims, y)
    print(f"fit over {len(runs)} run(s), dims {dims}")
    print(f"  a = {pa:.5f}, b = {pb:.5f}, c = {pc:.5f}, u = {pu:.2f}")
    print(f"  preset initialiser: {{{pa:.5f}, {pb:.5f}, {pc:.5f}, {pu:.2f}}}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
