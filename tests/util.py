"""Shared helpers for the tests: fixture loading and parity checks."""

import os

import numpy as np

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
LAYER_KEYS = oracle.LAYER_KEYS
SHARED_KEYS = oracle.SHARED_KEYS

# north_star tolerance for layer outputs (fp32 accumulation): max-abs <= 1e-3 * ||out||_inf
OUT_TOL = 1e-3


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


def oracle_layer(w: dict) -> oracle.LayerWeights:
    return oracle.layer_from_dict(w)


def rel_err(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


def assert_close(got, want, tol=OUT_TOL, what="out"):
    e = rel_err(got, want)
    assert e <= tol, f"{what}: max|diff|/||want||_inf = {e:.3e} > {tol:.1e}"
    return e
