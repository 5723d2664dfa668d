"""Error metrics (after the reference's tests/compare.hpp:86-137, vectorised)."""
from __future__ import annotations

import numpy as np


def compare(ref: np.ndarray, val: np.ndarray) -> dict:
    ref = np.asarray(ref, np.float64)
    val = np.asarray(val, np.float64)
    d = np.abs(val - ref)
    nz = np.abs(ref) > 1e-6
    rel = d[nz] / np.abs(ref[nz]) if nz.any() else np.zeros(1)
    return {
        "max_abs": float(d.max()) if d.size else 0.0,
        "mean_abs": float(d.mean()) if d.size else 0.0,
        "max_rel": float(rel.max()) if rel.size else 0.0,
        "rel_frob": float(np.linalg.norm(val - ref) / max(np.linalg.norm(ref), 1e-300)),
        "nan": int(np.isnan(val).sum()),
        "inf": int(np.isinf(val).sum()),
        "q99_abs": float(np.quantile(d, 0.99)) if d.size else 0.0,
    }


def fp16_ulp(x: np.ndarray) -> np.ndarray:
    """Spacing of binary16 at |x| (subnormal spacing 2^-24 at the bottom)."""
    a = np.abs(np.asarray(x, np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -14)))
    return 2.0 ** (e - 10)


def assert_fp16_close(ref, val, rel_frob=1e-3, abs_floor=1e-2, ulps=1.0, ctx=""):
    """HGEMM / attention gate: rel-Frobenius <= rel_frob and, element-wise,
    |val - ref| <= max(abs_floor, ulps * fp16 ulp(|ref|)) against the fp64 oracle."""
    m = compare(ref, val)
    assert m["nan"] == 0 and m["inf"] == 0, f"{ctx} NaN/Inf in output: {m}"
    assert m["rel_frob"] <= rel_frob, f"{ctx} rel_frob {m['rel_frob']:.3e} > {rel_frob}: {m}"
    tol = np.maximum(abs_floor, ulps * fp16_ulp(ref))
    bad = np.abs(np.asarray(val, np.float64) - ref) > tol
    assert not bad.any(), f"{ctx} {int(bad.sum())} elements beyond max({abs_floor}, {ulps} ulp): {m}"
    return m
