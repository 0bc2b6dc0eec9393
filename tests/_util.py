"""Shared test helpers: the reference's element-wise comparison and metric printing."""
from __future__ import annotations

import numpy as np

import oracle


def compare(actual, expected, atol: float, rtol: float, label: str) -> dict:
    """KernelTests.compare (Tests/AlpacaMetalTests/KernelTests.swift:30-36): every element must satisfy
    |a - e| <= atol + rtol * |e|. Prints the [metrics] line and returns the ErrorMetrics."""
    a = np.asarray(actual, np.float32).reshape(-1)
    e = np.asarray(expected, np.float64).reshape(-1)
    m = oracle.error_metrics(a, e)
    print(f"[metrics] {label}: {oracle.format_metrics(m)}")
    assert np.all(np.isfinite(a)), f"{label}: non-finite output"
    bad = np.abs(a.astype(np.float64) - e) > atol + rtol * np.abs(e)
    if bad.any():
        i = int(np.argmax(bad))
        raise AssertionError(f"{label}[{i}] gpu {a[i]} cpu {e[i]} (atol {atol}, rtol {rtol}); {oracle.format_metrics(m)}")
    return m


def max_abs_check(actual, expected, bound: float, label: str) -> dict:
    a = np.asarray(actual, np.float32).reshape(-1)
    m = oracle.error_metrics(a, np.asarray(expected, np.float64).reshape(-1))
    print(f"[metrics] {label}: {oracle.format_metrics(m)}")
    assert np.all(np.isfinite(a)), f"{label}: non-finite output"
    assert m["maxAbs"] < bound, f"{label}: maxAbs {m['maxAbs']:.3e} >= {bound:.1e}"
    return m
