"""Shared test helpers: the reference's LCG, seeded normals, tolerance checks,
ulp statistics and the golden known-answer loader."""

from __future__ import annotations

import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                      "reference_known_answers.json")

# Tolerances, in the reference's form |a - r| <= atol + rtol * |r|
# (docs/agents/specs/docs/05_TESTING_BENCHMARKS.md section 1), with atol
# scaled by the tensor's largest magnitude.
F32_RTOL = 1e-5
F32_ATOL_REL = 1e-6
F64_RTOL = 1e-12
F64_ATOL_REL = 1e-14
GELU_MAX_ULP = 4


def golden_case(name: str) -> dict:
    with open(GOLDEN, encoding="utf-8") as fh:
        doc = json.load(fh)
    for case in doc["cases"]:
        if case["name"] == name:
            return case
    raise KeyError(name)


def decode_value(v, dtype=np.float32):
    specials = {"-0.0": -0.0, "inf": np.inf, "-inf": -np.inf, "nan": np.nan,
                "f32::MAX": float(np.finfo(np.float32).max),
                "-f32::MAX": -float(np.finfo(np.float32).max)}
    if isinstance(v, str):
        return dtype(specials[v])
    return dtype(v)


def golden_tensor(case: dict, name: str) -> np.ndarray:
    t = case["tensors"][name]
    dtype = np.float32 if t["dtype"] == "f32" else np.float64
    return np.array([decode_value(v, dtype) for v in t["data"]], dtype=dtype)


def lcg_f32(state: int, n: int) -> tuple[np.ndarray, int]:
    """The reference tests' LCG (crates/tenferro-ext/src/layernorm.rs:313-316,
    crates/cpu-kernels/src/lib.rs lcg): state = state*6364136223846793005 + 1,
    value = (state >> 40) as f32 / 2^24 - 0.5, in f32 arithmetic."""
    out = np.empty(n, dtype=np.float32)
    m = (1 << 64) - 1
    for i in range(n):
        state = (state * 6364136223846793005 + 1) & m
        out[i] = np.float32(state >> 40) / np.float32(1 << 24) - np.float32(0.5)
    return out, state


def splitmix_normal(n: int, seed: int, mean: float = 0.0, std: float = 1.0,
                    dtype=np.float32) -> np.ndarray:
    """Seeded normals: SplitMix64 stream -> two 53-bit uniforms -> Box-Muller."""
    m = np.uint64(0xFFFFFFFFFFFFFFFF)
    pairs = (n + 1) // 2
    idx = np.arange(1, 2 * pairs + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = (np.uint64(seed) + idx * np.uint64(0x9E3779B97F4A7C15)) & m
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    u = ((z >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740992.0)
    u1, u2 = u[0::2], u[1::2]
    r = np.sqrt(-2.0 * np.log(u1))
    out = np.empty(2 * pairs, dtype=np.float64)
    out[0::2] = r * np.cos(2.0 * np.pi * u2)
    out[1::2] = r * np.sin(2.0 * np.pi * u2)
    return (mean + std * out[:n]).astype(dtype)


def splitmix_uniform(n: int, seed: int, lo: float, hi: float, dtype=np.float32) -> np.ndarray:
    m = np.uint64(0xFFFFFFFFFFFFFFFF)
    idx = np.arange(1, n + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = (np.uint64(seed) + idx * np.uint64(0x9E3779B97F4A7C15)) & m
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    u = (z >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    return (lo + (hi - lo) * u).astype(dtype)


def ulp_distance_f32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """|ulp distance| between float32 arrays (NaN==NaN counts as 0, NaN vs
    number as a huge distance)."""
    a = np.ascontiguousarray(a, dtype=np.float32).ravel().view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, dtype=np.float32).ravel().view(np.int32).astype(np.int64)
    # map sign-magnitude to a monotone integer line
    a = np.where(a < 0, -(a & 0x7FFFFFFF), a)
    b = np.where(b < 0, -(b & 0x7FFFFFFF), b)
    return np.abs(a - b)


def close_stats(actual: np.ndarray, expected: np.ndarray) -> dict:
    a = np.asarray(actual, dtype=np.float64).ravel()
    r = np.asarray(expected, dtype=np.float64).ravel()
    finite = np.isfinite(r)
    diff = np.abs(a - r)
    with np.errstate(divide="ignore", invalid="ignore"):
        rel = np.where(np.abs(r) > 0, diff / np.abs(r), diff)
    stats = {
        "max_abs": float(diff[finite].max()) if finite.any() else 0.0,
        "max_rel": float(rel[finite & (np.abs(r) > 1e-30)].max())
        if (finite & (np.abs(r) > 1e-30)).any() else 0.0,
    }
    if np.asarray(actual).dtype == np.float32:
        ulp = ulp_distance_f32(actual, expected)
        stats["max_ulp"] = int(ulp[finite].max()) if finite.any() else 0
        stats["exact_frac"] = float((ulp[finite] == 0).mean()) if finite.any() else 1.0
    return stats


def assert_close(actual, expected, rtol: float, atol_rel: float, what: str = "") -> dict:
    a = np.asarray(actual)
    r = np.asarray(expected)
    assert a.shape == r.shape, (what, a.shape, r.shape)
    an, rn = np.isnan(a), np.isnan(r)
    assert np.array_equal(an, rn), f"{what}: NaN pattern differs ({an.sum()} vs {rn.sum()})"
    ai, ri = np.isinf(a), np.isinf(r)
    assert np.array_equal(ai, ri) and np.array_equal(a[ai], r[ri]), f"{what}: inf pattern differs"
    fin = np.isfinite(r)
    if fin.any():
        scale = float(np.max(np.abs(r[fin].astype(np.float64))))
        atol = atol_rel * scale
        diff = np.abs(a[fin].astype(np.float64) - r[fin].astype(np.float64))
        bound = atol + rtol * np.abs(r[fin].astype(np.float64))
        bad = diff > bound
        if bad.any():
            i = int(np.argmax(diff - bound))
            raise AssertionError(
                f"{what}: {int(bad.sum())} of {diff.size} elements out of tolerance "
                f"(rtol={rtol}, atol={atol:.3g}); worst actual={a[fin][i]!r} "
                f"expected={r[fin][i]!r} diff={diff[i]:.3g}")
    return close_stats(a, r)


def assert_bitwise(actual, expected, what: str = "") -> None:
    a = np.ascontiguousarray(actual)
    r = np.ascontiguousarray(expected)
    assert a.shape == r.shape and a.dtype == r.dtype, (what, a.shape, r.shape, a.dtype, r.dtype)
    if a.size == 0:
        return
    both_nan = np.isnan(a) & np.isnan(r)
    same = (a.view(np.uint8).reshape(a.size, -1) == r.view(np.uint8).reshape(r.size, -1)).all(1)
    bad = ~(same | both_nan.ravel())
    if bad.any():
        i = int(np.flatnonzero(bad)[0])
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {a.size} elements differ bitwise; first at {i}: "
            f"actual={a.ravel()[i]!r} expected={r.ravel()[i]!r}")
