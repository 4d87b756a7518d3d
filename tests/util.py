"""Shared helpers for the tests: seeded inputs and the comparison metrics."""
from __future__ import annotations

import numpy as np

# Tolerances for floating-point outputs:
#   max relative error <= 1e-2, with the denominator max(|ref|, GUARD * rms(ref))
#   so that outputs near zero do not dominate; and cosine similarity >= 0.9999.
MAX_REL = 1e-2
GUARD = 1e-3
MIN_COS = 0.9999
# Attention outputs: the softmax turns a score's rounding (about 1e-5 of a score whose magnitude is
# ~|q||k| = tens, differing between any two summation orders of the same f32 products) into a relative
# change of the weights, so an output that cancels to near zero carries an absolute error of ~1e-5 x
# rms(v) whatever the implementation.  Their denominator floor is 1e-2 x rms (as the long-K GEMMs').
ATTN_GUARD = 1e-2


def rel_err(out, ref, guard: float = GUARD) -> float:
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    den = np.maximum(np.abs(ref), guard * rms)
    den = np.where(den == 0, 1.0, den)
    return float(np.max(np.abs(out - ref) / den)) if ref.size else 0.0


def cosine(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb + 1e-300))


def assert_close(out, ref, what: str = "", max_rel: float = MAX_REL, min_cos: float = MIN_COS,
                 guard: float = GUARD):
    e = rel_err(out, ref, guard)
    c = cosine(out, ref)
    assert e <= max_rel and c >= min_cos, \
        f"{what}: max rel err {e:.3e} (<= {max_rel}, guard {guard} x rms), cos {c:.6f} (>= {min_cos})"


def weights(N: int, K: int, seed: int = 0, std: float = 0.02) -> np.ndarray:
    """The configs' weight generator: W[N, K] ~ N(0, std), drawn first."""
    return (np.random.default_rng(seed).standard_normal((N, K)) * std).astype(np.float32)


def activations(M: int, K: int, seed: int = 1, std: float = 1.0) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal((M, K)) * std).astype(np.float32)
