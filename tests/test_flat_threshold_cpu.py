"""The gather threshold of the sampled exact flat search, restated on the host.

`chunk_threshold_kernel` (vicinity_b200/csrc/tc_select.cu) turns the binary16
chunk maxima of a sample of the columns into a per-query threshold slo; the
gather pass keeps the columns whose f32 tensor-core product s reaches slo, and
the finisher needs every column whose approximate distance fl(1 - s) lies
within 2 eps of the query's k-th smallest one (the exact top-k of
distance.rs:125-130 are among those).  This checks that rule on product rows
built to stress it: ties, values on binary16 rounding boundaries, negative and
subnormal-range products, and error bounds from zero to large.
"""
from __future__ import annotations

import numpy as np
import pytest

U20 = 2.0 ** -20


def f32_round_down(x: float) -> np.float32:
    y = np.float32(x)
    if float(y) > x:
        y = np.nextafter(y, np.float32(-np.inf))
    return y


def threshold(chunk_max_f16: np.ndarray, P: int, eps: float) -> np.float32:
    """The kernel's rule: m_P, the P-th largest maximum, bounds the P-th
    product from below after one binary16 rounding."""
    m = np.sort(chunk_max_f16.astype(np.float64)[np.isfinite(chunk_max_f16)])[::-1]
    if m.size < P or not eps < 1.0 or not abs(m[P - 1]) < 65536.0:
        return np.float32(-np.inf)
    mp = m[P - 1]
    S = mp - abs(mp) / 2048.0 - 2.0 ** -25
    return f32_round_down(S - 2.0 * eps - U20 * (1.0 + abs(1.0 - S) + 2.0 * eps))


def needed(s: np.ndarray, P: int, eps: float) -> np.ndarray:
    """Columns the finisher may need: fl(1 - s) within 2 eps of the P-th
    smallest, the limit rounded up as the finisher does."""
    a = (np.float32(1.0) - s).astype(np.float32)
    ap = np.sort(a)[P - 1]
    limit = np.float32(float(ap) + 2.0 * eps)
    if float(limit) < float(ap) + 2.0 * eps:
        limit = np.nextafter(limit, np.float32(np.inf))
    return a <= limit


def chunk_maxima(s: np.ndarray, stride_tiles: int) -> np.ndarray:
    """Binary16 maxima of the 32-column chunks of every stride-th 128-column tile."""
    tiles = s.size // 128
    keep = [t for t in range(0, tiles, stride_tiles)]
    cols = np.concatenate([np.arange(t * 128, t * 128 + 128) for t in keep])
    return s[cols].reshape(-1, 32).max(axis=1).astype(np.float16)


def rows(seed: int):
    g = np.random.default_rng(seed)
    n = 128 * 64
    yield (g.standard_normal(n) * 0.1).astype(np.float32)                 # unit-vector products
    s = (g.standard_normal(n) * 0.1).astype(np.float32)
    s[g.integers(0, n, 400)] = np.float32(0.3)                           # many ties at the top
    yield s
    edge = np.float32(0.5) - np.float32(2.0 ** -13) * np.arange(1, 8, dtype=np.float32)
    s = (g.standard_normal(n) * 0.05).astype(np.float32)
    s[g.integers(0, n, 300)] = g.choice(edge, 300)                       # just below a binade: rounds up to 0.5
    yield s
    yield (-np.abs(g.standard_normal(n)) * 3.0).astype(np.float32)        # every product negative
    yield (g.standard_normal(n) * 1e-6).astype(np.float32)                # binary16 subnormal range
    yield (g.standard_normal(n) * 40.0).astype(np.float32)                # long rows


@pytest.mark.parametrize("seed", [0, 1, 2])
@pytest.mark.parametrize("P", [1, 10, 100, 256])
@pytest.mark.parametrize("eps", [0.0, 1e-7, 1.1e-3, 0.05])
def test_threshold_keeps_every_needed_column(seed, P, eps):
    for s in rows(seed):
        slo = threshold(chunk_maxima(s, 4), P, eps)
        need = needed(s, P, eps)
        missed = np.nonzero(need & ~(s >= slo))[0]
        assert missed.size == 0, f"P={P} eps={eps}: column {missed[0]} s={s[missed[0]]!r} below slo={slo!r}"


def test_too_few_maxima_or_useless_bound_gathers_everything():
    s = (np.random.default_rng(3).standard_normal(128 * 4) * 0.1).astype(np.float32)
    cm = chunk_maxima(s, 4)  # one tile: 4 maxima
    assert threshold(cm, 5, 1e-3) == -np.inf
    assert threshold(cm, 4, 1.0) == -np.inf
    assert np.isfinite(threshold(cm, 4, 1e-3))
