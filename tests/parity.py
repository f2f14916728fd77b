"""Parity checks of a top-k result against exact scores (test helper).

The bar: every returned document's score within rtol 1e-5 of its
exact score; recall@10/100/1000 of 1.000 against the exhaustive ranking, where documents
whose exact scores tie within that tolerance at a cutoff are interchangeable; ids
distinct and scores non-increasing.
"""
from __future__ import annotations

import numpy as np

RTOL = 1e-5
ATOL = 1e-6


def exact_order(S_row: np.ndarray) -> np.ndarray:
    n = S_row.shape[0]
    return np.lexsort((np.arange(n), -S_row.astype(np.float64)))


def check_topk(got_s: np.ndarray, got_i: np.ndarray, S: np.ndarray, k: int,
               rtol: float = RTOL, atol: float = ATOL, cutoffs=(10, 100, 1000)) -> dict:
    """Assert parity of (got_s, got_i) [B, k'] with the exact score matrix S [B, N].
    Returns tie-aware recall at each cutoff (all 1.0 when the assertions pass)."""
    B, N = S.shape
    kk = min(k, N)
    assert got_s.shape == (B, kk), (got_s.shape, (B, kk))
    assert got_i.shape == (B, kk), (got_i.shape, (B, kk))
    recalls = {c: [] for c in cutoffs if c <= kk}
    for b in range(B):
        ids, sc = got_i[b].astype(np.int64), got_s[b].astype(np.float64)
        assert np.all((ids >= 0) & (ids < N)), f"row {b}: id out of range"
        assert len(np.unique(ids)) == kk, f"row {b}: duplicate ids"
        ex = S[b, ids].astype(np.float64)
        tol = rtol * np.abs(ex) + atol
        bad = np.abs(sc - ex) > tol
        assert not bad.any(), f"row {b}: score error {np.abs(sc - ex)[bad].max():.3g}"
        assert np.all(np.diff(sc) <= 0), f"row {b}: scores not descending"
        order = exact_order(S[b])
        for c in list(recalls) + [kk]:
            thr = float(S[b, order[c - 1]])
            tthr = rtol * abs(thr) + atol
            top_c = set(ids[:c].tolist())
            must = set(order[:c][S[b, order[:c]].astype(np.float64) > thr + 2 * tthr].tolist())
            missing = must - top_c
            assert not missing, f"row {b}: recall@{c} misses {sorted(missing)[:5]}"
            low = S[b, ids[:c]].astype(np.float64) < thr - 2 * tthr
            assert not low.any(), f"row {b}: a returned doc ranks below the top-{c} boundary"
            if c in recalls:
                exact_set = set(order[:c].tolist())
                tied = set(ids[:c][np.abs(S[b, ids[:c]] - thr) <= 2 * tthr].tolist())
                recalls[c].append(len(top_c & (exact_set | tied)) / c)
    return {c: float(np.mean(v)) if v else 1.0 for c, v in recalls.items()}


def assert_bit_exact(got_s, got_i, ref_s, ref_i):
    assert got_s.shape == ref_s.shape and got_i.shape == ref_i.shape
    assert np.array_equal(got_i, ref_i), \
        f"ids differ in {(got_i != ref_i).sum()} of {got_i.size} entries"
    assert np.array_equal(got_s.view(np.uint32), ref_s.view(np.uint32)), "scores differ bitwise"
