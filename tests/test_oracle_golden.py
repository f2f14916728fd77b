"""The CPU oracle pinned against outputs of the GPUSparse reference itself.

tests/golden/ holds what the reference produced (its Triton kernels under the CPU
interpreter, its numpy builders and plug-in helpers) on the seeded inputs below; see
tests/golden/make_golden.py.  These tests run without a GPU.
"""
import hashlib
import json
import os

import numpy as np
import pytest
import scipy.sparse as sp

from oracle import oracle as O
from parity import check_topk

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def sha(*arrs):
    h = hashlib.sha256()
    for a in arrs:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode()); h.update(str(a.shape).encode()); h.update(a.tobytes())
    return h.hexdigest()


@pytest.fixture(scope="module")
def gold():
    z = np.load(os.path.join(GOLD, "reference_outputs.npz"))
    meta = json.load(open(os.path.join(GOLD, "reference_meta.json")))
    return z, meta


@pytest.fixture(scope="module")
def corpus_a(gold):
    _, meta = gold
    c = meta["cases"]["A"]
    ip, ix, dt = O.synth_csr(c["N"], c["V"], seed=c["doc_seed"])
    return ip, ix, dt, c


def test_generator_reproduces_golden_inputs(gold, corpus_a):
    z, meta = gold
    ip, ix, dt, c = corpus_a
    assert sha(ip, ix, dt) == c["csr_sha256"]
    qi, qs = O.synth_queries(c["B"], c["V"], seed=c["query_seed"])
    assert sha(qi, qs) == c["queries_sha256"]
    assert np.array_equal(z["A_qi"][:c["B"]], qi)


def test_index_build_matches_reference(gold, corpus_a):
    z, meta = gold
    ip, ix, dt, c = corpus_a
    csr = sp.csr_matrix((dt, ix, ip), shape=(c["N"], c["V"]))
    ref = O.build_index_reference(csr, c["V"])
    fast = O.build_index(ip, ix, dt, c["V"])
    for f, h in c["index_sha256"].items():
        assert sha(getattr(ref, f)) == h, f
        assert sha(getattr(fast, f)) == h, f
    for f, h in c["plugin_index_sha256"].items():
        assert sha(getattr(fast, f)) == h, f


def test_small_index_arrays_match_reference(gold):
    z, meta = gold
    c = meta["cases"]["B"]
    ip, ix, dt = z["B_indptr"], z["B_indices"], z["B_data"]
    got = O.build_index(ip, ix, dt, c["V"])
    for f in ("doc_ids", "scores", "offsets", "lengths", "padded_lengths", "max_scores"):
        assert np.array_equal(getattr(got, f), z[f"B_index_{f}"]), f


@pytest.mark.parametrize("k", [10, 100, 1000])
def test_scores_match_reference_fused(gold, corpus_a, k):
    z, meta = gold
    ip, ix, dt, c = corpus_a
    idx = O.build_index(ip, ix, dt, c["V"])
    qi, qs = z["A_qi"], z["A_qs"]
    S = O.score_dense_f64(ip, ix, dt, c["V"], qi, qs)
    # the reference's own output passes the parity bar against the fp64 exhaustive scores
    rec = check_topk(z[f"A_fused_k{k}_s"], z[f"A_fused_k{k}_i"], S, k)
    assert all(v == 1.0 for v in rec.values())
    # and so does the oracle's canonical-order result
    s, i = O.score_topk(idx, qi, qs, k)
    check_topk(s, i, S, k)
    # identical id sets wherever no near-tie sits at the boundary
    for b in range(qi.shape[0]):
        ref_ids, got_ids = set(z[f"A_fused_k{k}_i"][b]), set(i[b])
        if ref_ids != got_ids:
            kth = np.sort(S[b])[::-1][k - 1]
            diff = np.array(sorted(ref_ids ^ got_ids))
            assert np.all(np.abs(S[b, diff] - kth) <= 1e-5 * abs(kth) + 1e-6), b


@pytest.mark.parametrize("dc", [256, 700])
def test_chunked_paths_and_bounds_match_reference(gold, corpus_a, dc):
    z, meta = gold
    ip, ix, dt, c = corpus_a
    idx = O.build_index(ip, ix, dt, c["V"])
    assert np.array_equal(O.chunk_bounds(idx, dc), z[f"A_bounds_{dc}"])
    S = O.score_dense_f64(ip, ix, dt, c["V"], z["A_qi"], z["A_qs"])
    for name in ("chunked", "cfused"):
        check_topk(z[f"A_{name}_{dc}_s"], z[f"A_{name}_{dc}_i"], S, 100)


def test_k_larger_than_corpus(gold):
    z, meta = gold
    c = meta["cases"]["B"]
    idx = O.build_index(z["B_indptr"], z["B_indices"], z["B_data"], c["V"])
    S = O.score_dense_f64(z["B_indptr"], z["B_indices"], z["B_data"], c["V"], z["B_qi"], z["B_qs"])
    assert z["B_fused_k500_s"].shape == (6, c["N"])           # k = min(k, N)
    check_topk(z["B_fused_k500_s"], z["B_fused_k500_i"], S, 500)
    s, i = O.score_topk(idx, z["B_qi"], z["B_qs"], 500)
    check_topk(s, i, S, 500)


def test_compacted_topk_matches_reference(gold):
    z, _ = gold
    S, tau = z["C_S"], z["C_tau"]
    v, i = O.compacted_topk(S, tau, 50)
    rv, ri = z["C_v"], z["C_i"]
    assert np.array_equal(np.isinf(v), np.isinf(rv))
    fin = ~np.isinf(rv)
    assert np.array_equal(v[fin], rv[fin])                     # same score multiset, in order
    assert np.array_equal(i[~fin], ri[~fin])                   # padding index 0
    for b in range(S.shape[0]):                                # ids agree up to exact ties
        for val in np.unique(rv[b][fin[b]]):
            assert set(i[b][v[b] == val]) <= set(np.nonzero(S[b] == val)[0])


def test_unsorted_lists_raise(gold, corpus_a):
    ip, ix, dt, c = corpus_a
    idx = O.build_index(ip, ix, dt, c["V"])
    t = int(np.argmax(idx.lengths))
    o = idx.offsets[t]
    idx.doc_ids[o], idx.doc_ids[o + 1] = idx.doc_ids[o + 1], idx.doc_ids[o]
    with pytest.raises(ValueError):
        O.chunk_bounds(idx, 512)
