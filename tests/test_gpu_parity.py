"""Scoring parity of the CUDA path against the CPU oracle.

fp32 mode is bit-exact against the oracle's canonical summation order (scores and ids);
bf16 / u8 modes are bit-exact against the oracle fed the dequantised weights; every
result also passes the tolerance / tie-aware recall bar against fp64 exhaustive scores
and against the reference's own golden outputs."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from parity import assert_bit_exact, check_topk

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = torch.device("cuda:0")
V = 30522


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def hd(g):
    """The GPU index's head terms: the oracle sums them first, as the scorer does."""
    return g.head_ids.cpu().numpy()


@pytest.fixture(scope="module")
def corpus():
    ip, ix, dt = O.synth_csr(20000, V, seed=0)
    return ip, ix, dt, O.build_index(ip, ix, dt, V)


@pytest.fixture(scope="module")
def gindex(corpus):
    import gpusparse
    ip, ix, dt, _ = corpus
    return gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV)


@pytest.mark.parametrize("k", [1, 10, 100, 1000, 5000])
def test_fp32_bit_exact(corpus, gindex, k):
    import gpusparse
    _, _, _, oidx = corpus
    qi, qs = O.synth_queries(96, V, seed=1)
    s, i = gpusparse.triton_fused_score(gindex, t(qi), t(qs), top_k=k)
    rs, ri = O.score_topk(oidx, qi, qs, k, head=hd(gindex))
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)


def test_tolerance_and_recall_vs_fp64(corpus, gindex):
    import gpusparse
    ip, ix, dt, _ = corpus
    qi, qs = O.synth_queries(24, V, seed=4)
    S = O.score_dense_f64(ip, ix, dt, V, qi, qs)
    s, i = gpusparse.triton_fused_score(gindex, t(qi), t(qs), top_k=1000)
    rec = check_topk(s.cpu().numpy(), i.cpu().numpy(), S, 1000)
    assert rec == {10: 1.0, 100: 1.0, 1000: 1.0}


def test_deterministic_run_to_run(gindex):
    import gpusparse
    qi, qs = O.synth_queries(200, V, seed=5)
    a = gpusparse.triton_fused_score(gindex, t(qi), t(qs), top_k=1000)
    b = gpusparse.triton_fused_score(gindex, t(qi), t(qs), top_k=1000)
    assert torch.equal(a[1], b[1]) and torch.equal(a[0].view(torch.int32), b[0].view(torch.int32))


def test_edge_queries(corpus, gindex):
    import gpusparse
    _, _, _, oidx = corpus
    W = 8
    qi = np.full((6, W), -1, dtype=np.int32)
    qs = np.zeros((6, W), dtype=np.float32)
    qi[0, :4] = [3, V + 5, 7, 2 * V]; qs[0, :4] = [0.5, 9.0, 1.25, 3.0]     # ids >= V skipped
    qi[1, :3] = [11, 11, 0]; qs[1, :3] = [0.75, 0.25, 0.125]                # duplicated term
    # row 2: all padding -> every score 0, ties by ascending doc id
    qi[3, :1] = [1]; qs[3, :1] = [2.0]                                     # one term
    qi[4, :] = np.arange(W); qs[4, :] = -1.0                               # negative weights
    qi[5, :2] = [29_000, 30_000]; qs[5, :2] = [1.0, 1.0]                   # rare terms
    for k in (10, 1000):
        s, i = gpusparse.triton_fused_score(gindex, t(qi), t(qs), top_k=k)
        rs, ri = O.score_topk(oidx, qi, qs, k, head=hd(gindex))
        assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)
    assert np.array_equal(i.cpu().numpy()[2], np.arange(1000))


def test_int64_query_ids_are_accepted(corpus, gindex):
    import gpusparse
    _, _, _, oidx = corpus
    qi, qs = O.synth_queries(8, V, seed=6)
    qi64 = qi.astype(np.int64)
    qi64[0, -1] = 2 ** 40                      # out of range, must be skipped not wrapped
    s, i = gpusparse.triton_fused_score(gindex, t(qi64), t(qs), top_k=50)
    qi[0, -1] = -1
    rs, ri = O.score_topk(oidx, qi, qs, 50, head=hd(gindex))
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)


@pytest.mark.parametrize("N,k", [(1, 5), (7, 1000), (33, 32), (4097, 1000), (100, 100)])
def test_small_corpora_k_at_least_n(N, k):
    import gpusparse
    ip, ix, dt = O.synth_csr(N, V, seed=N)
    oidx = O.build_index(ip, ix, dt, V)
    g = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV)
    qi, qs = O.synth_queries(40, V, seed=2)
    s, i = gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=k)
    rs, ri = O.score_topk(oidx, qi, qs, k, head=hd(g))
    assert s.shape == (40, min(k, N))
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)


@pytest.mark.parametrize("B", [1, 3, 31, 33, 257])
def test_batch_sizes(corpus, gindex, B):
    import gpusparse
    _, _, _, oidx = corpus
    qi, qs = O.synth_queries(B, V, seed=10 + B)
    s, i = gpusparse.triton_fused_score(gindex, t(qi), t(qs), top_k=100)
    rs, ri = O.score_topk(oidx, qi, qs, 100, head=hd(gindex))
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)


def test_wide_queries():
    """W beyond the synthetic maximum (fewer queries per warp slot)."""
    import gpusparse
    ip, ix, dt = O.synth_csr(5000, V, seed=3)
    oidx = O.build_index(ip, ix, dt, V)
    g = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV)
    rng = np.random.default_rng(0)
    qi = rng.integers(0, 2000, size=(10, 700)).astype(np.int32)
    qs = rng.random((10, 700)).astype(np.float32)
    s, i = gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=300)
    rs, ri = O.score_topk(oidx, qi, qs, 300, head=hd(g))
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)


@pytest.mark.parametrize("wd", ["bf16", "u8"])
def test_quantised_modes_bit_exact_vs_dequantised_oracle(corpus, wd):
    import gpusparse
    ip, ix, dt, oidx = corpus
    g = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV, weight_dtype=wd,
                                         keep_fp32=False)
    assert g.scores is None
    w = gpusparse.dequantized_weights(g).cpu().numpy()
    qi, qs = O.synth_queries(64, V, seed=8)
    s, i = gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=1000)
    rs, ri = O.score_topk(oidx, qi, qs, 1000, weights=w, head=hd(g))
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)


def test_reference_golden_outputs():
    """Against what the reference itself returned (tolerance + tie-aware)."""
    import gpusparse
    z = np.load(os.path.join(GOLD, "reference_outputs.npz"))
    c = json.load(open(os.path.join(GOLD, "reference_meta.json")))["cases"]["A"]
    ip, ix, dt = O.synth_csr(c["N"], c["V"], seed=c["doc_seed"])
    g = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), c["V"], DEV)
    qi, qs = z["A_qi"], z["A_qs"]
    S = O.score_dense_f64(ip, ix, dt, c["V"], qi, qs)
    for k in (10, 100, 1000):
        s, i = gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=k)
        s, i = s.cpu().numpy(), i.cpu().numpy()
        check_topk(s, i, S, k)
        rs = z[f"A_fused_k{k}_s"]
        assert np.allclose(s, rs, rtol=1e-5, atol=1e-6)        # same score sequence
    for dc in (256, 700):
        for fn, key in ((gpusparse.triton_chunked_score, "chunked"),
                        (gpusparse.triton_chunked_score_fused, "cfused")):
            s, i = fn(g, t(qi), t(qs), top_k=100, doc_chunk=dc)
            check_topk(s.cpu().numpy(), i.cpu().numpy(), S, 100)
            assert np.allclose(s.cpu().numpy(), z[f"A_{key}_{dc}_s"], rtol=1e-5, atol=1e-6)


def test_shards_merge_equals_unsharded(corpus):
    """The multi-GPU data flow emulated on one GPU: doc-range shards scored separately
    (local ids + doc_base), packed keys merged by the GPU merge kernel."""
    import gpusparse
    from gpusparse.distributed import ShardLayout
    ip, ix, dt, oidx = corpus
    N = len(ip) - 1
    qi, qs = O.synth_queries(50, V, seed=9)
    k = 1000
    full = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV)
    head = hd(full)        # one head set for every shard: the same summation order
    for world in (2, 3, 8):
        keys = []
        for r in range(world):
            lay = ShardLayout(N, world, r)
            sip = ip[lay.lo:lay.hi + 1] - ip[lay.lo]
            g = gpusparse.build_from_csr_tensors(t(sip), t(ix[ip[lay.lo]:ip[lay.hi]]),
                                                 t(dt[ip[lay.lo]:ip[lay.hi]]), V, DEV, doc_base=lay.lo,
                                                 head_ids=head)
            _, _, kk = gpusparse.score_topk(g, t(qi), t(qs), k, with_keys=True)
            keys.append(kk)
        allk = torch.stack(keys)
        s, i = gpusparse.merge_topk(allk, ShardLayout(N, world, 0).list_counts(k), k)
        rs, ri = O.score_topk(oidx, qi, qs, k, head=head)
        assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)


@pytest.mark.parametrize("k", [8192, 8193, 12000, 20000])
def test_large_k_is_exact(corpus, gindex, k):
    """top_k at and above the 8192 keys one CTA sorts in shared memory (the reference's
    torch.topk takes any k): above it every key is written out and each query's top-k is
    radix-selected and merge-sorted in global memory; k = 20000 is the whole corpus."""
    import gpusparse
    _, _, _, oidx = corpus
    qi, qs = O.synth_queries(12, V, seed=50)
    s, i = gpusparse.triton_fused_score(gindex, t(qi), t(qs), top_k=k)
    rs, ri = O.score_topk(oidx, qi, qs, k, head=hd(gindex))
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)


def test_large_k_through_the_shard_merge_and_compacted_topk(corpus):
    """k above 8192 in the other two selections: merging doc-range shards' keys
    (gsp_merge_topk) and compacted_topk over a dense score matrix."""
    import gpusparse
    from gpusparse.distributed import ShardLayout
    ip, ix, dt, oidx = corpus
    N, k = 20000, 9000
    qi, qs = O.synth_queries(6, V, seed=52)
    g0 = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV)
    head = g0.head_ids.cpu().numpy()
    keys = []
    for r in range(2):
        lay = ShardLayout(N, 2, r)
        g = gpusparse.build_from_csr_tensors(t(ip[lay.lo:lay.hi + 1] - ip[lay.lo]),
                                             t(ix[ip[lay.lo]:ip[lay.hi]]), t(dt[ip[lay.lo]:ip[lay.hi]]),
                                             V, DEV, doc_base=lay.lo, head_ids=head)
        keys.append(gpusparse.score_topk(g, t(qi), t(qs), k, with_keys=True)[2])
    s, i = gpusparse.merge_topk(torch.stack(keys), ShardLayout(N, 2, 0).list_counts(k), k)
    rs, ri = O.score_topk(oidx, qi, qs, k, head=head)
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)
    S = O.score_full(oidx, qi, qs, head=head)
    tau = np.full(6, -np.inf, dtype=np.float32)
    tau[1] = np.float32(np.sort(S[1])[-8500])   # fewer than k survive: padded with (-inf, 0)
    v, c = gpusparse.compacted_topk(t(S), t(tau), k)
    ov, oc = O.compacted_topk(S, tau, k)
    assert np.array_equal(v.cpu().numpy(), ov) and np.array_equal(c.cpu().numpy(), oc)


def test_wide_queries(corpus, gindex):
    """W = 16384 scored slots (the most one query plan sorts) stays exact; a batch padded
    wider than that is compacted to its longest query first (same result); a query with
    more than 16384 scored terms is refused."""
    import gpusparse
    _, _, _, oidx = corpus
    rng = np.random.default_rng(51)
    wi = rng.integers(0, V, size=(3, 16384)).astype(np.int32)
    ws = rng.random((3, 16384)).astype(np.float32)
    s, i = gpusparse.triton_fused_score(gindex, t(wi), t(ws), top_k=100)
    rs, ri = O.score_topk(oidx, wi, ws, 100, head=hd(gindex))
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)
    qi, qs = O.synth_queries(5, V, seed=53)
    pi = np.full((5, 20000), -1, dtype=np.int32)
    ps = np.zeros((5, 20000), dtype=np.float32)
    for b in range(5):   # the query's slots spread over the wide row, padding between them
        cols = np.sort(rng.choice(20000, size=qi.shape[1], replace=False))
        pi[b, cols], ps[b, cols] = qi[b], qs[b]
    s, i = gpusparse.triton_fused_score(gindex, t(pi), t(ps), top_k=1000)
    rs, ri = O.score_topk(oidx, qi, qs, 1000, head=hd(gindex))
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)
    with pytest.raises(RuntimeError):
        gpusparse.triton_fused_score(gindex, t(np.zeros((2, 16385), np.int32)),
                                     t(np.ones((2, 16385), np.float32)), top_k=10)


@pytest.mark.parametrize("N", [1, 4097, 20000])
def test_small_batch_merge_tree_matches_oracle(N):
    """Small batches with k' >= 256 take the per-tile top-k lists and the merge tree; the
    result is bit-exact against the oracle and equal to the shared-buffer path (forced by
    a tree limit of 0)."""
    import gpusparse
    import gpusparse._lib as L
    lib = L.lib()
    ip, ix, dt = O.synth_csr(N, V, seed=N + 3)
    oidx = O.build_index(ip, ix, dt, V)
    g = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV)
    default = lib.gsp_get_tree_limit()
    try:
        for B, k in [(1, 256), (3, 1000), (2, 1024), (6, 300)]:
            qi, qs = O.synth_queries(B, V, seed=B * 7 + N)
            s1, i1 = gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=k)
            rs, ri = O.score_topk(oidx, qi, qs, k, head=hd(g))
            assert_bit_exact(s1.cpu().numpy(), i1.cpu().numpy(), rs, ri)
            L.check(lib.gsp_set_tree_limit(0), "tree limit")
            s0, i0 = gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=k)
            L.check(lib.gsp_set_tree_limit(default), "tree limit")
            assert torch.equal(i1, i0) and torch.equal(s1.view(torch.int32), s0.view(torch.int32))
    finally:
        lib.gsp_set_tree_limit(default)


def test_empty_corpus_builds_and_scores_to_nothing():
    """A CSR with no rows builds an index with no postings; scoring it returns [B, 0]."""
    import gpusparse
    ip = np.zeros(1, dtype=np.int64)
    ix = np.zeros(0, dtype=np.int32)
    dt = np.zeros(0, dtype=np.float32)
    g = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV)
    assert g.num_docs == 0 and int(g.lengths.sum()) == 0
    qi, qs = O.synth_queries(4, V, seed=9)
    s, i = gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=10)
    assert s.shape == (4, 0) and i.shape == (4, 0)
