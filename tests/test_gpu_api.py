"""Reference API semantics on the GPU: compacted_topk, chunked entry points, the plug-in
and index objects built field by field as the reference's plug-in builds them."""
import json
import os
import sys
import types

import numpy as np
import pytest
import torch

from oracle import oracle as O
from parity import assert_bit_exact, check_topk

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = torch.device("cuda:0")


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def test_compacted_topk_matches_reference_and_oracle():
    import gpusparse
    z = np.load(os.path.join(GOLD, "reference_outputs.npz"))
    S, tau = z["C_S"], z["C_tau"]
    v, i = gpusparse.compacted_topk(t(S), t(tau), 50, max_cand=256, block=128)
    ov, oi = O.compacted_topk(S, tau, 50)
    assert np.array_equal(v.cpu().numpy(), ov) and np.array_equal(i.cpu().numpy(), oi)
    rv = z["C_v"]
    assert np.array_equal(v.cpu().numpy(), rv)            # identical score sequences
    fin = np.isinf(rv)
    assert np.array_equal(i.cpu().numpy()[fin], z["C_i"][fin])   # (-inf, 0) padding


def test_compacted_topk_strided_view():
    import gpusparse
    rng = np.random.default_rng(1)
    S = rng.standard_normal((7, 5000)).astype(np.float32)
    tau = np.full(7, 0.5, dtype=np.float32)
    big = t(S)
    v, i = gpusparse.compacted_topk(big[:, :3000], t(tau), 100)
    ov, oi = O.compacted_topk(S[:, :3000], tau, 100)
    assert np.array_equal(v.cpu().numpy(), ov) and np.array_equal(i.cpu().numpy(), oi)


def test_chunked_entry_points_equal_fused():
    import gpusparse
    ip, ix, dt = O.synth_csr(7000, 30522, seed=12)
    g = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), 30522, DEV)
    qi, qs = O.synth_queries(20, 30522, seed=13)
    a = gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=300)
    bnd = gpusparse.build_chunk_boundaries(g, 1000)
    b = gpusparse.triton_chunked_score(g, t(qi), t(qs), top_k=300, doc_chunk=1000, chunk_bounds=bnd)
    c = gpusparse.triton_chunked_score_fused(g, t(qi), t(qs), top_k=300, doc_chunk=1000, max_cand=16)
    for x in (b, c):
        assert torch.equal(a[0], x[0]) and torch.equal(a[1], x[1])
    with pytest.raises(ValueError):
        gpusparse.triton_chunked_score(g, t(qi), t(qs), chunk_bounds=bnd[:, :5])


def test_reference_style_index_without_blocks():
    """The reference plug-in creates the index with __new__ and sets six fields."""
    import gpusparse
    ip, ix, dt = O.synth_csr(3000, 30522, seed=14)
    ref = O.build_index(ip, ix, dt, 30522)
    idx = gpusparse.GPUInvertedIndex.__new__(gpusparse.GPUInvertedIndex)
    idx.doc_ids, idx.scores = t(ref.doc_ids), t(ref.scores)
    idx.offsets, idx.lengths = t(ref.offsets), t(ref.lengths)
    idx.num_docs, idx.vocab_size, idx.device = 3000, 30522, DEV
    qi, qs = O.synth_queries(16, 30522, seed=15)
    s, i = gpusparse.triton_fused_score(idx, t(qi), t(qs), top_k=200)
    rs, ri = O.score_topk(ref, qi, qs, 200, head=idx.head_ids.cpu().numpy())
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)


def test_errors_are_loud():
    import gpusparse
    ip, ix, dt = O.synth_csr(100, 30522, seed=16)
    g = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), 30522, DEV)
    qi, qs = O.synth_queries(4, 30522, seed=17)
    with pytest.raises(RuntimeError):                        # queries left on the host
        gpusparse.triton_fused_score(g, torch.from_numpy(qi), torch.from_numpy(qs))
    with pytest.raises(ValueError):
        gpusparse.triton_fused_score(g, t(qi), t(qs[:, :3]))
    with pytest.raises(ValueError):
        gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=0)
    with pytest.raises(RuntimeError):                        # more scored terms than a plan holds
        gpusparse.triton_fused_score(g, t(np.zeros((1, 16385), np.int32)),
                                     t(np.ones((1, 16385), np.float32)), top_k=5)


def _stub_harness():
    for name in ("lsr_benchmark", "lsr_benchmark.click", "lsr_benchmark.irds", "tirex_tracker"):
        sys.modules.pop(name, None)


def test_plugin_retrieve_matches_reference_golden():
    _stub_harness()
    from lsr_benchmark_engine import gpusparse_retrieval as P
    meta = json.load(open(os.path.join(GOLD, "reference_meta.json")))["plugin"]
    d_emb = [tuple(x) for x in meta["d_emb"]]
    q_emb = [tuple(x) for x in meta["q_emb"]]
    dim = P.determine_dimension(d_emb, q_emb)
    dids, dcsr = P.to_csr(d_emb, dim)
    qids, qcsr = P.to_csr(q_emb, dim)
    idx = P.build_index(dcsr, "cuda:0")
    ti, ts, _ = P.to_query_tensors(qcsr, "cuda:0")
    res = P.retrieve(idx, qids, ti, ts, dids, k=3)
    got = [[[q, float(s), d] for q, s, d in r] for r in res]
    assert got == meta["retrieve_k3"]


def test_plugin_retrieve_chunked_path_and_run_file(tmp_path):
    from lsr_benchmark_engine import gpusparse_retrieval as P
    ip, ix, dt = O.synth_csr(3000, 30522, seed=19)
    emb = [(f"d{d}", ix[ip[d]:ip[d + 1]], dt[ip[d]:ip[d + 1]]) for d in range(3000)]
    qi, qs = O.synth_queries(30, 30522, seed=20)
    qemb = [(f"q{b}", qi[b][qi[b] >= 0], qs[b][qi[b] >= 0]) for b in range(30)]
    dim = P.determine_dimension(emb, qemb)
    dids, dcsr = P.to_csr(emb, dim)
    qids, qcsr = P.to_csr(qemb, dim)
    idx = P.build_index(dcsr, "cuda:0")
    ti, ts, _ = P.to_query_tensors(qcsr, "cuda:0")
    mono = P.retrieve(idx, qids, ti, ts, dids, k=100, batch_size=7)
    chunk = P.retrieve(idx, qids, ti, ts, dids, k=100, batch_size=7, doc_chunk=512)
    assert mono == chunk
    oidx = O.build_index(ip, ix, dt, dim)
    rs, ri = O.score_topk(oidx, qi, qs, 100, head=idx.head_ids.cpu().numpy())
    for b in range(30):
        exp = [(f"q{b}", float(s), f"d{d}") for s, d in zip(rs[b], ri[b]) if s > 0]
        assert mono[b] == exp
    P.write_run(mono, tmp_path / "run.txt.gz")
    import gzip
    lines = gzip.open(tmp_path / "run.txt.gz", "rt").read().splitlines()
    assert lines[0].split()[:4] == ["q0", "Q0", mono[0][0][2], "1"]
    assert len(lines) == sum(len(r) for r in mono)


def _with_duplicates(ip, ix, dt, seed):
    """A copy of a CSR in which some rows list a term two or three times (adjacent and
    apart), with weights that do not sum exactly in fp32."""
    rng = np.random.default_rng(seed)
    ix, dt = ix.copy(), dt.copy()
    n = len(ip) - 1
    for r in rng.choice(n, size=max(1, n // 20), replace=False):
        e0, e1 = int(ip[r]), int(ip[r + 1])
        if e1 - e0 < 4:
            continue
        j = rng.integers(e0 + 1, e1)
        ix[j] = ix[e0]                          # a repeat of the row's first term
        dt[j] = np.float32(rng.random() * 3.0)
        if e1 - e0 > 40 and r % 2:
            ix[e1 - 1] = ix[e0]                 # and a third occurrence at the row's end
            dt[e1 - 1] = np.float32(0.1)
    return ix, dt


def test_duplicate_doc_term_entries_are_merged():
    """A term listed more than once in one CSR row: the reference keeps every entry as a
    posting and its scatter-add sums them.  The build merges them (first position, fp32 sum
    of the weights in row order); the index equals the oracle's build of the merged CSR,
    scores are bit-exact against the oracle and within tolerance of the fp64 scores of the
    original CSR, through the tensor builder, the streamed builder (chunk indptr not
    starting at 0) and the plug-in's scipy path."""
    import scipy.sparse as sp
    import gpusparse
    from run_correctness_verification import build_gpu_index_from_csr
    V = 30522
    ip, ix0, dt0 = O.synth_csr(3000, V, seed=21)
    ix, dt = _with_duplicates(ip, ix0, dt0, 5)
    mip, mix, mdt = O.merge_duplicates(ip, ix, dt)
    assert len(mix) < len(ix)
    oidx = O.build_index(mip, mix, mdt, V)
    qi, qs = O.synth_queries(40, V, seed=22)
    S = O.score_dense_f64(ip, ix, dt, V, qi, qs)
    ipd, ixd, dtd = t(ip), t(ix), t(dt)
    builds = {
        "tensors": gpusparse.build_from_csr_tensors(ipd, ixd, dtd, V, DEV),
        "streamed": gpusparse.build_streamed(
            3000, V, lambda lo, hi, wd: (ipd[lo:hi + 1], ixd, dtd if wd else None), DEV,
            chunk_docs=1024),
        "scipy": build_gpu_index_from_csr(sp.csr_matrix((dt, ix, ip), shape=(3000, V)), DEV),
    }
    for name, g in builds.items():
        assert np.array_equal(g.doc_ids.cpu().numpy(), oidx.doc_ids), name
        assert np.array_equal(g.scores.cpu().numpy().view(np.uint32), oidx.scores.view(np.uint32)), name
        s, i = gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=500)
        rs, ri = O.score_topk(oidx, qi, qs, 500, head=g.head_ids.cpu().numpy())
        assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)
        check_topk(s.cpu().numpy(), i.cpu().numpy(), S, 500)


@pytest.mark.parametrize("vocab", [0, 60])
def test_merge_duplicates_kernel_matches_oracle(vocab):
    """gsp_csr_dedup_* against the oracle's merge on rows of many lengths (up to 700
    entries, terms repeated up to 40 times) and a chunk whose indptr starts above 0; with
    the vocabulary size unknown (pairwise check) and known (vocabulary bitmap)."""
    from gpusparse.index import merge_duplicates
    rng = np.random.default_rng(7)
    lens = rng.integers(0, 700, size=400)
    lens[:5] = [0, 1, 33, 64, 65]
    ip = np.zeros(len(lens) + 1, dtype=np.int64)
    np.cumsum(lens, out=ip[1:])
    ix = rng.integers(0, 60, size=int(ip[-1])).astype(np.int32)     # many repeats per row
    dt = rng.random(int(ip[-1])).astype(np.float32)
    for lo, hi in [(0, 400), (37, 211)]:
        sub_ip = ip[lo:hi + 1]
        got = merge_duplicates(t(sub_ip), t(ix), t(dt), vocab)
        exp = O.merge_duplicates(sub_ip - sub_ip[0], ix[sub_ip[0]:sub_ip[-1]], dt[sub_ip[0]:sub_ip[-1]])
        assert np.array_equal(got[0].cpu().numpy(), exp[0])
        assert np.array_equal(got[1].cpu().numpy(), exp[1])
        assert np.array_equal(got[2].cpu().numpy().view(np.uint32), exp[2].view(np.uint32))
        only_ix = merge_duplicates(t(sub_ip), t(ix), None, vocab)
        assert np.array_equal(only_ix[1].cpu().numpy(), exp[1]) and only_ix[2] is None


def test_reference_style_index_with_repeated_doc_is_refused():
    import gpusparse
    ip, ix, dt = O.synth_csr(300, 30522, seed=22)
    ref = O.build_index(ip, ix, dt, 30522)
    d = ref.doc_ids.copy()
    t0 = int(np.argmax(ref.lengths))
    o = int(ref.offsets[t0])
    d[o + 1] = d[o]                                           # a repeated doc id in one list
    idx = gpusparse.GPUInvertedIndex.__new__(gpusparse.GPUInvertedIndex)
    idx.doc_ids, idx.scores = t(d), t(ref.scores)
    idx.offsets, idx.lengths = t(ref.offsets), t(ref.lengths)
    idx.num_docs, idx.vocab_size, idx.device = 300, 30522, DEV
    qi, qs = O.synth_queries(4, 30522, seed=23)
    with pytest.raises(ValueError, match="repeat"):
        gpusparse.triton_fused_score(idx, t(qi), t(qs), top_k=10)


@pytest.mark.parametrize("wd", ["fp32", "u8"])
def test_index_save_load_round_trip(tmp_path, wd):
    import gpusparse
    ip, ix, dt = O.synth_csr(6000, 30522, seed=30)
    g = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), 30522, DEV, weight_dtype=wd)
    qi, qs = O.synth_queries(20, 30522, seed=31)
    a = gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=500)
    gpusparse.save_index(g, tmp_path / "index.pt")
    h = gpusparse.load_index(tmp_path / "index.pt", DEV)
    for f in ("doc_ids", "offsets", "lengths", "block_starts", "head_ids", "head_rows"):
        assert torch.equal(getattr(h, f), getattr(g, f)), f
    b = gpusparse.triton_fused_score(h, t(qi), t(qs), top_k=500)
    assert torch.equal(a[1], b[1]) and torch.equal(a[0].view(torch.int32), b[0].view(torch.int32))
    torch.save({"x": 1}, tmp_path / "other.pt")
    with pytest.raises(ValueError):
        gpusparse.load_index(tmp_path / "other.pt", DEV)


def test_index_built_with_other_block_size_scores():
    import gpusparse
    ip, ix, dt = O.synth_csr(9000, 30522, seed=32)
    g = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), 30522, DEV, block_docs=4096)
    qi, qs = O.synth_queries(16, 30522, seed=33)
    s, i = gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=300)
    assert g.block_docs == 1024
    rs, ri = O.score_topk(O.build_index(ip, ix, dt, 30522), qi, qs, 300, head=g.head_ids.cpu().numpy())
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)


def test_captured_scorer_replays_equal_eager_calls():
    import gpusparse
    ip, ix, dt = O.synth_csr(20000, 30522, seed=34)
    g = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), 30522, DEV)
    qi0, _ = O.synth_queries(32, 30522, seed=35)
    cap = gpusparse.CapturedScorer(g, 32, qi0.shape[1] + 8, top_k=500)
    for seed in (35, 36, 37):
        qi, qs = O.synth_queries(32, 30522, seed=seed)
        W = cap.W
        pi = np.full((32, W), -1, dtype=np.int32)
        ps = np.zeros((32, W), dtype=np.float32)
        w = min(W, qi.shape[1])
        pi[:, :w], ps[:, :w] = qi[:, :w], qs[:, :w]
        s, i = cap.run(t(pi), t(ps))
        es, ei = gpusparse.triton_fused_score(g, t(pi), t(ps), top_k=500)
        torch.cuda.synchronize()
        assert torch.equal(i, ei) and torch.equal(s.view(torch.int32), es.view(torch.int32))
    with pytest.raises(ValueError):
        cap.run(t(pi[:5]), t(ps[:5]))
