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
from parity import assert_bit_exact

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
    big = O.synth_csr(20000, 30522, seed=18)
    gb = gpusparse.build_from_csr_tensors(t(big[0]), t(big[1]), t(big[2]), 30522, DEV)
    with pytest.raises(RuntimeError):                        # beyond the supported top-k
        gpusparse.triton_fused_score(gb, t(qi), t(qs), top_k=9000)


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


def test_duplicate_doc_term_entries_are_refused():
    """A term listed twice in one CSR row would repeat a doc id inside its posting list;
    the scorer updates a list's documents in parallel, so the build refuses it."""
    import gpusparse
    ip, ix, dt = O.synth_csr(50, 30522, seed=21)
    ix = ix.copy()
    ix[ip[3] + 1] = ix[ip[3]]                                 # doc 3 lists one term twice
    with pytest.raises(ValueError, match="twice"):
        gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), 30522, DEV)


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
