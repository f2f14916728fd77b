"""GPU generator and index builder against the CPU oracle (bit for bit)."""
import json
import os

import numpy as np
import pytest
import scipy.sparse as sp
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = torch.device("cuda:0")


def test_gpu_generator_equals_cpu_twin():
    from gpusparse import synth
    for (n, first, kind) in [(3000, 0, 0), (1777, 123_456, 0), (500, 0, 1)]:
        ip, ix, dt = synth.synth_csr(n, 30522, seed=7, kind=kind, first=first, device=DEV)
        cip, cix, cdt = O.synth_csr(n, 30522, seed=7, kind=kind, first=first)
        assert np.array_equal(ip.cpu().numpy(), cip)
        assert np.array_equal(ix.cpu().numpy(), cix)
        assert np.array_equal(dt.cpu().numpy().view(np.uint32), cdt.view(np.uint32))
    qi, qs = synth.synth_queries(64, 30522, seed=3, device=DEV)
    cqi, cqs = O.synth_queries(64, 30522, seed=3)
    assert np.array_equal(qi.cpu().numpy(), cqi) and np.array_equal(qs.cpu().numpy(), cqs)


def test_gpu_generator_small_vocab_and_completion():
    """Tiny vocabularies exercise the draw cap's deterministic completion."""
    from gpusparse import synth
    law = synth.Law(nnz_mean=40.0, nnz_sd=5.0, nnz_lo=30, nnz_hi=48)
    olaw = O.Law(nnz_mean=40.0, nnz_sd=5.0, nnz_lo=30, nnz_hi=48)
    ip, ix, dt = synth.synth_csr(200, 50, seed=9, law=law, device=DEV)
    cip, cix, cdt = O.synth_csr(200, 50, seed=9, law=olaw)
    assert np.array_equal(ix.cpu().numpy(), cix) and np.array_equal(ip.cpu().numpy(), cip)


@pytest.mark.parametrize("N,V,block_docs", [(2000, 30522, 4096), (9000, 30522, 1024), (120, 300, 32)])
def test_gpu_index_equals_reference_layout(N, V, block_docs):
    import gpusparse
    ip, ix, dt = O.synth_csr(N, V, seed=1)
    csr = sp.csr_matrix((dt, ix, ip), shape=(N, V))
    ref = O.build_index_reference(csr, V)
    t = lambda a: torch.from_numpy(a).to(DEV)  # noqa: E731
    idx = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV, block_docs=block_docs)
    for f in ("doc_ids", "scores", "offsets", "lengths", "padded_lengths", "max_scores"):
        assert np.array_equal(getattr(idx, f).cpu().numpy(), getattr(ref, f)), f
    nb = (N + block_docs - 1) // block_docs
    bounds = O.chunk_bounds(ref, block_docs)
    assert idx.block_starts.shape == (nb + 1, V)
    assert np.array_equal(idx.block_starts.cpu().numpy().astype(np.int64),
                          bounds - ref.offsets[None, :])


def test_gpu_index_matches_golden_small_case():
    import gpusparse
    z = np.load(os.path.join(GOLD, "reference_outputs.npz"))
    meta = json.load(open(os.path.join(GOLD, "reference_meta.json")))["cases"]["B"]
    csr = sp.csr_matrix((z["B_data"], z["B_indices"], z["B_indptr"]), shape=(meta["N"], meta["V"]))
    idx = gpusparse.build_index_from_scipy(csr, DEV, meta["V"])
    for f in ("doc_ids", "scores", "offsets", "lengths", "padded_lengths", "max_scores"):
        assert np.array_equal(getattr(idx, f).cpu().numpy(), z[f"B_index_{f}"]), f


def test_gpu_builders_agree():
    import gpusparse
    ip, ix, dt = O.synth_csr(300, 1000, seed=2, law=O.Law(nnz_mean=20.0, nnz_sd=5.0, nnz_lo=5, nnz_hi=60))
    ids = [ix[ip[d]:ip[d + 1]].tolist() for d in range(300)]
    scs = [dt[ip[d]:ip[d + 1]].tolist() for d in range(300)]
    a = gpusparse.build_gpu_inverted_index(ids, scs, 1000, DEV)
    dense = torch.zeros(300, 1000)
    for d in range(300):
        dense[d, ids[d]] = torch.tensor(scs[d])
    b = gpusparse.build_gpu_inverted_index_from_sparse(dense, DEV)
    nz = dt != 0                                       # from_sparse keeps only nonzeros
    c = O.build_index(*_drop_zeros(ip, ix, dt), 1000)
    for f in ("doc_ids", "scores", "offsets", "lengths"):
        assert np.array_equal(getattr(b, f).cpu().numpy(), getattr(c, f)), f
    ref = O.build_index(ip, ix, dt, 1000)
    for f in ("doc_ids", "scores", "offsets", "lengths"):
        assert np.array_equal(getattr(a, f).cpu().numpy(), getattr(ref, f)), f
    assert nz.sum() < len(dt)


def _drop_zeros(ip, ix, dt):
    keep = dt != 0
    rows = np.repeat(np.arange(len(ip) - 1), np.diff(ip))[keep]
    nip = np.zeros(len(ip), dtype=np.int64)
    np.cumsum(np.bincount(rows, minlength=len(ip) - 1), out=nip[1:])
    order = np.lexsort((ix[keep], rows))                 # dense nonzero order: ascending column
    return nip, ix[keep][order], dt[keep][order]


def test_duplicate_terms_in_a_document_are_merged():
    """The reference's builder keeps both postings of a term a row lists twice (a list that
    repeats doc 0) and its scatter-add sums them; this build merges them first (weights
    summed in row order), which gives the index of the scipy-summed CSR."""
    import gpusparse
    ip = np.array([0, 3, 5], dtype=np.int64)
    ix = np.array([4, 4, 1, 4, 2], dtype=np.int32)
    dt = np.array([0.5, 0.25, 1.0, 2.0, 3.0], dtype=np.float32)
    t = lambda a: torch.from_numpy(a).to(DEV)  # noqa: E731
    idx = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), 8, DEV)
    m = sp.csr_matrix((dt, ix, ip), shape=(2, 8))
    m.sum_duplicates()
    ref = O.build_index_reference(m, 8)
    assert np.array_equal(idx.doc_ids.cpu().numpy(), ref.doc_ids)
    assert np.array_equal(idx.scores.cpu().numpy(), ref.scores)
    o4 = int(idx.offsets.cpu().numpy()[4])                    # term 4: docs 0 and 1
    assert idx.doc_ids.cpu().numpy()[o4] == 0
    assert float(idx.scores.cpu().numpy()[o4]) == 0.75        # doc 0: 0.5 + 0.25


def test_bad_column_id_raises():
    import gpusparse
    t = lambda a: torch.from_numpy(a).to(DEV)  # noqa: E731
    with pytest.raises(ValueError):
        gpusparse.build_from_csr_tensors(t(np.array([0, 2], dtype=np.int64)),
                                         t(np.array([1, 9], dtype=np.int32)),
                                         t(np.array([1.0, 1.0], dtype=np.float32)), 5, DEV)


def test_quantisation_matches_oracle():
    import gpusparse
    ip, ix, dt = O.synth_csr(3000, seed=5)
    t = lambda a: torch.from_numpy(a).to(DEV)  # noqa: E731
    idx = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), 30522, DEV, weight_dtype="u8")
    ref = O.build_index(ip, ix, dt, 30522)
    q, scale = O.quantize_u8(ref)
    assert np.array_equal(idx.weights_q.cpu().numpy(), q)
    assert np.array_equal(idx.term_scale.cpu().numpy(), scale)
    deq = gpusparse.dequantized_weights(idx).cpu().numpy()
    assert np.array_equal(deq, O.dequantize_u8(q, scale, ref.offsets, ref.lengths, ref.padded_lengths))
    gpusparse.quantize_(idx, "bf16")
    bf = idx.weights_q.float().cpu().numpy()
    assert np.array_equal(bf, torch.from_numpy(ref.scores).bfloat16().float().numpy())


def test_chunk_bounds_and_unsorted_error():
    import gpusparse
    z = np.load(os.path.join(GOLD, "reference_outputs.npz"))
    meta = json.load(open(os.path.join(GOLD, "reference_meta.json")))["cases"]["A"]
    ip, ix, dt = O.synth_csr(meta["N"], meta["V"], seed=meta["doc_seed"])
    t = lambda a: torch.from_numpy(a).to(DEV)  # noqa: E731
    idx = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), meta["V"], DEV)
    for dc in (256, 700):
        assert np.array_equal(gpusparse.build_chunk_boundaries(idx, dc).cpu().numpy(), z[f"A_bounds_{dc}"])
    tt = int(torch.argmax(idx.lengths))
    o = int(idx.offsets[tt])
    idx.doc_ids[o:o + 2] = idx.doc_ids[o:o + 2].flip(0)
    with pytest.raises(ValueError):
        gpusparse.build_chunk_boundaries(idx, 512)


def _same_index(a, b):
    for f in ("doc_ids", "offsets", "lengths", "padded_lengths", "block_starts", "head_ids",
              "head_slot"):
        assert torch.equal(getattr(a, f), getattr(b, f)), f
    for f in ("scores", "max_scores", "head_rows"):
        assert torch.equal(getattr(a, f).view(torch.int32), getattr(b, f).view(torch.int32)), f
    assert (a.num_docs, a.doc_base, a.block_docs) == (b.num_docs, b.doc_base, b.block_docs)


@pytest.mark.parametrize("chunk_docs", [1024, 3 * 1024, 5000])
def test_streamed_build_equals_whole_csr(chunk_docs):
    """Counting and filling chunk by chunk gives the same index, bit for bit, as one pass
    over the whole CSR (5000 rounds down to whole 1024-document blocks)."""
    from gpusparse import synth
    N = 20_000
    whole = synth.synth_index(N, seed=2, device=DEV, chunk_docs=1 << 30)
    _same_index(whole, synth.synth_index(N, seed=2, device=DEV, chunk_docs=chunk_docs))
    shard = synth.synth_index(N, seed=2, doc_range=(7168, N), device=DEV, chunk_docs=1 << 30)
    _same_index(shard, synth.synth_index(N, seed=2, doc_range=(7168, N), device=DEV,
                                         chunk_docs=chunk_docs))


def test_host_csr_streamed_build_equals_oracle():
    import gpusparse
    N, V = 9000, 30522
    ip, ix, dt = O.synth_csr(N, V, seed=4)
    idx = gpusparse.build_from_host_csr(ip, ix, dt, V, DEV, chunk_docs=2048)
    ref = O.build_index(ip, ix, dt, V)
    for f in ("doc_ids", "scores", "offsets", "lengths", "padded_lengths", "max_scores"):
        assert np.array_equal(getattr(idx, f).cpu().numpy(), getattr(ref, f)), f
    t = lambda a: torch.from_numpy(a).to(DEV)  # noqa: E731
    _same_index(idx, gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV))


def test_streamed_build_refuses_rows_other_than_counted():
    """The fill pass of chunk [1024, 2048) is handed the rows of documents [0, 1024): every
    write stays inside its block's counted slice of a list, and the surplus is reported."""
    from gpusparse.index import build_streamed
    N, V = 4096, 30522
    ip, ix, dt = O.synth_csr(N, V, seed=3)

    def get_chunk(lo, hi, with_data):
        src = 0 if (with_data and lo == 1024) else lo
        e0, e1 = ip[src], ip[src + hi - lo]
        return (torch.from_numpy(ip[src:src + hi - lo + 1] - e0), torch.from_numpy(ix[e0:e1]),
                torch.from_numpy(dt[e0:e1]))

    with pytest.raises(ValueError, match="other rows"):
        build_streamed(N, V, get_chunk, DEV, chunk_docs=1024)
