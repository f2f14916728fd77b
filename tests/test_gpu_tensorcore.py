"""The tensor-core head phase (tcgen05, 3xTF32) against fp64 exhaustive scores and the oracle.

With the head terms on the tensor cores a document's head sum is one dense product, so
scores are no longer bitwise equal to the canonical fp32 order; the bar is the north
star's: every returned score within 1e-5 relative of the exact score, tie-aware
recall@10/100/1000 = 1.000 against the fp64 exhaustive ranking, and top-k lists equal to
the oracle's except where scores tie within that tolerance.  Results must still be
bitwise reproducible run to run.  Sizes cover partial 64-query units, partial tiles,
repeated head terms in a query, the uint8 weight mode, the dense (large-k) selection and
the benchmark configs 0 and 1.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from parity import check_topk

pytestmark = [pytest.mark.gpu, pytest.mark.tensorcore]
DEV = torch.device("cuda:0")
V = 30522
RTOL, ATOL = 1e-5, 1e-6


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def assert_topk_close(gs, gi, rs, ri):
    """Two top-k lists of the same queries agree within the tolerance: sorted scores equal to
    rtol 1e-5, and an id may differ only where its score ties the k-th within tolerance."""
    assert gs.shape == rs.shape and gi.shape == ri.shape
    assert np.allclose(gs, rs, rtol=RTOL, atol=ATOL), float(np.abs(gs - rs).max())
    for b in range(gs.shape[0]):
        kth = float(rs[b, -1])
        tol = 2 * (RTOL * abs(kth) + ATOL)
        sure = set(ri[b][rs[b] > kth + tol].tolist())
        assert sure <= set(gi[b].tolist()), f"row {b}: missing {sorted(sure - set(gi[b].tolist()))[:5]}"
        sure_g = set(gi[b][gs[b] > kth + tol].tolist())
        assert sure_g <= set(ri[b].tolist()), f"row {b}: extra {sorted(sure_g - set(ri[b].tolist()))[:5]}"


def tc_used(index):
    """The tensor-core path ran: its view of the index carried the head rows' low parts
    (built on first use in the tensor-core mode) over at least 16 head terms."""
    return index.head_lo is not None and index.head_ids.numel() >= 16


@pytest.fixture(scope="module")
def corpus():
    ip, ix, dt = O.synth_csr(20000, V, seed=0)
    return ip, ix, dt, O.build_index(ip, ix, dt, V)


@pytest.fixture(scope="module")
def gindex(corpus):
    import gpusparse
    ip, ix, dt, _ = corpus
    return gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV)


@pytest.mark.parametrize("B", [1, 63, 64, 100, 257])
@pytest.mark.parametrize("k", [10, 1000])
def test_tensor_cores_vs_fp64_and_oracle(corpus, gindex, B, k):
    import gpusparse
    ip, ix, dt, oidx = corpus
    qi, qs = O.synth_queries(B, V, seed=B + k)
    s, i = gpusparse.triton_fused_score(gindex, t(qi), t(qs), top_k=k)
    assert tc_used(gindex)
    s, i = s.cpu().numpy(), i.cpu().numpy()
    S = O.score_dense_f64(ip, ix, dt, V, qi, qs)
    rec = check_topk(s, i, S, k)
    assert all(v == 1.0 for v in rec.values()), rec
    rs, ri = O.score_topk(oidx, qi, qs, k, head=gindex.head_ids.cpu().numpy())
    assert_topk_close(s, i, rs, ri)


def test_tensor_cores_are_deterministic_and_close_to_canonical(gindex):
    import gpusparse
    import gpusparse._lib as L
    qi, qs = O.synth_queries(200, V, seed=5)
    a = gpusparse.triton_fused_score(gindex, t(qi), t(qs), top_k=1000)
    b = gpusparse.triton_fused_score(gindex, t(qi), t(qs), top_k=1000)
    assert torch.equal(a[1], b[1]) and torch.equal(a[0].view(torch.int32), b[0].view(torch.int32))
    L.check(L.lib().gsp_set_head_mode(L.HEAD_CUDA_CORES), "mode")
    c = gpusparse.triton_fused_score(gindex, t(qi), t(qs), top_k=1000)
    L.check(L.lib().gsp_set_head_mode(L.HEAD_TENSOR_CORES), "mode")
    assert_topk_close(a[0].cpu().numpy(), a[1].cpu().numpy(), c[0].cpu().numpy(), c[1].cpu().numpy())
    # the two orders really differ somewhere (otherwise the tensor cores did not run)
    assert not torch.equal(a[0].view(torch.int32), c[0].view(torch.int32))


def test_repeated_head_terms_partial_tile_and_negative_weights():
    """A query that lists a head term twice (its weights are added before the product), a
    corpus whose last tile is partial, and negative query weights."""
    import gpusparse
    N = 5000 + 321
    ip, ix, dt = O.synth_csr(N, V, seed=11)
    g = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV)
    head = g.head_ids.cpu().numpy()
    qi, qs = O.synth_queries(70, V, seed=12)
    qi, qs = qi.copy(), qs.copy()
    qi[0, :4] = [head[0], head[0], head[3], head[3]]
    qs[0, :4] = [0.75, 0.5, 1.25, -0.25]
    qs[1] = -qs[1]
    s, i = gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=300)
    S = O.score_dense_f64(ip, ix, dt, V, qi, qs)
    rec = check_topk(s.cpu().numpy(), i.cpu().numpy(), S, 300)
    assert all(v == 1.0 for v in rec.values()), rec


def test_large_k_on_tensor_cores(corpus, gindex):
    import gpusparse
    ip, ix, dt, oidx = corpus
    qi, qs = O.synth_queries(70, V, seed=13)
    s, i = gpusparse.triton_fused_score(gindex, t(qi), t(qs), top_k=9000)
    S = O.score_dense_f64(ip, ix, dt, V, qi, qs)
    rec = check_topk(s.cpu().numpy(), i.cpu().numpy(), S, 9000)
    assert all(v == 1.0 for v in rec.values()), rec


@pytest.mark.slow
def test_config0_whole_batch_on_tensor_cores():
    import gpusparse
    from gpusparse import synth
    N, B = 100_000, 500
    ip, ix, dt = O.synth_csr(N, V, seed=0)
    g = synth.synth_index(N, V, seed=0, device=DEV)
    qi, qs = synth.synth_queries(B, V, seed=1, device=DEV)
    qi_h, qs_h = qi.cpu().numpy(), qs.cpu().numpy()
    S = O.score_dense_f64(ip, ix, dt, V, qi_h, qs_h)
    oidx = O.build_index(ip, ix, dt, V)
    rs, ri = O.score_topk(oidx, qi_h, qs_h, 1000, head=g.head_ids.cpu().numpy())
    for k in (10, 100, 1000):
        s, i = gpusparse.triton_fused_score(g, qi, qs, top_k=k)
        s, i = s.cpu().numpy(), i.cpu().numpy()
        rec = check_topk(s, i, S, k)
        assert all(v == 1.0 for v in rec.values()), rec
        assert_topk_close(s, i, rs[:, :k], ri[:, :k])


@pytest.mark.slow
@pytest.mark.parametrize("wd", ["fp32", "u8"])
def test_config1_batch_1000_on_tensor_cores(wd):
    import gpusparse
    from gpusparse import synth
    N = 1_000_000
    ip, ix, dt = O.synth_csr(N, V, seed=0)
    oidx = O.build_index(ip, ix, dt, V)
    g = synth.synth_index(N, V, seed=0, device=DEV, weight_dtype=wd)
    qi, qs = synth.synth_queries(1000, V, seed=1, device=DEV)
    s, i = gpusparse.triton_fused_score(g, qi, qs, top_k=1000)
    s, i = s.cpu().numpy(), i.cpu().numpy()
    w, dt_eff = None, dt
    if wd == "u8":
        q, scale = O.quantize_u8(oidx)
        w = O.dequantize_u8(q, scale, oidx.offsets, oidx.lengths, oidx.padded_lengths)
        sc = scale[ix]
        with np.errstate(divide="ignore", invalid="ignore"):
            qd = np.where(sc > 0, np.clip(np.rint(dt / sc), 0, 255), 0).astype(np.float32)
        dt_eff = (qd * sc).astype(np.float32)
    sel = np.r_[0:100, 900:1000]
    qi_h, qs_h = qi.cpu().numpy(), qs.cpu().numpy()
    rs, ri = O.score_topk(oidx, qi_h[sel], qs_h[sel], 1000, weights=w, head=g.head_ids.cpu().numpy())
    assert_topk_close(s[sel], i[sel], rs, ri)
    few = sel[::8][:24]
    S = O.score_dense_f64(ip, ix, dt_eff, V, qi_h[few], qs_h[few])
    rec = check_topk(s[few], i[few], S, 1000)
    assert rec == {10: 1.0, 100: 1.0, 1000: 1.0}


def test_exhausted_waits_on_tensor_cores_report_a_fault(corpus, gindex):
    """With a wait limit of 0 the tensor-core kernel's stage, accumulator and unit waits give
    up at their first poll: the call reports the fault (NaN scores, ids -1) after its copies
    and products in flight have landed and its tensor memory is released, and the next call
    on the same context, with the default limit, is correct again."""
    import gpusparse
    import gpusparse._lib as L
    lib = L.lib()
    ip, ix, dt, oidx = corpus
    qi, qs = O.synth_queries(130, V, seed=21)
    default = lib.gsp_get_wait_limit()
    L.check(lib.gsp_set_wait_limit(0), "wait limit")
    try:
        s, i = gpusparse.triton_fused_score(gindex, t(qi), t(qs), top_k=100)
        torch.cuda.synchronize()
    finally:
        L.check(lib.gsp_set_wait_limit(default), "wait limit")
    assert tc_used(gindex)
    assert bool(torch.isnan(s).all()) and bool((i == -1).all())
    s, i = gpusparse.triton_fused_score(gindex, t(qi), t(qs), top_k=100)
    rs, ri = O.score_topk(oidx, qi, qs, 100, head=gindex.head_ids.cpu().numpy())
    assert_topk_close(s.cpu().numpy(), i.cpu().numpy(), rs, ri)
