"""gsp_score_topk_noalloc: scoring for callers that cannot allocate device memory.

Such callers (a serving loop in which a cudaMalloc would synchronise the device, or a host
program that hands the library only its input and output buffers through a C FFI) use
this entry point; its scratch is a fixed array compiled into the library.  The test calls
it through the C ABI twice in a row, with different batches and top-k, and requires the
results of the workspace entry point gsp_score_topk bit for bit (the tolerance this
suite uses for fp32 scoring); it also checks that a batch too large for the fixed
scratch is refused with an error instead of being run.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
V = 30522


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def noalloc(index, qi, qs, k):
    import gpusparse._lib as L
    from gpusparse.index import view
    B, W = qi.shape
    kk = min(k, index.num_docs)
    s = torch.full((B, kk), float("nan"), device=DEV)
    i = torch.full((B, kk), -7, dtype=torch.int64, device=DEV)
    v = view(index)
    rc = L.lib().gsp_score_topk_noalloc(ctypes.byref(v), L.ptr(qi), L.ptr(qs), B, W, kk,
                                        L.ptr(s), L.ptr(i), None, L.stream_of(DEV))
    return rc, s, i


def test_noalloc_equals_workspace_entry_on_consecutive_calls():
    import gpusparse
    import gpusparse._lib as L
    ip, ix, dt = O.synth_csr(20000, V, seed=21)
    index = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV)
    batches = [(O.synth_queries(64, V, seed=22), 100), (O.synth_queries(48, V, seed=23), 1000)]
    for (qi_h, qs_h), k in batches:
        qi, qs = t(qi_h), t(qs_h)
        ref_s, ref_i = gpusparse.score_topk(index, qi, qs, k)
        rc, s, i = noalloc(index, qi, qs, k)
        L.check(rc, "gsp_score_topk_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(i, ref_i)
        assert torch.equal(s.view(torch.int32), ref_s.view(torch.int32))


def test_noalloc_refuses_batches_beyond_its_scratch():
    import gpusparse
    import gpusparse._lib as L
    ip, ix, dt = O.synth_csr(5000, V, seed=24)
    index = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV)
    qi_h, qs_h = O.synth_queries(4000, V, seed=25)
    rc, s, i = noalloc(index, t(qi_h), t(qs_h), 1000)
    assert rc == L.GSP_ERR_UNSUPPORTED
    assert b"scratch" in L.lib().gsp_last_error()
    torch.cuda.synchronize()
    assert torch.isnan(s).all()                 # nothing ran


def test_noalloc_minimum_capacity_stresses_the_candidate_protocol():
    """A large batch (300 queries, k = 1000) at the minimum candidate capacity (k + 1024
    keys, which at k = 1000 is also the default), so a buffer fills after about one tile
    of candidates: many compactions, generations and retries against raised thresholds.
    The result must still equal the workspace entry point bit for bit."""
    import gpusparse
    import gpusparse._lib as L
    from gpusparse import synth
    ip, ix, dt = synth.synth_csr(200_000, V, seed=26, device=DEV)
    index = gpusparse.build_from_csr_tensors(ip, ix, dt, V, DEV)
    qi, qs = synth.synth_queries(300, V, seed=27, device=DEV)
    ref_s, ref_i = gpusparse.score_topk(index, qi, qs, 1000)
    rc, s, i = noalloc(index, qi, qs, 1000)
    L.check(rc, "gsp_score_topk_noalloc")
    torch.cuda.synchronize()
    assert not torch.isnan(s).any()
    assert torch.equal(i, ref_i)
    assert torch.equal(s.view(torch.int32), ref_s.view(torch.int32))


def test_noalloc_shrinks_candidate_buffers_above_k_2048():
    """k = 4096: the default candidate capacity (k + k/2) is above the minimum (k + 1024),
    and 130 queries fit the fixed scratch only once the buffers shrink to that minimum; the
    shrunken buffers compact more often and must still give the workspace result bit for
    bit."""
    import gpusparse
    import gpusparse._lib as L
    from gpusparse import synth
    ip, ix, dt = synth.synth_csr(60_000, V, seed=28, device=DEV)
    index = gpusparse.build_from_csr_tensors(ip, ix, dt, V, DEV)
    qi, qs = synth.synth_queries(130, V, seed=29, device=DEV)
    ref_s, ref_i = gpusparse.score_topk(index, qi, qs, 4096)
    rc, s, i = noalloc(index, qi, qs, 4096)
    L.check(rc, "gsp_score_topk_noalloc")
    torch.cuda.synchronize()
    assert not torch.isnan(s).any()
    assert torch.equal(i, ref_i)
    assert torch.equal(s.view(torch.int32), ref_s.view(torch.int32))
