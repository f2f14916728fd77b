"""The canonical summation order must not depend on scheduling.

With a schedule jitter set (lane 0 of every scoring warp sleeps a few microseconds at the
start of half of its work items), the lanes of a warp and the warps of an SM interleave
differently from an undisturbed run, and results must stay bit-exact against the CPU
oracle.  Two consecutive long tail runs of a query may hold the same document in different
lanes; without a warp barrier between them the later term's contribution can land first,
which shows here as scores one ulp off on a few percent of the queries at 1M documents.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from parity import assert_bit_exact

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
V = 30522


@pytest.fixture
def jitter():
    import gpusparse._lib as L
    lib = L.lib()
    assert lib.gsp_get_schedule_jitter() == 0
    L.check(lib.gsp_set_schedule_jitter(3000), "jitter")
    try:
        yield
    finally:
        L.check(lib.gsp_set_schedule_jitter(0), "jitter")


def test_jitter_control_validates():
    import gpusparse._lib as L
    lib = L.lib()
    assert lib.gsp_set_schedule_jitter(-1) != 0
    assert lib.gsp_set_schedule_jitter(1000001) != 0
    assert lib.gsp_get_schedule_jitter() == 0


@pytest.mark.parametrize("wd", ["fp32", "u8", "bf16"])
def test_config1_batch_bit_exact_under_jitter(jitter, wd):
    """Config 1 (1M documents, 1000 queries, k = 1000), the whole batch, shared candidate
    buffers."""
    import gpusparse
    from gpusparse import synth
    N, B, k = 1_000_000, 1000, 1000
    ip, ix, dt = O.synth_csr(N, V, seed=0)
    oidx = O.build_index(ip, ix, dt, V)
    g = synth.synth_index(N, V, seed=0, device=DEV, weight_dtype=wd)
    qi, qs = synth.synth_queries(B, V, seed=1, device=DEV)
    s, i = gpusparse.triton_fused_score(g, qi, qs, top_k=k)
    w = None
    if wd == "u8":
        q, scale = O.quantize_u8(oidx)
        w = O.dequantize_u8(q, scale, oidx.offsets, oidx.lengths, oidx.padded_lengths)
    elif wd == "bf16":
        w = torch.from_numpy(oidx.scores).bfloat16().float().numpy()
    rs, ri = O.score_topk(oidx, qi.cpu().numpy(), qs.cpu().numpy(), k, weights=w,
                          head=g.head_ids.cpu().numpy())
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)


def test_small_batch_tree_mode_bit_exact_under_jitter(jitter):
    """A small batch takes per-tile lists and the merge tree."""
    import gpusparse
    N, B, k = 200_000, 8, 500
    ip, ix, dt = O.synth_csr(N, V, seed=3)
    g = gpusparse.build_from_csr_tensors(*(torch.from_numpy(a).to(DEV) for a in (ip, ix, dt)), V, DEV)
    qi, qs = O.synth_queries(B, V, seed=4)
    s, i = gpusparse.triton_fused_score(g, torch.from_numpy(qi).to(DEV), torch.from_numpy(qs).to(DEV),
                                        top_k=k)
    rs, ri = O.score_topk(O.build_index(ip, ix, dt, V), qi, qs, k, head=g.head_ids.cpu().numpy())
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)


@pytest.mark.parametrize("k", [256, 600])
def test_frequent_compactions_bit_exact_under_jitter(jitter, shared_buffers_only, k):
    """Small k over 200K documents through the shared candidate buffers: each query's buffer
    fills every tile or two early on, so generations open, compact and are zeroed back to
    back while other warps append, under the jitter."""
    import gpusparse
    N, B = 200_000, 96
    ip, ix, dt = O.synth_csr(N, V, seed=7)
    g = gpusparse.build_from_csr_tensors(*(torch.from_numpy(a).to(DEV) for a in (ip, ix, dt)), V, DEV)
    qi, qs = O.synth_queries(B, V, seed=8)
    oidx = O.build_index(ip, ix, dt, V)
    rs, ri = O.score_topk(oidx, qi, qs, k, head=g.head_ids.cpu().numpy())
    for _ in range(2):
        s, i = gpusparse.triton_fused_score(g, torch.from_numpy(qi).to(DEV), torch.from_numpy(qs).to(DEV),
                                            top_k=k)
        assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)
