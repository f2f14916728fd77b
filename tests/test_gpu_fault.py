"""The scorer's bounded waits, made to run out: with a wait limit of 0 every wait of the
candidate buffers gives up at once, and the call must report that (NaN scores, ids -1)
instead of a result or a hang; the next call, with the default limit, must be exact
again on the same context."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from parity import assert_bit_exact

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("shared_buffers_only")]
DEV = torch.device("cuda:0")
V = 30522


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def test_exhausted_waits_report_a_fault_and_the_context_stays_usable():
    import gpusparse
    import gpusparse._lib as L
    lib = L.lib()
    ip, ix, dt = O.synth_csr(20000, V, seed=40)
    g = gpusparse.build_from_csr_tensors(t(ip), t(ix), t(dt), V, DEV)
    qi, qs = O.synth_queries(64, V, seed=41)
    default = lib.gsp_get_wait_limit()
    assert default > 0
    L.check(lib.gsp_set_wait_limit(0), "wait limit")
    try:
        # 20 tiles of candidates per query overflow its buffer, so compactions (and their
        # waits) happen
        s, i = gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=1000)
        torch.cuda.synchronize()
    finally:
        L.check(lib.gsp_set_wait_limit(default), "wait limit")
    assert bool(torch.isnan(s).all()) and bool((i == -1).all())
    s, i = gpusparse.triton_fused_score(g, t(qi), t(qs), top_k=1000)
    rs, ri = O.score_topk(O.build_index(ip, ix, dt, V), qi, qs, 1000, head=g.head_ids.cpu().numpy())
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)
