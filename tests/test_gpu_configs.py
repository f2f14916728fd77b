"""Parity at the sizes of the benchmark configs (1 and 3).

The CUDA path and the CPU oracle score the same seeded corpus and batch (the GPU and CPU
generators are byte-identical): every compared query's top-k must equal the oracle's bit
for bit, and a sample must also pass the north-star bar against fp64 exhaustive scores
(per-document relative error <= 1e-5, tie-aware recall@10/100/1000 = 1.000).
* config 0: 100K documents, the whole batch of 500, k = 10, 100 and 1000;
* config 1: 1M documents, batch 1000, k = 1000 (the GPU scores the whole batch; 200 of
  its queries are compared with the oracle, 24 with fp64);
* config 3's weight modes at 1M documents: uint8 impacts with per-term scale and bf16
  weights, against the oracle fed the same dequantised weights (and the quantisation
  itself against the oracle's).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from parity import assert_bit_exact, check_topk

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
DEV = torch.device("cuda:0")
V = 30522


def _gpu_queries(B):
    from gpusparse import synth
    qi, qs = synth.synth_queries(B, V, seed=1, device=DEV)
    return qi, qs


def test_config0_whole_batch():
    import gpusparse
    from gpusparse import synth
    N, B = 100_000, 500
    ip, ix, dt = O.synth_csr(N, V, seed=0)
    oidx = O.build_index(ip, ix, dt, V)
    g = synth.synth_index(N, V, seed=0, device=DEV)
    assert np.array_equal(g.doc_ids.cpu().numpy(), oidx.doc_ids)
    qi, qs = _gpu_queries(B)
    qi_h, qs_h = qi.cpu().numpy(), qs.cpu().numpy()
    head = g.head_ids.cpu().numpy()
    rs, ri = O.score_topk(oidx, qi_h, qs_h, 1000, head=head)
    S = O.score_dense_f64(ip, ix, dt, V, qi_h, qs_h)
    for k in (10, 100, 1000):
        s, i = gpusparse.triton_fused_score(g, qi, qs, top_k=k)
        s, i = s.cpu().numpy(), i.cpu().numpy()
        assert_bit_exact(s, i, rs[:, :k], ri[:, :k])
        rec = check_topk(s, i, S, k)
        assert all(v == 1.0 for v in rec.values()), rec


@pytest.fixture(scope="module")
def config1():
    from gpusparse import synth
    N = 1_000_000
    ip, ix, dt = O.synth_csr(N, V, seed=0)
    oidx = O.build_index(ip, ix, dt, V)
    qi, qs = _gpu_queries(1000)
    return N, (ip, ix, dt), oidx, qi, qs, synth


def test_config1_batch_1000(config1):
    import gpusparse
    N, (ip, ix, dt), oidx, qi, qs, synth = config1
    g = synth.synth_index(N, V, seed=0, device=DEV)
    s, i = gpusparse.triton_fused_score(g, qi, qs, top_k=1000)
    s, i = s.cpu().numpy(), i.cpu().numpy()
    sel = np.r_[0:100, 900:1000]            # query 0 (107+ terms) and the batch's end
    qi_h, qs_h = qi.cpu().numpy()[sel], qs.cpu().numpy()[sel]
    rs, ri = O.score_topk(oidx, qi_h, qs_h, 1000, head=g.head_ids.cpu().numpy())
    assert_bit_exact(s[sel], i[sel], rs, ri)
    few = sel[::8][:24]
    S = O.score_dense_f64(ip, ix, dt, V, qi.cpu().numpy()[few], qs.cpu().numpy()[few])
    rec = check_topk(s[few], i[few], S, 1000)
    assert rec == {10: 1.0, 100: 1.0, 1000: 1.0}


@pytest.mark.parametrize("wd", ["u8", "bf16"])
def test_config3_weight_modes_at_1m(config1, wd):
    import gpusparse
    N, (ip, ix, dt), oidx, qi, qs, synth = config1
    g = synth.synth_index(N, V, seed=0, device=DEV, weight_dtype=wd)
    if wd == "u8":
        q, scale = O.quantize_u8(oidx)
        assert np.array_equal(g.weights_q.cpu().numpy(), q)
        assert np.array_equal(g.term_scale.cpu().numpy().view(np.uint32), scale.view(np.uint32))
        w = O.dequantize_u8(q, scale, oidx.offsets, oidx.lengths, oidx.padded_lengths)
        sc = scale[ix]
        with np.errstate(divide="ignore", invalid="ignore"):
            qd = np.where(sc > 0, np.clip(np.rint(dt / sc), 0, 255), 0).astype(np.float32)
        dt_deq = (qd * sc).astype(np.float32)
    else:
        w = torch.from_numpy(oidx.scores).bfloat16().float().numpy()
        assert np.array_equal(g.weights_q.float().cpu().numpy().view(np.uint32), w.view(np.uint32))
        dt_deq = torch.from_numpy(dt).bfloat16().float().numpy()
    s, i = gpusparse.triton_fused_score(g, qi, qs, top_k=1000)
    s, i = s.cpu().numpy(), i.cpu().numpy()
    sel = np.r_[0:100, 500:600]
    qi_h, qs_h = qi.cpu().numpy()[sel], qs.cpu().numpy()[sel]
    rs, ri = O.score_topk(oidx, qi_h, qs_h, 1000, weights=w, head=g.head_ids.cpu().numpy())
    assert_bit_exact(s[sel], i[sel], rs, ri)
    few = sel[::12][:16]
    S = O.score_dense_f64(ip, ix, dt_deq, V, qi.cpu().numpy()[few], qs.cpu().numpy()[few])
    rec = check_topk(s[few], i[few], S, 1000)
    assert rec == {10: 1.0, 100: 1.0, 1000: 1.0}
