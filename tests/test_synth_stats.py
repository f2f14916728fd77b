"""The synthetic corpus has the shape the benchmark configs describe (CPU).

The seeded generator stands in for MS MARCO SPLADE.  Its law follows BASELINE.json
(Zipf s = 1.1 term ids over V = 30522, log-normal nnz with mean 180 / sd 80 clipped to
[20, 600], weights log1p(relu(N(0.8, 0.7))) with explicit zeros; queries with mean 30,
clipped to [5, 128], query 0 at >= 107 terms).  A successive-sampling restatement of that
law (numpy ``default_rng(0)``, ``choice(replace=False, p)``) measured these statistics at
config 0 (100K documents): 17.98M postings, every document holding the top term, 43 lists
of at least N/2 documents, 12.7 % explicit zero weights, 2.6 % pad-to-32 overhead, and a
batch's unique terms owning 0.713 / 0.785 / 0.909 of the postings at B = 500 / 1000 / 4096
with about 11.6 * B * N (query term, posting) contributions.  This generator draws the
same law with a counter-based stream, so the figures agree to within sampling noise.
"""
import numpy as np
import pytest

from oracle import oracle as O

V = 30522


@pytest.fixture(scope="module")
def config0():
    ip, ix, dt = O.synth_csr(100_000, V, seed=0)
    return ip, ix, dt, np.bincount(ix, minlength=V)


def test_config0_corpus_statistics(config0):
    ip, ix, dt, lengths = config0
    n = len(ip) - 1
    assert abs(len(ix) - 17.98e6) / 17.98e6 < 0.01
    nnz = np.diff(ip)
    assert nnz.min() >= 20 and nnz.max() <= 600 and abs(nnz.mean() - 180) < 2
    assert lengths.max() == n                      # the top term is in every document
    assert 38 <= int((lengths >= n // 2).sum()) <= 48
    assert abs(float((dt == 0).mean()) - 0.127) < 0.005
    padded = ((lengths + 31) // 32) * 32
    assert abs((1.0 - len(ix) / padded.sum()) - 0.026) < 0.002


@pytest.mark.parametrize("B,frac", [(500, 0.713), (1000, 0.785), (4096, 0.909)])
def test_config0_batch_statistics(config0, B, frac):
    _, ix, _, lengths = config0
    qi, _ = O.synth_queries(B, V, seed=1)
    uniq = np.unique(qi[qi >= 0])
    assert abs(lengths[uniq].sum() / len(ix) - frac) < 0.01
    contrib = (lengths[np.where(qi >= 0, qi, 0)] * (qi >= 0)).sum()
    assert abs(contrib / (B * 100_000) - 11.6) < 0.2
    nq = (qi >= 0).sum(axis=1)
    assert nq[0] >= 107 and nq.max() <= 128 and nq.min() >= 5 and abs(nq.mean() - 30) < 1.5
