"""Seeded synthetic SPLADE-shaped corpora and query batches, generated on the GPU.

This is the benchmark configs' stand-in for MS MARCO SPLADE (no dataset travels with the
repo): term ids Zipf(s) over the vocabulary (rank r <-> id r-1); per item a clipped,
rounded log-normal number of *distinct* terms drawn by successive sampling; weights
log1p(relu(N(0.8, 0.7))) with exact zeros kept as explicit entries.  Documents use
nnz ~ LogNormal(mean 180, sd 80) clipped to [20, 600]; queries LogNormal(mean 30, sd 15)
clipped to [5, 128], with query 0 forced to at least 107 terms.

Generation is counter-based (seed, stream, item, counter) and every floating-point step
is an explicitly rounded IEEE operation (csrc/synth.cu), so any item range -- e.g. one
GPU's doc-range shard -- is generated independently and bit-identically.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from functools import lru_cache

import numpy as np
import torch

from . import _lib as L
from .index import GPUInvertedIndex, build_streamed

WTAB_SEGS = 65536
GUIDE = 65536


@dataclass(frozen=True)
class Law:
    zipf_s: float = 1.1
    nnz_mean: float = 180.0
    nnz_sd: float = 80.0
    nnz_lo: int = 20
    nnz_hi: int = 600
    w_mu: float = 0.8
    w_sd: float = 0.7
    min_nnz_item0: int = 0


DOC_LAW = Law()
QUERY_LAW = Law(nnz_mean=30.0, nnz_sd=15.0, nnz_lo=5, nnz_hi=128, min_nnz_item0=107)

# (num_docs, batch, zipf_s)
CONFIGS = {
    0: dict(num_docs=100_000, batch=500, zipf_s=1.1),
    1: dict(num_docs=1_000_000, batch=1000, zipf_s=1.1),
    2: dict(num_docs=8_800_000, batch=1000, zipf_s=1.1),
    3: dict(num_docs=8_800_000, batch=1000, zipf_s=1.1),
    4: dict(num_docs=50_000_000, batch=4096, zipf_s=1.2),
}


def _term_cdf(V: int, s: float) -> np.ndarray:
    r = np.arange(1, V + 1, dtype=np.float64)
    c = np.cumsum(r ** (-s))
    c /= c[-1]
    c[-1] = 1.0
    return c


def _nnz_cdf(law: Law) -> np.ndarray:
    s2 = math.log(1.0 + law.nnz_sd ** 2 / law.nnz_mean ** 2)
    mu, sig = math.log(law.nnz_mean) - s2 / 2.0, math.sqrt(s2)
    c = np.array([0.5 * (1.0 + math.erf((math.log(n + 0.5) - mu) / (sig * math.sqrt(2.0))))
                  for n in range(law.nnz_lo, law.nnz_hi + 1)], dtype=np.float64)
    c[-1] = 1.0
    return c


def _term_guide(cdf: np.ndarray) -> np.ndarray:
    g = np.searchsorted(cdf, np.arange(GUIDE + 1, dtype=np.float64) / GUIDE, side="right")
    return np.minimum(g, len(cdf) - 1).astype(np.int32)


def _weight_table(law: Law) -> np.ndarray:
    from scipy.special import ndtri
    u = np.arange(WTAB_SEGS + 1, dtype=np.float64) / WTAB_SEGS
    u[-1] = 1.0 - 2.0 ** -20
    return np.log1p(np.maximum(law.w_mu + law.w_sd * ndtri(u), 0.0))


@lru_cache(maxsize=16)
def _tables(V: int, law: Law, device_index: int):
    dev = torch.device("cuda", device_index)
    tc = _term_cdf(V, law.zipf_s)
    return (torch.from_numpy(_nnz_cdf(law)).to(dev), torch.from_numpy(tc).to(dev),
            torch.from_numpy(_term_guide(tc)).to(dev), torch.from_numpy(_weight_table(law)).to(dev))


def synth_csr(n: int, V: int = 30522, seed: int = 0, kind: int = 0, first: int = 0,
              law: Law | None = None, device=None):
    """Items [first, first+n) as device CSR (indptr int64, indices int32, data fp32)."""
    law = law or (DOC_LAW if kind == 0 else QUERY_LAW)
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    nc, tc, gd, wt = _tables(int(V), law, dev.index)
    lib = L.lib()
    with torch.cuda.device(dev):
        st = L.stream_of(dev)
        nnz = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
        L.check(lib.gsp_synth_nnz(int(seed), int(kind), int(first), int(n), int(V), L.ptr(nc),
                                  nc.numel(), law.nnz_lo, law.min_nnz_item0, L.ptr(nnz), st),
                "synth")
        indptr = torch.empty(n + 1, dtype=torch.int64, device=dev)
        ws = L.workspace(lib.gsp_scan_ws_bytes(n), dev)
        L.check(lib.gsp_scan_i32(L.ptr(nnz), int(n), L.ptr(indptr), L.ptr(ws), ws.numel(), st),
                "synth")
        total = int(indptr[-1].item())
        indices = torch.empty(max(total, 1), dtype=torch.int32, device=dev)[:total]
        data = torch.empty(max(total, 1), dtype=torch.float32, device=dev)[:total]
        L.check(lib.gsp_synth_fill(int(seed), int(kind), int(first), int(n), int(V), L.ptr(tc),
                                   L.ptr(gd), L.ptr(wt), L.ptr(indptr), L.ptr(indices),
                                   L.ptr(data), st),
                "synth")
    return indptr, indices, data


def synth_queries(B: int, V: int = 30522, seed: int = 1, law: Law | None = None, device=None):
    """(qi int32 [B, W] padded with -1, qs fp32 [B, W] padded with 0), W = max nnz."""
    indptr, indices, data = synth_csr(B, V, seed, kind=1, law=law or QUERY_LAW, device=device)
    dev = indptr.device
    nnz = indptr[1:] - indptr[:-1]
    W = int(nnz.max().item()) if B else 1
    rows = torch.repeat_interleave(torch.arange(B, device=dev), nnz)
    cols = torch.arange(indices.numel(), device=dev) - indptr[rows]
    qi = torch.full((B, W), -1, dtype=torch.int32, device=dev)
    qs = torch.zeros((B, W), dtype=torch.float32, device=dev)
    qi[rows, cols] = indices
    qs[rows, cols] = data
    return qi, qs


def shard_range(num_docs: int, world: int, rank: int):
    """Contiguous doc-range shard [lo, hi) of rank `rank` out of `world`."""
    return num_docs * rank // world, num_docs * (rank + 1) // world


def synth_index(num_docs: int, V: int = 30522, seed: int = 0, law: Law | None = None,
                doc_range=None, device=None, weight_dtype: str = "fp32",
                keep_fp32: bool = True, head_ids=None,
                chunk_docs: int = 1 << 21) -> GPUInvertedIndex:
    """Index of documents [lo, hi) of the seeded corpus (local ids, doc_base = lo).

    The CSR is generated and consumed ``chunk_docs`` documents at a time (each chunk is
    generated twice, for the count and the fill pass), so the device holds the index and
    one chunk of rows, never the whole CSR."""
    lo, hi = doc_range if doc_range is not None else (0, num_docs)
    law = law or DOC_LAW
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())

    def get_chunk(a, b, with_data):
        return synth_csr(b - a, V, seed, kind=0, first=lo + a, law=law, device=dev)

    return build_streamed(hi - lo, V, get_chunk, dev, chunk_docs=chunk_docs,
                          weight_dtype=weight_dtype, doc_base=lo, keep_fp32=keep_fp32,
                          head_ids=head_ids)
