"""CPU oracle for the exact learned-sparse scoring path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline / reference arm of
``bench.py`` may import this module.  The product (``gpu-sparse_b200/``) never does.

What is restated here (reference paths are relative to the GPUSparse checkout):

* ``build_index_reference``: ``src/run_correctness_verification.py:32-84``
  (``build_gpu_index_from_csr``) line for line in numpy: stable argsort of the COO
  columns, ``np.unique`` counts, pad to 32, exclusive cumsum -> offsets, -1/0 fill,
  per-term max.  ``build_index`` is the same algorithm as a C counting sort
  (``oracle.c``) for large inputs; a test pins the two against each other.
* ``chunk_bounds``: ``src/triton_kernel_chunked.py:83-122`` (ascending check raising
  ``ValueError`` :96-108, per-term ``searchsorted`` :110-121).
* ``compacted_topk``: ``src/fused_topk.py:71-103`` (keep ``score >= tau``, top-k of
  the survivors padded with (-inf, 0), exact fallback on overflow).
* ``score_topk`` / ``score_full``: ``src/triton_kernel.py:93-156,199`` in the
  canonical summation order documented in ``oracle.c``.
* ``score_dense_f64``: the exhaustive dense reference
  (``src/remeasure_2026_09.py:238-258``) in fp64.
* ``dense_reference_topk``: that same dense path as the reference runs it (fp32 ``Q @ D^T``
  per chunk of densified documents, ``torch.topk`` and a running cat/topk/gather merge),
  on the CPU -- the CPU baseline the benchmark reports beside the C port.
* ``sequential_score``: ``cpu_sequential_score`` (``src/gpu_scoring.py:221-259``), the
  reference's pure-Python posting-list loop.
* ``synth_*``: the seeded synthetic SPLADE-shaped generator (twin of the GPU one).
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "liboracle.so")
BLOCK = 32
WTAB_SEGS = 65536


def build_lib(force: bool = False) -> str:
    """Compile oracle.c into oracle/liboracle.so (no implicit FMA contraction; the scorer's
    explicit fmaf is the canonical arithmetic)."""
    src = os.path.join(_HERE, "oracle.c")
    if force or not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.check_call(["gcc", "-O3", "-ffp-contract=off", "-fno-fast-math", "-fPIC",
                               "-shared", "-pthread", src, "-o", _SO, "-lm"])
    return _SO


_lib = None


def lib():
    global _lib
    if _lib is None:
        build_lib()
        L = ctypes.CDLL(_SO)
        i32, i64, u32, u64 = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint64
        p = ctypes.c_void_p
        L.orc_synth_nnz.argtypes = [u64, u32, u64, i64, i32, p, i32, i32, i32, p]
        L.orc_synth_fill.argtypes = [u64, u32, u64, i64, i32, p, p, p, p, p, p, i32]
        L.orc_build_lengths.argtypes = [i64, i32, p, p]
        L.orc_build_fill.argtypes = [i64, i32, p, p, p, p, p, p, p]
        L.orc_score_topk.argtypes = [i64, i32, p, p, p, p, i64, i64, p, p, i64, i64, i32, p, p, p]
        L.orc_score_full.argtypes = [i64, i32, p, p, p, p, i64, i64, p, p, i32, p, p]
        L.orc_score_dense_f64.argtypes = [i64, i32, p, p, p, i64, i64, p, p, p, i32]
        for f in ("orc_synth_nnz", "orc_synth_fill", "orc_build_lengths", "orc_build_fill",
                  "orc_score_topk", "orc_score_full", "orc_score_dense_f64"):
            getattr(L, f).restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)


def nthreads_default() -> int:
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:  # pragma: no cover
        return max(1, os.cpu_count() or 1)


# ---------------------------------------------------------------- synthetic law tables

@dataclass(frozen=True)
class Law:
    """One item law (documents or queries) of the synthetic SPLADE-shaped corpus."""
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


def term_cdf(V: int, s: float) -> np.ndarray:
    """CDF over term ids of p(rank r) ~ r^-s, rank r <-> term id r-1."""
    r = np.arange(1, V + 1, dtype=np.float64)
    c = np.cumsum(r ** (-s))
    c /= c[-1]
    c[-1] = 1.0
    return c


def nnz_cdf(law: Law) -> np.ndarray:
    """CDF of clip(round(LogNormal(mean, sd)), lo, hi) over n = lo..hi."""
    s2 = math.log(1.0 + law.nnz_sd ** 2 / law.nnz_mean ** 2)
    mu, sig = math.log(law.nnz_mean) - s2 / 2.0, math.sqrt(s2)
    ns = np.arange(law.nnz_lo, law.nnz_hi + 1)
    c = np.array([0.5 * (1.0 + math.erf((math.log(n + 0.5) - mu) / (sig * math.sqrt(2.0))))
                  for n in ns], dtype=np.float64)
    c[-1] = 1.0
    return c


GUIDE = 65536


def term_guide(cdf: np.ndarray) -> np.ndarray:
    """guide[j] = first i with cdf[i] > j / GUIDE, j = 0..GUIDE (last clamped to V-1)."""
    g = np.searchsorted(cdf, np.arange(GUIDE + 1, dtype=np.float64) / GUIDE, side="right")
    return np.minimum(g, len(cdf) - 1).astype(np.int32)


def weight_table(law: Law) -> np.ndarray:
    """Quantiles of log1p(relu(N(mu, sd))) at u = i / 65536 (last point at 1 - 2^-20)."""
    from scipy.special import ndtri
    u = np.arange(WTAB_SEGS + 1, dtype=np.float64) / WTAB_SEGS
    u[-1] = 1.0 - 2.0 ** -20
    x = law.w_mu + law.w_sd * ndtri(u)
    return np.log1p(np.maximum(x, 0.0))


def synth_csr(n: int, V: int = 30522, seed: int = 0, kind: int = 0, first: int = 0,
              law: Law | None = None, nthreads: int | None = None):
    """Items [first, first+n) of the seeded generator as (indptr i64, indices i32, data f32)."""
    law = law or (DOC_LAW if kind == 0 else QUERY_LAW)
    L = lib()
    nc = nnz_cdf(law)
    nnz = np.empty(n, dtype=np.int32)
    rc = L.orc_synth_nnz(seed, kind, first, n, V, _p(nc), len(nc), law.nnz_lo,
                         law.min_nnz_item0, _p(nnz))
    assert rc == 0
    indptr = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(nnz, out=indptr[1:])
    indices = np.empty(int(indptr[-1]), dtype=np.int32)
    data = np.empty(int(indptr[-1]), dtype=np.float32)
    tc, wt = term_cdf(V, law.zipf_s), weight_table(law)
    gd = term_guide(tc)
    rc = L.orc_synth_fill(seed, kind, first, n, V, _p(tc), _p(gd), _p(wt), _p(indptr),
                          _p(indices), _p(data), nthreads or nthreads_default())
    assert rc == 0
    return indptr, indices, data


def synth_queries(B: int, V: int = 30522, seed: int = 0, law: Law | None = None):
    """(qi int32 [B, W] padded with -1, qs fp32 [B, W] padded with 0), W = max nnz."""
    indptr, indices, data = synth_csr(B, V, seed, kind=1, law=law or QUERY_LAW)
    nnz = np.diff(indptr)
    W = int(nnz.max()) if B else 1
    qi = np.full((B, W), -1, dtype=np.int32)
    qs = np.zeros((B, W), dtype=np.float32)
    for b in range(B):
        qi[b, :nnz[b]] = indices[indptr[b]:indptr[b + 1]]
        qs[b, :nnz[b]] = data[indptr[b]:indptr[b + 1]]
    return qi, qs


# ---------------------------------------------------------------- index build

@dataclass
class Index:
    doc_ids: np.ndarray
    scores: np.ndarray
    offsets: np.ndarray
    lengths: np.ndarray
    padded_lengths: np.ndarray
    max_scores: np.ndarray
    num_docs: int
    vocab_size: int


def build_index_reference(csr, vocab_size: int | None = None) -> Index:
    """src/run_correctness_verification.py:32-84 restated in numpy (V from the matrix
    width when not given; the reference hard-codes VOCAB_SIZE = 30522 at :28)."""
    num_docs = csr.shape[0]
    V = int(vocab_size if vocab_size is not None else csr.shape[1])
    coo = csr.tocoo()
    rows = coo.row.astype(np.int32)
    cols = coo.col.astype(np.int32)
    vals = coo.data.astype(np.float32)
    sort_idx = np.argsort(cols, kind="stable")
    sorted_terms, sorted_docs, sorted_scores = cols[sort_idx], rows[sort_idx], vals[sort_idx]
    unique_terms, counts = np.unique(sorted_terms, return_counts=True)
    lengths = np.zeros(V, dtype=np.int32)
    lengths[unique_terms] = counts
    padded = ((lengths + BLOCK - 1) // BLOCK) * BLOCK
    offsets = np.zeros(V, dtype=np.int64)
    np.cumsum(padded[:-1], out=offsets[1:])
    total = int(offsets[-1] + padded[-1])
    all_docs = np.full(total, -1, dtype=np.int32)
    all_scores = np.zeros(total, dtype=np.float32)
    max_scores = np.zeros(V, dtype=np.float32)
    src = 0
    for i, t in enumerate(unique_terms):
        n = counts[i]
        off = offsets[t]
        all_docs[off:off + n] = sorted_docs[src:src + n]
        all_scores[off:off + n] = sorted_scores[src:src + n]
        max_scores[t] = sorted_scores[src:src + n].max()
        src += n
    return Index(all_docs, all_scores, offsets, lengths, padded.astype(np.int32), max_scores,
                 num_docs, V)


def merge_duplicates(indptr: np.ndarray, indices: np.ndarray, data: np.ndarray):
    """CSR rows with every term once, as the library's builders see them.  The reference
    keeps a term that one row lists twice as two postings and sums both in its scatter-add
    (``lsr_benchmark_engine/gpusparse_retrieval.py:84-105`` builds from the raw CSR;
    ``src/triton_kernel.py:127-156`` adds every posting); here the first occurrence keeps
    its place and its weight becomes the fp32 sum of all occurrences, left to right in
    row order.  Rows without repeats are returned as they are."""
    indptr = np.asarray(indptr, dtype=np.int64)
    indices = np.asarray(indices, dtype=np.int32)
    data = np.asarray(data, dtype=np.float32)
    n = len(indptr) - 1
    if n <= 0 or len(indices) == 0:
        return indptr, indices, data
    rows = np.repeat(np.arange(n, dtype=np.int64), np.diff(indptr))
    lo = min(0, int(indices.min()))
    span = int(indices.max()) + 1 - lo
    sk = np.sort(rows * span + (indices.astype(np.int64) - lo))
    dup_rows = np.unique(sk[1:][sk[1:] == sk[:-1]] // span)
    if len(dup_rows) == 0:
        return indptr, indices, data
    keep = np.ones(len(indices), dtype=bool)
    out_data = data.copy()
    for r in dup_rows:
        e0, e1 = int(indptr[r]), int(indptr[r + 1])
        first = {}
        for e in range(e0, e1):
            t = int(indices[e])
            if t in first:
                f = first[t]
                out_data[f] = np.float32(out_data[f] + data[e])
                keep[e] = False
            else:
                first[t] = e
    new_nnz = np.bincount(rows[keep], minlength=n)
    new_ip = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(new_nnz, out=new_ip[1:])
    return new_ip, indices[keep], out_data[keep]


def build_index(indptr: np.ndarray, indices: np.ndarray, data: np.ndarray, V: int) -> Index:
    """The same layout as build_index_reference via the C stable counting sort."""
    L = lib()
    N = len(indptr) - 1
    indptr = np.ascontiguousarray(indptr, dtype=np.int64)
    indices = np.ascontiguousarray(indices, dtype=np.int32)
    data = np.ascontiguousarray(data, dtype=np.float32)
    lengths = np.empty(V, dtype=np.int32)
    assert L.orc_build_lengths(len(indices), V, _p(indices), _p(lengths)) == 0
    padded = ((lengths + BLOCK - 1) // BLOCK) * BLOCK
    offsets = np.zeros(V, dtype=np.int64)
    np.cumsum(padded[:-1], out=offsets[1:])
    total = int(offsets[-1] + padded[-1]) if V else 0
    doc_ids = np.full(total, -1, dtype=np.int32)
    scores = np.zeros(total, dtype=np.float32)
    max_scores = np.zeros(V, dtype=np.float32)
    assert L.orc_build_fill(N, V, _p(indptr), _p(indices), _p(data), _p(offsets), _p(doc_ids),
                            _p(scores), _p(max_scores)) == 0
    return Index(doc_ids, scores, offsets, lengths, padded.astype(np.int32), max_scores, N, V)


def chunk_bounds(index: Index, doc_chunk: int) -> np.ndarray:
    """src/triton_kernel_chunked.py:83-122: int64 [n_chunks+1, V] posting offsets."""
    doc_ids, offsets = index.doc_ids, index.offsets.astype(np.int64)
    lengths = index.lengths.astype(np.int64)
    V, N = int(index.vocab_size), int(index.num_docs)
    n_chunks = (N + doc_chunk - 1) // doc_chunk
    n_bad = 0
    for t in np.nonzero(lengths)[0]:
        if np.any(np.diff(doc_ids[offsets[t]:offsets[t] + lengths[t]]) < 0):
            n_bad += 1
    if n_bad:
        raise ValueError(f"{n_bad} posting lists are not ascending in doc_id")
    bounds = np.zeros((n_chunks + 1, V), dtype=np.int64)
    edges = [c * doc_chunk for c in range(n_chunks)] + [N]
    for t in range(V):
        L = lengths[t]
        if L == 0:
            bounds[:, t] = offsets[t]
            continue
        seg = doc_ids[offsets[t]:offsets[t] + L]
        first = int(np.searchsorted(seg, 0, side="left"))
        rel = np.searchsorted(seg[first:], edges, side="left")
        bounds[:, t] = offsets[t] + first + rel
    return bounds


# ---------------------------------------------------------------- scoring

def fkey(x: np.ndarray) -> np.ndarray:
    """Order-preserving uint32 key of fp32 values (-0 folded onto +0)."""
    b = (np.asarray(x, dtype=np.float32) + np.float32(0.0)).view(np.uint32)
    return np.where(b & 0x80000000, ~b, b | 0x80000000).astype(np.uint32)


def topk_rows(S: np.ndarray, k: int, id_base: int = 0):
    """Exact top-k of each row of S by (score desc, index asc)."""
    B, N = S.shape
    k = min(k, N)
    key = fkey(S).astype(np.uint64)
    comp = (key << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - np.arange(N, dtype=np.uint64))[None, :]
    idx = np.empty((B, k), dtype=np.int64)
    for b in range(B):
        idx[b] = np.argsort(comp[b])[::-1][:k]   # composite keys are unique
    vals = np.take_along_axis(S, idx, axis=1)
    return vals.astype(np.float32), idx + id_base


def _head_mask(V: int, head):
    if head is None:
        return None
    m = np.zeros(V, dtype=np.uint8)
    m[np.asarray(head, dtype=np.int64)] = 1
    return m


def score_topk(index: Index, qi: np.ndarray, qs: np.ndarray, k: int, weights=None,
               id_base: int = 0, nthreads: int | None = None, head=None):
    """Exact top-k (fp32 scores [B,k], int64 ids [B,k]) in the canonical order; `head`
    lists the term ids summed first (the scorer's dense head rows)."""
    L = lib()
    qi = np.ascontiguousarray(qi, dtype=np.int32)
    qs = np.ascontiguousarray(qs, dtype=np.float32)
    B, W = qi.shape
    N = int(index.num_docs)
    kk = min(k, N)
    w = np.ascontiguousarray(index.scores if weights is None else weights, dtype=np.float32)
    out_s = np.zeros((B, kk), dtype=np.float32)
    out_i = np.zeros((B, kk), dtype=np.int64)
    hm = _head_mask(int(index.vocab_size), head)
    rc = L.orc_score_topk(N, int(index.vocab_size), _p(index.doc_ids), _p(w), _p(index.offsets),
                          _p(index.lengths), B, W, _p(qi), _p(qs), kk, id_base,
                          nthreads or nthreads_default(), _p(out_s), _p(out_i),
                          _p(hm) if hm is not None else None)
    assert rc == 0
    return out_s, out_i


def score_full(index: Index, qi: np.ndarray, qs: np.ndarray, weights=None,
               nthreads: int | None = None, head=None) -> np.ndarray:
    """The whole fp32 [B, N] score matrix in the canonical order."""
    L = lib()
    qi = np.ascontiguousarray(qi, dtype=np.int32)
    qs = np.ascontiguousarray(qs, dtype=np.float32)
    B, W = qi.shape
    N = int(index.num_docs)
    w = np.ascontiguousarray(index.scores if weights is None else weights, dtype=np.float32)
    out = np.zeros((B, N), dtype=np.float32)
    hm = _head_mask(int(index.vocab_size), head)
    rc = L.orc_score_full(N, int(index.vocab_size), _p(index.doc_ids), _p(w), _p(index.offsets),
                          _p(index.lengths), B, W, _p(qi), _p(qs), nthreads or nthreads_default(),
                          _p(out), _p(hm) if hm is not None else None)
    assert rc == 0
    return out


def score_dense_f64(indptr, indices, data, V: int, qi, qs, nthreads: int | None = None) -> np.ndarray:
    L = lib()
    indptr = np.ascontiguousarray(indptr, dtype=np.int64)
    indices = np.ascontiguousarray(indices, dtype=np.int32)
    data = np.ascontiguousarray(data, dtype=np.float32)
    qi = np.ascontiguousarray(qi, dtype=np.int32)
    qs = np.ascontiguousarray(qs, dtype=np.float32)
    B, W = qi.shape
    N = len(indptr) - 1
    out = np.zeros((B, N), dtype=np.float64)
    assert L.orc_score_dense_f64(N, V, _p(indptr), _p(indices), _p(data), B, W, _p(qi), _p(qs),
                                 _p(out), nthreads or nthreads_default()) == 0
    return out


def compacted_topk(scores: np.ndarray, tau: np.ndarray, k: int):
    """src/fused_topk.py:71-103 semantics: top-min(k, L) of the entries >= tau per row,
    padded with (-inf, 0) when fewer survive; ties by ascending column."""
    B, L = scores.shape
    kk = min(k, L)
    v = np.full((B, kk), -np.inf, dtype=np.float32)
    ix = np.zeros((B, kk), dtype=np.int64)
    for b in range(B):
        keep = np.nonzero(scores[b] >= tau[b])[0]
        if len(keep) == 0:
            continue
        sv, si = topk_rows(scores[b:b + 1, keep], kk)
        n = sv.shape[1]
        v[b, :n] = sv[0]
        ix[b, :n] = keep[si[0]]
    return v, ix


def dequantize_u8(q: np.ndarray, scale: np.ndarray, offsets, lengths, padded) -> np.ndarray:
    """fp32 weights q * scale_t of a uint8 posting array (one fp32 rounding)."""
    term_of = np.repeat(np.arange(len(padded)), padded)
    return (q.astype(np.float32) * scale[term_of].astype(np.float32)).astype(np.float32)


def quantize_u8(index: Index):
    """uint8 impacts with per-term fp32 scale max_t / 255, round-to-nearest (ties to
    even), the config-3 weight law; returns (q uint8 [P_pad], scale fp32 [V])."""
    V = index.vocab_size
    scale = (index.max_scores.astype(np.float32) / np.float32(255.0)).astype(np.float32)
    scale[index.lengths == 0] = 0.0
    term_of = np.repeat(np.arange(V), index.padded_lengths)
    st = scale[term_of]
    with np.errstate(divide="ignore", invalid="ignore"):
        r = np.where(st > 0, index.scores / st, 0.0).astype(np.float32)
    q = np.clip(np.rint(r), 0, 255).astype(np.uint8)
    return q, scale


# ---------------------------------------------------------------- the reference's CPU paths

def dense_query_matrix(qi: np.ndarray, qs: np.ndarray, V: int) -> np.ndarray:
    """fp32 [B, V] query matrix (term ids outside [0, V) dropped, repeats summed)."""
    B, W = qi.shape
    Q = np.zeros((B, V), dtype=np.float32)
    ok = (qi >= 0) & (qi < V)
    rows = np.repeat(np.arange(B), W).reshape(B, W)
    np.add.at(Q, (rows[ok], qi[ok]), qs[ok].astype(np.float32))
    return Q


def dense_reference_topk(indptr, indices, data, V: int, Q: np.ndarray, k: int, doc_lo: int = 0,
                         doc_hi: int | None = None, chunk: int = 16384):
    """``src/remeasure_2026_09.py:238-258`` (dense_reference_topk) on the CPU: for every chunk
    of documents, densify the chunk, S = Q @ D_chunk^T in fp32, torch.topk of each row, and
    merge into the running top-k with torch.cat / topk / gather.  The reference densifies
    200 000 documents per chunk on the GPU; ``chunk`` only bounds the dense block's memory.
    Covers documents [doc_lo, doc_hi); returns (scores fp32 [B, k'], ids int64 [B, k'])."""
    import torch
    doc_hi = len(indptr) - 1 if doc_hi is None else doc_hi
    Qt = torch.from_numpy(np.ascontiguousarray(Q, dtype=np.float32))
    nq = Qt.shape[0]
    best_s = torch.zeros((nq, 0), dtype=torch.float32)
    best_i = torch.zeros((nq, 0), dtype=torch.long)
    for start in range(doc_lo, doc_hi, chunk):
        stop = min(doc_hi, start + chunk)
        e0, e1 = int(indptr[start]), int(indptr[stop])
        rows = np.repeat(np.arange(stop - start), np.diff(indptr[start:stop + 1]))
        Db = torch.zeros((stop - start, V), dtype=torch.float32)
        Db.index_put_((torch.from_numpy(rows), torch.from_numpy(indices[e0:e1].astype(np.int64))),
                      torch.from_numpy(data[e0:e1].astype(np.float32)), accumulate=True)
        sc = Qt @ Db.t()
        kk = min(k, sc.shape[1])
        vs, ix = torch.topk(sc, kk, dim=1)
        best_s = torch.cat([best_s, vs], dim=1)
        best_i = torch.cat([best_i, ix + start], dim=1)
        vs2, ix2 = torch.topk(best_s, min(k, best_s.shape[1]), dim=1)
        best_s, best_i = vs2, torch.gather(best_i, 1, ix2)
        del Db, sc
    return best_s.numpy(), best_i.numpy()


def sequential_score(indptr, indices, data, qi: np.ndarray, qs: np.ndarray, num_docs: int,
                     top_k: int = 10):
    """``cpu_sequential_score`` (``src/gpu_scoring.py:221-259``): a Python dict inverted index
    of (doc, score) lists, then per query a float32 accumulator filled posting by posting and
    an argpartition top-k.  Returns the (scores, doc ids) lists and the scoring time in
    seconds (the index build excluded)."""
    import time
    inv = {}
    for d in range(num_docs):
        for e in range(int(indptr[d]), int(indptr[d + 1])):
            inv.setdefault(int(indices[e]), []).append((d, float(data[e])))
    out_s, out_i = [], []
    t0 = time.perf_counter()
    for b in range(qi.shape[0]):
        doc_scores = np.zeros(num_docs, dtype=np.float32)
        for t, w in zip(qi[b].tolist(), qs[b].tolist()):
            if t >= 0 and t in inv:
                for d, ds in inv[t]:
                    doc_scores[d] += w * ds
        kk = min(top_k, num_docs)
        top = np.argpartition(doc_scores, -kk)[-kk:]
        top = top[np.argsort(doc_scores[top])[::-1]]
        out_s.append(doc_scores[top].tolist())
        out_i.append(top.tolist())
    return out_s, out_i, time.perf_counter() - t0
