"""Reference-named scoring API over the sm_100a kernels (drop-in for src/triton_kernel.py,
src/triton_kernel_chunked.py and src/fused_topk.py).

All three reference scorers (monolithic, chunked, chunked + threshold-compacted) return
the same exact top-k, so here they share one fused kernel path (csrc/score.cu): a batch
is scored tile by tile in shared memory and selected on chip, with no [B, N] matrix.
Their tuning arguments are validated exactly as the reference validates them
(``block_pl`` must be a positive power of two -> AssertionError; a supplied
``chunk_bounds`` must have V columns) and otherwise have no effect on the result.

Results: fp32 scores [B, k'] descending and int64 global doc ids [B, k'], k' =
min(top_k, num_docs), ties broken by ascending doc id, bitwise reproducible.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib as L
from .index import GPUInvertedIndex, view


def _check_block_pl(block_pl: int) -> None:
    # src/triton_kernel.py:175 (and :276, triton_kernel_chunked.py:135)
    assert block_pl > 0 and (block_pl & (block_pl - 1)) == 0, \
        f"block_pl must be a positive power of 2, got {block_pl}"


def _prep_queries(index: GPUInvertedIndex, qi: torch.Tensor, qs: torch.Tensor):
    dev = index.device
    if qi.dim() != 2 or qs.shape != qi.shape:
        raise ValueError(f"query tensors must be [B, W] of equal shape, got {tuple(qi.shape)} "
                         f"and {tuple(qs.shape)}")
    L.require_cuda(qi, "query_term_ids")
    L.require_cuda(qs, "query_term_scores")
    if qi.device != dev or qs.device != dev:
        raise ValueError(f"query tensors must live on the index device {dev}")
    if qi.dtype != torch.int32:
        if qi.dtype.is_floating_point:
            raise ValueError("query_term_ids must be an integer tensor")
        V = int(index.vocab_size)
        qi = torch.where((qi < 0) | (qi >= V), torch.full_like(qi, -1), qi).to(torch.int32)
    if qs.dtype != torch.float32:
        qs = qs.to(torch.float32)
    if qi.shape[1] > MAX_WIDTH:
        qi, qs = _compact_queries(qi, qs, int(index.vocab_size))
    return qi.contiguous(), qs.contiguous()


MAX_WIDTH = 16384   # query slots one plan sorts (kMaxWidth in csrc/score.cu)


def _compact_queries(qi: torch.Tensor, qs: torch.Tensor, V: int):
    """Moves every query's scored entries (term id in [0, V)) to the front, keeping their
    slot order, so that a batch padded wider than MAX_WIDTH needs only its longest query's
    width; the canonical order (term id, then slot) and so the result are unchanged."""
    valid = (qi >= 0) & (qi < V)
    width = int(valid.sum(dim=1).max().item()) if qi.shape[0] else 1
    if width > MAX_WIDTH:
        raise RuntimeError(f"a query has {width} scored terms; at most {MAX_WIDTH} are supported")
    order = torch.sort((~valid).to(torch.int8), dim=1, stable=True).indices[:, :max(width, 1)]
    keep = torch.gather(valid, 1, order)
    qi = torch.where(keep, torch.gather(qi, 1, order), torch.full_like(order, -1, dtype=qi.dtype))
    qs = torch.where(keep, torch.gather(qs, 1, order), torch.zeros_like(order, dtype=qs.dtype))
    return qi.to(torch.int32), qs


def score_topk(index: GPUInvertedIndex, query_term_ids: torch.Tensor,
               query_term_scores: torch.Tensor, top_k: int = 10, with_keys: bool = False,
               out: Optional[Tuple[torch.Tensor, ...]] = None, board: Optional[int] = None,
               shard: int = 0, peer_boards=()):
    """Exact top-k of every query over the whole index (see module docstring).

    with_keys=True also returns the packed uint64 candidate keys (as int64) used by the
    multi-GPU merge.  ``out`` may pass preallocated (scores, ids[, keys]) tensors.

    ``board`` (a device address, or a CUDA int64 tensor of n_shards * B entries) turns
    this into shard ``shard`` of n_shards = len(peer_boards) + 1 doc-range shards scoring
    the batch at the same time: row s of a board holds, per query, a key that shard s has
    at least ceil(k / n_shards) candidates at or above; the minimum over the rows bounds
    the corpus-wide k-th best key from below and lets every shard drop candidates early.
    This call writes its own row of its board and of ``peer_boards`` (device addresses of
    the other shards' boards) and never clears them.  The shard may return fewer than k
    real entries; merging all shards' keys gives the exact corpus top-k.
    """
    if top_k < 1:
        raise ValueError("top_k must be >= 1")
    qi, qs = _prep_queries(index, query_term_ids, query_term_scores)
    B, W = qi.shape
    N = int(index.num_docs)
    k = min(int(top_k), N)
    dev = index.device
    lib = L.lib()
    with torch.cuda.device(dev):
        v = view(index)
        if out is not None:
            s_out, i_out = out[0], out[1]
            k_out = out[2] if with_keys else None
        else:
            s_out = torch.empty((B, k), dtype=torch.float32, device=dev)
            i_out = torch.empty((B, k), dtype=torch.int64, device=dev)
            k_out = torch.empty((B, k), dtype=torch.int64, device=dev) if with_keys else None
        if B == 0 or k == 0:
            return (s_out, i_out, k_out) if with_keys else (s_out, i_out)
        ws_bytes = lib.gsp_score_ws_bytes(ctypes.byref(v), B, max(W, 1), k)
        if ws_bytes < 0:
            L.check(int(-ws_bytes), "score_topk")
        ws = L.workspace(ws_bytes, dev)
        if board is None:
            L.check(lib.gsp_score_topk(ctypes.byref(v), L.ptr(qi), L.ptr(qs), B, max(W, 1), k,
                                       L.ptr(s_out), L.ptr(i_out), L.ptr(k_out), L.ptr(ws),
                                       ws_bytes, L.stream_of(dev)), "score_topk")
        else:
            addr = board.data_ptr() if isinstance(board, torch.Tensor) else int(board)
            peers = [p.data_ptr() if isinstance(p, torch.Tensor) else int(p) for p in peer_boards]
            arr = (ctypes.c_void_p * max(len(peers), 1))(*peers)
            L.check(lib.gsp_score_topk_shared(ctypes.byref(v), L.ptr(qi), L.ptr(qs), B, max(W, 1),
                                              k, L.ptr(s_out), L.ptr(i_out), L.ptr(k_out),
                                              L.ptr(ws), ws_bytes, ctypes.c_void_p(addr),
                                              int(shard), len(peers) + 1, arr,
                                              L.stream_of(dev)), "score_topk")
    return (s_out, i_out, k_out) if with_keys else (s_out, i_out)


def triton_fused_score(index, query_term_ids: torch.Tensor, query_term_scores: torch.Tensor,
                       top_k: int = 10, block_pl: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """src/triton_kernel.py:159-200 -- exact scoring + top-k (fp32 [B,k'], int64 [B,k'])."""
    _check_block_pl(block_pl)
    return score_topk(index, query_term_ids, query_term_scores, top_k)


def triton_wand_score(index, query_term_ids: torch.Tensor, query_term_scores: torch.Tensor,
                      top_k: int = 10, block_pl: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """src/triton_kernel.py:260-307.  The reference's WAND scorer runs with threshold 0
    (:290) and so prunes nothing; its result is the exhaustive one, returned here."""
    _check_block_pl(block_pl)
    return score_topk(index, query_term_ids, query_term_scores, top_k)


def build_chunk_boundaries(index, doc_chunk: int) -> torch.Tensor:
    """src/triton_kernel_chunked.py:83-122: int64 [n_chunks+1, V] posting offsets of
    every (chunk boundary, term); ValueError if any list is not ascending in doc id."""
    if doc_chunk <= 0:
        raise ValueError("doc_chunk must be positive")
    dev = index.device if isinstance(index.device, torch.device) else torch.device(index.device)
    N, V = int(index.num_docs), int(index.vocab_size)
    n_chunks = (N + doc_chunk - 1) // doc_chunk
    out = torch.empty((n_chunks + 1, V), dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        ws = L.workspace(L.CHECK_WS_BYTES, dev)
        L.check(L.lib().gsp_chunk_bounds(N, V, int(doc_chunk), L.ptr(index.doc_ids),
                                         L.ptr(index.offsets), L.ptr(index.lengths), L.ptr(out),
                                         L.ptr(ws), ws.numel(), L.stream_of(dev)),
                "build_chunk_boundaries")
    return out


def _check_chunk_bounds(index, chunk_bounds, doc_chunk):
    if doc_chunk <= 0:
        raise ValueError("doc_chunk must be positive")
    if chunk_bounds is None:
        # the reference derives (and validates) the bounds when none are passed
        build_chunk_boundaries(index, doc_chunk)
        return
    if chunk_bounds.dim() != 2 or chunk_bounds.shape[1] != int(index.vocab_size):
        raise ValueError(f"chunk_bounds must be [n_chunks+1, V], got {tuple(chunk_bounds.shape)}")


def triton_chunked_score(index, query_term_ids, query_term_scores, top_k=10, doc_chunk=131072,
                         block_pl=128, chunk_bounds=None):
    """src/triton_kernel_chunked.py:125-170.  Same result as triton_fused_score; the
    doc-chunking the reference does on the host happens on chip here."""
    _check_block_pl(block_pl)
    _check_chunk_bounds(index, chunk_bounds, doc_chunk)
    return score_topk(index, query_term_ids, query_term_scores, top_k)


def triton_chunked_score_fused(index, query_term_ids, query_term_scores, top_k=10,
                               doc_chunk=131072, block_pl=128, chunk_bounds=None, max_cand=8192):
    """src/fused_topk.py:106-160.  Threshold-compacted selection is the scorer's own
    selection here (a running per-query threshold with exact compaction)."""
    _check_block_pl(block_pl)
    _check_chunk_bounds(index, chunk_bounds, doc_chunk)
    if max_cand < 0:
        raise ValueError("max_cand must be >= 0")
    return score_topk(index, query_term_ids, query_term_scores, top_k)


def compacted_topk(scores: torch.Tensor, tau: torch.Tensor, k: int, max_cand: int = 8192,
                   block: int = 1024):
    """src/fused_topk.py:71-103: top-min(k, L) of the entries >= tau[b] of each row of
    ``scores`` [B, L] (column indices, int64), padded with (-inf, 0) when fewer survive.
    The answer does not depend on max_cand/block (the reference's overflow fallback makes
    it exact too); ties break by ascending column."""
    if scores.dim() != 2:
        raise ValueError("scores must be [B, L]")
    L.require_cuda(scores, "scores")
    B, Lc = scores.shape
    kk = min(int(k), Lc)
    dev = scores.device
    if scores.dtype != torch.float32:
        scores = scores.float()
    if scores.stride(1) != 1:
        scores = scores.contiguous()
    tau = tau.to(device=dev, dtype=torch.float32).contiguous()
    if tau.numel() != B:
        raise ValueError("tau must have one entry per row")
    v = torch.empty((B, kk), dtype=torch.float32, device=dev)
    i = torch.empty((B, kk), dtype=torch.int64, device=dev)
    if B == 0 or kk == 0:
        return v, i
    lib = L.lib()
    with torch.cuda.device(dev):
        nb = lib.gsp_compacted_ws_bytes(B, Lc, kk, max_cand)
        ws = L.workspace(nb, dev)
        L.check(lib.gsp_compacted_topk(L.ptr(scores), B, Lc, scores.stride(0), L.ptr(tau), kk,
                                       int(max_cand), L.ptr(v), L.ptr(i), L.ptr(ws), nb,
                                       L.stream_of(dev)), "compacted_topk")
    return v, i


def merge_topk(keys: torch.Tensor, counts, k: int, stride_r: Optional[int] = None):
    """Exact top-k over R candidate lists per query.  keys: int64 [R, B, kin] packed keys
    (as returned by score_topk(with_keys=True)), counts: R valid-entry counts."""
    R, B, kin = keys.shape
    dev = keys.device
    cnt = (ctypes.c_int32 * R)(*[int(c) for c in counts])
    k = int(k)
    s = torch.empty((B, k), dtype=torch.float32, device=dev)
    i = torch.empty((B, k), dtype=torch.int64, device=dev)
    lib = L.lib()
    with torch.cuda.device(dev):
        nb = lib.gsp_merge_ws_bytes(B, k)
        if nb < 0:
            L.check(int(-nb), "merge_topk")
        ws = L.workspace(nb, dev) if nb > 0 else None
        L.check(lib.gsp_merge_topk(L.ptr(keys), B, R, kin, B * kin, cnt, k, L.ptr(s), L.ptr(i),
                                   None, L.ptr(ws), int(nb), L.stream_of(dev)), "merge_topk")
    return s, i


class CapturedScorer:
    """Exact top-k of fixed-shape query batches replayed from one CUDA graph (no reference
    counterpart).  The query, output and workspace buffers are allocated once, one call of
    the fused path (query plan, scorer, merge) is captured after a first call outside the
    capture, and every ``run`` copies a batch in and replays the graph on the current
    stream; the launch cost is then paid once per batch instead of once per kernel.  Meant
    for serving loops with small batches.

    ``run`` returns the scorer's own output tensors, which the next ``run`` overwrites.
    """

    def __init__(self, index: GPUInvertedIndex, batch: int, width: int, top_k: int = 10):
        if batch < 1 or width < 1 or top_k < 1:
            raise ValueError("batch, width and top_k must be positive")
        self.index = index
        self.B, self.W = int(batch), int(width)
        self.k = min(int(top_k), int(index.num_docs))
        dev = index.device
        self.qi = torch.full((self.B, self.W), -1, dtype=torch.int32, device=dev)
        self.qs = torch.zeros((self.B, self.W), dtype=torch.float32, device=dev)
        self.s = torch.empty((self.B, self.k), dtype=torch.float32, device=dev)
        self.i = torch.empty((self.B, self.k), dtype=torch.int64, device=dev)
        lib = L.lib()
        with torch.cuda.device(dev):
            self._v = view(index)                     # block and head rows exist from here on
            nbytes = lib.gsp_score_ws_bytes(ctypes.byref(self._v), self.B, self.W, self.k)
            if nbytes < 0:
                L.check(int(-nbytes), "CapturedScorer")
            self.ws = L.workspace(nbytes, dev)
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                self._launch()                        # first call: attributes, symbol set-up
            torch.cuda.current_stream(dev).wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=side):
                self._launch()

    def _launch(self) -> None:
        dev = self.index.device
        L.check(L.lib().gsp_score_topk(ctypes.byref(self._v), L.ptr(self.qi), L.ptr(self.qs), self.B,
                                       self.W, self.k, L.ptr(self.s), L.ptr(self.i), None,
                                       L.ptr(self.ws), self.ws.numel(), L.stream_of(dev)),
                "CapturedScorer")

    def run(self, query_term_ids: torch.Tensor, query_term_scores: torch.Tensor):
        """Scores one batch of exactly (batch, width) queries; returns (scores, ids)."""
        qi, qs = _prep_queries(self.index, query_term_ids, query_term_scores)
        if tuple(qi.shape) != (self.B, self.W):
            raise ValueError(f"batch must be {(self.B, self.W)}, got {tuple(qi.shape)}")
        with torch.cuda.device(self.index.device):
            self.qi.copy_(qi)
            self.qs.copy_(qs)
            self.graph.replay()
        return self.s, self.i
