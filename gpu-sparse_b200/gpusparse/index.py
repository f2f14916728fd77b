"""GPU-resident term-major inverted index (src/gpu_inverted_index.py:21-35 layout).

Postings of all terms are concatenated, each list ascending in doc id and padded to a
multiple of 32 entries (doc id -1, weight 0), so every list starts on a 128-byte boundary
and 32-wide warp loads of a list are aligned.  Besides the reference's fields the index
keeps:

* ``weight_dtype`` ("fp32" | "bf16" | "u8") and ``weights_q`` (bf16 or uint8 postings) with
  ``term_scale`` (uint8 mode: weight = q * term_scale[t]);
* ``block_starts`` int32 [n_blocks+1, V]: postings of term t with doc id < b*block_docs,
  the doc-range blocks a scorer uses to start mid-list without searching;
* ``doc_base``: global id of local document 0 when the index is one doc-range shard;
* ``head_ids`` / ``head_slot`` / ``head_rows``: the N_HEAD terms with the longest posting
  lists, also stored as dense rows [n_head, ld] (the weight of the term in every document,
  0 where absent) that the scorer sums as one dense product per tile instead of scattering
  their postings; ``head_lo`` (fp32 rows only) holds each element minus its tf32
  truncation, so that the tensor cores carry the full fp32 value (3xTF32).

Builders run on the GPU (csrc/build.cu); the CSR is only copied host -> device, in chunks
of rows when it comes from the host (``build_from_host_csr``, ``build_streamed``).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional, Tuple

import numpy as np
import torch

from . import _lib as L

BLOCK_SIZE = 32          # posting lists are padded to a warp (src/gpu_inverted_index.py:18)
BLOCK_DOCS = 1024        # documents per block_starts row = the scorer's document tile
N_HEAD = 128             # densest terms scored from dense rows instead of posting lists
HEAD_PAD = 4096          # head rows cover a multiple of this many documents
VOCAB_SIZE = 30522       # src/run_correctness_verification.py:28


@dataclass
class GPUInvertedIndex:
    """GPU-resident index with block-aligned posting lists (reference fields first)."""
    doc_ids: torch.Tensor
    scores: Optional[torch.Tensor]
    offsets: torch.Tensor
    lengths: torch.Tensor
    padded_lengths: torch.Tensor
    max_scores: torch.Tensor
    num_docs: int
    vocab_size: int
    device: torch.device
    weight_dtype: str = "fp32"
    weights_q: Optional[torch.Tensor] = None
    term_scale: Optional[torch.Tensor] = None
    block_starts: Optional[torch.Tensor] = None
    block_docs: int = BLOCK_DOCS
    doc_base: int = 0
    head_ids: Optional[torch.Tensor] = None
    head_slot: Optional[torch.Tensor] = None
    head_rows: Optional[torch.Tensor] = None
    head_ld: int = 0
    head_wdtype: int = 0          # dtype code of head_rows (fp32 rows for uint8 postings)
    head_lo: Optional[torch.Tensor] = None   # fp32 rows: low tf32 parts for the tensor cores
    _view: object = field(default=None, repr=False, compare=False)


def _dev(device) -> torch.device:
    d = torch.device(device)
    if d.type != "cuda":
        raise RuntimeError("GPUSparse requires a CUDA device; no CPU path exists")
    if d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return d


def build_from_csr_tensors(indptr: torch.Tensor, indices: torch.Tensor, data: torch.Tensor,
                           vocab_size: int, device=None, weight_dtype: str = "fp32",
                           doc_base: int = 0, keep_fp32: bool = True,
                           block_docs: int = BLOCK_DOCS, head_ids=None) -> GPUInvertedIndex:
    """Build from device CSR tensors (indptr int64 [N+1], indices int32, data fp32)."""
    device = _dev(device if device is not None else indptr.device)
    indptr = indptr.to(device=device, dtype=torch.int64).contiguous()
    indices = indices.to(device=device, dtype=torch.int32).contiguous()
    data = data.to(device=device, dtype=torch.float32).contiguous()
    N = indptr.numel() - 1
    return build_streamed(N, vocab_size, lambda lo, hi, with_data: (indptr, indices, data),
                          device, chunk_docs=max(N, 1), weight_dtype=weight_dtype,
                          doc_base=doc_base, keep_fp32=keep_fp32, block_docs=block_docs,
                          head_ids=head_ids)


def build_streamed(num_docs: int, vocab_size: int, get_chunk, device,
                   chunk_docs: int = 1 << 21, weight_dtype: str = "fp32", doc_base: int = 0,
                   keep_fp32: bool = True, block_docs: int = BLOCK_DOCS,
                   head_ids=None) -> GPUInvertedIndex:
    """Build from CSR rows delivered in chunks, so that only the index and one chunk of rows
    are on the device at a time (a corpus whose CSR and index do not fit together).

    ``get_chunk(lo, hi, with_data)`` returns ``(indptr, indices, data)`` for documents
    [lo, hi): indptr has hi - lo + 1 entries indexing the returned indices/data; data may be
    None when ``with_data`` is False.  Every chunk is requested twice, once for the count
    pass (without data) and once for the fill pass, with the same bounds.  Chunks hold
    ``chunk_docs`` documents (rounded down to whole ``block_docs`` blocks) except the last.
    The result is identical to building from the whole CSR at once.
    """
    device = _dev(device)
    N, V = int(num_docs), int(vocab_size)
    if V <= 0:
        raise ValueError("vocab_size must be positive")
    if N < 0:
        raise ValueError("num_docs must be >= 0")
    step = N if chunk_docs >= N else max(block_docs, int(chunk_docs) // block_docs * block_docs)
    bounds = [(lo, min(N, lo + step)) for lo in range(0, N, max(step, 1))]
    lib = L.lib()

    # chunks whose count pass found no repeated terms skip the check in the fill pass (the
    # same rows by contract)
    clean = set()

    def fetch(lo, hi, with_data):
        ip, ix, dt = get_chunk(lo, hi, with_data)
        ip = torch.as_tensor(ip).to(device=device, dtype=torch.int64).contiguous()
        ix = torch.as_tensor(ix).to(device=device, dtype=torch.int32).contiguous()
        if ip.numel() != hi - lo + 1:
            raise ValueError(f"chunk [{lo}, {hi}): indptr has {ip.numel()} entries, "
                             f"expected {hi - lo + 1}")
        if with_data:
            dt = torch.as_tensor(dt).to(device=device, dtype=torch.float32).contiguous()
            if dt.numel() != ix.numel():
                raise ValueError(f"chunk [{lo}, {hi}): {ix.numel()} indices but {dt.numel()} "
                                 "weights")
        else:
            dt = None
        if (lo, hi) in clean:
            return ip, ix, dt
        out = merge_duplicates(ip, ix, dt, V)
        if out[1] is ix and not with_data:
            clean.add((lo, hi))
        return out

    with torch.cuda.device(device):
        st = L.stream_of(device)
        nb = (N + block_docs - 1) // block_docs
        ws = L.workspace(lib.gsp_index_ws_bytes(N, V, block_docs), device)
        lengths = torch.empty(V, dtype=torch.int32, device=device)
        padded = torch.empty(V, dtype=torch.int32, device=device)
        offsets = torch.empty(V, dtype=torch.int64, device=device)
        block_starts = torch.empty((nb + 1, V), dtype=torch.int32, device=device)
        for lo, hi in bounds:
            ip, ix, _ = fetch(lo, hi, False)
            L.check(lib.gsp_index_count_chunk(N, V, block_docs, lo, hi - lo, L.ptr(ip), L.ptr(ix),
                                              L.ptr(block_starts), L.ptr(ws), ws.numel(), st),
                    "index build")
            del ip, ix
        total = ctypes.c_int64(0)
        L.check(lib.gsp_index_count_finish(N, V, block_docs, L.ptr(lengths), L.ptr(padded),
                                           L.ptr(offsets), L.ptr(block_starts),
                                           ctypes.byref(total), L.ptr(ws), ws.numel(), st),
                "index build")
        P = int(total.value)
        doc_ids = torch.empty(max(P, 0), dtype=torch.int32, device=device)
        scores = torch.empty(max(P, 0), dtype=torch.float32, device=device)
        max_scores = torch.empty(V, dtype=torch.float32, device=device)
        for lo, hi in bounds:
            ip, ix, dt = fetch(lo, hi, True)
            L.check(lib.gsp_index_fill_chunk(N, V, block_docs, lo, hi - lo, L.ptr(ip), L.ptr(ix),
                                             L.ptr(dt), L.ptr(offsets), L.ptr(block_starts),
                                             L.ptr(doc_ids), L.ptr(scores), L.ptr(ws),
                                             ws.numel(), st), "index build")
            del ip, ix, dt
        L.check(lib.gsp_index_fill_finish(N, V, L.ptr(offsets), L.ptr(lengths), L.ptr(doc_ids),
                                          L.ptr(scores), L.ptr(max_scores), L.ptr(ws),
                                          ws.numel(), st), "index build")
        idx = GPUInvertedIndex(doc_ids=doc_ids, scores=scores, offsets=offsets, lengths=lengths,
                               padded_lengths=padded, max_scores=max_scores, num_docs=N,
                               vocab_size=V, device=device, block_starts=block_starts,
                               block_docs=block_docs, doc_base=int(doc_base))
        if weight_dtype != "fp32":
            quantize_(idx, weight_dtype, keep_fp32=keep_fp32)
        if block_docs == BLOCK_DOCS:
            ensure_head(idx, head_ids=head_ids)
    return idx


def merge_duplicates(indptr: torch.Tensor, indices: torch.Tensor, data=None, vocab_size: int = 0):
    """Device CSR rows with every term once: a term that a row lists more than once keeps
    its first position and the fp32 sum of its weights in row order (the reference keeps
    both entries as postings and its scatter-add sums them per document).  Returns the
    inputs unchanged when no row repeats a term; ``indptr`` may start above 0.
    ``vocab_size`` (if known) lets the check use a vocabulary bitmap."""
    n = indptr.numel() - 1
    dev = indptr.device
    lib = L.lib()
    if n <= 0 or indices.numel() == 0:
        return indptr, indices, data
    nnz = torch.empty(n, dtype=torch.int32, device=dev)
    dropped = ctypes.c_int64(0)
    ws = L.workspace(8, dev)
    st = L.stream_of(dev)
    L.check(lib.gsp_csr_dedup_count(n, int(vocab_size), L.ptr(indptr), L.ptr(indices), L.ptr(nnz),
                                    ctypes.byref(dropped), L.ptr(ws), ws.numel(), st),
            "merge duplicate entries")
    if dropped.value == 0:
        return indptr, indices, data
    new_ip = torch.empty(n + 1, dtype=torch.int64, device=dev)
    sws = L.workspace(lib.gsp_scan_ws_bytes(n), dev)
    L.check(lib.gsp_scan_i32(L.ptr(nnz), n, L.ptr(new_ip), L.ptr(sws), sws.numel(), st),
            "merge duplicate entries")
    total = int(indptr[-1].item() - indptr[0].item()) - int(dropped.value)
    out_ix = torch.empty(total, dtype=torch.int32, device=dev)
    out_dt = torch.empty(total, dtype=torch.float32, device=dev) if data is not None else None
    L.check(lib.gsp_csr_dedup_fill(n, L.ptr(indptr), L.ptr(indices), L.ptr(data), L.ptr(new_ip),
                                   L.ptr(out_ix), L.ptr(out_dt), st), "merge duplicate entries")
    return new_ip, out_ix, out_dt


def build_from_host_csr(indptr, indices, data, vocab_size: int, device,
                        chunk_docs: int = 1 << 21, **kw) -> GPUInvertedIndex:
    """Build from a host (numpy) CSR, copying it to the device one chunk of rows at a time."""
    indptr = np.asarray(indptr, dtype=np.int64)

    def get_chunk(lo, hi, with_data):
        e0, e1 = int(indptr[lo]), int(indptr[hi])
        ip = torch.from_numpy(indptr[lo:hi + 1] - e0)
        ix = torch.from_numpy(np.ascontiguousarray(indices[e0:e1], dtype=np.int32))
        dt = (torch.from_numpy(np.ascontiguousarray(data[e0:e1], dtype=np.float32))
              if with_data else None)
        return ip, ix, dt

    return build_streamed(len(indptr) - 1, vocab_size, get_chunk, device, chunk_docs=chunk_docs,
                          **kw)


def quantize_(index: GPUInvertedIndex, weight_dtype: str, keep_fp32: bool = True) -> None:
    """Convert the posting weights to bf16 or uint8-with-per-term-scale in place."""
    if weight_dtype not in ("bf16", "u8"):
        raise ValueError(f"weight_dtype must be fp32, bf16 or u8, got {weight_dtype!r}")
    if index.scores is None:
        raise ValueError("index has no fp32 weights to quantise")
    dev = index.device
    P = index.doc_ids.numel()
    if weight_dtype == "bf16":
        q = torch.empty(P, dtype=torch.bfloat16, device=dev)
        scale = None
        code = L.W_BF16
    else:
        q = torch.empty(P, dtype=torch.uint8, device=dev)
        scale = torch.empty(index.vocab_size, dtype=torch.float32, device=dev)
        code = L.W_U8
    with torch.cuda.device(dev):
        L.check(L.lib().gsp_index_quantize(index.vocab_size, P, L.ptr(index.offsets),
                                           L.ptr(index.padded_lengths), L.ptr(index.max_scores),
                                           L.ptr(index.scores), code, L.ptr(q), L.ptr(scale),
                                           L.stream_of(dev)), "quantize")
    index.weights_q, index.term_scale, index.weight_dtype = q, scale, weight_dtype
    if not keep_fp32:
        index.scores = None
    index.head_rows = None          # rebuilt in the new weight dtype on next use
    index.head_lo = None
    index._view = None


def dequantized_weights(index: GPUInvertedIndex) -> torch.Tensor:
    """fp32 weights the scorer effectively uses (q * scale_t with one fp32 rounding)."""
    if index.weight_dtype == "fp32":
        return index.scores
    if index.weight_dtype == "bf16":
        return index.weights_q.float()
    term_of = torch.repeat_interleave(torch.arange(index.vocab_size, device=index.device),
                                      index.padded_lengths.long())
    return index.weights_q.float() * index.term_scale[term_of]


def ensure_blocks(index: GPUInvertedIndex) -> None:
    """Derive the scorer's block rows (1024-document blocks) for an index constructed
    without them (e.g. field by field, as the reference's plug-in does) or built with
    another block size; validates that lists strictly ascend (ValueError for a
    descending step or a repeated doc id)."""
    if getattr(index, "block_starts", None) is not None and \
            (getattr(index, "block_docs", None) or BLOCK_DOCS) == BLOCK_DOCS:
        return
    from .scoring import build_chunk_boundaries
    bd = BLOCK_DOCS
    dev = index.device if isinstance(index.device, torch.device) else torch.device(index.device)
    n_bad, n_dup = ctypes.c_int64(0), ctypes.c_int64(0)
    with torch.cuda.device(dev):
        ws = L.workspace(L.CHECK_WS_BYTES, dev)
        L.check(L.lib().gsp_check_sorted(int(index.vocab_size), L.ptr(index.doc_ids),
                                         L.ptr(index.offsets), L.ptr(index.lengths),
                                         ctypes.byref(n_bad), ctypes.byref(n_dup), L.ptr(ws),
                                         ws.numel(), L.stream_of(dev)),
                "index check")
    if n_dup.value:
        raise ValueError(f"{n_dup.value} posting lists repeat a doc id (a term listed twice in one "
                         "document); merge duplicate (doc, term) entries first")
    b = build_chunk_boundaries(index, bd)
    index.block_starts = (b - index.offsets.unsqueeze(0)).to(torch.int32).contiguous()
    index.block_docs = bd


def ensure_head(index: GPUInvertedIndex, n_head: int = N_HEAD, head_ids=None) -> None:
    """Build the dense head rows if missing: by default the n_head terms with the longest
    lists; doc-range shards of one corpus pass the same explicit `head_ids` so that every
    shard sums each document's terms in the same order."""
    if getattr(index, "head_rows", None) is not None and head_ids is None:
        return
    dev = index.device
    V = int(index.vocab_size)
    # rows padded to a multiple of HEAD_PAD documents, whole scoring tiles
    ld = ((int(index.num_docs) + HEAD_PAD - 1) // HEAD_PAD) * HEAD_PAD
    H = min(int(n_head), V)
    lengths = index.lengths
    H = min(H, int((lengths > 0).sum().item()))
    wd = getattr(index, "weight_dtype", "fp32")
    with torch.cuda.device(dev):
        if wd == "fp32":
            w, code, dt = index.scores, L.W_F32, torch.float32
        elif wd == "bf16":
            w, code, dt = index.weights_q, L.W_BF16, torch.bfloat16
        else:
            # uint8 postings: the head rows hold the dequantised weights q * scale_t (the
            # exact values the scorer computes), so the dense phase needs no decode
            w, code, dt = dequantized_weights(index), L.W_F32, torch.float32
        if head_ids is not None:
            ids = torch.as_tensor(head_ids, dtype=torch.int64).to(dev).unique().to(torch.int32)
            H = int(ids.numel())
        elif H > 0:
            # longest lists first, ties to the lower term id (deterministic), then id order
            top = torch.sort(-lengths.long(), stable=True).indices[:H]
            ids = top.sort().values.to(torch.int32).contiguous()
        else:
            ids = torch.zeros(0, dtype=torch.int32, device=dev)
        slot = torch.full((V,), -1, dtype=torch.int32, device=dev)
        slot[ids.long()] = torch.arange(H, dtype=torch.int32, device=dev)
        rows = torch.zeros((max(H, 1), max(ld, 1)), dtype=dt, device=dev)
        L.check(L.lib().gsp_index_head_rows(H, L.ptr(ids), L.ptr(index.offsets), L.ptr(lengths),
                                            L.ptr(index.doc_ids), L.ptr(w), code, ld, L.ptr(rows),
                                            L.stream_of(dev)), "head rows")
    index.head_ids, index.head_slot, index.head_rows, index.head_ld = ids, slot, rows, ld
    index.head_wdtype = code
    index.head_lo = None


def ensure_head_lo(index: GPUInvertedIndex) -> None:
    """The tf32 low parts of fp32 head rows (``head_lo``), which only the tensor-core head
    mode reads: built on first use in that mode, since they cost as much memory as the rows
    (4.5 GB at 8.8M documents)."""
    if getattr(index, "head_lo", None) is not None or getattr(index, "head_rows", None) is None:
        return
    if getattr(index, "head_wdtype", L.W_F32) != L.W_F32 or index.head_ids.numel() == 0:
        return
    rows = index.head_rows
    lo = torch.empty_like(rows)
    with torch.cuda.device(index.device):
        L.check(L.lib().gsp_index_head_lo(rows.numel(), L.ptr(rows), L.ptr(lo), L.stream_of(index.device)),
                "head rows")
    index.head_lo = lo


# ------------------------------------------------------------------ persistence
# The reference rebuilds its index from the CSR on every run; a built index (posting
# arrays, block rows and head rows) can be written once and loaded straight to a device.
_FORMAT = "gpusparse-index-v1"
_ARRAYS = ("doc_ids", "scores", "offsets", "lengths", "padded_lengths", "max_scores", "weights_q",
           "term_scale", "block_starts", "head_ids", "head_slot", "head_rows", "head_lo")
_SCALARS = ("num_docs", "vocab_size", "weight_dtype", "block_docs", "doc_base", "head_ld",
            "head_wdtype")


def save_index(index: GPUInvertedIndex, path) -> None:
    """Write every array of a built index (with its block and head rows) to one file."""
    ensure_blocks(index)
    ensure_head(index)
    state = {"format": _FORMAT}
    for f in _SCALARS:
        v = getattr(index, f)
        state[f] = v if isinstance(v, str) else int(v)
    state["arrays"] = {f: getattr(index, f).cpu() for f in _ARRAYS if getattr(index, f, None) is not None}
    torch.save(state, path)


def load_index(path, device) -> GPUInvertedIndex:
    """Load an index written by save_index onto `device` (ValueError for other files)."""
    device = _dev(device)
    state = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(state, dict) or state.get("format") != _FORMAT:
        raise ValueError(f"{path}: not a {_FORMAT} file")
    arr = {f: t.to(device) for f, t in state["arrays"].items()}
    idx = GPUInvertedIndex(doc_ids=arr["doc_ids"], scores=arr.get("scores"), offsets=arr["offsets"],
                           lengths=arr["lengths"], padded_lengths=arr["padded_lengths"],
                           max_scores=arr["max_scores"], num_docs=state["num_docs"],
                           vocab_size=state["vocab_size"], device=device,
                           weight_dtype=state["weight_dtype"], block_docs=state["block_docs"],
                           doc_base=state["doc_base"])
    for f in ("weights_q", "term_scale", "block_starts", "head_ids", "head_slot", "head_rows", "head_lo"):
        setattr(idx, f, arr.get(f))
    idx.head_ld = state["head_ld"]
    idx.head_wdtype = state["head_wdtype"]
    return idx


def view(index: GPUInvertedIndex) -> L.IndexView:
    ensure_blocks(index)
    ensure_head(index)
    if L.lib().gsp_get_head_mode() == L.HEAD_TENSOR_CORES:
        ensure_head_lo(index)
    wd = getattr(index, "weight_dtype", "fp32")
    if wd == "fp32":
        w, code = index.scores, L.W_F32
    elif wd == "bf16":
        w, code = index.weights_q, L.W_BF16
    else:
        w, code = index.weights_q, L.W_U8
    v = L.IndexView()
    v.n_docs = int(index.num_docs)
    v.doc_base = int(getattr(index, "doc_base", 0))
    v.V = int(index.vocab_size)
    v.block_docs = int(index.block_docs)
    v.wdtype = code
    v.doc_ids = index.doc_ids.data_ptr()
    v.weights = w.data_ptr()
    ts = getattr(index, "term_scale", None)
    v.term_scale = ts.data_ptr() if ts is not None else 0
    v.offsets = index.offsets.data_ptr()
    v.lengths = index.lengths.data_ptr()
    v.block_starts = index.block_starts.data_ptr()
    v.n_head = int(index.head_ids.numel())
    v.head_slot = index.head_slot.data_ptr()
    v.head_rows = index.head_rows.data_ptr()
    v.head_ld = int(index.head_ld)
    v.head_wdtype = int(getattr(index, "head_wdtype", code))
    lo = getattr(index, "head_lo", None)
    v.head_lo = lo.data_ptr() if lo is not None else 0
    return v


# ------------------------------------------------------------------ reference builders

def build_index_from_scipy(csr_mat, device, vocab_size: int, **kw) -> GPUInvertedIndex:
    csr = csr_mat.tocsr()
    return build_from_host_csr(csr.indptr, csr.indices, csr.data, vocab_size, device, **kw)


def build_gpu_index_from_csr(csr_mat, device, **kw) -> GPUInvertedIndex:
    """src/run_correctness_verification.py:32-84 (vocabulary fixed at VOCAB_SIZE)."""
    return build_index_from_scipy(csr_mat, device, VOCAB_SIZE, **kw)


def build_gpu_inverted_index(doc_term_ids: list, doc_term_scores: list, vocab_size: int,
                             device: torch.device = torch.device("cuda:0"),
                             **kw) -> GPUInvertedIndex:
    """src/gpu_inverted_index.py:38-113: lists of per-document term ids / scores."""
    lens = np.fromiter((len(t) for t in doc_term_ids), dtype=np.int64, count=len(doc_term_ids))
    indptr = np.zeros(len(lens) + 1, dtype=np.int64)
    np.cumsum(lens, out=indptr[1:])
    indices = (np.concatenate([np.asarray(t, dtype=np.int64) for t in doc_term_ids])
               if len(lens) and indptr[-1] else np.zeros(0, dtype=np.int64))
    data = (np.concatenate([np.asarray(s, dtype=np.float32) for s in doc_term_scores])
            if len(lens) and indptr[-1] else np.zeros(0, dtype=np.float32))
    if indices.size and (indices.min() < 0 or indices.max() >= vocab_size):
        raise IndexError("term id outside [0, vocab_size)")
    return build_from_host_csr(indptr, indices.astype(np.int32), data, vocab_size, device, **kw)


def build_gpu_inverted_index_from_sparse(sparse_matrix: torch.Tensor,
                                         device: torch.device = torch.device("cuda:0"),
                                         **kw) -> GPUInvertedIndex:
    """src/gpu_inverted_index.py:116-134: dense or torch-sparse [num_docs, vocab] matrix;
    entries that are exactly zero are not postings (np.nonzero semantics)."""
    m = sparse_matrix.to_dense() if sparse_matrix.is_sparse else sparse_matrix
    m = m.to(device=_dev(device), dtype=torch.float32)
    N, V = m.shape
    nz = m != 0
    counts = nz.sum(dim=1, dtype=torch.int64)
    indptr = torch.zeros(N + 1, dtype=torch.int64, device=m.device)
    torch.cumsum(counts, 0, out=indptr[1:])
    rows, cols = torch.nonzero(nz, as_tuple=True)      # row-major, columns ascending
    return build_from_csr_tensors(indptr, cols.to(torch.int32), m[rows, cols], V, device, **kw)


def generate_synthetic_splade_data(num_docs: int, vocab_size: int = 30522,
                                   avg_terms_per_doc: int = 150,
                                   score_range: Tuple[float, float] = (0.1, 3.0),
                                   zipf_a: float = 1.5, seed: int = 42) -> Tuple[list, list]:
    """src/gpu_inverted_index.py:137-174: Zipf(zipf_a) terms without replacement,
    Poisson(avg) term counts floored at 10, uniform scores, numpy RandomState(seed)."""
    rng = np.random.RandomState(seed)
    ranks = np.arange(1, vocab_size + 1, dtype=np.float64)
    probs = 1.0 / np.power(ranks, zipf_a)
    probs /= probs.sum()
    ids, scs = [], []
    for _ in range(num_docs):
        n_terms = min(max(10, rng.poisson(avg_terms_per_doc)), vocab_size)
        terms = rng.choice(vocab_size, size=n_terms, replace=False, p=probs)
        scores = rng.uniform(score_range[0], score_range[1], size=n_terms).astype(np.float32)
        ids.append(terms.tolist())
        scs.append(scores.tolist())
    return ids, scs


def index_memory_stats(index: GPUInvertedIndex) -> dict:
    """src/gpu_inverted_index.py:177-196 (plus the quantised weights when present)."""
    def nbytes(t):
        return 0 if t is None else t.nelement() * t.element_size()
    doc_ids_bytes = nbytes(index.doc_ids)
    scores_bytes = nbytes(index.scores) + nbytes(index.weights_q) + nbytes(index.term_scale)
    meta_bytes = (nbytes(index.offsets) + nbytes(index.lengths) + nbytes(index.padded_lengths)
                  + nbytes(index.max_scores) + nbytes(index.block_starts)
                  + nbytes(getattr(index, "head_rows", None)) + nbytes(getattr(index, "head_lo", None)))
    n = int(index.lengths.sum().item())
    npad = int(index.padded_lengths.sum().item()) if index.padded_lengths is not None else n
    return {"doc_ids_MB": doc_ids_bytes / 1e6, "scores_MB": scores_bytes / 1e6,
            "metadata_MB": meta_bytes / 1e6,
            "total_MB": (doc_ids_bytes + scores_bytes + meta_bytes) / 1e6,
            "num_postings": n, "num_padded": npad,
            "padding_overhead": 1.0 - n / max(1, npad)}
