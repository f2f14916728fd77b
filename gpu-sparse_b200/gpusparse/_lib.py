"""ctypes binding of the C ABI declared in include/gpusparse.h.

Loading never falls back to anything: if libgpusparse.so is missing the import of an
entry point raises, and every status code other than GSP_OK raises the exception type the
reference raises in the same situation (ValueError for bad input or unsorted posting
lists, AssertionError for a non-power-of-two block_pl, RuntimeError otherwise).
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libgpusparse.so")

GSP_OK = 0
GSP_ERR_ARG = 1
GSP_ERR_UNSORTED = 2
GSP_ERR_OVERFLOW = 3
GSP_ERR_CUDA = 4
GSP_ERR_TIMEOUT = 5
GSP_ERR_UNSUPPORTED = 6
GSP_ERR_BLOCK_PL = 7

W_F32, W_BF16, W_U8 = 0, 1, 2
HEAD_AUTO, HEAD_CUDA_CORES, HEAD_TENSOR_CORES = 0, 1, 2   # gsp_set_head_mode
CHECK_WS_BYTES = 16     # GSP_CHECK_WS_BYTES

# every symbol include/gpusparse.h declares
EXPORTS = (
    "gsp_last_error", "gsp_version", "gsp_scan_i32", "gsp_scan_ws_bytes", "gsp_synth_nnz",
    "gsp_synth_fill", "gsp_index_ws_bytes", "gsp_index_count", "gsp_index_fill",
    "gsp_index_count_chunk", "gsp_index_count_finish", "gsp_index_fill_chunk",
    "gsp_index_fill_finish", "gsp_csr_dedup_count", "gsp_csr_dedup_fill",
    "gsp_index_quantize", "gsp_index_head_rows", "gsp_index_head_lo", "gsp_set_head_mode",
    "gsp_get_head_mode", "gsp_check_sorted", "gsp_chunk_bounds", "gsp_score_ws_bytes",
    "gsp_score_topk", "gsp_score_topk_noalloc", "gsp_score_topk_shared", "gsp_board_alloc",
    "gsp_board_free", "gsp_board_open", "gsp_board_close", "gsp_board_clear", "gsp_profile_enable", "gsp_profile_collect", "gsp_set_wait_limit", "gsp_get_wait_limit", "gsp_set_schedule_jitter", "gsp_get_schedule_jitter", "gsp_set_tree_limit", "gsp_get_tree_limit", "gsp_merge_ws_bytes", "gsp_merge_topk",
    "gsp_compacted_ws_bytes", "gsp_compacted_topk",
)


class IndexView(ctypes.Structure):
    """struct gsp_index_view"""
    _fields_ = [
        ("n_docs", ctypes.c_int64), ("doc_base", ctypes.c_int64), ("V", ctypes.c_int32),
        ("block_docs", ctypes.c_int32), ("wdtype", ctypes.c_int32), ("pad_", ctypes.c_int32),
        ("doc_ids", ctypes.c_void_p), ("weights", ctypes.c_void_p),
        ("term_scale", ctypes.c_void_p), ("offsets", ctypes.c_void_p),
        ("lengths", ctypes.c_void_p), ("block_starts", ctypes.c_void_p),
        ("n_head", ctypes.c_int32), ("head_wdtype", ctypes.c_int32), ("head_slot", ctypes.c_void_p),
        ("head_rows", ctypes.c_void_p), ("head_ld", ctypes.c_int64), ("head_lo", ctypes.c_void_p),
    ]


_lock = threading.Lock()
_lib = None


def lib_path() -> str:
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(_LIB_PATH):
            raise RuntimeError(
                f"libgpusparse.so is not built ({_LIB_PATH}); run __graft_entry__.build() or "
                "python -m gpusparse._build. There is no CPU fallback.")
        L = ctypes.CDLL(_LIB_PATH)
        i32, i64, u32, u64, p = (ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32,
                                 ctypes.c_uint64, ctypes.c_void_p)
        sig = {
            "gsp_last_error": (ctypes.c_char_p, []),
            "gsp_version": (ctypes.c_int, []),
            "gsp_scan_i32": (ctypes.c_int, [p, i64, p, p, i64, p]),
            "gsp_scan_ws_bytes": (i64, [i64]),
            "gsp_synth_nnz": (ctypes.c_int, [u64, u32, u64, i64, i32, p, i32, i32, i32, p, p]),
            "gsp_synth_fill": (ctypes.c_int, [u64, u32, u64, i64, i32, p, p, p, p, p, p, p]),
            "gsp_index_ws_bytes": (i64, [i64, i32, i32]),
            "gsp_index_count": (ctypes.c_int, [i64, i32, i32, p, p, p, p, p, p,
                                               ctypes.POINTER(i64), p, i64, p]),
            "gsp_index_fill": (ctypes.c_int, [i64, i32, i32, p, p, p, p, p, p, i64, p, p, p, p,
                                              i64, p]),
            "gsp_index_count_chunk": (ctypes.c_int, [i64, i32, i32, i64, i64, p, p, p, p, i64,
                                                     p]),
            "gsp_index_count_finish": (ctypes.c_int, [i64, i32, i32, p, p, p, p,
                                                      ctypes.POINTER(i64), p, i64, p]),
            "gsp_index_fill_chunk": (ctypes.c_int, [i64, i32, i32, i64, i64, p, p, p, p, p, p, p,
                                                    p, i64, p]),
            "gsp_index_fill_finish": (ctypes.c_int, [i64, i32, p, p, p, p, p, p, i64, p]),
            "gsp_csr_dedup_count": (ctypes.c_int, [i64, i32, p, p, p, ctypes.POINTER(i64), p, i64, p]),
            "gsp_csr_dedup_fill": (ctypes.c_int, [i64, p, p, p, p, p, p, p]),
            "gsp_index_quantize": (ctypes.c_int, [i32, i64, p, p, p, p, i32, p, p, p]),
            "gsp_index_head_rows": (ctypes.c_int, [i32, p, p, p, p, p, i32, i64, p, p]),
            "gsp_index_head_lo": (ctypes.c_int, [i64, p, p, p]),
            "gsp_set_head_mode": (ctypes.c_int, [i32]),
            "gsp_get_head_mode": (i32, []),
            "gsp_check_sorted": (ctypes.c_int, [i32, p, p, p, ctypes.POINTER(i64),
                                                ctypes.POINTER(i64), p, i64, p]),
            "gsp_chunk_bounds": (ctypes.c_int, [i64, i32, i64, p, p, p, p, p, i64, p]),
            "gsp_score_ws_bytes": (i64, [ctypes.POINTER(IndexView), i64, i64, i64]),
            "gsp_score_topk": (ctypes.c_int, [ctypes.POINTER(IndexView), p, p, i64, i64, i64, p,
                                              p, p, p, i64, p]),
            "gsp_score_topk_noalloc": (ctypes.c_int, [ctypes.POINTER(IndexView), p, p, i64, i64,
                                                      i64, p, p, p, p]),
            "gsp_score_topk_shared": (ctypes.c_int, [ctypes.POINTER(IndexView), p, p, i64, i64,
                                                     i64, p, p, p, p, i64, p, i32, i32, p, p]),
            "gsp_board_alloc": (ctypes.c_int, [i64, ctypes.POINTER(p), p]),
            "gsp_board_free": (ctypes.c_int, [p]),
            "gsp_board_open": (ctypes.c_int, [p, ctypes.POINTER(p)]),
            "gsp_board_close": (ctypes.c_int, [p]),
            "gsp_board_clear": (ctypes.c_int, [p, i64, p]),
            "gsp_profile_enable": (ctypes.c_int, [ctypes.c_int]),
            "gsp_set_wait_limit": (ctypes.c_int, [ctypes.c_int32]),
            "gsp_get_wait_limit": (ctypes.c_int32, []),
            "gsp_set_schedule_jitter": (ctypes.c_int, [ctypes.c_int32]),
            "gsp_get_schedule_jitter": (ctypes.c_int32, []),
            "gsp_set_tree_limit": (ctypes.c_int, [i64]),
            "gsp_get_tree_limit": (i64, []),
            "gsp_profile_collect": (ctypes.c_int, [ctypes.POINTER(ctypes.c_double),
                                                   ctypes.POINTER(i64)]),
            "gsp_merge_ws_bytes": (i64, [i64, i64]),
            "gsp_merge_topk": (ctypes.c_int, [p, i64, i64, i64, i64, p, i64, p, p, p, p, i64, p]),
            "gsp_compacted_ws_bytes": (i64, [i64, i64, i64, i64]),
            "gsp_compacted_topk": (ctypes.c_int, [p, i64, i64, i64, p, i64, i64, p, p, p, i64,
                                                  p]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
        return L


def check(rc: int, what: str) -> None:
    if rc == GSP_OK:
        return
    msg = lib().gsp_last_error().decode(errors="replace")
    text = f"{what}: {msg}"
    if rc in (GSP_ERR_ARG, GSP_ERR_UNSORTED):
        raise ValueError(text)
    if rc == GSP_ERR_BLOCK_PL:
        raise AssertionError(text)
    raise RuntimeError(text)


def ptr(t: torch.Tensor | None):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def stream_of(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (GPUSparse has no CPU path)")


def workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)
