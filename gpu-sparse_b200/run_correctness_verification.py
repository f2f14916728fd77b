"""Module-name shim for the helpers callers import from the reference's
src/run_correctness_verification.py (:32 build_gpu_index_from_csr, :87
prepare_queries_from_meta, :110 compute_recall_exact)."""
import numpy as np
import torch

from gpusparse.index import VOCAB_SIZE, build_gpu_index_from_csr  # noqa: F401


def prepare_queries_from_meta(meta, max_terms=128, device="cuda:0"):
    """Query tensors [nq, max_terms] from a dense query matrix, terms sorted by
    descending weight and truncated to max_terms (the reference's :87-107)."""
    query_dense = meta["query_dense"]
    if isinstance(query_dense, torch.Tensor):
        query_dense = query_dense.numpy()
    n = query_dense.shape[0]
    term_ids = np.full((n, max_terms), -1, dtype=np.int32)
    term_scores = np.zeros((n, max_terms), dtype=np.float32)
    for i in range(n):
        nz = np.nonzero(query_dense[i])[0]
        vals = query_dense[i, nz]
        order = np.argsort(-vals)[:max_terms]
        term_ids[i, :len(order)] = nz[order]
        term_scores[i, :len(order)] = vals[order]
    return (torch.from_numpy(term_ids).to(device), torch.from_numpy(term_scores).to(device),
            query_dense)


def compute_recall_exact(gpu_ids, cpu_ids, k_values=(10, 100, 1000)):
    """Set recall of gpu_ids against cpu_ids at each k (the reference's :110-125)."""
    out = {}
    for k in k_values:
        if k > gpu_ids.shape[1] or k > cpu_ids.shape[1]:
            continue
        hit = tot = 0
        for q in range(gpu_ids.shape[0]):
            gt = set(cpu_ids[q, :k].tolist())
            hit += len(gt & set(gpu_ids[q, :k].tolist()))
            tot += len(gt)
        out[f"recall@{k}"] = hit / tot if tot else 0.0
    return out
