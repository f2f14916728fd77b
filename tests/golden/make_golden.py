"""Regenerate the golden fixtures in this directory from the GPUSparse reference itself.

Run in a container that has the reference checkout (read-only) and Triton; the
reference's Triton kernels execute on CPU tensors under TRITON_INTERPRET=1:

    GPUSPARSE_REF=/path/to/gpu-sparse python tests/golden/make_golden.py

Inputs are the seeded synthetic corpus and queries of ``oracle/oracle.py`` (the
fixtures store the sha256 of the generated CSR so the tests can prove they rebuild
exactly the inputs the reference saw).  Outputs recorded per case:

* ``build_gpu_index_from_csr`` (src/run_correctness_verification.py:32-84) and the
  plug-in ``build_index`` (lsr_benchmark_engine/gpusparse_retrieval.py:81-115):
  sha256 of every index array, plus the full arrays for the smallest corpus;
* ``triton_fused_score`` (src/triton_kernel.py:159-200) at k = 10 / 100 / 1000;
* ``triton_chunked_score`` (src/triton_kernel_chunked.py:125-170) and
  ``triton_chunked_score_fused`` (src/fused_topk.py:106-160) with small doc chunks so
  several chunks, the running merge and the compaction path all run;
* ``build_chunk_boundaries`` (src/triton_kernel_chunked.py:83-122);
* ``compacted_topk`` (src/fused_topk.py:71-103), including an overflowing row;
* the plug-in helpers ``to_csr``, ``determine_dimension``, ``to_query_tensors`` and
  ``retrieve`` (lsr_benchmark_engine/gpusparse_retrieval.py:56-172) with stub modules
  standing in for its absent third-party imports.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402
import scipy.sparse as sp  # noqa: E402
import torch  # noqa: E402

from oracle import oracle as O  # noqa: E402

REF = os.environ.get("GPUSPARSE_REF", "")


def sha(*arrs) -> str:
    h = hashlib.sha256()
    for a in arrs:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode()); h.update(str(a.shape).encode()); h.update(a.tobytes())
    return h.hexdigest()


def import_reference():
    if not REF or not os.path.isdir(os.path.join(REF, "src")):
        raise SystemExit("set GPUSPARSE_REF to the reference checkout (the directory holding src/)")
    sys.path.insert(0, os.path.join(REF, "src"))
    sys.path.insert(0, REF)
    import triton_kernel, triton_kernel_chunked, fused_topk  # noqa: E401
    from src.run_correctness_verification import build_gpu_index_from_csr
    # stubs for the plug-in's third-party imports (not part of the scoring path)
    tt = types.ModuleType("tirex_tracker")
    tt.ExportFormat = types.SimpleNamespace(IR_METADATA="ir_metadata")
    tt.register_metadata = lambda *a, **k: None
    class _T:  # noqa: E306
        def __init__(self, *a, **k): pass
        def __enter__(self): return self
        def __exit__(self, *a): return False
    tt.tracking = _T
    lb = types.ModuleType("lsr_benchmark")
    lb.register_to_ir_datasets = lambda *a, **k: None
    lbc = types.ModuleType("lsr_benchmark.click")
    lbc.retrieve_command = lambda *a, **k: (lambda f: f)
    lbi = types.ModuleType("lsr_benchmark.irds")
    lbi.embeddings = lambda *a, **k: []
    lb.click, lb.irds = lbc, lbi
    for name, mod in [("tirex_tracker", tt), ("lsr_benchmark", lb), ("lsr_benchmark.click", lbc),
                      ("lsr_benchmark.irds", lbi)]:
        sys.modules[name] = mod
    os.environ["GPUSPARSE_SRC"] = os.path.join(REF, "src")
    sys.path.insert(0, os.path.join(REF, "lsr_benchmark_engine"))
    import gpusparse_retrieval as plug
    return triton_kernel, triton_kernel_chunked, fused_topk, build_gpu_index_from_csr, plug


def index_arrays(idx, fields=("doc_ids", "scores", "offsets", "lengths", "padded_lengths",
                              "max_scores")):
    return {f: getattr(idx, f).cpu().numpy() for f in fields if hasattr(idx, f)}


def main():
    tk, tkc, ftk, build_ref, plug = import_reference()
    out: dict[str, np.ndarray] = {}
    meta: dict = {"reference": "ashutoshuiuc/gpu-sparse", "generator": "oracle/oracle.py synth v1",
                  "cases": {}}
    V = 30522

    # ---------------- corpus A: 2000 docs, full vocabulary (the reference hard-codes V)
    N = 2000
    ip, ix, dt = O.synth_csr(N, V, seed=0)
    csr = sp.csr_matrix((dt, ix, ip), shape=(N, V))
    qi, qs = O.synth_queries(16, V, seed=1)
    # edge rows: out-of-range ids, duplicated term, all padding, one term
    qi_e = np.full((4, qi.shape[1]), -1, dtype=np.int32)
    qs_e = np.zeros_like(qs[:4])
    qi_e[0, :4] = [3, V + 5, 7, 2 * V]; qs_e[0, :4] = [0.5, 9.0, 1.25, 3.0]
    qi_e[1, :3] = [11, 11, 0]; qs_e[1, :3] = [0.75, 0.25, 0.125]
    qi_e[3, :1] = [1]; qs_e[3, :1] = [2.0]
    qi_all = np.concatenate([qi, qi_e]); qs_all = np.concatenate([qs, qs_e])
    meta["cases"]["A"] = {"N": N, "V": V, "doc_seed": 0, "query_seed": 1, "B": 16,
                          "csr_sha256": sha(ip, ix, dt), "queries_sha256": sha(qi, qs)}
    out["A_qi"], out["A_qs"] = qi_all, qs_all

    idx = build_ref(csr, "cpu")
    arrs = index_arrays(idx)
    meta["cases"]["A"]["index_sha256"] = {k: sha(v) for k, v in arrs.items()}
    pidx = plug.build_index(csr, "cpu")
    meta["cases"]["A"]["plugin_index_sha256"] = {
        k: sha(v) for k, v in index_arrays(pidx, ("doc_ids", "scores", "offsets", "lengths")).items()}

    tqi, tqs = torch.from_numpy(qi_all), torch.from_numpy(qs_all)
    for k in (10, 100, 1000):
        s, i = tk.triton_fused_score(idx, tqi, tqs, top_k=k)
        out[f"A_fused_k{k}_s"], out[f"A_fused_k{k}_i"] = s.numpy(), i.numpy()
    for dc in (256, 700):
        b = tkc.build_chunk_boundaries(idx, dc)
        out[f"A_bounds_{dc}"] = b.numpy()
        s, i = tkc.triton_chunked_score(idx, tqi, tqs, top_k=100, doc_chunk=dc, chunk_bounds=b)
        out[f"A_chunked_{dc}_s"], out[f"A_chunked_{dc}_i"] = s.numpy(), i.numpy()
        s, i = ftk.triton_chunked_score_fused(idx, tqi, tqs, top_k=100, doc_chunk=dc,
                                              chunk_bounds=b, max_cand=64)
        out[f"A_cfused_{dc}_s"], out[f"A_cfused_{dc}_i"] = s.numpy(), i.numpy()

    # ---------------- corpus B: 120 docs, small vocabulary, full index arrays stored
    Nb, Vb = 120, 300
    ipb, ixb, dtb = O.synth_csr(Nb, Vb, seed=5, law=O.Law(nnz_mean=12.0, nnz_sd=6.0, nnz_lo=2,
                                                          nnz_hi=40))
    csrb = sp.csr_matrix((dtb, ixb, ipb), shape=(Nb, Vb))
    out["B_indptr"], out["B_indices"], out["B_data"] = ipb, ixb, dtb
    sys.modules["src.run_correctness_verification"].VOCAB_SIZE = Vb
    idxb = build_ref(csrb, "cpu")
    sys.modules["src.run_correctness_verification"].VOCAB_SIZE = V
    for k, v in index_arrays(idxb).items():
        out[f"B_index_{k}"] = v
    qib, qsb = O.synth_queries(6, Vb, seed=6, law=O.Law(nnz_mean=5.0, nnz_sd=2.0, nnz_lo=1,
                                                        nnz_hi=12))
    out["B_qi"], out["B_qs"] = qib, qsb
    s, i = tk.triton_fused_score(idxb, torch.from_numpy(qib), torch.from_numpy(qsb), top_k=500)
    out["B_fused_k500_s"], out["B_fused_k500_i"] = s.numpy(), i.numpy()   # k > N -> k = N
    meta["cases"]["B"] = {"N": Nb, "V": Vb, "doc_seed": 5, "query_seed": 6}

    # ---------------- compacted_topk on a dense matrix, one row overflowing max_cand
    rng = np.random.default_rng(7)
    S = rng.standard_normal((5, 3000)).astype(np.float32)
    S[2, :] = np.round(S[2, :], 1)          # many exact ties
    tau = np.array([1.5, 0.5, 0.0, 3.5, -10.0], dtype=np.float32)
    v, ii = ftk.compacted_topk(torch.from_numpy(S), torch.from_numpy(tau), 50, max_cand=256,
                               block=128)
    out["C_S"], out["C_tau"], out["C_v"], out["C_i"] = S, tau, v.numpy(), ii.numpy()

    # ---------------- plug-in helpers on a handful of embeddings
    d_emb = [("d0", [3, 5, 9], [0.5, 1.0, 2.0]), ("d1", [5, 9], [1.5, 0.25]),
             ("d2", [], []), ("d3", [1, 3, 12], [0.75, 0.5, 0.125])]
    q_emb = [("q0", [5, 3], [1.0, 2.0]), ("q1", [12], [1.0]), ("q2", [7], [1.0])]
    dim = plug.determine_dimension(d_emb, q_emb)
    dids, dcsr = plug.to_csr(d_emb, dim)
    qids, qcsr = plug.to_csr(q_emb, dim)
    pidx = plug.build_index(dcsr, "cpu")
    ti, ts, mx = plug.to_query_tensors(qcsr, "cpu")
    res = plug.retrieve(pidx, qids, ti, ts, dids, k=3)
    meta["plugin"] = {"dim": dim, "max_nnz": mx, "ti": ti.numpy().tolist(),
                      "ts": ts.numpy().tolist(),
                      "retrieve_k3": [[[q, float(s), d] for q, s, d in r] for r in res],
                      "d_emb": d_emb, "q_emb": q_emb}

    np.savez_compressed(os.path.join(HERE, "reference_outputs.npz"), **out)
    with open(os.path.join(HERE, "reference_meta.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()
