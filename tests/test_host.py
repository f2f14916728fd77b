"""Host-side logic that needs no GPU: the C ABI library loads and exports every declared
symbol, reference argument validation, plug-in helpers, shard layout, key decoding and
the synthetic generator's law."""
import ctypes
import json
import os
import re

import numpy as np
import pytest
import torch

from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden")


def header_symbols():
    txt = open(os.path.join(ROOT, "include", "gpusparse.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(gsp_[a-z0-9_]+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    import gpusparse._lib as L
    lib = L.lib()
    syms = header_symbols()
    assert syms, "no declarations parsed"
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(L.EXPORTS)
    assert lib.gsp_version() == 1


def test_no_cpu_fallback():
    import gpusparse
    with pytest.raises(RuntimeError):
        gpusparse.build_from_csr_tensors(torch.zeros(2, dtype=torch.int64),
                                         torch.zeros(0, dtype=torch.int32),
                                         torch.zeros(0), 10, device="cpu")


@pytest.mark.parametrize("bad", [0, -4, 3, 96])
def test_block_pl_must_be_power_of_two(bad):
    import gpusparse
    with pytest.raises(AssertionError):
        gpusparse.triton_fused_score(None, None, None, top_k=10, block_pl=bad)
    with pytest.raises(AssertionError):
        gpusparse.triton_chunked_score(None, None, None, block_pl=bad)
    with pytest.raises(AssertionError):
        gpusparse.triton_chunked_score_fused(None, None, None, block_pl=bad)


def test_plugin_helpers_match_reference():
    meta = json.load(open(os.path.join(GOLD, "reference_meta.json")))["plugin"]
    from lsr_benchmark_engine import gpusparse_retrieval as P
    d_emb = [tuple(x) for x in meta["d_emb"]]
    q_emb = [tuple(x) for x in meta["q_emb"]]
    dim = P.determine_dimension(d_emb, q_emb)
    assert dim == meta["dim"]
    qids, qcsr = P.to_csr(q_emb, dim)
    ti, ts, mx = P.to_query_tensors(qcsr, "cpu")
    assert mx == meta["max_nnz"]
    assert ti.tolist() == meta["ti"] and ts.tolist() == meta["ts"]


def test_shard_layout_and_counts():
    from gpusparse.distributed import ShardLayout
    for N, G in [(10, 3), (8_800_000, 8), (5, 8)]:
        sizes = ShardLayout(N, G, 0).sizes()
        assert sum(sizes) == N and max(sizes) - min(sizes) <= 1
        lo = [ShardLayout(N, G, r).lo for r in range(G)]
        assert lo == sorted(lo) and lo[0] == 0
        assert ShardLayout(N, G, G - 1).hi == N
    lay = ShardLayout(5, 8, 0)
    assert lay.sizes() == [0, 1, 0, 1, 1, 0, 1, 1]
    assert lay.list_counts(3) == [0, 1, 0, 1, 1, 0, 1, 1]
    assert ShardLayout(100, 2, 1).list_counts(30) == [30, 30]


def test_key_packing_orders_like_reference_ranking():
    from gpusparse.distributed import decode_keys
    rng = np.random.default_rng(3)
    s = rng.standard_normal(500).astype(np.float32)
    s[::7] = 0.0
    s[1::11] = s[0]
    d = rng.permutation(500).astype(np.uint64)
    keys = (O.fkey(s).astype(np.uint64) << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - d)
    order = np.argsort(keys)[::-1]
    ref = np.lexsort((d, -s.astype(np.float64)))
    assert np.array_equal(order, ref)
    ds, di = decode_keys(torch.from_numpy(keys.view(np.int64)))
    assert np.array_equal(ds.numpy(), s) and np.array_equal(di.numpy(), d.astype(np.int64))


def test_generator_law_and_range_independence():
    ip, ix, dt = O.synth_csr(4000, seed=11)
    nnz = np.diff(ip)
    assert 20 <= nnz.min() and nnz.max() <= 600 and 170 < nnz.mean() < 190
    assert 0.11 < (dt == 0).mean() < 0.14                  # P(N(0.8,0.7) < 0) = 0.1265
    for r in range(0, 4000, 997):                          # distinct terms per document
        row = ix[ip[r]:ip[r + 1]]
        assert len(np.unique(row)) == len(row)
    a = O.synth_csr(1500, seed=11, first=2500)             # any item range on its own
    assert np.array_equal(a[1], ix[ip[2500]:]) and np.array_equal(a[2], dt[ip[2500]:])
    qi, qs = O.synth_queries(300, seed=2)
    n = (qi >= 0).sum(1)
    assert n[0] >= 107 and 5 <= n.min() and n.max() <= 128 and 25 < n.mean() < 35


def test_oracle_quantisation_roundtrip():
    ip, ix, dt = O.synth_csr(500, seed=4)
    idx = O.build_index(ip, ix, dt, 30522)
    q, scale = O.quantize_u8(idx)
    w = O.dequantize_u8(q, scale, idx.offsets, idx.lengths, idx.padded_lengths)
    real = idx.doc_ids >= 0
    err = np.abs(w[real] - idx.scores[real])
    term_of = np.repeat(np.arange(30522), idx.padded_lengths)[real]
    assert np.all(err <= scale[term_of] * 0.5 + 1e-7)


def test_plugin_retrieve_pipeline_with_a_stand_in_scorer(monkeypatch):
    """The plug-in's batch pipeline (score batch i+1 while batch i is formatted) on the CPU
    with a stand-in scorer: batches are collected in order, rows keep the scorer's order,
    scores <= 0 are dropped and doc ids are mapped to the caller's names."""
    import torch
    from lsr_benchmark_engine import gpusparse_retrieval as P

    class Idx:
        num_docs = 50

    def fake_score(index, qi, qs, top_k=10, block_pl=128):
        B = qi.shape[0]
        base = qi[:, 0].to(torch.float32)                 # row identity from the query
        s = base[:, None] - torch.arange(top_k, dtype=torch.float32)[None, :]
        ids = (qi[:, :1].long() + torch.arange(top_k)[None, :]) % Idx.num_docs
        return s, ids

    class Ev:
        def record(self, stream=None):
            pass

        def synchronize(self):
            pass

    monkeypatch.setattr(P, "triton_fused_score", fake_score)
    monkeypatch.setattr(P.torch.cuda, "Event", lambda *a, **k: Ev())
    monkeypatch.setattr(P.torch.cuda, "current_stream", lambda *a, **k: None)
    monkeypatch.setattr(P.torch.cuda, "is_available", lambda: False)
    n = 23
    qi = torch.arange(n, dtype=torch.int32)[:, None].repeat(1, 3)
    qs = torch.ones((n, 3))
    names = [f"doc{d}" for d in range(Idx.num_docs)]
    res = P.retrieve(Idx(), [f"q{j}" for j in range(n)], qi, qs, names, k=5, batch_size=4)
    assert len(res) == n
    for j, row in enumerate(res):
        exp = [(f"q{j}", float(j - r), f"doc{(j + r) % 50}") for r in range(5) if j - r > 0]
        assert row == exp


def test_index_view_layout_matches_the_header(tmp_path):
    """gsp_index_view as the C compiler lays it out (sizeof, offsetof) equals the ctypes
    binding's layout, so a caller of the C ABI and the Python wrapper agree."""
    import ctypes
    import shutil
    import subprocess
    import gpusparse._lib as L
    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    inc = os.path.join(ROOT, "include")
    names = [f[0] for f in L.IndexView._fields_]
    src = tmp_path / "layout.c"
    src.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "gpusparse.h"\nint main(void) {\n'
                   '  printf("size %zu\\n", sizeof(gsp_index_view));\n'
                   + "".join(f'  printf("{n} %zu\\n", offsetof(gsp_index_view, {n}));\n' for n in names)
                   + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.check_call(["gcc", "-I", inc, str(src), "-o", str(exe)])
    got = dict(line.split() for line in subprocess.check_output([str(exe)], text=True).splitlines())
    assert int(got["size"]) == ctypes.sizeof(L.IndexView)
    for n in names:
        assert int(got[n]) == getattr(L.IndexView, n).offset, n


def test_streamed_build_chunk_arguments_are_checked_on_the_host():
    """A chunk must be a run of whole blocks inside the corpus and the workspace large
    enough; these calls fail their argument checks before any device work (the pointers
    they get are never dereferenced)."""
    import gpusparse._lib as L
    lib = L.lib()
    N, V, bd = 5000, 30522, 1024
    need = int(lib.gsp_index_ws_bytes(N, V, bd))
    ws = ctypes.create_string_buffer(need)
    fake = ctypes.c_void_p(256)
    for first, n, ws_bytes in [(100, 1024, need), (1024, 1000, need), (4096, 1000, need),
                               (0, 1024, 8), (-1024, 1024, need)]:
        rc = lib.gsp_index_count_chunk(N, V, bd, first, n, fake, fake, fake, ws, ws_bytes, None)
        assert rc == L.GSP_ERR_ARG, (first, n, ws_bytes)
        rc = lib.gsp_index_fill_chunk(N, V, bd, first, n, fake, fake, fake, fake, fake, fake,
                                      fake, ws, ws_bytes, None)
        assert rc == L.GSP_ERR_ARG, (first, n, ws_bytes)
    assert b"whole" in lib.gsp_last_error() or b"workspace" in lib.gsp_last_error()


def test_tree_limit_knob_round_trips_on_the_host():
    """The small-batch mode's size limit is a process-wide host setting (no device work)."""
    import gpusparse._lib as L
    lib = L.lib()
    default = lib.gsp_get_tree_limit()
    assert default == 256 << 20
    try:
        assert lib.gsp_set_tree_limit(0) == L.GSP_OK and lib.gsp_get_tree_limit() == 0
        assert lib.gsp_set_tree_limit(-1) == L.GSP_ERR_ARG
    finally:
        lib.gsp_set_tree_limit(default)
    assert lib.gsp_get_tree_limit() == default


def test_small_batch_mode_is_chosen_by_the_documented_rules():
    """Workspace sizing (host-only) includes the per-tile lists exactly when the
    small-batch mode applies: 256 <= k' <= 1024, at most 24576 query-tiles, lists within
    the size limit."""
    import ctypes
    import gpusparse._lib as L
    lib = L.lib()
    v = L.IndexView()
    v.n_docs, v.V, v.block_docs, v.wdtype, v.n_head = 8_800_000, 30522, 1024, 0, 0
    tiles = (v.n_docs + 1023) // 1024

    def ws(B, k):
        n = lib.gsp_score_ws_bytes(ctypes.byref(v), B, 128, k)
        assert n > 0, lib.gsp_last_error()
        return n

    lists = lambda B, k: B * tiles * k * 8  # noqa: E731
    assert ws(1, 1000) >= lists(1, 1000)            # one query, k = 1000: tree
    assert ws(2, 1000) >= lists(2, 1000)            # 17 188 query-tiles: tree
    assert ws(4, 1000) < lists(4, 1000)             # 34 376 query-tiles: shared buffers
    assert ws(1, 255) < lists(1, 255)               # k' below 256: shared buffers
    assert ws(1, 2000) < lists(1, 1024)             # k' above one tile: shared buffers
    default = lib.gsp_get_tree_limit()
    try:
        L.check(lib.gsp_set_tree_limit(lists(1, 1000) - 1), "tree limit")
        assert ws(1, 1000) < lists(1, 1000)         # lists above the limit: shared buffers
    finally:
        lib.gsp_set_tree_limit(default)


def test_shared_scoring_and_board_arguments_are_checked_on_the_host():
    """Bad shard arguments and bad board calls fail their checks before any device work
    (the pointers below are never dereferenced)."""
    import ctypes
    import gpusparse._lib as L
    lib = L.lib()
    fake = ctypes.c_void_p(256)
    v = L.IndexView()
    v.n_docs, v.V, v.block_docs, v.wdtype, v.n_head = 5000, 30522, 1024, 0, 0
    for f in ("doc_ids", "weights", "offsets", "lengths", "block_starts"):
        setattr(v, f, 256)
    B, W, k = 4, 8, 10
    nb = lib.gsp_score_ws_bytes(ctypes.byref(v), B, W, k)
    ws = ctypes.create_string_buffer(int(nb))
    peers = (ctypes.c_void_p * 9)(*([256] * 9))
    for board, shard, n_shards in [(fake, 0, 10), (fake, 2, 2), (fake, -1, 2),
                                   (ctypes.c_void_p(0), 0, 2)]:
        rc = lib.gsp_score_topk_shared(ctypes.byref(v), fake, fake, B, W, k, fake, fake, None, ws,
                                       nb, board, shard, n_shards, peers, None)
        assert rc == L.GSP_ERR_ARG, (shard, n_shards)
    out = ctypes.c_void_p()
    assert lib.gsp_board_alloc(0, ctypes.byref(out), None) == L.GSP_ERR_ARG
    assert lib.gsp_board_clear(None, 4, None) == L.GSP_ERR_ARG
    assert lib.gsp_board_open(None, ctypes.byref(out)) == L.GSP_ERR_ARG


def test_run_file_is_the_reference_text(tmp_path):
    """write_run produces the reference's TREC lines ("qid Q0 docno rank score gpusparse",
    ranks from 1, Python's float text) in a gzip stream any reader accepts."""
    import gzip
    from lsr_benchmark_engine import gpusparse_retrieval as P
    results = [[("q1", 3.5, "d7"), ("q1", 1.25, "d2")], [], [("q2", 0.1 + 0.2, "d0")]]
    P.write_run(results, tmp_path / "run.txt.gz")
    lines = gzip.open(tmp_path / "run.txt.gz", "rt").read().splitlines()
    assert lines == ["q1 Q0 d7 1 3.5 gpusparse", "q1 Q0 d2 2 1.25 gpusparse",
                     f"q2 Q0 d0 1 {0.1 + 0.2} gpusparse"]
