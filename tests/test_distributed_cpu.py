"""The multi-GPU exchange on CPU ranks (gloo, world size 2): each rank scores its
doc-range shard with the oracle, packs its local top-k into keys, the real
gather_candidates collective moves them, and merging the gathered keys reproduces the
oracle's unsharded top-k exactly.  (On GPUs the local scorer and the merge are the CUDA
kernels; the collective and the bookkeeping are this code.)"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

N, V, B, K = 3000, 30522, 12, 200


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _keys(s, ids):
    from oracle import oracle as O
    return ((O.fkey(s).astype(np.uint64) << np.uint64(32))
            | (np.uint64(0xFFFFFFFF) - ids.astype(np.uint64))).view(np.int64)


def _worker(rank, world, port, out_path):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "gpu-sparse_b200")]
    from oracle import oracle as O
    from gpusparse.distributed import ShardLayout, gather_candidates
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        lay = ShardLayout(N, world, rank)
        ip, ix, dt = O.synth_csr(lay.hi - lay.lo, V, seed=0, first=lay.lo)
        idx = O.build_index(ip, ix, dt, V)
        qi, qs = O.synth_queries(B, V, seed=1)
        s, i = O.score_topk(idx, qi, qs, K, id_base=lay.lo, nthreads=2)
        allk = gather_candidates(torch.from_numpy(_keys(s, i)), K)
        if rank == 0:
            np.save(out_path, allk.numpy())
            np.save(out_path + ".counts.npy", np.array(lay.list_counts(K)))
    finally:
        dist.destroy_process_group()


def test_gather_and_merge_equals_unsharded(tmp_path):
    from oracle import oracle as O
    out = str(tmp_path / "keys.npy")
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    allk = np.load(out).view(np.uint64)               # [world, B, K]
    counts = np.load(out + ".counts.npy")
    assert allk.shape == (2, B, K)
    merged = np.empty((B, K), dtype=np.uint64)
    for b in range(B):
        cand = np.concatenate([allk[r, b, :counts[r]] for r in range(2)])
        merged[b] = np.sort(cand)[::-1][:K]
    ip, ix, dt = O.synth_csr(N, V, seed=0)
    idx = O.build_index(ip, ix, dt, V)
    qi, qs = O.synth_queries(B, V, seed=1)
    s, i = O.score_topk(idx, qi, qs, K)
    assert np.array_equal(merged, _keys(s, i).view(np.uint64))


def test_gather_pads_short_shards():
    """A shard with fewer than k documents contributes min(k, size) keys (zero padded)."""
    from gpusparse.distributed import ShardLayout
    lay = ShardLayout(150, 2, 0)
    assert lay.list_counts(100) == [75, 75]
    assert ShardLayout(150, 2, 0).list_counts(50) == [50, 50]


def _worker_blocks(rank, world, port, out_path):
    """Like _worker, through the query-block exchange: all_to_all of the candidate keys,
    a merge of this rank's block (numpy here, the CUDA merge kernel on GPUs), and the
    all-gather of the merged results."""
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "gpu-sparse_b200")]
    from oracle import oracle as O
    from gpusparse.distributed import ShardLayout, exchange_candidates, gather_results
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        lay = ShardLayout(N, world, rank)
        ip, ix, dt = O.synth_csr(lay.hi - lay.lo, V, seed=0, first=lay.lo)
        idx = O.build_index(ip, ix, dt, V)
        Bq = B - 1                                   # not a multiple of the world size
        qi, qs = O.synth_queries(Bq, V, seed=1)
        s, i = O.score_topk(idx, qi, qs, K, id_base=lay.lo, nthreads=2)
        blk = exchange_candidates(torch.from_numpy(_keys(s, i)), K).numpy().view(np.uint64)
        counts = lay.list_counts(K)
        ms = np.empty((blk.shape[1], K), dtype=np.uint64)
        for b in range(blk.shape[1]):
            cand = np.concatenate([blk[r, b, :counts[r]] for r in range(world)])
            ms[b] = np.sort(cand)[::-1][:K]
        gs, gi = gather_results(torch.from_numpy(ms.view(np.int64)), torch.from_numpy(ms.view(np.int64)), Bq)
        if rank == 0:
            np.save(out_path, gs.numpy())
    finally:
        dist.destroy_process_group()


def test_query_block_exchange_and_merge_equals_unsharded(tmp_path):
    from oracle import oracle as O
    out = str(tmp_path / "blocks.npy")
    mp.start_processes(_worker_blocks, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    got = np.load(out).view(np.uint64)
    ip, ix, dt = O.synth_csr(N, V, seed=0)
    idx = O.build_index(ip, ix, dt, V)
    qi, qs = O.synth_queries(B - 1, V, seed=1)
    s, i = O.score_topk(idx, qi, qs, K)
    assert got.shape == (B - 1, K)
    assert np.array_equal(got, _keys(s, i).view(np.uint64))
