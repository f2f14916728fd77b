"""Threshold boards of the sharded scorer, exercised on one GPU with plain device arrays
in place of the IPC mappings: a shard that starts from another shard's published row
still merges into the exact corpus top-k, a shard writes only its own row (the same keys
into its board and its peers'), an absent bound changes nothing, and a bound above every
score empties the shard without a fault."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from parity import assert_bit_exact

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("shared_buffers_only")]
DEV = torch.device("cuda:0")
N, V, B = 60_000, 30522, 48


def u64(x: torch.Tensor) -> np.ndarray:
    return x.cpu().numpy().view(np.uint64)


def pack_keys(scores: np.ndarray, ids: np.ndarray) -> np.ndarray:
    """The scorer's packed keys: order-preserving score bits << 32 | (2^32 - 1 - doc id)."""
    b = (np.asarray(scores, dtype=np.float32) + np.float32(0)).view(np.uint32).astype(np.uint64)
    fk = np.where(b & 0x80000000, ~b & 0xFFFFFFFF, b | 0x80000000).astype(np.uint64)
    return (fk << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - ids.astype(np.uint64))


@pytest.fixture(scope="module")
def shards():
    from gpusparse import synth
    whole = synth.synth_index(N, V, seed=0, device=DEV)
    head = whole.head_ids
    a = synth.synth_index(N, V, seed=0, doc_range=(0, 33 * 1024), device=DEV, head_ids=head)
    b = synth.synth_index(N, V, seed=0, doc_range=(33 * 1024, N), device=DEV, head_ids=head)
    qi, qs = synth.synth_queries(B, V, seed=4, device=DEV)
    ip, ix, dt = O.synth_csr(N, V, seed=0)
    return a, b, qi, qs, O.build_index(ip, ix, dt, V), head.cpu().numpy()


@pytest.mark.parametrize("k", [10, 100, 1000])
def test_seeded_board_merges_to_exact_topk(shards, k):
    """Shard b (index 1 of 2) starts with shard a's row: a's ceil(k/2)-th best keys."""
    from gpusparse.scoring import merge_topk, score_topk
    a, b, qi, qs, oidx, head = shards
    c = -(-k // 2)
    _, _, ka = score_topk(a, qi, qs, k, with_keys=True)
    _, _, kb0 = score_topk(b, qi, qs, k, with_keys=True)
    board = torch.zeros((2, B), dtype=torch.int64, device=DEV)
    board[0] = ka[:, c - 1]
    seed = board[0].clone()
    peer = torch.zeros((2, B), dtype=torch.int64, device=DEV)
    sb, ib, kb = score_topk(b, qi, qs, k, with_keys=True, board=board, shard=1, peer_boards=[peer])
    s, i = merge_topk(torch.stack([ka, kb]), [k, k], k)
    rs, ri = O.score_topk(oidx, qi.cpu().numpy(), qs.cpu().numpy(), k, head=head)
    assert_bit_exact(s.cpu().numpy(), i.cpu().numpy(), rs, ri)
    # b wrote only its own row, the same into both boards, and only keys its keep list
    # reached; the bound (minimum over rows) stayed below the corpus k-th best key
    assert torch.equal(board[0], seed) and torch.equal(peer[0], torch.zeros_like(peer[0]))
    assert torch.equal(board[1], peer[1])
    row = u64(board[1])
    assert np.all(row <= u64(kb0[:, c - 1]))
    kth = pack_keys(rs[:, k - 1], ri[:, k - 1])
    assert np.all(np.minimum(u64(board[0]), row) <= kth)


@pytest.mark.parametrize("k", [10, 300])
def test_published_rows_without_a_bound_change_nothing(shards, k):
    """With the other shard's row still empty there is no bound: the result equals the
    plain call, and the shard's row (in its board and the peer's) holds, for every query,
    a key at most its ceil(k/2)-th best."""
    from gpusparse.scoring import score_topk
    a, b, qi, qs, _, _ = shards
    c = -(-k // 2)
    _, _, kb = score_topk(b, qi, qs, k, with_keys=True)
    board = torch.zeros((2, B), dtype=torch.int64, device=DEV)
    peers = [torch.zeros((2, B), dtype=torch.int64, device=DEV)]
    _, _, kb1 = score_topk(b, qi, qs, k, with_keys=True, board=board, shard=1, peer_boards=peers)
    assert torch.equal(kb1, kb)
    row = u64(board[1])
    assert np.all(row > 0)                           # every query compacted at least once
    assert np.all(row <= u64(kb[:, c - 1]))
    assert torch.equal(peers[0][1], board[1]) and not bool(board[0].any())


def test_board_above_every_score_empties_the_shard(shards):
    from gpusparse.scoring import score_topk
    a, b, qi, qs, _, _ = shards
    board = torch.full((2, B), -1, dtype=torch.int64, device=DEV)   # all ones: above every key
    peer = torch.zeros((2, B), dtype=torch.int64, device=DEV)
    s, i = score_topk(b, qi, qs, 100, board=board, shard=0, peer_boards=[peer])
    assert torch.all(i == -1)
    assert not torch.isnan(s).any()
