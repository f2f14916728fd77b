"""Doc-range sharded scoring across the GPUs of one node.

One process per GPU (torchrun), NCCL over NVLink/NVSwitch.  Rank r holds the index of
documents [r*N/G, (r+1)*N/G) with local ids and doc_base = r*N/G, scores the full query
batch against it and keeps its exact local top-k as packed uint64 keys
(fkey(score) << 32 | ~global doc id).  The batch is split into G blocks of queries: one
all_to_all_single sends rank r every rank's keys of block r (B*k*8/G bytes per pair), the
GPU merge kernel reduces the G*k candidates of each of its B/G queries to the exact
global top-k (ties -> lower global doc id), and one all_gather per output (scores, ids)
gives every rank the whole result -- each rank merges 1/G of the batch and receives
about 1/G of what an all-gather of every candidate list would move.

While the shards score, they share a threshold: every rank has a board of G rows (one key
per query and shard, CUDA IPC-mapped into the other ranks).  After each compaction a
shard writes into its row of every board, with remote atomics over NVLink, a key that at
least ceil(k/G) of its candidates reach; the minimum over the G rows is then a lower bound
of the corpus's k-th best key (the shards hold at least k candidates at or above it), so
every shard drops candidates below it -- a bound no single shard's own k-th best reaches
until it has seen the whole corpus.  Nothing waits on a peer, and the result is the same
bit for bit (GSP_SHARED_THRESHOLDS=0 turns the sharing off).

This replaces the reference's 2-GPU experiments, which merged shard results on the host
(src/comprehensive_benchmark.py:416-489, src/run_remeasure_audit.py:164-186).
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import List

import torch
import torch.distributed as dist

from . import _lib as L
from .synth import shard_range


@dataclass
class ShardLayout:
    num_docs: int
    world: int
    rank: int

    @property
    def lo(self) -> int:
        return shard_range(self.num_docs, self.world, self.rank)[0]

    @property
    def hi(self) -> int:
        return shard_range(self.num_docs, self.world, self.rank)[1]

    def sizes(self) -> List[int]:
        return [shard_range(self.num_docs, self.world, r)[1] - shard_range(self.num_docs, self.world, r)[0]
                for r in range(self.world)]

    def list_counts(self, k: int) -> List[int]:
        """Valid candidates each rank contributes: min(k, shard size)."""
        return [min(k, s) for s in self.sizes()]


def global_head(index, n_head: int, group=None) -> torch.Tensor:
    """The corpus-wide head set (the n_head longest posting lists summed over all shards,
    ties to the lower term id), so every shard sums a document's terms in the same order."""
    lengths = index.lengths.to(torch.int64).clone()
    dist.all_reduce(lengths, group=group)
    top = torch.sort(-lengths, stable=True).indices[:n_head]
    return top.sort().values.to(torch.int32)


def gather_candidates(local_keys: torch.Tensor, k: int, group=None) -> torch.Tensor:
    """All-gather each rank's [B, k_local] int64 keys, zero-padded to [B, k], into
    [world, B, k] on every rank (one collective): every rank can then merge the whole
    batch itself.  sharded_score_topk uses the query-block exchange below instead, which
    moves and merges 1/world of this per rank."""
    world = dist.get_world_size(group)
    B, kl = local_keys.shape
    if kl < k:
        pad = torch.zeros((B, k - kl), dtype=local_keys.dtype, device=local_keys.device)
        local_keys = torch.cat([local_keys, pad], dim=1)
    local_keys = local_keys.contiguous()
    out = torch.empty((world * B, k), dtype=local_keys.dtype, device=local_keys.device)
    dist.all_gather_into_tensor(out, local_keys, group=group)
    return out.view(world, B, k)


class ThresholdBoards:
    """This rank's threshold boards and IPC mappings of every other rank's (collective:
    every rank of the group constructs, uses and closes them together).

    Two boards per rank, used by alternate batches.  A batch clears its own board on its
    stream before scoring; a raise from another rank's previous batch can only target the
    other board, because a rank starts a batch only after the previous batch's exchange
    (the all-to-all of candidate keys), which no rank finishes before every rank's scoring
    kernel of that batch has ended.
    Raises of the current batch that land before the clear are lost, which only weakens a
    bound.  If a peer's board cannot be mapped, this rank scores without any board: it
    neither reads a bound nor publishes one, so its row stays 0 (no bound) everywhere."""

    def __init__(self, device: torch.device, capacity: int, group=None):
        """capacity: queries per batch the boards hold (G rows of capacity keys each)."""
        lib = L.lib()
        self.device, self.capacity, self.group = device, int(capacity), group
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        self.world, self.rank = world, rank
        self.own: List[int] = []
        self.peers: List[List[int]] = [[], []]
        self.epoch = 0
        hb = (ctypes.c_ubyte * (2 * 64))()
        with torch.cuda.device(device):
            for e in range(2):
                ptr = ctypes.c_void_p()
                L.check(lib.gsp_board_alloc(world * self.capacity, ctypes.byref(ptr),
                                            ctypes.byref(hb, 64 * e)), "threshold board")
                self.own.append(int(ptr.value))
            mine = torch.tensor(list(hb), dtype=torch.uint8, device=device)
            allh = torch.empty(world * 2 * 64, dtype=torch.uint8, device=device)
            dist.all_gather_into_tensor(allh, mine, group=group)
            allh = bytes(allh.cpu().numpy().tobytes())
            opened = [[], []]
            ok = True
            for r in range(world):
                if r == rank or not ok:
                    continue
                for e in range(2):
                    h = (ctypes.c_ubyte * 64).from_buffer_copy(allh, (2 * r + e) * 64)
                    ptr = ctypes.c_void_p()
                    if lib.gsp_board_open(ctypes.byref(h), ctypes.byref(ptr)) != L.GSP_OK:
                        ok = False
                        break
                    opened[e].append(int(ptr.value))
            if ok:
                self.peers = opened
            else:
                for e in range(2):
                    for ptr in opened[e]:
                        lib.gsp_board_close(ctypes.c_void_p(ptr))

    def next(self, B: int):
        """(own board, peer boards) for the next batch of B queries; clears the own board's
        G rows of B keys on the current stream."""
        e = self.epoch & 1
        self.epoch += 1
        L.check(L.lib().gsp_board_clear(ctypes.c_void_p(self.own[e]), self.world * int(B),
                                        L.stream_of(self.device)), "threshold board")
        return self.own[e], self.peers[e]

    def close(self) -> None:
        """Unmap the peers' boards and free this rank's (collective)."""
        lib = L.lib()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            for e in range(2):
                for ptr in self.peers[e]:
                    lib.gsp_board_close(ctypes.c_void_p(ptr))
            self.peers = [[], []]
            dist.barrier(group=self.group)
            for ptr in self.own:
                lib.gsp_board_free(ctypes.c_void_p(ptr))
            self.own = []


_BOARDS = {}


def _boards(device: torch.device, B: int, group) -> "ThresholdBoards":
    key = (device.index, id(group))
    b = _BOARDS.get(key)
    if b is None or b.capacity < B:
        if b is not None:
            b.close()
        b = ThresholdBoards(device, max(B, 4096), group)
        _BOARDS[key] = b
    return b


def release_threshold_boards() -> None:
    """Close every threshold board of this process (collective; call before
    destroy_process_group)."""
    for b in list(_BOARDS.values()):
        b.close()
    _BOARDS.clear()


def shared_thresholds_enabled() -> bool:
    return os.environ.get("GSP_SHARED_THRESHOLDS", "1") != "0"


def exchange_candidates(local_keys: torch.Tensor, k: int, group=None) -> torch.Tensor:
    """One all_to_all_single of query blocks: each rank's [B, k_local] int64 keys,
    zero-padded to [Bp, k] (Bp = B rounded up to a multiple of the world size), are cut
    into world blocks of Bp/world queries; rank r receives block r of every rank, as
    [world, Bp/world, k]."""
    world = dist.get_world_size(group)
    B, kl = local_keys.shape
    Bp = -(-B // world) * world
    if kl < k or Bp != B:
        padded = torch.zeros((Bp, k), dtype=local_keys.dtype, device=local_keys.device)
        padded[:B, :kl] = local_keys
        local_keys = padded
    local_keys = local_keys.contiguous()
    out = torch.empty_like(local_keys)
    dist.all_to_all_single(out, local_keys, group=group)
    return out.view(world, Bp // world, k)


def gather_results(scores: torch.Tensor, ids: torch.Tensor, B: int, group=None):
    """Every rank's merged block [Bp/world, k] of scores and ids into the whole batch on
    every rank (two all-gathers), cut back to B queries."""
    world = dist.get_world_size(group)
    bb, k = scores.shape
    s_all = torch.empty((world * bb, k), dtype=scores.dtype, device=scores.device)
    i_all = torch.empty((world * bb, k), dtype=ids.dtype, device=ids.device)
    dist.all_gather_into_tensor(s_all, scores.contiguous(), group=group)
    dist.all_gather_into_tensor(i_all, ids.contiguous(), group=group)
    return s_all[:B], i_all[:B]


def exchange_mode() -> str:
    """``blocks`` (default): one all-to-all of query blocks, each rank merges B/G queries,
    two all-gathers of the results; ``allgather`` (GSP_EXCHANGE=allgather): one all-gather
    of every rank's keys, every rank merges the whole batch."""
    return "allgather" if os.environ.get("GSP_EXCHANGE", "blocks") == "allgather" else "blocks"


def sharded_score_topk(index, layout: ShardLayout, query_term_ids: torch.Tensor,
                       query_term_scores: torch.Tensor, top_k: int, group=None, events=None):
    """Exact global top-k of the batch over all shards; every rank gets the result.

    ``events`` (a list, optional) receives (phase name, CUDA event recorded after it) on the
    current stream: score, exchange, merge, gather -- a diagnostic of where a step's time
    goes."""
    from .scoring import merge_topk, score_topk
    k = min(int(top_k), layout.num_docs)

    def mark(name):
        if events is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            events.append((name, e))

    if layout.world == 1:
        out = score_topk(index, query_term_ids, query_term_scores, k)
        mark("score")
        return out
    if shared_thresholds_enabled():
        dev = index.device if isinstance(index.device, torch.device) else torch.device(index.device)
        boards = _boards(dev, int(query_term_ids.shape[0]), group)
        own, peers = boards.next(int(query_term_ids.shape[0]))
        if len(peers) == layout.world - 1:
            _, _, keys = score_topk(index, query_term_ids, query_term_scores, k, with_keys=True,
                                    board=own, shard=layout.rank, peer_boards=peers)
        else:   # the peers' boards could not be mapped: score alone
            _, _, keys = score_topk(index, query_term_ids, query_term_scores, k, with_keys=True)
    else:
        _, _, keys = score_topk(index, query_term_ids, query_term_scores, k, with_keys=True)
    mark("score")
    if exchange_mode() == "allgather":
        allk = gather_candidates(keys, k, group)
        mark("exchange")
        out = merge_topk(allk, layout.list_counts(k), k)
        mark("merge")
        return out
    blk = exchange_candidates(keys, k, group)
    mark("exchange")
    s, i = merge_topk(blk, layout.list_counts(k), k)
    mark("merge")
    out = gather_results(s, i, int(query_term_ids.shape[0]), group)
    mark("gather")
    return out


def decode_keys(keys: torch.Tensor):
    """(scores fp32, global doc ids int64) of packed keys (host or device tensors)."""
    u = keys.to(torch.int64)
    hi = (u >> 32) & 0xFFFFFFFF
    lo = u & 0xFFFFFFFF
    bits = torch.where(hi >= 0x80000000, hi & 0x7FFFFFFF, (~hi) & 0xFFFFFFFF).to(torch.int64)
    scores = bits.to(torch.int32).view(torch.float32)
    ids = 0xFFFFFFFF - lo
    return scores, ids
