"""Doc-range sharded scoring across the GPUs of one node.

One process per GPU (torchrun), NCCL over NVLink/NVSwitch.  Rank r holds the index of
documents [r*N/G, (r+1)*N/G) with local ids and doc_base = r*N/G, scores the full query
batch against it and keeps its exact local top-k as packed uint64 keys
(fkey(score) << 32 | ~global doc id).  One all_gather_into_tensor moves the G lists
(B*k*8 bytes per rank) into every rank's memory, and the GPU merge kernel reduces the G*k
candidates of each query to the exact global top-k (ties -> lower global doc id).  No
device ever reads another GPU's memory directly.

This replaces the reference's 2-GPU experiments, which merged shard results on the host
(src/comprehensive_benchmark.py:416-489, src/run_remeasure_audit.py:164-186).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List

import torch
import torch.distributed as dist

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
    [world, B, k] on every rank (one collective)."""
    world = dist.get_world_size(group)
    B, kl = local_keys.shape
    if kl < k:
        pad = torch.zeros((B, k - kl), dtype=local_keys.dtype, device=local_keys.device)
        local_keys = torch.cat([local_keys, pad], dim=1)
    local_keys = local_keys.contiguous()
    out = torch.empty((world * B, k), dtype=local_keys.dtype, device=local_keys.device)
    dist.all_gather_into_tensor(out, local_keys, group=group)
    return out.view(world, B, k)


def sharded_score_topk(index, layout: ShardLayout, query_term_ids: torch.Tensor,
                       query_term_scores: torch.Tensor, top_k: int, group=None):
    """Exact global top-k of the batch over all shards; every rank gets the result."""
    from .scoring import merge_topk, score_topk
    k = min(int(top_k), layout.num_docs)
    if layout.world == 1:
        return score_topk(index, query_term_ids, query_term_scores, k)
    _, _, keys = score_topk(index, query_term_ids, query_term_scores, k, with_keys=True)
    allk = gather_candidates(keys, k, group)
    return merge_topk(allk, layout.list_counts(k), k)


def decode_keys(keys: torch.Tensor):
    """(scores fp32, global doc ids int64) of packed keys (host or device tensors)."""
    u = keys.to(torch.int64)
    hi = (u >> 32) & 0xFFFFFFFF
    lo = u & 0xFFFFFFFF
    bits = torch.where(hi >= 0x80000000, hi & 0x7FFFFFFF, (~hi) & 0xFFFFFFFF).to(torch.int64)
    scores = bits.to(torch.int32).view(torch.float32)
    ids = 0xFFFFFFFF - lo
    return scores, ids
