"""Multi-GPU placement of the hot path: one process per GPU, no collective inside a decode step except the output
gather of KV-head sharding.

The reference has no multi-GPU code of its own (tensor parallelism comes from vLLM, kushkash README "Tensor
parallel"); decode work units (sequence, kv head, split) and quantize-on-write units (sequence, page, head) are
independent, so they shard without communication:

  request partitioning  rank r owns whole sequences (their pages, block-table rows and tail slots); a step needs no
                        collective.  partition_requests balances the ranks by cached tokens (the decode's bytes).
  kv-head partitioning  for a few very long sequences: rank r owns kv heads [h0, h1) of every
                        sequence and the q heads h0*G .. h1*G; after the local split-KV decode, the [S, Hq/N, D]
                        outputs are gathered over NCCL (NVLink) into [S, Hq, D] -- the only data-path collective.
"""
from __future__ import annotations

import heapq

import torch


def partition_requests(seq_lens: list[int], world: int) -> list[list[int]]:
    """Sequence indices per rank, balanced by cached tokens (longest first onto the least-loaded rank; ties by rank,
    so every rank computes the same assignment)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    heap = [(0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(seq_lens)), key=lambda i: (-seq_lens[i], i)):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + int(seq_lens[i]), r))
    return [sorted(x) for x in out]


def kv_head_range(num_kv_heads: int, rank: int, world: int) -> tuple[int, int]:
    """[h0, h1) of the kv heads rank `rank` owns; heads must divide evenly (8 kv heads over 1, 2, 4 or 8 GPUs)."""
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} kv heads do not split over {world} ranks")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def gather_heads(local_out: torch.Tensor, group=None) -> torch.Tensor:
    """[S, Hq/N, D] outputs of this rank's q heads -> [S, Hq, D] on every rank (all_gather over the process group:
    NCCL over NVLink on GPUs, gloo on CPU), heads in rank order."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if world == 1:
        return local_out
    parts = [torch.empty_like(local_out) for _ in range(world)]
    dist.all_gather(parts, local_out.contiguous(), group=group)
    return torch.cat(parts, dim=1)
