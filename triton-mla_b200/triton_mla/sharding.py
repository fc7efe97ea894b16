"""Batch sharding of decode requests over the GPUs of one node.

Requests are independent in MLA decode (no data crosses requests), so the batch
is partitioned by request and every rank runs ``mla_decode`` on its own requests
with its own page pool and block table; no collective touches the decode path.

* ``contiguous_requests``: equal contiguous slices (uniform lengths).
* ``balance_requests``: longest-first greedy onto the least-loaded rank, by token
  count, since the decode time of a rank grows with the tokens it streams.
* ``rank_local_batch``: the rank's q rows, lengths, a compact page pool holding
  only its requests' pages, and a block table renumbered into that pool.

The reference has one GPU and no partitioning; this module has no counterpart there.
"""

from __future__ import annotations

import heapq
from typing import List, Sequence

import torch


def contiguous_requests(batch: int, world_size: int) -> List[List[int]]:
    """Equal contiguous slices of ``range(batch)`` (the first ``batch % world`` ranks get one more)."""
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    base, extra = divmod(batch, world_size)
    out, at = [], 0
    for r in range(world_size):
        n = base + (1 if r < extra else 0)
        out.append(list(range(at, at + n)))
        at += n
    return out


def balance_requests(seqlens: Sequence[int], world_size: int) -> List[List[int]]:
    """Longest-processing-time assignment of requests to ranks by token count.

    Requests are taken longest first (ties: lower index first) and each goes to the
    rank with the fewest tokens so far (ties: lower rank).  Each rank's list is
    returned in increasing request order.  The largest rank load is at most the
    average load plus the longest request.
    """
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    lens = [int(x) for x in seqlens]
    order = sorted(range(len(lens)), key=lambda i: (-lens[i], i))
    heap = [(0, r) for r in range(world_size)]
    shards: List[List[int]] = [[] for _ in range(world_size)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + lens[i], r))
    return [sorted(s) for s in shards]


def rank_local_batch(q: torch.Tensor, kv_cache: torch.Tensor, cache_seqlens: torch.Tensor,
                     block_table: torch.Tensor, requests: Sequence[int], page_size: int | None = None):
    """The inputs of one rank: ``(q, kv_cache, cache_seqlens, block_table)`` for ``requests``.

    The rank's pool holds, in order, the pages its requests use (their first
    ``ceil(len / page_size)`` block-table entries); the block table is renumbered into
    it and padded with page 0.  Results of ``mla_decode`` on these inputs equal the
    rows ``requests`` of a decode of the whole batch.
    """
    if kv_cache.dim() == 4:
        kv_cache = kv_cache.squeeze(2)
    page_size = int(page_size or kv_cache.shape[1])
    idx = torch.as_tensor(list(requests), dtype=torch.long)
    lens = cache_seqlens.to(torch.long).cpu()[idx]
    need = (lens + page_size - 1) // page_size
    width = max(1, int(need.max())) if len(idx) else 1
    bt_cpu = block_table.cpu().to(torch.long)
    pages, local_bt = [], torch.zeros(len(idx), width, dtype=torch.int32)
    for row, (b, k) in enumerate(zip(idx.tolist(), need.tolist())):
        local_bt[row, :k] = torch.arange(len(pages), len(pages) + k, dtype=torch.int32)
        pages.extend(bt_cpu[b, :k].tolist())
    page_idx = torch.as_tensor(pages if pages else [0], dtype=torch.long, device=kv_cache.device)
    local_kv = kv_cache.index_select(0, page_idx).contiguous()
    return (q.index_select(0, idx.to(q.device)).contiguous(), local_kv,
            lens.to(torch.int32).to(cache_seqlens.device), local_bt.to(block_table.device))
