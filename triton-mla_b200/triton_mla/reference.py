"""PyTorch MLA decode functions kept for API parity with the reference package.

The reference exports ``mla_decode_ref`` and ``mla_decode_torch``
(src/triton_mla/reference.py:16-44, re-exported by __init__.py:3) as its
correctness oracle and eager baseline; user code that imports them keeps
working.  They are plain PyTorch, run on any device, and are NOT used by
``mla_decode`` (which runs only the CUDA library).  This package's own tests
check the CUDA path against the separate numpy oracle and golden vectors
produced by the reference itself, not against these functions.
"""

from __future__ import annotations

import torch


def gather_kv(kv_cache, cache_seqlens, block_table=None):
    """Contiguous ``[batch, max_blocks * page, D]`` view of a paged or dense cache."""
    if kv_cache.dim() == 4:
        kv_cache = kv_cache.squeeze(2)
    if block_table is None:
        return kv_cache
    rows = kv_cache.index_select(0, block_table.reshape(-1).long())
    return rows.view(block_table.shape[0], -1, kv_cache.shape[-1])


def mla_decode_ref(q, kv_cache, cache_seqlens, block_table=None, head_dim_v=512, softmax_scale=None):
    """Per-request fp32 attention; returns ``(out in q.dtype, lse fp32)``."""
    scale = q.shape[-1] ** -0.5 if softmax_scale is None else softmax_scale
    kv = gather_kv(kv_cache, cache_seqlens, block_table)
    batch, heads = q.shape[0], q.shape[1]
    out = q.new_zeros(batch, heads, head_dim_v, dtype=torch.float32)
    lse = q.new_full((batch, heads), float("-inf"), dtype=torch.float32)
    for b, n in enumerate(cache_seqlens.tolist()):
        if n == 0:
            continue
        k = kv[b, :n].float()
        logits = (q[b].float() @ k.t()) * scale
        lse[b] = logits.logsumexp(-1)
        out[b] = logits.softmax(-1) @ k[:, :head_dim_v]
    return out.to(q.dtype), lse


def mla_decode_torch(q, kv_cache, cache_seqlens, block_table=None, head_dim_v=512, softmax_scale=None):
    """Batched masked attention in PyTorch (no LSE), the eager baseline."""
    scale = q.shape[-1] ** -0.5 if softmax_scale is None else softmax_scale
    kv = gather_kv(kv_cache, cache_seqlens, block_table)
    logits = torch.matmul(q, kv.transpose(1, 2)).float() * scale
    positions = torch.arange(kv.shape[1], device=q.device)
    invalid = positions[None, :] >= cache_seqlens[:, None]
    logits = logits.masked_fill(invalid[:, None, :], float("-inf"))
    probs = logits.softmax(-1).to(q.dtype)
    return torch.matmul(probs, kv[..., :head_dim_v])
