"""DeepSeek-V2/V3 MLA layer whose decode step runs the B200 decode kernel.

API-compatible with the reference's ``triton_mla.model`` (src/triton_mla/model.py):
``MLAConfig`` has the same fields, defaults and properties (model.py:13-31);
``MLA`` has the same parameter names and shapes (``wq_a``, ``q_norm``, ``wq_b``,
``wkv_a``, ``kv_norm``, ``wkv_b``, ``wo``), so a state dict moves between the two
unchanged; ``MLA.forward(x, kv_cache, cache_seqlens, block_table=None,
num_splits=None) -> (out, seqlens)`` appends the new token in place and runs
the absorbed decode (model.py:101-124); ``MLA.forward_naive`` is the
decompressed form (model.py:126-144).

The attention step is ``mla_decode`` (CUDA library).  For up to 64 tokens of one
16-bit dtype the large projections (``wq_b``, ``wo``) are the library's
weight-streaming tcgen05 GEMM (``layer_ops.linear``), the others cuBLAS (``wq_a``
and ``wkv_a`` as one GEMM).  The rest
of a decode step runs as three fused CUDA launches (``layer_ops``): the kv_norm,
k_pe RoPE and cache append, with q_norm in the same launch; the q_pe RoPE,
absorption by W_UK and concatenation into the decode query; and the W_UV
projection of the decode output.  Steps whose tensors do not share one dtype take
the PyTorch-op form of the same math.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import layer_ops
from .kernel import mla_decode
from .reference import gather_kv


@dataclass
class MLAConfig:
    hidden_size: int = 7168
    num_heads: int = 128
    q_lora_rank: int = 1536
    kv_lora_rank: int = 512
    qk_nope_head_dim: int = 128
    qk_rope_head_dim: int = 64
    v_head_dim: int = 128
    rope_theta: float = 10000.0
    rms_norm_eps: float = 1e-6

    @property
    def qk_head_dim(self):
        return self.qk_nope_head_dim + self.qk_rope_head_dim

    @property
    def kv_cache_dim(self):
        return self.kv_lora_rank + self.qk_rope_head_dim


class RMSNorm(nn.Module):
    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        return F.rms_norm(x, (x.shape[-1],), self.weight, self.eps)


def apply_rope(x, positions, theta):
    """Half-split rotary embedding at integer ``positions`` (computed in fp32)."""
    half = x.shape[-1] // 2
    exponent = torch.arange(half, device=x.device, dtype=torch.float32) * (2.0 / x.shape[-1])
    angle = positions.float()[..., None] * theta ** (-exponent)
    c, s = angle.cos(), angle.sin()
    a, b = x.float()[..., :half], x.float()[..., half:]
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1).to(x.dtype)


class MLA(nn.Module):
    """Multi-head Latent Attention; caches only the 512-d latent and the 64-d RoPE key per token."""

    def __init__(self, cfg: MLAConfig):
        super().__init__()
        self.cfg = cfg
        h = cfg.num_heads
        self.wq_a = nn.Linear(cfg.hidden_size, cfg.q_lora_rank, bias=False)
        self.q_norm = RMSNorm(cfg.q_lora_rank, cfg.rms_norm_eps)
        self.wq_b = nn.Linear(cfg.q_lora_rank, h * cfg.qk_head_dim, bias=False)
        self.wkv_a = nn.Linear(cfg.hidden_size, cfg.kv_cache_dim, bias=False)
        self.kv_norm = RMSNorm(cfg.kv_lora_rank, cfg.rms_norm_eps)
        self.wkv_b = nn.Linear(cfg.kv_lora_rank, h * (cfg.qk_nope_head_dim + cfg.v_head_dim), bias=False)
        self.wo = nn.Linear(h * cfg.v_head_dim, cfg.hidden_size, bias=False)
        self.softmax_scale = cfg.qk_head_dim ** -0.5

    def _project(self, x, positions):
        cfg = self.cfg
        q = self.wq_b(self.q_norm(self.wq_a(x))).view(x.shape[0], cfg.num_heads, cfg.qk_head_dim)
        q_nope, q_pe = q.split([cfg.qk_nope_head_dim, cfg.qk_rope_head_dim], dim=-1)
        q_pe = apply_rope(q_pe, positions[:, None], cfg.rope_theta)
        c_kv, k_pe = self.wkv_a(x).split([cfg.kv_lora_rank, cfg.qk_rope_head_dim], dim=-1)
        return q_nope, q_pe, self.kv_norm(c_kv), apply_rope(k_pe, positions, cfg.rope_theta)

    @staticmethod
    def _append_kv(kv_cache, c_kv, k_pe, cache_seqlens, block_table):
        row = torch.cat([c_kv, k_pe], dim=-1).to(kv_cache.dtype)
        pos = cache_seqlens.long()
        req = torch.arange(pos.shape[0], device=pos.device)
        if kv_cache.dim() == 4:
            kv_cache = kv_cache.squeeze(2)
        if block_table is None:
            kv_cache[req, pos] = row
        else:
            page = kv_cache.shape[1]
            kv_cache[block_table[req, pos // page].long(), pos % page] = row

    def _wkv_b(self):
        cfg = self.cfg
        w = self.wkv_b.weight.view(cfg.num_heads, cfg.qk_nope_head_dim + cfg.v_head_dim, cfg.kv_lora_rank)
        return w[:, : cfg.qk_nope_head_dim], w[:, cfg.qk_nope_head_dim:]

    def forward(self, x, kv_cache, cache_seqlens, block_table=None, num_splits=None):
        """One decode step for x [batch, hidden]; returns (out [batch, hidden], cache_seqlens + 1)."""
        cfg = self.cfg
        weights = (self.wq_a.weight, self.q_norm.weight, self.wq_b.weight, self.wkv_a.weight, self.kv_norm.weight,
                   self.wkv_b.weight, self.wo.weight)
        if layer_ops.fusable(x, kv_cache, weights, cfg.kv_lora_rank, cfg.qk_nope_head_dim, cfg.qk_rope_head_dim):
            return self._forward_fused(x, kv_cache, cache_seqlens, block_table, num_splits)
        return self._forward_ops(x, kv_cache, cache_seqlens, block_table, num_splits)

    def _w_a(self):
        """``[wq_a.weight; wkv_a.weight]``: both down-projections of x as one GEMM.  The copy
        is cached and remade when either weight changes (storage or in-place version); a
        captured CUDA graph keeps the copy it was captured with."""
        wq, wkv = self.wq_a.weight, self.wkv_a.weight
        key = (wq.data_ptr(), wq._version, wkv.data_ptr(), wkv._version, wq.dtype, wq.device)
        if getattr(self, "_w_a_key", None) != key:
            self._w_a_cat = torch.cat([wq.detach(), wkv.detach()], dim=0)
            self._w_a_key = key
        return self._w_a_cat

    def _linear_ws(self):
        """The projection kernel's workspace of this layer (its steps run on one stream at a time)."""
        ws = self.__dict__.get("_linear_workspace")
        if ws is None:
            ws = self.__dict__["_linear_workspace"] = layer_ops.LinearWorkspace()
        return ws

    # Bytes of wo brought into L2 during the decode (with all of W_UV); negative: no prefetch.
    # Config 5 (B200): none 174.5-175.6 µs per step, W_UV only 173.9, + 32 MB of wo 170.3,
    # + 64 MB 170.9-172.7, + 96 MB 174.2 (more is evicted by the decode's cache stream).
    l2_prefetch_wo_bytes = 32 << 20

    def _side_stream(self, device):
        """A stream of this layer for work beside the decode (made once per device)."""
        streams = self.__dict__.setdefault("_side_streams", {})
        if device not in streams:
            streams[device] = torch.cuda.Stream(device)
        return streams[device]

    def _prefetch_after_decode(self, device):
        """On a side stream that starts with the decode: W_UV (the rows of wkv_b that o_unabsorb
        reads) and the first ``l2_prefetch_wo_bytes`` of wo into L2.  The decode is latency-bound
        and leaves HBM bandwidth and 20 SMs idle; the two products after it stream these weights.
        Returns the side stream (joined by the caller), or None."""
        if self.l2_prefetch_wo_bytes < 0:
            return None
        cfg = self.cfg
        side = self._side_stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        w = self.wkv_b.weight
        row = w.shape[1] * w.element_size()
        wo = self.wo.weight
        with torch.cuda.stream(side):
            layer_ops.l2_prefetch(w[cfg.qk_nope_head_dim:], cfg.v_head_dim * row,
                                  (cfg.qk_nope_head_dim + cfg.v_head_dim) * row, cfg.num_heads)
            nbytes = min(self.l2_prefetch_wo_bytes, wo.numel() * wo.element_size()) // 16 * 16
            if nbytes > 0:
                layer_ops.l2_prefetch(wo, nbytes)
        return side

    def _proj(self, inp, weight, overlap):
        """``F.linear(inp, weight)``: the weight-streaming tcgen05 kernel for up to 64 tokens and
        a large weight (``layer_ops.linear_preferred``), else cuBLAS.  ``overlap`` as in
        ``layer_ops.linear``."""
        if layer_ops.linear_preferred(inp, weight):
            return layer_ops.linear(inp, weight, overlap=overlap, workspace=self._linear_ws())
        return F.linear(inp, weight)

    def _forward_fused(self, x, kv_cache, cache_seqlens, block_table, num_splits):
        cfg = self.cfg
        batch = x.shape[0]
        # The first GEMM is an ordinary launch: the kernel before it may have written a weight.
        qa, kva = self._proj(x, self._w_a(), False).split([cfg.q_lora_rank, cfg.kv_cache_dim], dim=-1)
        positions = cache_seqlens.to(torch.int32).contiguous()
        bt = None if block_table is None else block_table.to(torch.int32).contiguous()
        seqlens = torch.empty_like(positions)
        # The layer ops launch as programmatic dependents of the kernel before them (their
        # weight loads and launch overlap its end): none of those kernels writes a weight.
        # One launch appends the cache row and applies q_norm to the other half of the GEMM.
        qn = layer_ops.kv_norm_rope_append(kva, self.kv_norm.weight, positions, kv_cache, bt, self.kv_norm.eps,
                                           cfg.rope_theta, seqlens_out=seqlens, overlap=True, q_in=qa,
                                           q_norm_weight=self.q_norm.weight, q_eps=self.q_norm.eps)
        q = self._proj(qn, self.wq_b.weight, True).view(batch, cfg.num_heads, cfg.qk_head_dim)
        q_full = layer_ops.q_absorb_rope(q, self.wkv_b.weight, positions, cfg.qk_nope_head_dim, cfg.v_head_dim,
                                         cfg.rope_theta, overlap=True)
        side = self._prefetch_after_decode(x.device)
        o = mla_decode(q_full, kv_cache, seqlens, bt, head_dim_v=cfg.kv_lora_rank, softmax_scale=self.softmax_scale,
                       num_splits=num_splits)
        o = layer_ops.o_unabsorb(o, self.wkv_b.weight, cfg.qk_nope_head_dim, cfg.v_head_dim, overlap=True)
        y = self._proj(o, self.wo.weight, True)
        if side is not None:
            torch.cuda.current_stream(x.device).wait_stream(side)
        return y, seqlens.to(cache_seqlens.dtype)

    def _forward_ops(self, x, kv_cache, cache_seqlens, block_table, num_splits):
        """The decode step as PyTorch ops around ``mla_decode`` (mixed dtypes)."""
        q_nope, q_pe, c_kv, k_pe = self._project(x, cache_seqlens)
        self._append_kv(kv_cache, c_kv, k_pe, cache_seqlens, block_table)
        seqlens = cache_seqlens + 1
        w_uk, w_uv = self._wkv_b()
        q_abs = torch.einsum("bhd,hdc->bhc", q_nope, w_uk)
        q = torch.cat([q_abs, q_pe], dim=-1).to(kv_cache.dtype).contiguous()
        o = mla_decode(q, kv_cache, seqlens, block_table, head_dim_v=self.cfg.kv_lora_rank,
                       softmax_scale=self.softmax_scale, num_splits=num_splits)
        o = torch.einsum("bhc,hdc->bhd", o.to(w_uv.dtype), w_uv)
        return self.wo(o.flatten(1)), seqlens

    def forward_naive(self, x, kv_cache, cache_seqlens, block_table=None):
        """The same decode step without absorption: per-head K/V decompressed from the cache."""
        cfg = self.cfg
        q_nope, q_pe, c_kv, k_pe = self._project(x, cache_seqlens)
        self._append_kv(kv_cache, c_kv, k_pe, cache_seqlens, block_table)
        seqlens = cache_seqlens + 1
        kv = gather_kv(kv_cache, seqlens, block_table).to(x.dtype)
        latent, kpe = kv.split([cfg.kv_lora_rank, cfg.qk_rope_head_dim], dim=-1)
        kvb = self.wkv_b(latent).view(*latent.shape[:2], cfg.num_heads, -1)
        k_nope, v = kvb.split([cfg.qk_nope_head_dim, cfg.v_head_dim], dim=-1)
        k = torch.cat([k_nope, kpe[:, :, None].expand(-1, -1, cfg.num_heads, -1)], dim=-1)
        q = torch.cat([q_nope, q_pe], dim=-1)
        logits = torch.einsum("bhd,bshd->bhs", q.float(), k.float()) * self.softmax_scale
        invalid = torch.arange(kv.shape[1], device=x.device)[None, :] >= seqlens[:, None]
        probs = logits.masked_fill(invalid[:, None, :], float("-inf")).softmax(-1)
        o = torch.einsum("bhs,bshd->bhd", probs, v.float()).to(x.dtype)
        return self.wo(o.flatten(1)), seqlens


class MLADecodeGraph:
    """One ``MLA.forward`` decode step captured in a CUDA graph for fixed shapes.

    The projections, norms, RoPE, cache append, absorption, decode kernels and output
    projection replay as one graph launch, so a step costs no per-op launch or Python
    time.  The graph reads the new tokens from ``self.x`` (or the ``x`` given to the
    call, copied there) and the lengths from ``cache_seqlens`` as they are at replay
    time (update it in place between steps), appends to ``kv_cache`` in place and
    writes ``self.out`` [batch, hidden] and ``self.next_seqlens`` (= lengths + 1).
    ``num_splits=None`` is sized at capture for the longest request the cache holds.
    No counterpart in the reference, which runs the step eagerly.
    """

    def __init__(self, layer: MLA, kv_cache, cache_seqlens, block_table=None, num_splits=None):
        param = next(layer.parameters())
        batch = cache_seqlens.shape[0]
        self.x = torch.zeros(batch, layer.cfg.hidden_size, dtype=param.dtype, device=param.device)
        self.graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(param.device)
        side.wait_stream(torch.cuda.current_stream(param.device))
        with torch.no_grad(), torch.cuda.stream(side):
            layer(self.x, kv_cache, cache_seqlens, block_table, num_splits=num_splits)  # warm-up outside capture
        torch.cuda.current_stream(param.device).wait_stream(side)
        with torch.no_grad(), torch.cuda.graph(self.graph):
            self.out, self.next_seqlens = layer(self.x, kv_cache, cache_seqlens, block_table, num_splits=num_splits)

    def __call__(self, x=None):
        """Replay the step (after copying ``x`` into the graph's input when given); returns ``self.out``."""
        if x is not None:
            self.x.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.out

