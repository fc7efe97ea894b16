"""CPU oracle for absorbed-MLA single-token decode.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (``triton-mla_b200/``) imports
this module; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg (``cpu_baseline`` / ``--impl reference``) may use it, and there only
as the checker or as the timed CPU restatement of the reference.

It restates, in numpy, the reference algorithm of luvadlamudi/triton-mla
(``src/triton_mla/reference.py`` and ``src/triton_mla/model.py``):

* ``gather_kv``         <- reference.py:6-13
* ``mla_decode_ref``    <- reference.py:16-31 (per-request fp32 softmax attention
                           over the shared latent cache; V = first head_dim_v dims)
* ``mla_decode_masked`` <- reference.py:34-44 (batched masked form)
* ``get_num_splits_ref``<- kernel.py:190-201 (the reference's H100 split heuristic)
* ``rms_norm``, ``apply_rope``, ``mla_project``, ``append_kv``,
  ``mla_layer_forward_naive``, ``mla_layer_forward_absorbed``
                        <- model.py:34-144 (MLA layer, naive and absorbed forms)

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function above
against golden vectors that ``tests/golden/make_golden.py`` produced by running
the reference's own Python code on identical seeded inputs.

bf16 values travel as raw ``uint16`` bit patterns (numpy has no bfloat16);
``bf16_to_f32`` widens them exactly.
"""

from __future__ import annotations

import math

import numpy as np

LOG2E = 1.4426950408889634


# ----------------------------------------------------------------------------- bf16 helpers
def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """Exact widening of bf16 bit patterns (uint16) to float32."""
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even narrowing of float32 to bf16 bit patterns (NaN kept quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    rounded = u + 0x7FFF + ((u >> 16) & 1)
    out = (rounded >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = 0x7FC0
    return out


# ----------------------------------------------------------------------------- attention
def gather_kv(kv_cache: np.ndarray, block_table: np.ndarray | None) -> np.ndarray:
    """[batch, max_blocks*page, D] view of a paged cache (reference.py:6-13).

    A 4-D ``[N, P, 1, D]`` cache is squeezed first; a dense cache is returned as is.
    """
    if kv_cache.ndim == 4:
        kv_cache = kv_cache[:, :, 0, :]
    if block_table is None:
        return kv_cache
    batch = block_table.shape[0]
    return kv_cache[block_table.astype(np.int64)].reshape(batch, -1, kv_cache.shape[-1])


def _kv_rows(kv_cache: np.ndarray, block_table: np.ndarray | None, b: int, n: int) -> np.ndarray:
    """The first ``n`` cache rows of request ``b`` without materialising the whole batch."""
    if kv_cache.ndim == 4:
        kv_cache = kv_cache[:, :, 0, :]
    if block_table is None:
        return kv_cache[b, :n]
    page = kv_cache.shape[1]
    pages = block_table[b, : -(-n // page)].astype(np.int64)
    return kv_cache[pages].reshape(-1, kv_cache.shape[-1])[:n]


def mla_decode_ref(q, kv_cache, cache_seqlens, block_table=None, head_dim_v=512,
                   softmax_scale=None, dtype=np.float64):
    """Per-request softmax attention over the latent cache (reference.py:16-31).

    ``q`` [B, H, D] and ``kv_cache`` are float arrays (already widened from bf16).
    Returns ``(out [B, H, head_dim_v], lse [B, H])`` in ``dtype``; rows with
    length 0 give out 0 and lse -inf, as the reference does.
    """
    if softmax_scale is None:
        softmax_scale = q.shape[-1] ** -0.5
    batch, heads = q.shape[0], q.shape[1]
    out = np.zeros((batch, heads, head_dim_v), dtype=dtype)
    lse = np.full((batch, heads), -np.inf, dtype=dtype)
    for b in range(batch):
        n = int(cache_seqlens[b])
        if n == 0:
            continue
        k = _kv_rows(kv_cache, block_table, b, n).astype(dtype)
        s = (q[b].astype(dtype) @ k.T) * dtype(softmax_scale)
        m = s.max(axis=-1, keepdims=True)
        p = np.exp(s - m)
        l = p.sum(axis=-1, keepdims=True)
        lse[b] = (m + np.log(l))[:, 0]
        out[b] = (p / l) @ k[:, :head_dim_v]
    return out, lse


def mla_decode_masked(q, kv_cache, cache_seqlens, block_table=None, head_dim_v=512,
                      softmax_scale=None, dtype=np.float64):
    """Batched masked attention (reference.py:34-44); returns only ``out``.

    Like the reference, a request with length 0 has every score masked and its
    softmax is undefined (NaN); callers avoid zero lengths here.
    """
    if softmax_scale is None:
        softmax_scale = q.shape[-1] ** -0.5
    kv = gather_kv(kv_cache, block_table).astype(dtype)
    scores = np.einsum("bhd,bsd->bhs", q.astype(dtype), kv) * dtype(softmax_scale)
    pos = np.arange(kv.shape[1])
    mask = pos[None, :] >= np.asarray(cache_seqlens)[:, None]
    scores = np.where(mask[:, None, :], -np.inf, scores)
    with np.errstate(invalid="ignore"):
        m = scores.max(axis=-1, keepdims=True)
        p = np.exp(scores - m)
        p = p / p.sum(axis=-1, keepdims=True)
    return np.einsum("bhs,bsd->bhd", p, kv[..., :head_dim_v])


def get_num_splits_ref(batch, num_heads, max_seqlen, num_sms, min_tokens_per_split=128):
    """The reference's split-count heuristic (kernel.py:190-201), restated."""
    head_groups = -(-num_heads // 64)
    target = num_sms // max(batch * head_groups, 1)
    max_by_len = -(-max_seqlen // min_tokens_per_split)
    splits = max(min(target, max_by_len, 64), 1)
    return 1 << (splits.bit_length() - 1)


# ----------------------------------------------------------------------------- MLA layer
def rms_norm(x, weight, eps):
    """RMSNorm as ``F.rms_norm`` computes it (model.py:34-41)."""
    x = x.astype(np.float64)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * weight


def apply_rope(x, positions, theta):
    """Half-split rotary embedding (model.py:44-50)."""
    d = x.shape[-1]
    inv_freq = 1.0 / (theta ** (np.arange(0, d, 2, dtype=np.float64) / d))
    freqs = np.asarray(positions, dtype=np.float64)[..., None] * inv_freq
    cos, sin = np.cos(freqs), np.sin(freqs)
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    return np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], axis=-1)


def mla_project(w, cfg, x, positions):
    """q/kv LoRA projections, norms and RoPE (model.py:74-82).

    ``w`` maps parameter names (``wq_a``, ``q_norm``, ``wq_b``, ``wkv_a``,
    ``kv_norm``, ``wkv_b``, ``wo``) to float arrays in ``nn.Linear`` layout
    ([out_features, in_features]).
    """
    h, dn, dr = cfg["num_heads"], cfg["qk_nope_head_dim"], cfg["qk_rope_head_dim"]
    eps, theta = cfg["rms_norm_eps"], cfg["rope_theta"]
    qa = rms_norm(x @ w["wq_a"].T, w["q_norm"], eps)
    q = (qa @ w["wq_b"].T).reshape(x.shape[0], h, dn + dr)
    q_nope, q_pe = q[..., :dn], q[..., dn:]
    q_pe = apply_rope(q_pe, np.asarray(positions)[:, None], theta)
    kva = x @ w["wkv_a"].T
    c_kv = rms_norm(kva[:, : cfg["kv_lora_rank"]], w["kv_norm"], eps)
    k_pe = apply_rope(kva[:, cfg["kv_lora_rank"]:], positions, theta)
    return q_nope, q_pe, c_kv, k_pe


def append_kv(kv_cache, c_kv, k_pe, cache_seqlens, block_table):
    """Write the new token's ``[c_kv | k_pe]`` row into the cache in place (model.py:84-94)."""
    entry = np.concatenate([c_kv, k_pe], axis=-1)
    pos = np.asarray(cache_seqlens, dtype=np.int64)
    rows = np.arange(pos.shape[0])
    if block_table is None:
        kv_cache[rows, pos] = entry
    else:
        page = kv_cache.shape[1]
        pages = block_table[rows, pos // page].astype(np.int64)
        kv_cache[pages, pos % page] = entry


def _attend_naive(w, cfg, q_nope, q_pe, kv_cache, seqlens, block_table):
    h, dn, dv = cfg["num_heads"], cfg["qk_nope_head_dim"], cfg["v_head_dim"]
    r = cfg["kv_lora_rank"]
    scale = (dn + cfg["qk_rope_head_dim"]) ** -0.5
    wkv_b = w["wkv_b"].reshape(h, dn + dv, r)
    out = np.zeros((q_nope.shape[0], h, dv))
    for b in range(q_nope.shape[0]):
        n = int(seqlens[b])
        if n == 0:
            continue
        kv = _kv_rows(kv_cache, block_table, b, n).astype(np.float64)
        latent, kpe = kv[:, :r], kv[:, r:]
        kvb = np.einsum("sr,hdr->shd", latent, wkv_b)
        k_nope, v = kvb[..., :dn], kvb[..., dn:]
        s = (np.einsum("hd,shd->hs", q_nope[b], k_nope) + q_pe[b] @ kpe.T) * scale
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        out[b] = np.einsum("hs,shd->hd", p, v)
    return out


def mla_layer_forward_naive(w, cfg, x, kv_cache, cache_seqlens, block_table=None):
    """One non-absorbed decode step (model.py:126-144): decompress K/V per head.

    Appends the new token to ``kv_cache`` in place and returns
    ``(out [B, hidden], seqlens + 1)``.
    """
    x = x.astype(np.float64)
    q_nope, q_pe, c_kv, k_pe = mla_project(w, cfg, x, cache_seqlens)
    append_kv(kv_cache, c_kv, k_pe, cache_seqlens, block_table)
    seqlens = np.asarray(cache_seqlens) + 1
    o = _attend_naive(w, cfg, q_nope, q_pe, kv_cache, seqlens, block_table)
    return o.reshape(o.shape[0], -1) @ w["wo"].T, seqlens


def mla_layer_forward_absorbed(w, cfg, x, kv_cache, cache_seqlens, block_table=None):
    """One weight-absorbed decode step (model.py:101-124) with ``mla_decode_ref`` inside."""
    h, dn, dv = cfg["num_heads"], cfg["qk_nope_head_dim"], cfg["v_head_dim"]
    r = cfg["kv_lora_rank"]
    x = x.astype(np.float64)
    q_nope, q_pe, c_kv, k_pe = mla_project(w, cfg, x, cache_seqlens)
    append_kv(kv_cache, c_kv, k_pe, cache_seqlens, block_table)
    seqlens = np.asarray(cache_seqlens) + 1
    wkv_b = w["wkv_b"].reshape(h, dn + dv, r)
    w_uk, w_uv = wkv_b[:, :dn], wkv_b[:, dn:]
    q_abs = np.einsum("bhd,hdc->bhc", q_nope, w_uk)
    q = np.concatenate([q_abs, q_pe], axis=-1)
    o, _ = mla_decode_ref(q, kv_cache, seqlens, block_table, head_dim_v=r,
                          softmax_scale=(dn + cfg["qk_rope_head_dim"]) ** -0.5)
    o = np.einsum("bhc,hdc->bhd", o, w_uv)
    return o.reshape(o.shape[0], -1) @ w["wo"].T, seqlens


# ----------------------------------------------------------------------------- measurement helpers
def decode_flops(total_tokens: int, num_heads: int, d_qk: int = 576, d_v: int = 512) -> float:
    """Algorithmic FLOPs of one decode call (the reference bench's model, bench.py:81)."""
    return float(total_tokens) * num_heads * 2 * (d_qk + d_v)


def decode_bytes(total_tokens: int, batch: int, num_heads: int, elt: int = 2,
                 d_qk: int = 576, d_v: int = 512) -> float:
    """Algorithmic bytes of one decode call: cache rows + q + out (bench.py:80)."""
    return float(total_tokens * d_qk + batch * num_heads * d_qk + batch * num_heads * d_v) * elt


def log2_lse_to_ln(lse2):
    return lse2 * math.log(2.0)
