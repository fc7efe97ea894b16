"""The MLA layer's per-step operations around the decode kernel, one CUDA launch each
(C ABI: ``tmla_q_absorb_rope``, ``tmla_kv_norm_rope_append``, ``tmla_o_unabsorb``).

They replace the PyTorch glue of the reference's ``MLA.forward``
(src/triton_mla/model.py:74-94 and 111-123): RoPE of q_pe and k_pe, kv_norm, the
paged-cache append, the absorption einsums by W_UK / W_UV and the concatenation.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .kernel import _DTYPE_CODES, _status_word


def _stream(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _ptr(t):
    return None if t is None else t.data_ptr()


def fusable(x: torch.Tensor, kv_cache: torch.Tensor, weights, rank: int, d_nope: int, d_rope: int) -> bool:
    """Whether the fused operations take this layer step: CUDA tensors of one dtype
    (bf16, fp16 or fp32), a latent rank that is a multiple of 16 (<= 2048), d_nope <= 512,
    an even RoPE width and row-major weights."""
    dt = x.dtype
    if not x.is_cuda or dt not in _DTYPE_CODES or kv_cache.dtype != dt:
        return False
    if any(w.dtype != dt or not w.is_contiguous() or w.device != x.device for w in weights):
        return False
    return rank % 16 == 0 and rank <= 2048 and 0 < d_nope <= 512 and d_rope % 2 == 0


def q_absorb_rope(q_in: torch.Tensor, w_kv_b: torch.Tensor, positions: torch.Tensor, d_nope: int, d_v: int,
                  rope_theta: float, overlap: bool = False) -> torch.Tensor:
    """``[q_in[..., :d_nope] . W_UK | rope(q_in[..., d_nope:])]`` for q_in [batch, heads, d_nope + d_rope].

    ``overlap``: launch as a programmatic dependent of the preceding kernel in the stream
    (``TMLA_LAYER_FLAG_PDL``); that kernel must not write ``w_kv_b``."""
    batch, heads, d = q_in.shape
    rank = w_kv_b.shape[1]
    assert q_in.stride(-1) == 1 and positions.dtype == torch.int32 and positions.is_contiguous()
    q_out = torch.empty(batch, heads, rank + d - d_nope, dtype=q_in.dtype, device=q_in.device)
    p = _lib.TmlaQPrepParams(q_in.data_ptr(), q_in.stride(0), q_in.stride(1), w_kv_b.data_ptr(), positions.data_ptr(),
                             q_out.data_ptr(), q_out.stride(0), q_out.stride(1), batch, heads, d_nope, d - d_nope,
                             d_v, rank, _DTYPE_CODES[q_in.dtype], float(rope_theta),
                             _lib.LAYER_FLAG_PDL if overlap else 0)
    _lib.check(_lib.load().tmla_q_absorb_rope(ctypes.byref(p), _stream(q_in)), "tmla_q_absorb_rope")
    return q_out


def kv_norm_rope_append(kv_in: torch.Tensor, norm_weight: torch.Tensor, positions: torch.Tensor,
                        kv_cache: torch.Tensor, block_table, eps: float, rope_theta: float,
                        seqlens_out: torch.Tensor | None = None, overlap: bool = False,
                        q_in: torch.Tensor | None = None, q_norm_weight: torch.Tensor | None = None,
                        q_eps: float = 1e-6):
    """Write ``[rmsnorm(kv_in[:, :rank]) | rope(kv_in[:, rank:])]`` at each request's position.
    ``overlap`` as in ``q_absorb_rope`` (the preceding kernel must not write a norm weight).
    With ``q_in`` [batch, q_rank] the same launch also returns ``rmsnorm(q_in) * q_norm_weight``
    (contiguous); otherwise it returns None."""
    if kv_cache.dim() == 4:
        kv_cache = kv_cache.squeeze(2)
    batch, width = kv_in.shape
    rank = norm_weight.shape[0]
    assert kv_in.stride(-1) == 1 and kv_cache.stride(-1) == 1 and positions.dtype == torch.int32
    assert kv_cache.shape[-1] == width
    if block_table is not None:
        assert block_table.dtype == torch.int32 and block_table.stride(-1) == 1
    q_out = None
    if q_in is not None:
        assert q_in.dim() == 2 and q_in.shape[0] == batch and q_in.stride(-1) == 1 and q_in.dtype == kv_in.dtype
        assert q_norm_weight is not None and q_norm_weight.shape == (q_in.shape[1],)
        q_out = torch.empty(q_in.shape, dtype=q_in.dtype, device=q_in.device)
    p = _lib.TmlaKvAppendParams(
        kv_in.data_ptr(), kv_in.stride(0), norm_weight.data_ptr(), positions.data_ptr(), _ptr(seqlens_out),
        kv_cache.data_ptr(), kv_cache.stride(0), kv_cache.stride(1), kv_cache.shape[0], kv_cache.shape[1],
        _ptr(block_table), 0 if block_table is None else block_table.stride(0),
        0 if block_table is None else block_table.shape[1], _status_word(kv_in.device).data_ptr(),
        batch, rank, width - rank, _DTYPE_CODES[kv_in.dtype], float(eps), float(rope_theta),
        _lib.LAYER_FLAG_PDL if overlap else 0,
        _ptr(q_in), 0 if q_in is None else q_in.stride(0), _ptr(q_norm_weight), _ptr(q_out),
        0 if q_out is None else q_out.stride(0), 0 if q_in is None else q_in.shape[1], float(q_eps))
    _lib.check(_lib.load().tmla_kv_norm_rope_append(ctypes.byref(p), _stream(kv_in)), "tmla_kv_norm_rope_append")
    return q_out


def o_unabsorb(o: torch.Tensor, w_kv_b: torch.Tensor, d_nope: int, d_v: int, overlap: bool = False) -> torch.Tensor:
    """``o . W_UV`` per head for o [batch, heads, rank]; returns [batch, heads * d_v].
    ``overlap`` as in ``q_absorb_rope``."""
    batch, heads, rank = o.shape
    assert o.stride(-1) == 1
    out = torch.empty(batch, heads * d_v, dtype=o.dtype, device=o.device)
    p = _lib.TmlaOUnabsorbParams(o.data_ptr(), o.stride(0), o.stride(1), w_kv_b.data_ptr(), out.data_ptr(),
                                 out.stride(0), batch, heads, d_nope, d_v, rank, _DTYPE_CODES[o.dtype],
                                 _lib.LAYER_FLAG_PDL if overlap else 0)
    _lib.check(_lib.load().tmla_o_unabsorb(ctypes.byref(p), _stream(o)), "tmla_o_unabsorb")
    return out
