"""The MLA layer's per-step operations around the decode kernel, one CUDA launch each
(C ABI: ``tmla_q_absorb_rope``, ``tmla_kv_norm_rope_append``, ``tmla_o_unabsorb``,
``tmla_linear``), and an L2 prefetch of the weights the step reads after its decode
(``tmla_l2_prefetch``).

They replace the PyTorch glue of the reference's ``MLA.forward``
(src/triton_mla/model.py:74-94 and 111-123): RoPE of q_pe and k_pe, kv_norm, the
paged-cache append, the absorption einsums by W_UK / W_UV and the concatenation;
and, for decode batches of up to 64 tokens, the projections' GEMMs (model.py:104-108, 124).
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


# ----------------------------------------------------------------------------- projections
LINEAR_MAX_TOKENS = 64


def linear_ok(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether ``linear`` takes ``x @ weight.T``: CUDA tensors of one 16-bit dtype, at most 64
    rows of x, 16-byte aligned rows (k a multiple of 8) and a row-major weight."""
    if not (x.is_cuda and x.dim() == 2 and weight.dim() == 2 and x.dtype in (torch.bfloat16, torch.float16)):
        return False
    if weight.dtype != x.dtype or weight.device != x.device or x.shape[1] != weight.shape[1]:
        return False
    m, k = x.shape
    return (0 < m <= LINEAR_MAX_TOKENS and k % 8 == 0 and x.stride(-1) == 1 and x.stride(0) % 8 == 0
            and weight.stride(-1) == 1 and weight.stride(0) % 8 == 0
            and x.data_ptr() % 16 == 0 and weight.data_ptr() % 16 == 0)


# From this many weight bytes up a layer step takes the projection kernel (all of the DeepSeek-V3
# layer's projections: [wq_a; wkv_a] 30 MB, wq_b 75 MB, wo 235 MB); smaller weights go to
# cuBLAS.  Measured on B200 in the layer graph: wq_b and wo on this kernel beat cuBLAS;
# [wq_a; wkv_a] (9 split-K pieces per tile, first kernel of the step, nothing to overlap its
# cold start) costs about 1 us more than cuBLAS there (169.1-169.4 against 168.4 us), which the
# step pays so that it runs on this library's kernels alone.
LINEAR_MIN_WEIGHT_BYTES = 16 << 20


def linear_preferred(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether a layer step should take ``linear`` for ``x @ weight.T`` rather than cuBLAS."""
    return linear_ok(x, weight) and weight.numel() * weight.element_size() >= LINEAR_MIN_WEIGHT_BYTES


def linear_workspace_bytes(m: int, n: int, k: int, num_sms: int, groups: int = 1) -> int:
    """Workspace bytes of ``linear`` for x [m, k], weight [n, k] (per group) spread over
    ``num_sms`` SMs."""
    need = _lib.load().tmla_linear_workspace_bytes(m, n, k, groups, num_sms)
    if need < 0:
        _lib.check(-need, "tmla_linear_workspace_bytes")
    return need


class LinearWorkspace:
    """Counters and partial sums of ``linear`` for calls on one stream at a time.  Grows on
    demand; a grown-out buffer is kept alive, because a captured CUDA graph may still use it.
    The kernel leaves the counters at zero, so the buffer is zero-filled only when made."""

    def __init__(self):
        self.buf = None
        self._retired = []

    def clear(self) -> None:
        """Zero the buffer: needed only after a call that set ``STATUS_TIMEOUT`` (read with
        ``read_status``), whose pieces that gave up were never counted."""
        if self.buf is not None:
            self.buf.zero_()

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        if self.buf is None or self.buf.device != device or self.buf.numel() < nbytes:
            if self.buf is not None:
                self._retired.append(self.buf)
            self.buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        return self.buf


_stream_ws = {}


def _linear_launch(x, x_stride, x_gstride, w, w_stride, w_gstride, w_layout, y, y_stride, y_gstride,
                   m, n, k, groups, overlap, workspace):
    sms = torch.cuda.get_device_properties(x.device).multi_processor_count
    need = linear_workspace_bytes(m, n, k, sms, groups)
    if workspace is None:
        key = (x.device.index, torch.cuda.current_stream(x.device).cuda_stream)
        workspace = _stream_ws.setdefault(key, LinearWorkspace())
    ws = workspace.get(x.device, need)
    p = _lib.TmlaLinearParams(x.data_ptr(), x_stride, w.data_ptr(), w_stride, y.data_ptr(), y_stride,
                              m, n, k, _DTYPE_CODES[x.dtype], ws.data_ptr(), ws.numel(), sms,
                              _lib.LAYER_FLAG_PDL if overlap else 0, _status_word(x.device).data_ptr(),
                              groups, w_layout, x_gstride, w_gstride, y_gstride)
    _lib.check(_lib.load().tmla_linear(ctypes.byref(p), _stream(x)), "tmla_linear")


def linear(x: torch.Tensor, weight: torch.Tensor, overlap: bool = False,
           workspace: LinearWorkspace | None = None) -> torch.Tensor:
    """``x @ weight.T`` (``F.linear`` without bias) for a decode batch of at most 64 rows, with
    the weight streamed once through tcgen05 MMAs on every SM (C ABI: ``tmla_linear``).
    ``overlap``: launch as a programmatic dependent of the preceding kernel in the stream,
    whose end then overlaps the first weight loads; that kernel must not write ``weight``.
    ``workspace``: a ``LinearWorkspace`` not used by another stream at the same time
    (default: one per device and stream)."""
    assert linear_ok(x, weight), "linear: 16-bit CUDA x [m <= 64, k] and weight [n, k], 16-byte aligned rows"
    m, k = x.shape
    n = weight.shape[0]
    y = torch.empty(m, n, dtype=x.dtype, device=x.device)
    _linear_launch(x, x.stride(0), 0, weight, weight.stride(0), 0, _lib.W_NK, y, n, 0, m, n, k, 1, overlap,
                   workspace)
    return y


def l2_prefetch(t: torch.Tensor, chunk_bytes: int = None, stride_bytes: int = None, count: int = 1,
                ctas: int = 16) -> None:
    """Bring ``count`` chunks of ``chunk_bytes`` starting at ``t``'s data, ``stride_bytes``
    apart, into L2 (bulk prefetches on the current stream; nothing waits for them).  Defaults:
    one chunk of the whole tensor.  A hint with no effect on any result."""
    nbytes = t.numel() * t.element_size()
    chunk = nbytes if chunk_bytes is None else int(chunk_bytes)
    stride = chunk if stride_bytes is None else int(stride_bytes)
    assert t.is_cuda and 0 < chunk and stride >= chunk and (count - 1) * stride + chunk <= nbytes
    _lib.check(_lib.load().tmla_l2_prefetch(ctypes.c_void_p(t.data_ptr()), chunk, stride, int(count), int(ctas),
                                             _stream(t)), "tmla_l2_prefetch")
