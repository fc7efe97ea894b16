"""Host wrapper of the B200 MLA decode kernels: the drop-in ``mla_decode``.

Same signature, argument meaning, defaults and error behaviour as the
reference's ``triton_mla.mla_decode`` (src/triton_mla/kernel.py:204-323):

* a 4-D ``[N, P, 1, D]`` cache (FlashMLA layout) is squeezed (kernel.py:235-237);
* the same ``AssertionError`` checks on ranks, widths, unit inner strides,
  power-of-two ``head_dim_v`` / RoPE width and equal dtypes (kernel.py:238-245);
* ``softmax_scale`` defaults to ``d_qk ** -0.5`` (kernel.py:247-248);
* ``block_table is None`` selects the dense ``[B, S_max, D]`` layout (kernel.py:257-262);
* ``num_splits=None`` costs one host sync to read the longest request
  (kernel.py:264-266); an explicit value keeps the call sync-free (CUDA-graph safe).
  Inside CUDA-graph capture, where the reference's sync would fail, ``None`` plans the
  splits on the GPU from the lengths at replay time (tcgen05 kernel;
  ``make_device_split_plan``), or sizes the split count for the longest request the cache
  can hold (generic kernel).  Either way the captured call stays valid when the lengths
  change between replays;
* returns ``out [B, H, head_dim_v]`` in ``q.dtype`` and, with ``return_lse``,
  the natural-log LSE ``[B, H]`` fp32; zero-length requests give 0 and -inf.

Underneath, everything runs in the CUDA library through its C ABI
(``include/triton_mla_b200.h``); non-CUDA tensors raise ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

_DTYPE_CODES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_FP16, torch.float32: _lib.DTYPE_FP32}
_KERNELS = {"auto": _lib.KERNEL_AUTO, "generic": _lib.KERNEL_GENERIC, "sm100": _lib.KERNEL_SM100}

B200_NUM_SMS = 148
FP8_ROW_BYTES = 656  # an FP8 cache row: 512 e4m3 latent values, 4 fp32 scales, 64 bf16 RoPE values


def _is_pow2(v: int) -> bool:
    return v > 0 and (v & (v - 1)) == 0


def _num_sms(device) -> int:
    """SM count of ``device`` (148 on B200); B200's count when not on CUDA."""
    if device.type == "cuda":
        return torch.cuda.get_device_properties(device).multi_processor_count
    return B200_NUM_SMS


def plan_units(seqlens, num_heads: int, num_sms: int = B200_NUM_SMS):
    """Per-request split plan for a batch (``tmla_plan_units``; host only, no GPU).

    Returns ``(units, req_first)`` as int32 numpy arrays: ``units[u] = (request, split,
    splits of that request, partial slot or -1)``, longest unit first, and
    ``req_first[b]`` the first partial slot of request b (``req_first[-1]`` slots in all).
    """
    import numpy as np

    lens = np.ascontiguousarray(np.asarray(seqlens, dtype=np.int32).reshape(-1))
    batch = lens.shape[0]
    cap = max(1, batch * 64)
    units = np.zeros((cap, 4), dtype=np.int32)
    req_first = np.zeros(batch + 1, dtype=np.int32)
    n = _lib.load().tmla_plan_units(lens.ctypes.data, batch, int(num_heads), int(num_sms), cap, units.ctypes.data,
                                    req_first.ctypes.data)
    if n < 0:
        raise _lib.LibraryError(-n, "tmla_plan_units")
    return units[:n].copy(), req_first


class SplitPlan:
    """A per-request split plan in device memory, for ``mla_decode(..., plan=...)``.

    It says how many splits each request gets and in which order the work units run, not
    where the splits start: the kernels cut each request's tokens from its length on the
    device.  So a plan stays valid when the lengths change (a decode loop can plan once per
    batch composition) and a call with a plan needs no host sync (CUDA-graph safe).

    A host plan (``make_split_plan``) holds exactly its units.  A device plan
    (``make_device_split_plan``) holds a fixed number of entries (``num_units`` is its
    capacity, padding entries do no work) and ``num_slots`` partial slots, and
    ``refresh`` re-plans it on the GPU for new lengths.
    """

    def __init__(self, units, req_first, device):
        self.batch = int(req_first.shape[0]) - 1
        self.num_units = int(units.shape[0])
        self.num_slots = int(req_first[-1])
        self.units = torch.from_numpy(units).to(device)
        self.req_first = torch.from_numpy(req_first).to(device)
        self.num_heads = None

    @classmethod
    def empty(cls, batch: int, num_heads: int, capacity: int, slot_capacity: int, device) -> "SplitPlan":
        plan = cls.__new__(cls)
        plan.batch, plan.num_units, plan.num_slots, plan.num_heads = batch, capacity, slot_capacity, num_heads
        plan.units = torch.empty(capacity, 4, dtype=torch.int32, device=device)
        plan.req_first = torch.empty(batch + 1, dtype=torch.int32, device=device)
        return plan

    def refresh(self, cache_seqlens: torch.Tensor) -> "SplitPlan":
        """Re-plan a device plan for the lengths now in ``cache_seqlens`` (int32, on the plan's
        device), on the current stream: one small kernel, no host sync, capturable."""
        if self.num_heads is None:
            raise ValueError("refresh() re-plans a device plan (make_device_split_plan)")
        assert cache_seqlens.shape == (self.batch,) and cache_seqlens.device == self.units.device
        lens = cache_seqlens.to(torch.int32).contiguous()
        dev = self.units.device
        _lib.check(_lib.load().tmla_plan_units_device(
            lens.data_ptr(), self.batch, self.num_heads, _num_sms(dev), self.num_units, self.num_slots,
            self.units.data_ptr(), self.req_first.data_ptr(),
            ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)), "tmla_plan_units_device")
        return self


def make_device_split_plan(cache_seqlens: torch.Tensor, num_heads: int, capacity: int | None = None,
                           slot_capacity: int | None = None) -> SplitPlan:
    """Plan per-request splits on the GPU from the lengths in device memory
    (``tmla_plan_units_device``): no host sync, so the planning can sit in a CUDA graph with
    the decode.  ``capacity`` work units (default: batch + 2 x the clusters that run at once)
    and ``slot_capacity`` partial slots (default: 2 x those clusters) bound the plan and the
    workspace; a plan that needs more falls back to fewer splits."""
    dev = cache_seqlens.device
    batch = int(cache_seqlens.shape[0])
    machines = max(1, _num_sms(dev) // 2 // ((int(num_heads) + 127) // 128))
    capacity = min(65535, batch + 2 * machines) if capacity is None else int(capacity)
    slot_capacity = 2 * machines if slot_capacity is None else int(slot_capacity)
    plan = SplitPlan.empty(batch, int(num_heads), capacity, slot_capacity, dev)
    return plan.refresh(cache_seqlens)


def make_split_plan(cache_seqlens, num_heads: int, device=None) -> SplitPlan:
    """Plan per-request splits for the lengths ``cache_seqlens`` (a tensor or a sequence) with
    ``tmla_plan_units`` on the host, and put the plan on ``device``."""
    import numpy as np

    if isinstance(cache_seqlens, torch.Tensor):
        device = cache_seqlens.device if device is None else device
        lens = cache_seqlens.detach().to("cpu", torch.int32).numpy()
    else:
        lens = np.asarray(cache_seqlens, dtype=np.int32)
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    units, req_first = plan_units(lens, num_heads, _num_sms(device))
    return SplitPlan(units, req_first, device)


def _num_splits_rule(batch, num_heads, max_seqlen, num_sms):
    """``tmla_num_splits`` restated for torch.compile, which cannot trace the ctypes call (the
    same estimate: waves x (rows per split + fixed rows) + merge traffic, smallest count within
    2% of the best)."""
    if batch <= 0 or num_heads <= 0 or max_seqlen <= 0:
        return 1
    clusters = max(num_sms // 2, 1)
    units = batch * ((num_heads + 127) // 128)
    tiles = (max_seqlen + 63) // 64
    merge = batch * num_heads * 512.0 * 2.0 / (clusters * 1152.0) + 8.0
    cost = {}
    for s in range(1, min(tiles, 64) + 1):
        waves = (units * s + clusters - 1) // clusters
        cost[s] = waves * (((tiles + s - 1) // s) * 64.0 + 256.0) + (merge * s if s > 1 else 0.0)
    best = min(cost.values())
    return next(s for s in sorted(cost) if cost[s] <= best * 1.02)


def get_num_splits(batch, num_heads, max_seqlen, num_sms, min_tokens_per_split=128):
    """Split count for one decode call on B200.

    Replaces the reference's one-wave power-of-two rule (kernel.py:190-201).
    The tcgen05 kernel runs one 2-SM cluster per (request, 128-head tile,
    split), so a 148-SM B200 holds 74 of them per wave; the C library picks the
    count that minimises waves x (rows per split + fixed cost) + the merge's
    cost per split (the 16-bit partials written, plus a fixed latency).
    ``min_tokens_per_split`` caps the count as in the reference.
    """
    if batch <= 0 or max_seqlen <= 0:
        return 1
    s = int(_lib.load().tmla_num_splits(int(batch), int(num_heads), int(max_seqlen), int(num_sms)))
    cap = max(-(-int(max_seqlen) // int(min_tokens_per_split)), 1)
    return max(1, min(s, cap))


# ----------------------------------------------------------------------------- device status word
_status = {}


def _status_word(device: torch.device) -> torch.Tensor:
    t = _status.get(device.index)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _status[device.index] = t
    return t


def read_status(device=None, reset: bool = True) -> int:
    """Read (and by default clear) the device status word of ``device``.

    Bits: ``_lib.STATUS_BAD_PAGE`` (a block-table entry outside the page pool
    or a length beyond the cache; those tokens were masked),
    ``_lib.STATUS_TIMEOUT`` (a bounded pipeline wait gave up) and ``_lib.STATUS_RANGE``
    (FP8 rows on the tcgen05 kernel: a query, RoPE value or row scale beyond the range of its
    fp16 products; ``kernel="generic"`` computes such rows in fp32).  Synchronises.
    """
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    t = _status_word(device)
    v = int(t.item())
    if reset and v:
        t.zero_()
    return v


_CHECK = os.environ.get("TRITON_MLA_CHECK", "0") == "1"
_DECODE_OP = _lib.load_torch_op()


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "triton_mla (B200) runs only on CUDA tensors; there is no CPU implementation "
                f"(got a tensor on {t.device})")


def _ptr(t):
    return None if t is None else t.data_ptr()


def mla_decode(
    q: torch.Tensor,
    kv_cache: torch.Tensor,
    cache_seqlens: torch.Tensor,
    block_table: torch.Tensor = None,
    head_dim_v: int = 512,
    softmax_scale: float = None,
    num_splits: int = None,
    return_lse: bool = False,
    *,
    kernel: str = "auto",
    out: torch.Tensor = None,
    plan: "SplitPlan" = None,
):
    """Weight-absorbed MLA decode attention over a shared latent KV cache.

    Args:
        q: [batch, num_heads, head_dim_v + rope_dim]; the first head_dim_v dims
            are the W_UK-absorbed nope query, the rest the RoPE query.  Extension: a 4-D
            q [batch, q_len, num_heads, d] holds q_len new tokens per request (the last q_len
            of its cache_seqlens rows, e.g. multi-token prediction); token i attends causally
            to the first cache_seqlens - (q_len - 1 - i) rows, and out / lse gain the same
            q_len axis.
        kv_cache: paged [num_blocks, page_size, D] when block_table is given,
            otherwise contiguous [batch, max_seqlen, D]; [..., 1, D] accepted.
        cache_seqlens: [batch] number of valid tokens per sequence.
        block_table: optional [batch, max_blocks_per_seq] page indices.
        head_dim_v: latent rank (512 for DeepSeek-V2/V3).
        softmax_scale: defaults to q.shape[-1] ** -0.5.
        num_splits: KV splits; None picks one (one host sync); pass it
            explicitly for CUDA-graph capture.
        return_lse: also return the natural-log log-sum-exp per head.
        plan: keyword-only, a ``SplitPlan`` (``make_split_plan``) to follow instead of
            ``num_splits``: per-request split counts, no host sync (tcgen05 kernel only).
        kernel: keyword-only, "auto" (tcgen05 kernel where the shape allows),
            "sm100" (require it) or "generic" (CUDA-core kernel).
        out: keyword-only preallocated [batch, num_heads, head_dim_v] output.

    Returns:
        out [batch, num_heads, head_dim_v] (and lse [batch, num_heads] fp32).
    """
    q_len, q4 = 1, None
    if q.dim() == 4:
        q4 = q.shape
        q_len = q4[1]
        assert q_len >= 1 and q.stride(-1) == 1
        if q.stride(1) != q4[2] * q.stride(2):
            q = q.contiguous()
        q = q.view(q4[0], q_len * q4[2], q4[3])
        if out is not None:
            assert out.dim() == 4 and out.shape[:3] == q4[:3]
            out = out.view(q4[0], q_len * q4[2], out.shape[3])
    if kv_cache.dim() == 4:
        assert kv_cache.shape[2] == 1, "MLA uses a single shared latent KV head"
        kv_cache = kv_cache.squeeze(2)
    assert q.dim() == 3 and kv_cache.dim() == 3
    batch, num_heads, d_qk = q.shape
    d_rope = d_qk - head_dim_v
    # Extension: a uint8 cache of FP8 rows (``fp8_cache``: 656 bytes per token, DeepSeek dims).
    kv_format = _lib.KV_FP8_E4M3 if kv_cache.dtype == torch.uint8 else _lib.KV_SAME
    if kv_format == _lib.KV_FP8_E4M3:
        assert kv_cache.shape[-1] == FP8_ROW_BYTES and d_qk == 576 and head_dim_v == 512
        assert q.dtype in (torch.bfloat16, torch.float16)
    else:
        assert kv_cache.shape[-1] == d_qk
    assert q.stride(-1) == 1 and kv_cache.stride(-1) == 1
    assert _is_pow2(head_dim_v)
    assert _is_pow2(d_rope)
    if kv_format == _lib.KV_SAME:
        assert q.dtype == kv_cache.dtype
    if block_table is None:
        assert kv_cache.shape[0] == batch
    _require_cuda(q, kv_cache, cache_seqlens, block_table)
    if q.dtype not in _DTYPE_CODES:
        raise TypeError(f"unsupported dtype {q.dtype}; use bfloat16, float16 or float32")
    if kernel not in _KERNELS:
        raise ValueError(f"kernel must be one of {sorted(_KERNELS)}")

    if softmax_scale is None:
        softmax_scale = d_qk ** -0.5
    cache_seqlens = cache_seqlens.to(torch.int32)
    if cache_seqlens.stride(0) != 1:
        cache_seqlens = cache_seqlens.contiguous()

    paged = block_table is not None
    if paged:
        block_table = block_table.to(torch.int32)
        if block_table.stride(-1) != 1:
            block_table = block_table.contiguous()
        page_size = kv_cache.shape[1]
        num_pages = kv_cache.shape[0]
        bt_width = block_table.shape[1]
        bt_stride = block_table.stride(0)
    else:
        assert kv_cache.shape[0] == batch
        page_size = kv_cache.shape[1]
        num_pages = batch
        bt_width = 0
        bt_stride = 0

    device = q.device
    compiling = torch.compiler.is_compiling()
    if plan is not None:
        assert plan.batch == batch, "the split plan was made for another batch size"
        num_splits = 1
    elif num_splits is None and compiling:
        # Under torch.compile the split count comes from the host-side rule on the longest
        # request the cache can hold (no sync on the lengths, no graph break).
        max_seqlen = bt_width * page_size if paged else kv_cache.shape[1]
        num_splits = _num_splits_rule(batch, num_heads, max_seqlen, _num_sms(device))
    elif num_splits is None:
        if batch > 0 and torch.cuda.is_current_stream_capturing():
            # No host sync during capture.  The tcgen05 kernel follows a plan made on the GPU
            # from the lengths at replay time; the generic kernel's split count is sized for
            # the longest request the cache holds.
            if kernel != "generic" and selected_kernel(q, kv_cache, block_table, head_dim_v, num_splits=1,
                                                       kernel=kernel, q_len=q_len) == "sm100":
                plan = make_device_split_plan(cache_seqlens, num_heads)
                num_splits = 1
            else:
                max_seqlen = bt_width * page_size if paged else kv_cache.shape[1]
                num_splits = get_num_splits(batch, num_heads, max_seqlen, _num_sms(device))
        elif batch > 0:
            # The one host sync (the reference reads max(cache_seqlens) here, kernel.py:264-266).
            lens_host = cache_seqlens.cpu()
            if kernel != "generic" and selected_kernel(q, kv_cache, block_table, head_dim_v, num_splits=1,
                                                       kernel=kernel, q_len=q_len) == "sm100":
                # The tcgen05 kernel takes a split count per request: the planner's choice.
                units, req_first = plan_units(lens_host.numpy(), num_heads, _num_sms(device))
                counts = units[:, 2]
                tiles = (lens_host + 63) // 64
                if counts.min() == counts.max() and int(tiles.min()) == int(tiles.max()):
                    num_splits = int(counts[0])  # equal requests split the same way: the uniform grid
                else:
                    plan = SplitPlan(units, req_first, device)
                    num_splits = 1
            if num_splits is None:
                num_splits = get_num_splits(batch, num_heads, int(lens_host.max()), _num_sms(device))
        else:
            num_splits = 1
    num_splits = int(num_splits)

    if out is None:
        out = torch.empty(batch, num_heads, head_dim_v, dtype=q.dtype, device=device)
    else:
        assert out.shape == (batch, num_heads, head_dim_v) and out.dtype == q.dtype and out.stride(-1) == 1
    lse = torch.empty(batch, num_heads, dtype=torch.float32, device=device)

    def _shaped(o, l):
        if q4 is not None:
            o = o.view(q4[0], q_len, q4[2], o.shape[-1])
            l = l.view(q4[0], q_len, q4[2])
        return (o, l) if return_lse else o

    if batch == 0:
        return _shaped(out, lse)

    if plan is None:
        # One operator call: torch.ops.triton_mla.decode (C ABI tmla_decode underneath), on the
        # current stream, workspace from the caching allocator.
        _DECODE_OP(q, kv_cache, cache_seqlens, block_table, out, lse, num_splits, float(softmax_scale),
                   _KERNELS[kernel], q_len, None if compiling else _status_word(device))
        if _CHECK and not compiling and not torch.cuda.is_current_stream_capturing():
            st = read_status(device)
            if st:
                raise RuntimeError(f"mla_decode device status 0x{st:x} (bad page id / length, or a wait timed out)")
        return _shaped(out, lse)

    lib = _lib.load()
    slots = plan.num_slots
    ws_bytes = lib.tmla_units_workspace_bytes(slots, num_heads, head_dim_v)
    o_bytes = (slots * num_heads * head_dim_v * 4 + 255) & ~255
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device) if ws_bytes else None
    ws_o = ws_lse = None
    if ws is not None:
        ws_o = ws.data_ptr()
        ws_lse = ws_o + o_bytes

    p = _lib.TmlaDecodeParams(
        q.data_ptr(), q.stride(0), q.stride(1),
        kv_cache.data_ptr(), kv_cache.stride(0), kv_cache.stride(1), num_pages, page_size,
        cache_seqlens.data_ptr(), _ptr(block_table), bt_stride, bt_width,
        out.data_ptr(), out.stride(0), out.stride(1),
        lse.data_ptr(), lse.stride(0),
        ws_o, ws_lse, _status_word(device).data_ptr(),
        batch, num_heads, d_qk, head_dim_v, num_splits,
        _DTYPE_CODES[q.dtype], _KERNELS[kernel], 0, float(softmax_scale), q_len, kv_format,
    )
    prev = torch.cuda.current_device()
    if prev != device.index:
        torch.cuda.set_device(device)
    try:
        stream = torch.cuda.current_stream(device).cuda_stream
        _lib.check(lib.tmla_decode_units(ctypes.byref(p), plan.units.data_ptr(), plan.req_first.data_ptr(),
                                         plan.num_units, plan.num_slots, ctypes.c_void_p(stream)),
                   "tmla_decode_units")
    finally:
        if prev != device.index:
            torch.cuda.set_device(prev)
    if _CHECK and not torch.cuda.is_current_stream_capturing():
        st = read_status(device)
        if st:
            raise RuntimeError(f"mla_decode device status 0x{st:x} (bad page id / length, or a wait timed out)")
    return _shaped(out, lse)


def selected_kernel(q, kv_cache, block_table=None, head_dim_v=512, num_splits=1, kernel="auto", q_len=1) -> str:
    """Which kernel ``mla_decode`` runs for these tensors: "sm100" or "generic"."""
    if kv_cache.dim() == 4:
        kv_cache = kv_cache.squeeze(2)
    if q.dim() == 4:
        q_len = q.shape[1]
        q = q.reshape(q.shape[0], q.shape[1] * q.shape[2], q.shape[3])
    batch, num_heads, d_qk = q.shape
    p = _lib.TmlaDecodeParams()
    p.q, p.q_stride_b, p.q_stride_h = q.data_ptr(), q.stride(0), q.stride(1)
    p.kv, p.kv_stride_page, p.kv_stride_tok = kv_cache.data_ptr(), kv_cache.stride(0), kv_cache.stride(1)
    p.page_size = kv_cache.shape[1]
    if block_table is not None:
        p.block_table, p.bt_stride, p.bt_width = block_table.data_ptr(), block_table.stride(0), block_table.shape[1]
        p.num_pages = kv_cache.shape[0]
    else:
        p.num_pages = batch
    p.seqlens = p.out = p.ws_o = p.ws_lse = 256  # only checked for being non-null and aligned
    p.out_stride_b, p.out_stride_h = num_heads * head_dim_v, head_dim_v
    p.batch, p.num_heads, p.d_qk, p.d_v, p.num_splits = batch, num_heads, d_qk, head_dim_v, num_splits
    p.dtype, p.kernel, p.q_len = _DTYPE_CODES[q.dtype], _KERNELS[kernel], int(q_len)
    p.kv_format = _lib.KV_FP8_E4M3 if kv_cache.dtype == torch.uint8 else _lib.KV_SAME
    k = _lib.load().tmla_select_kernel(ctypes.byref(p))
    if k < 0:
        raise _lib.LibraryError(-k, "tmla_select_kernel")
    return {_lib.KERNEL_SM100: "sm100", _lib.KERNEL_GENERIC: "generic"}[k]
