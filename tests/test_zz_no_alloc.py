"""The decode entry point that allocates nothing (`tmla_decode_noalloc`).

It is for C-ABI callers that cannot allocate device memory (an FFI host
without a device allocator of its own, or a serving loop that must not call
cudaMalloc): the split partials go to a fixed 32 MiB array of device memory
owned by the library.  Its results must match `tmla_decode`, which takes the
workspace from the caller, on consecutive calls that reuse the array.  This
file is collected last (test_zz_*) so a failure here stops a `-x` run only
after every other test has run.
"""

import ctypes

import numpy as np
import pytest
import torch

import recipes
from oracle import mla_oracle as orc
from triton_mla import _lib

OUT_TOL = 2e-2
LSE_TOL = 1e-3


def _params(q, kv, lens, bt, out, lse, splits, scale, ws=None):
    B, H = q.shape[0], q.shape[1]
    ws_o = ws_lse = None
    if ws is not None:
        o_bytes = (B * H * splits * 512 * 4 + 255) & ~255
        ws_o, ws_lse = ws.data_ptr(), ws.data_ptr() + o_bytes
    return _lib.TmlaDecodeParams(
        q.data_ptr(), q.stride(0), q.stride(1), kv.data_ptr(), kv.stride(0), kv.stride(1), kv.shape[0], kv.shape[1],
        lens.data_ptr(), bt.data_ptr(), bt.stride(0), bt.shape[1], out.data_ptr(), out.stride(0), out.stride(1),
        lse.data_ptr(), lse.stride(0), ws_o, ws_lse, None, B, H, 576, 512, splits, _lib.DTYPE_BF16,
        _lib.KERNEL_AUTO, 0, scale)


def test_noalloc_rejects_workspace_beyond_its_array():
    lib = _lib.load()
    p = _lib.TmlaDecodeParams()
    p.batch, p.num_heads, p.d_qk, p.d_v, p.num_splits = 1024, 128, 576, 512, 64  # 1 GiB of partials
    p.dtype, p.page_size, p.softmax_scale = _lib.DTYPE_BF16, 64, 0.07
    assert lib.tmla_workspace_bytes(1024, 128, 64, 512) > _lib.NOALLOC_SCRATCH_BYTES
    assert lib.tmla_decode_noalloc(ctypes.byref(p), None) == _lib.ERR_WORKSPACE


@pytest.mark.gpu
def test_noalloc_matches_tmla_decode_on_consecutive_calls(device):
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    for seed, lens, splits in ((3, [4096, 1000, 0, 65], 5), (4, [777, 2048, 64], 3)):
        case = recipes.paged_case(lens, 128, 64, seed=seed)
        q, kv, sl, bt = (case[k].to(device) for k in ("q", "kv", "seqlens", "block_table"))
        B = q.shape[0]
        ref_out = torch.empty(B, 128, 512, dtype=torch.bfloat16, device=device)
        ref_lse = torch.empty(B, 128, dtype=torch.float32, device=device)
        ws = torch.empty(lib.tmla_workspace_bytes(B, 128, splits, 512), dtype=torch.uint8, device=device)
        assert 0 < ws.numel() <= _lib.NOALLOC_SCRATCH_BYTES
        p_ref = _params(q, kv, sl, bt, ref_out, ref_lse, splits, case["scale"], ws)
        assert lib.tmla_decode(ctypes.byref(p_ref), stream) == 0
        out = torch.full_like(ref_out, float("nan"))
        lse = torch.full_like(ref_lse, float("nan"))
        p = _params(q, kv, sl, bt, out, lse, splits, case["scale"])
        assert lib.tmla_decode_noalloc(ctypes.byref(p), stream) == 0
        torch.cuda.synchronize(device)
        assert (out.float() - ref_out.float()).abs().max().item() <= OUT_TOL
        valid = sl > 0
        assert (lse[valid] - ref_lse[valid]).abs().max().item() <= LSE_TOL
        assert torch.all(out[~valid] == 0) and torch.all(torch.isneginf(lse[~valid]))
        # And against the reference algorithm (numpy oracle) on the same inputs.
        o_np, l_np = orc.mla_decode_ref(case["q"].float().numpy(), case["kv"].float().numpy(),
                                        case["seqlens"].numpy(), case["block_table"].numpy(),
                                        softmax_scale=case["scale"])
        assert np.abs(out.float().cpu().numpy() - o_np).max() <= OUT_TOL


@pytest.mark.gpu
def test_noalloc_ignores_the_partial_only_flag(device):
    """With one split and TMLA_FLAG_PARTIAL_ONLY set, the call still decodes whole (the flag
    is stage-1 semantics, which tmla_decode ignores too) instead of asking for a workspace."""
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    case = recipes.paged_case([300, 64], 128, 64, seed=6)
    q, kv, sl, bt = (case[k].to(device) for k in ("q", "kv", "seqlens", "block_table"))
    out = torch.empty(2, 128, 512, dtype=torch.bfloat16, device=device)
    lse = torch.empty(2, 128, dtype=torch.float32, device=device)
    ref_out, ref_lse = torch.empty_like(out), torch.empty_like(lse)
    p_ref = _params(q, kv, sl, bt, ref_out, ref_lse, 1, case["scale"])
    p = _params(q, kv, sl, bt, out, lse, 1, case["scale"])
    p_ref.flags = p.flags = _lib.FLAG_PARTIAL_ONLY
    assert lib.tmla_decode(ctypes.byref(p_ref), stream) == 0
    assert lib.tmla_decode_noalloc(ctypes.byref(p), stream) == 0
    torch.cuda.synchronize(device)
    assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)
