"""Host-side checks that need no GPU: the C library loads and exports every
symbol the header declares, the ctypes mirror matches the C struct, argument
validation and kernel selection, the split heuristic, and the Python wrapper's
drop-in error behaviour (kernel.py:235-245 of the reference)."""

import ctypes
import re

import pytest
import torch

from conftest import ROOT
from triton_mla import _lib, get_num_splits, mla_decode
from triton_mla.kernel import selected_kernel

HEADER = ROOT / "include" / "triton_mla_b200.h"


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    declared = set(re.findall(r"\b(tmla_[a-z_0-9]+)\s*\(", HEADER.read_text()))
    assert declared == set(_lib.EXPORTED), declared ^ set(_lib.EXPORTED)
    for name in declared:
        assert hasattr(lib, name), name


def test_library_exports_nothing_the_header_does_not_declare():
    """The other direction: every tmla_ function the library exports is in the header."""
    import shutil
    import subprocess

    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("nm (binutils) not available")
    out = subprocess.run([nm, "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.split()[-1].startswith("tmla")}
    declared = set(re.findall(r"\b(tmla_[a-z_0-9]+)\s*\(", HEADER.read_text()))
    assert exported == declared, exported ^ declared


def test_abi_version_and_struct_layout():
    lib = _lib.load()
    assert lib.tmla_abi_version() == _lib.ABI_VERSION
    assert lib.tmla_params_bytes() == ctypes.sizeof(_lib.TmlaDecodeParams)
    # Header constants match the binding's.
    text = HEADER.read_text()
    for name in ("OK", "ERR_INVALID_ARG", "ERR_UNSUPPORTED", "ERR_MISALIGNED", "ERR_CUDA", "ERR_WORKSPACE",
                 "STATUS_BAD_PAGE", "STATUS_TIMEOUT", "STATUS_RANGE", "DTYPE_BF16", "DTYPE_FP16", "DTYPE_FP32", "KERNEL_AUTO",
                 "KERNEL_GENERIC", "KERNEL_SM100", "FLAG_PARTIAL_ONLY", "MAX_BATCH"):
        m = re.search(rf"#define TMLA_{name}\s+(0x[0-9a-fA-F]+|\d+)", text)
        assert m and int(m.group(1), 0) == getattr(_lib, name), name


def test_error_strings():
    for code in range(6):
        assert _lib.error_string(code)
    assert _lib.error_string(99) == "unknown error"


def _params(**kw):
    p = _lib.TmlaDecodeParams()
    p.q = p.kv = p.seqlens = p.out = 16
    p.q_stride_b, p.q_stride_h = 128 * 576, 576
    p.kv_stride_page, p.kv_stride_tok = 64 * 576, 576
    p.num_pages, p.page_size = 10, 64
    p.block_table, p.bt_stride, p.bt_width = 16, 4, 4
    p.out_stride_b, p.out_stride_h = 128 * 512, 512
    p.batch, p.num_heads, p.d_qk, p.d_v, p.num_splits = 2, 128, 576, 512, 1
    p.dtype, p.kernel, p.softmax_scale = _lib.DTYPE_BF16, _lib.KERNEL_AUTO, 0.07
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize("bad", [
    dict(d_v=500), dict(d_qk=512 + 48), dict(d_qk=512), dict(num_heads=0), dict(num_splits=0),
    dict(batch=-1), dict(dtype=7), dict(page_size=0), dict(q=None), dict(block_table=None, num_pages=3),
])
def test_select_kernel_rejects_invalid(bad):
    rc = _lib.load().tmla_select_kernel(ctypes.byref(_params(**bad)))
    assert rc == -_lib.ERR_INVALID_ARG


def test_batches_beyond_the_grid_limit_are_refused():
    # One decode call covers at most TMLA_MAX_BATCH requests and splits (a grid dimension's
    # limit); beyond it the call is refused before any launch.
    lib = _lib.load()
    big = dict(batch=_lib.MAX_BATCH + 1, num_pages=10)
    assert lib.tmla_select_kernel(ctypes.byref(_params(**big))) == -_lib.ERR_UNSUPPORTED
    assert lib.tmla_decode(ctypes.byref(_params(**big)), None) == _lib.ERR_UNSUPPORTED
    ws = dict(num_splits=_lib.MAX_BATCH + 1, ws_o=16, ws_lse=16)
    assert lib.tmla_select_kernel(ctypes.byref(_params(**ws))) == -_lib.ERR_UNSUPPORTED
    assert lib.tmla_select_kernel(ctypes.byref(_params(batch=_lib.MAX_BATCH))) >= 0


def test_select_kernel_needs_workspace_for_splits():
    rc = _lib.load().tmla_select_kernel(ctypes.byref(_params(num_splits=4)))
    assert rc == -_lib.ERR_WORKSPACE


def test_select_kernel_generic_for_other_dims():
    lib = _lib.load()
    assert lib.tmla_select_kernel(ctypes.byref(_params(d_qk=256 + 32, d_v=256))) == _lib.KERNEL_GENERIC
    assert lib.tmla_select_kernel(ctypes.byref(_params(dtype=_lib.DTYPE_FP32))) == _lib.KERNEL_GENERIC
    assert lib.tmla_select_kernel(ctypes.byref(_params(kernel=_lib.KERNEL_GENERIC))) == _lib.KERNEL_GENERIC


def test_workspace_bytes():
    lib = _lib.load()
    assert lib.tmla_workspace_bytes(4, 128, 1, 512) == 0
    n = lib.tmla_workspace_bytes(4, 128, 3, 512)
    assert n >= 4 * 128 * 3 * 513 * 4 and n % 256 == 0


@pytest.mark.parametrize("batch,heads,seqlen", [(1, 128, 65536), (4, 128, 65536), (32, 128, 4096),
                                                (128, 128, 8192), (256, 128, 16384), (2, 16, 1024), (1, 16, 1)])
def test_num_splits_properties(batch, heads, seqlen):
    s = get_num_splits(batch, heads, seqlen, 148)
    assert 1 <= s <= 64
    assert s <= max(-(-seqlen // 128), 1)
    # A batch that already fills the machine is split at most to even out the last wave.
    if batch * ((heads + 127) // 128) >= 148:
        assert s <= 2


def test_num_splits_b200_configs():
    # BASELINE configs on a 148-SM B200: the long-context case splits to about one wave of clusters.
    s3 = get_num_splits(4, 128, 65536, 148)
    assert 4 * s3 <= 74 and 4 * s3 >= 60
    assert get_num_splits(32, 128, 4096, 148) == 2
    assert get_num_splits(0, 128, 4096, 148) == 1


@pytest.mark.parametrize("batch,seqlen,want", [
    (32, 4096, 2),     # config 2
    (4, 65536, 18),    # config 3
    (16, 8192, 4),     # config 5's decode
    (4, 4096, 16),     # a rank's share of config 2 at N = 8
    (1, 1024, 8),
    (24, 1024, 3),
    (128, 16384, 4),
    (256, 8192, 2),
])
def test_num_splits_matches_the_measured_choices(batch, seqlen, want):
    # The split counts the rule gives for shapes whose call times were measured on a B200
    # (each the fastest count measured, or within 0.13% of it).
    assert get_num_splits(batch, 128, seqlen, 148) == want


def test_wrapper_assertions_match_reference():
    q = torch.zeros(2, 16, 576, dtype=torch.bfloat16)
    kv = torch.zeros(2, 64, 576, dtype=torch.bfloat16)
    lens = torch.tensor([3, 4], dtype=torch.int32)
    with pytest.raises(AssertionError):
        mla_decode(q, torch.zeros(2, 64, 2, 576, dtype=torch.bfloat16), lens)   # kv head dim != 1
    with pytest.raises(AssertionError):
        mla_decode(q[0], kv, lens)                                                # q not 3-D
    with pytest.raises(AssertionError):
        mla_decode(q, kv[..., :575], lens)                                         # width mismatch
    with pytest.raises(AssertionError):
        mla_decode(q, kv, lens, head_dim_v=500)                                    # not a power of two
    with pytest.raises(AssertionError):
        mla_decode(q, kv.half(), lens)                                             # dtype mismatch
    with pytest.raises(AssertionError):
        mla_decode(q, torch.zeros(3, 64, 576, dtype=torch.bfloat16), lens)        # dense batch mismatch
    with pytest.raises(AssertionError):
        mla_decode(q.transpose(1, 2).contiguous().transpose(1, 2), kv, lens)       # inner stride != 1


def test_wrapper_refuses_cpu_tensors():
    q = torch.zeros(2, 16, 576, dtype=torch.bfloat16)
    kv = torch.zeros(2, 64, 576, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        mla_decode(q, kv, torch.tensor([3, 4], dtype=torch.int32))


def test_selected_kernel_reports_generic_for_non_deepseek_dims_on_cpu_tensors():
    q = torch.zeros(2, 16, 256 + 32, dtype=torch.bfloat16)
    kv = torch.zeros(2, 64, 256 + 32, dtype=torch.bfloat16)
    assert selected_kernel(q, kv, head_dim_v=256) == "generic"


# ----------------------------------------------------------------------------- per-request split plan
def _check_plan(lens, units, req_first):
    import numpy as np
    lens = np.asarray(lens)
    tiles = (np.maximum(lens, 0) + 63) // 64
    seen = {}
    for b, s, ns, slot in units.tolist():
        assert 1 <= ns <= 64 and 0 <= s < ns
        assert (b, s) not in seen
        seen[(b, s)] = ns
        if ns == 1:
            assert slot == -1
        else:
            assert slot == req_first[b] + s
    for b in range(len(lens)):
        ns = seen[(b, 0)]
        assert all(seen[(b, s)] == ns for s in range(ns))
        assert req_first[b + 1] - req_first[b] == (ns if ns > 1 else 0)
    # longest unit first (tiles of each split as split_range cuts them)
    sizes = []
    for b, s, ns, _ in units.tolist():
        per = -(-int(tiles[b]) // ns)
        sizes.append(max(0, min(int(tiles[b]), (s + 1) * per) - min(int(tiles[b]), s * per)))
    assert sizes == sorted(sizes, reverse=True)


def test_plan_units_reproduces_uniform_splits_for_uniform_batches():
    from triton_mla.kernel import plan_units
    units, first = plan_units([4096] * 32, 128, 148)
    assert set(units[:, 2].tolist()) == {2} and len(units) == 64
    _check_plan([4096] * 32, units, first)
    units, first = plan_units([65536] * 4, 128, 148)
    assert set(units[:, 2].tolist()) == {18}
    _check_plan([65536] * 4, units, first)


def test_plan_units_on_ragged_batches():
    import numpy as np
    from triton_mla.kernel import plan_units
    rng = np.random.default_rng(0)
    for trial in range(20):
        lens = rng.integers(0, 16385, size=int(rng.integers(1, 300))).tolist()
        units, first = plan_units(lens, 128 if trial % 2 else 256, 148)
        _check_plan(lens, units, first)
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(1, 16385, (256,), generator=g).tolist()
    units, first = plan_units(lens, 128, 148)
    _check_plan(lens, units, first)
    lens = [65536] + [100] * 300  # one long request among many short ones is split, the short ones not
    units, first = plan_units(lens, 128, 148)
    _check_plan(lens, units, first)
    assert units[units[:, 0] == 0][0, 2] > 1 and set(units[units[:, 0] > 0][:, 2].tolist()) == {1}


def test_plan_units_edge_cases():
    import numpy as np
    from triton_mla.kernel import plan_units
    units, first = plan_units([], 128, 148)
    assert units.shape == (0, 4) and first.tolist() == [0]
    units, first = plan_units([0, 0, 0], 128, 148)
    assert units[:, 2].tolist() == [1, 1, 1] and first.tolist() == [0, 0, 0, 0]
    lib = _lib.load()
    bad = np.zeros(4, dtype=np.int32)
    assert lib.tmla_plan_units(None, 2, 128, 148, 8, bad.ctypes.data, bad.ctypes.data) < 0


def test_plan_units_device_rejects_bad_arguments():
    """tmla_plan_units_device checks its arguments before it launches anything."""
    lib = _lib.load()
    p = ctypes.c_void_p(256)  # never dereferenced: every call below is rejected first
    bad = [
        (p, 4, 128, 148, 3, 0, p, p),        # capacity below the batch (one unit per request at least)
        (p, 4, 128, 148, 65536, 0, p, p),    # capacity above the grid limit
        (p, 4, 128, 148, 8, -1, p, p),       # negative slot capacity
        (p, 4, 0, 148, 8, 0, p, p),          # no heads
        (p, 4, 128, 148, 8, 0, p, None),     # no req_first
        (None, 4, 128, 148, 8, 0, p, p),     # no lengths
        (p, -1, 128, 148, 8, 0, p, p),       # negative batch
    ]
    for args in bad:
        assert lib.tmla_plan_units_device(*args, None) == _lib.ERR_INVALID_ARG, args


def _linear_plan(m, n, k, sms, groups=1):
    """The projection kernel's work split, restated: units (group, 128-row tile, 128-column
    k-step), in that order, cut into min(sms, units) equal contiguous ranges."""
    tiles, steps = -(-n // 128) * groups, -(-k // 128)
    units = tiles * steps
    grid = min(sms, units)
    owner = lambda u: ((u + 1) * grid - 1) // units  # noqa: E731
    parts = max(owner(t * steps + steps - 1) - owner(t * steps) + 1 for t in range(tiles))
    tok = 16 if m <= 16 else (32 if m <= 32 else 64)
    counters = 65536 * 4  # TMLA_LINEAR_MAX_TILES counters, whatever the shape
    return counters + (tiles * parts * tok * 128 * 4 if parts > 1 else 0)


@pytest.mark.parametrize("m,n,k,sms,groups", [(16, 2112, 7168, 148, 1), (16, 24576, 1536, 148, 1),
                                              (16, 7168, 16384, 148, 1), (1, 100, 64, 148, 1), (33, 257, 72, 148, 1),
                                              (64, 1000, 512, 7, 1), (16, 128, 512, 148, 128), (16, 512, 128, 148, 128),
                                              (3, 200, 72, 5, 9)])
def test_linear_workspace_bytes(m, n, k, sms, groups):
    assert _lib.load().tmla_linear_workspace_bytes(m, n, k, groups, sms) == _linear_plan(m, n, k, sms, groups)


def test_linear_workspace_bytes_rejects_bad_shapes():
    lib = _lib.load()
    for args in [(0, 8, 8, 1, 148), (65, 8, 8, 1, 148), (4, 0, 8, 1, 148), (4, 8, 0, 1, 148), (4, 8, 8, 0, 148)]:
        assert lib.tmla_linear_workspace_bytes(*args) == -_lib.ERR_INVALID_ARG


def test_linear_workspace_bytes_default_sm_count():
    """num_sms <= 0 means the current device's SM count, in the size query as in the launch;
    without a device the query reports the CUDA error instead of a size."""
    lib = _lib.load()
    got = lib.tmla_linear_workspace_bytes(16, 2112, 7168, 1, 0)
    if torch.cuda.is_available():
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        assert got == lib.tmla_linear_workspace_bytes(16, 2112, 7168, 1, sms) > 0
    else:
        assert got == -_lib.ERR_CUDA and lib.tmla_last_cuda_error()


def _linear_params(**kw):
    """TmlaLinearParams with fake (aligned, never dereferenced) pointers: every case below is
    rejected by the argument checks before any CUDA call."""
    p = _lib.TmlaLinearParams()
    p.x, p.w, p.y = 4096, 8192, 12288
    p.m, p.n, p.k, p.groups = 16, 256, 512, 1
    p.x_stride, p.w_stride, p.y_stride = 512, 512, 256
    p.dtype, p.w_layout, p.num_sms = _lib.DTYPE_BF16, _lib.W_NK, 148
    for key, value in kw.items():
        setattr(p, key, value)
    return p


@pytest.mark.parametrize("kw,code", [
    (dict(x=None), _lib.ERR_INVALID_ARG),
    (dict(dtype=_lib.DTYPE_FP32), _lib.ERR_UNSUPPORTED),
    (dict(m=0), _lib.ERR_INVALID_ARG),
    (dict(m=65), _lib.ERR_INVALID_ARG),
    (dict(groups=0), _lib.ERR_INVALID_ARG),
    (dict(w_layout=7), _lib.ERR_INVALID_ARG),
    (dict(x_stride=256), _lib.ERR_INVALID_ARG),
    (dict(w_layout=_lib.W_KN, w_stride=128), _lib.ERR_INVALID_ARG),
    (dict(x=4104), _lib.ERR_MISALIGNED),
    (dict(x_stride=516), _lib.ERR_MISALIGNED),
    (dict(groups=2, w_group_stride=4), _lib.ERR_MISALIGNED),
    (dict(), _lib.ERR_WORKSPACE),  # no workspace: 256 x 512 on 148 SMs cuts tiles
])
def test_linear_rejects_bad_arguments_before_any_launch(kw, code):
    p = _linear_params(**kw)
    assert _lib.load().tmla_linear(ctypes.byref(p), None) == code


def test_linear_helpers_refuse_cpu_tensors():
    from triton_mla import layer_ops
    x, w = torch.zeros(4, 64, dtype=torch.bfloat16), torch.zeros(64, 64, dtype=torch.bfloat16)
    assert not layer_ops.linear_ok(x, w) and not layer_ops.linear_preferred(x, w)
    with pytest.raises(AssertionError):
        layer_ops.linear(x, w)


def test_split_rule_restated_for_torch_compile_matches_the_library():
    from triton_mla.kernel import _num_splits_rule
    lib = _lib.load()
    for b in (1, 2, 3, 4, 16, 32, 64, 256, 1024):
        for h in (16, 128, 256):
            for s in (1, 64, 100, 4096, 16384, 65536):
                for sms in (132, 148):
                    assert _num_splits_rule(b, h, s, sms) == lib.tmla_num_splits(b, h, s, sms), (b, h, s, sms)


def test_decode_is_a_registered_torch_operator_with_a_meta_kernel():
    """torch.ops.triton_mla.decode exists with the documented schema, and its Meta kernel
    accepts meta tensors (what torch.compile's tracing runs)."""
    op = torch.ops.triton_mla.decode
    schema = str(op.default._schema)
    assert "Tensor(a!) out" in schema and "Tensor(b!) lse" in schema and "int num_splits" in schema
    meta = torch.device("meta")
    q = torch.empty(4, 128, 576, dtype=torch.bfloat16, device=meta)
    kv = torch.empty(64, 64, 576, dtype=torch.bfloat16, device=meta)
    lens = torch.empty(4, dtype=torch.int32, device=meta)
    bt = torch.empty(4, 16, dtype=torch.int32, device=meta)
    out = torch.empty(4, 128, 512, dtype=torch.bfloat16, device=meta)
    lse = torch.empty(4, 128, dtype=torch.float32, device=meta)
    op(q, kv, lens, bt, out, lse, 2, 0.07, 0, 1, None)


@pytest.mark.parametrize("args, code", [
    ((256, 32, 32, 1, 1), _lib.OK),                    # count 0 below: nothing to do, nothing launched
    ((0, 32, 32, 1, 1), _lib.ERR_INVALID_ARG),         # null base
    ((256, 0, 32, 1, 1), _lib.ERR_INVALID_ARG),        # empty chunk
    ((256, 32, 16, 1, 1), _lib.ERR_INVALID_ARG),       # chunks overlap (stride < chunk)
    ((256, 32, 32, 1, 0), _lib.ERR_INVALID_ARG),       # no CTAs
    ((256, 32, 32, -1, 1), _lib.ERR_INVALID_ARG),      # negative count
    ((264, 32, 32, 1, 1), _lib.ERR_MISALIGNED),        # base not 16-byte aligned
    ((256, 24, 32, 1, 1), _lib.ERR_MISALIGNED),        # chunk not a multiple of 16
    ((256, 32, 40, 1, 1), _lib.ERR_MISALIGNED),        # stride not a multiple of 16
])
def test_l2_prefetch_rejects_bad_arguments_before_any_launch(args, code):
    """tmla_l2_prefetch checks its arguments before it launches anything (the first case has
    count 0, which returns at once)."""
    base, chunk, stride, count, ctas = args
    if code == _lib.OK:
        count = 0
    rc = _lib.load().tmla_l2_prefetch(ctypes.c_void_p(base), chunk, stride, count, ctas, None)
    assert rc == code


def test_l2_prefetch_helper_refuses_cpu_tensors():
    from triton_mla import layer_ops
    with pytest.raises(AssertionError):
        layer_ops.l2_prefetch(torch.zeros(64, dtype=torch.bfloat16))
