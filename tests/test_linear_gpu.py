"""The weight-streaming projection (``tmla_linear``, ``layer_ops.linear``) against a plain
PyTorch fp32 matmul of the same operands: ``F.linear`` without bias, the op behind the
reference layer's ``wq_a``, ``wkv_a``, ``wq_b`` and ``wo`` (src/triton_mla/model.py:104-108,124)."""

import pytest
import torch
import torch.nn.functional as F

from triton_mla import layer_ops, read_status

pytestmark = pytest.mark.gpu

# The DeepSeek-V3 layer's projections at 16 tokens per GPU, then ragged shapes: a tile and
# k-step tail, one CTA per unit, MMA widths 16 / 32 / 64.
SHAPES = [
    (16, 2112, 7168),    # [wq_a; wkv_a]
    (16, 24576, 1536),   # wq_b
    (16, 7168, 16384),   # wo
    (1, 100, 64),
    (5, 130, 200),
    (33, 257, 72),
    (64, 1000, 512),
    (17, 4096, 4104),
]


def _check(y, x, w):
    ref = x.float() @ w.float().T
    err = (y.float() - ref).abs()
    # One rounding of the fp32 sum to 16 bits (2^-8 relative for bf16), plus the difference of
    # two fp32 summation orders.
    bound = ref.abs() * (2.0 ** -8 if y.dtype == torch.bfloat16 else 2.0 ** -11) + 1e-4 * float(ref.abs().max())
    bad = err > bound
    assert not bool(bad.any()), f"{int(bad.sum())} elements off; worst {float((err - bound).max()):.3e}"


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_linear_matches_fp32_matmul(device, m, n, k, dtype):
    g = torch.Generator(device=device).manual_seed(m * 7919 + n * 31 + k)
    x = torch.randn(m, k, generator=g, device=device).to(dtype)
    w = (torch.randn(n, k, generator=g, device=device) * 0.02).to(dtype)
    y = layer_ops.linear(x, w)
    assert y.shape == (m, n) and y.dtype == dtype
    _check(y, x, w)
    assert read_status(device) == 0


def test_linear_is_deterministic_and_leaves_counters_zero(device):
    g = torch.Generator(device=device).manual_seed(5)
    x = torch.randn(16, 7168, generator=g, device=device).to(torch.bfloat16)
    w = (torch.randn(2112, 7168, generator=g, device=device) * 0.02).to(torch.bfloat16)
    ws = layer_ops.LinearWorkspace()
    y0 = layer_ops.linear(x, w, workspace=ws)
    for _ in range(3):
        assert torch.equal(layer_ops.linear(x, w, workspace=ws), y0), "partials must be summed in a fixed order"
    torch.cuda.synchronize()
    assert int(ws.buf[: 4 * 65536].view(torch.int32).abs().sum()) == 0
    # Shapes with more tiles through the same workspace right after (the earlier partial sums
    # must not be taken for counters), with the partials poisoned in between.
    ws.buf[4 * 65536:].fill_(0x7F)
    for n, k in [(24576, 1536), (7168, 16384), (2112, 7168)]:
        x2 = torch.randn(3, k, generator=g, device=device).to(torch.bfloat16)
        w2 = (torch.randn(n, k, generator=g, device=device) * 0.02).to(torch.bfloat16)
        _check(layer_ops.linear(x2, w2, workspace=ws), x2, w2)


def test_linear_strided_input_and_programmatic_launch(device):
    g = torch.Generator(device=device).manual_seed(11)
    big = torch.randn(16, 3 * 1024, generator=g, device=device).to(torch.bfloat16)
    x = big[:, 1024:2048]                      # row stride 3072
    w = (torch.randn(640, 1024, generator=g, device=device) * 0.02).to(torch.bfloat16)
    a = torch.randn(4096, 4096, device=device)
    _ = a @ a                                  # a kernel for the programmatic launch to follow
    y = layer_ops.linear(x, w, overlap=True)
    _check(y, x, w)
    torch.testing.assert_close(y.float(), F.linear(x, w).float(), rtol=2 ** -7, atol=1e-3)


def test_linear_in_cuda_graph(device):
    g = torch.Generator(device=device).manual_seed(3)
    x = torch.randn(16, 1536, generator=g, device=device).to(torch.bfloat16)
    w = (torch.randn(24576, 1536, generator=g, device=device) * 0.02).to(torch.bfloat16)
    ws = layer_ops.LinearWorkspace()
    layer_ops.linear(x, w, workspace=ws)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = layer_ops.linear(x, w, overlap=True, workspace=ws)
    for seed in range(3):
        x.copy_(torch.randn(16, 1536, generator=g, device=device).to(torch.bfloat16))
        graph.replay()
        torch.cuda.synchronize()
        _check(y, x, w)


def test_linear_rejects_unsupported_inputs(device):
    w = torch.zeros(64, 64, device=device, dtype=torch.bfloat16)
    assert not layer_ops.linear_ok(torch.zeros(65, 64, device=device, dtype=torch.bfloat16), w)
    assert not layer_ops.linear_ok(torch.zeros(4, 64, device=device, dtype=torch.float32), w.float())
    assert not layer_ops.linear_ok(torch.zeros(4, 64, device=device, dtype=torch.float16), w)
    assert not layer_ops.linear_ok(torch.zeros(4, 60, device=device, dtype=torch.bfloat16)[:, :60], w[:, :60])
    with pytest.raises(AssertionError):
        layer_ops.linear(torch.zeros(65, 64, device=device, dtype=torch.bfloat16), w)


@pytest.mark.parametrize("layout", ["nk", "kn"])
@pytest.mark.parametrize("m,n,k,groups", [(16, 128, 512, 128), (16, 512, 128, 128), (5, 200, 72, 9), (40, 64, 264, 3)])
def test_grouped_linear_matches_per_group_matmul(device, layout, m, n, k, groups):
    """Per-group products over strided views, as the absorption einsums use them: x rows of
    several groups interleaved ([m, groups, k]), y written into [m, groups * n]."""
    from triton_mla import _lib
    g = torch.Generator(device=device).manual_seed(m * 13 + n + groups)
    x = torch.randn(m, groups, k, generator=g, device=device).to(torch.bfloat16)
    if layout == "nk":
        w = (torch.randn(groups, n, k, generator=g, device=device) * 0.05).to(torch.bfloat16)
        ref = torch.einsum("mgk,gnk->mgn", x.float(), w.float())
        w_stride, w_gstride, code = k, n * k, _lib.W_NK
    else:
        w = (torch.randn(groups, k, n, generator=g, device=device) * 0.05).to(torch.bfloat16)
        ref = torch.einsum("mgk,gkn->mgn", x.float(), w.float())
        w_stride, w_gstride, code = n, k * n, _lib.W_KN
    y = torch.full((m, groups * n), float("nan"), device=device, dtype=torch.bfloat16)
    layer_ops._linear_launch(x, groups * k, k, w, w_stride, w_gstride, code, y, groups * n, n, m, n, k, groups,
                             False, None)
    err = (y.view(m, groups, n).float() - ref).abs()
    bound = ref.abs() * 2.0 ** -8 + 1e-4 * float(ref.abs().max())
    assert not bool((err > bound).any()), f"max excess {float((err - bound).max()):.3e}"
    assert read_status(device) == 0


def test_timed_out_wait_returns_cleanly_and_heals_the_workspace(device):
    """A bounded wait that runs out (the test-only stall: the first CTA never loads its first
    stage, a barrier that nothing completes) sets TMLA_STATUS_TIMEOUT and the kernel returns:
    the call reports success, the device stays usable, the tile counters end at zero, the tiles
    of the CTAs that finished are right and the stalled CTA's tile is left unwritten.  The next
    call on the same workspace is exact."""
    import ctypes

    from triton_mla import _lib
    from triton_mla.kernel import _status_word

    g = torch.Generator(device=device).manual_seed(11)
    m, n, k = 16, 2112, 7168  # 17 tiles x 56 k-steps over 148 CTAs: tile 0 is cut between CTAs 0 and 1
    x = torch.randn(m, k, generator=g, device=device).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device=device) * 0.02).to(torch.bfloat16)
    lib = _lib.load()
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    ws = torch.zeros(int(lib.tmla_linear_workspace_bytes(m, n, k, 1, sms)), dtype=torch.uint8, device=device)
    counters = ws[: 4 * _lib.LINEAR_MAX_TILES].view(torch.int32)
    status = _status_word(device)
    read_status(device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)

    def call(y, flags, wait_ns):
        p = _lib.TmlaLinearParams(x.data_ptr(), k, w.data_ptr(), k, y.data_ptr(), n, m, n, k, _lib.DTYPE_BF16,
                                  ws.data_ptr(), ws.numel(), sms, flags, status.data_ptr(), 1, _lib.W_NK, 0, 0, 0,
                                  wait_ns)
        return lib.tmla_linear(ctypes.byref(p), stream)

    y = torch.full((m, n), float("nan"), device=device, dtype=torch.bfloat16)
    assert call(y, _lib.LINEAR_FLAG_TEST_STALL, 20_000_000) == 0
    torch.cuda.synchronize()
    assert read_status(device) & _lib.STATUS_TIMEOUT
    assert int(counters.abs().sum()) == 0, "every tile counter back at zero after the timeout"
    assert bool(torch.isnan(y[:, :128].float()).all()), "the stalled CTA's tile is not written"
    _check(y[:, 128:], x, w[128:])
    y2 = torch.empty(m, n, device=device, dtype=torch.bfloat16)
    assert call(y2, 0, 0) == 0
    torch.cuda.synchronize()
    assert read_status(device) == 0
    _check(y2, x, w)
    assert int(counters.abs().sum()) == 0
