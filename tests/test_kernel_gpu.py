"""Parity of the CUDA decode path (called through the C ABI by ``mla_decode``)
with the reference: golden vectors made by the reference's own code, the numpy
oracle on the same seeded inputs, and size-independent properties at the
BASELINE configs' full sizes.

Tolerances: output max-abs <= 2e-2 and LSE max-abs <= 1e-3
against the fp32 reference for 16-bit inputs; zero-length rows exactly 0 / -inf.
"""

import math

import numpy as np
import pytest
import torch

import recipes
from conftest import load_golden
from oracle import mla_oracle as orc
from triton_mla import _lib, mla_decode, read_status, selected_kernel

pytestmark = pytest.mark.gpu

OUT_TOL = 2e-2
LSE_TOL = 1e-3
KERNELS = ["auto", "generic"]


def to_dev(case, device):
    out = dict(case)
    for k in ("q", "kv", "seqlens", "block_table"):
        if case.get(k) is not None:
            out[k] = case[k].to(device)
    return out


def oracle_of(case, **kw):
    bt = case["block_table"]
    return orc.mla_decode_ref(case["q"].float().numpy(), case["kv"].float().numpy(), case["seqlens"].numpy(),
                              None if bt is None else bt.numpy(), softmax_scale=case["scale"], dtype=np.float64, **kw)


def check(out, lse, ref_out, ref_lse, seqlens, out_tol=OUT_TOL, lse_tol=LSE_TOL):
    out = out.float().cpu().numpy()
    lse = lse.cpu().numpy()
    valid = np.asarray(seqlens) > 0
    err = np.abs(out - ref_out).max() if out.size else 0.0
    assert err <= out_tol, f"output max-abs error {err:.3e} > {out_tol}"
    if valid.any():
        lerr = np.abs(lse[valid] - ref_lse[valid]).max()
        assert lerr <= lse_tol, f"LSE max-abs error {lerr:.3e} > {lse_tol}"
    assert np.all(out[~valid] == 0), "zero-length rows must be exactly 0"
    assert np.all(np.isneginf(lse[~valid])), "zero-length rows must have LSE -inf"


def run(case, device, **kw):
    c = to_dev(case, device)
    return mla_decode(c["q"], c["kv"], c["seqlens"], c["block_table"], softmax_scale=c["scale"],
                      return_lse=True, **kw)


# ----------------------------------------------------------------------------- reference test grid
@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("num_heads", [16, 128])
@pytest.mark.parametrize("num_splits", [1, 4, 16])
@pytest.mark.parametrize("paged", [False, True])
def test_matches_reference(device, kernel, num_heads, num_splits, paged):
    """tests/test_kernel.py:29-51 of the reference: seqlens [0, 1, 513, 4096], seed 0."""
    case = recipes.ref_grid(num_heads, paged)
    gold = load_golden(f"ref_grid_h{num_heads}")
    pg = recipes.ref_grid(num_heads, True)  # the golden file was made from the paged layout
    assert str(gold["digest"]) == recipes.tensor_digest(pg["q"], pg["kv"], pg["seqlens"], pg["block_table"])
    out, lse = run(case, device, num_splits=num_splits, kernel=kernel)
    check(out, lse, gold["out"], gold["lse"], case["seqlens"])


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("name,make", [("cfg1", recipes.cfg1), ("edge_p16_h20", recipes.edge_p16_h20)])
def test_golden_cases(device, kernel, name, make):
    case = make()
    gold = load_golden(name)
    assert str(gold["digest"]) == recipes.tensor_digest(case["q"], case["kv"], case["seqlens"], case["block_table"])
    for splits in (None, 1, 3):
        out, lse = run(case, device, num_splits=splits, kernel=kernel)
        check(out, lse, gold["out"], gold["lse"], case["seqlens"])


def test_default_splits_and_flashmla_layout(device):
    """tests/test_kernel.py:54-61: num_splits=None, 4-D [B, S, 1, 576] cache, default scale."""
    case = recipes.flashmla_layout()
    gold = load_golden("flashmla_layout")
    c = to_dev(case, device)
    out = mla_decode(c["q"], c["kv"], c["seqlens"])
    assert out.shape == (2, 16, 512) and out.dtype == torch.bfloat16
    err = (out.float().cpu().numpy() - gold["out"]).__abs__().max()
    assert err <= OUT_TOL
    err_t = (out.float().cpu().numpy() - gold["out_torch"]).__abs__().max()
    assert err_t <= OUT_TOL


# ----------------------------------------------------------------------------- shapes, dtypes, layouts
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("kernel", KERNELS)
def test_dtypes(device, dtype, kernel):
    case = recipes.paged_case([0, 1, 64, 65, 700, 2048], 128, 64, seed=11, dtype=dtype)
    ref_out, ref_lse = oracle_of(case)
    out, lse = run(case, device, num_splits=2, kernel=kernel)
    assert out.dtype == dtype
    check(out, lse, ref_out, ref_lse, case["seqlens"])


def test_fp32_generic(device):
    case = recipes.paged_case([0, 5, 300], 16, 64, seed=12, dtype=torch.float32)
    ref_out, ref_lse = oracle_of(case)
    out, lse = run(case, device, num_splits=2)
    check(out, lse, ref_out, ref_lse, case["seqlens"], out_tol=1e-4, lse_tol=1e-4)


@pytest.mark.parametrize("page_size", [1, 3, 16, 48, 64, 100, 128, 256])
def test_page_sizes(device, page_size):
    case = recipes.paged_case([1, 63, 64, 129, 1000], 128, page_size, seed=20 + page_size)
    ref_out, ref_lse = oracle_of(case)
    for kernel in KERNELS:
        out, lse = run(case, device, num_splits=3, kernel=kernel)
        check(out, lse, ref_out, ref_lse, case["seqlens"])


@pytest.mark.parametrize("num_heads", [1, 20, 64, 129, 256])
def test_head_counts(device, num_heads):
    case = recipes.paged_case([0, 77, 640], num_heads, 64, seed=30 + num_heads)
    ref_out, ref_lse = oracle_of(case)
    for kernel in KERNELS:
        out, lse = run(case, device, num_splits=2, kernel=kernel)
        check(out, lse, ref_out, ref_lse, case["seqlens"])


@pytest.mark.parametrize("d_v,d_rope", [(256, 32), (128, 64), (512, 32), (64, 16)])
def test_other_latent_dims(device, d_v, d_rope):
    g = torch.Generator().manual_seed(d_v + d_rope)
    lens = torch.tensor([0, 9, 300], dtype=torch.int32)
    q = torch.randn(3, 16, d_v + d_rope, generator=g).bfloat16()
    kv = torch.randn(3, 320, d_v + d_rope, generator=g).bfloat16()
    assert selected_kernel(q.to(device), kv.to(device), head_dim_v=d_v) == "generic"
    ref_out, ref_lse = orc.mla_decode_ref(q.float().numpy(), kv.float().numpy(), lens.numpy(), None, head_dim_v=d_v)
    out, lse = mla_decode(q.to(device), kv.to(device), lens.to(device), head_dim_v=d_v, num_splits=2, return_lse=True)
    check(out, lse, ref_out, ref_lse, lens)


def test_strided_inputs(device):
    """q with padded head stride, cache pages with padded rows, block table a column slice."""
    g = torch.Generator().manual_seed(5)
    lens = torch.tensor([100, 1, 257], dtype=torch.int32)
    q_big = torch.randn(3, 128, 640, generator=g).bfloat16()
    q = q_big[:, :, :576]
    pool = torch.randn(40, 64, 584, generator=g).bfloat16()
    kv = pool[:, :, :576]
    bt_big = torch.randperm(40, generator=g)[:30].view(3, 10).int()
    bt_full = torch.zeros(3, 12, dtype=torch.int32)
    bt_full[:, 1:11] = bt_big
    bt = bt_full[:, 1:11]
    case = dict(q=q, kv=kv, seqlens=lens, block_table=bt, scale=192 ** -0.5)
    ref_out, ref_lse = orc.mla_decode_ref(q.float().numpy(), kv.float().numpy(), lens.numpy(), bt.numpy(),
                                          softmax_scale=case["scale"])
    for kernel in KERNELS:
        out, lse = mla_decode(q.to(device), kv.to(device), lens.to(device), bt.to(device), softmax_scale=case["scale"],
                              num_splits=2, return_lse=True, kernel=kernel)
        check(out, lse, ref_out, ref_lse, lens)


@pytest.mark.parametrize("num_splits", [1, 3])
def test_strided_out_view_and_partial_head_tile(device, num_splits):
    """The tcgen05 kernel writes its output with tensor-tile stores: a padded ``out=`` view
    receives exactly its own rows and columns (the padding around it is untouched), and the
    rows past H in the last 128-head tile are not written."""
    lens = [300, 0, 129]
    case = recipes.paged_case(lens, 129, 64, seed=31)
    c = to_dev(case, device)
    big = torch.full((3, 136, 520), 7.0, dtype=torch.bfloat16, device=device)
    view = big[:, 3:132, 8:]
    assert selected_kernel(c["q"], c["kv"], c["block_table"], num_splits=num_splits) == "sm100"
    out, lse = mla_decode(c["q"], c["kv"], c["seqlens"], c["block_table"], softmax_scale=c["scale"],
                          num_splits=num_splits, return_lse=True, out=view)
    assert out.data_ptr() == view.data_ptr()
    ref_out, ref_lse = oracle_of(case)
    check(out, lse, ref_out, ref_lse, lens)
    pad = torch.ones(big.shape, dtype=torch.bool, device=device)
    pad[:, 3:132, 8:] = False
    assert bool((big[pad] == 7.0).all()), "the output store wrote outside the out= view"
    assert read_status(device) == 0


def test_cuda_graph_capture_with_default_splits(device):
    """mla_decode(num_splits=None) captured in a CUDA graph (no host sync inside capture)
    and replayed after the lengths and the query changed in place."""
    case = recipes.paged_case([300, 4096, 17, 1000], 128, 64, seed=41)
    c = to_dev(case, device)
    q, lens, bt, kv = c["q"].clone(), c["seqlens"].clone(), c["block_table"], c["kv"]
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):  # warm-up outside the capture, as torch.cuda.graphs asks
        mla_decode(q, kv, lens, bt, softmax_scale=c["scale"], return_lse=True)
    torch.cuda.current_stream(device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out, lse = mla_decode(q, kv, lens, bt, softmax_scale=c["scale"], return_lse=True)
    g = torch.Generator().manual_seed(42)
    for new_lens in ([300, 4096, 17, 1000], [4096, 1, 0, 2500], [64, 65, 4000, 3]):
        q_new = torch.randn(q.shape, generator=g).to(q.dtype)
        q.copy_(q_new.to(device))
        lens.copy_(torch.tensor(new_lens, dtype=torch.int32, device=device))
        graph.replay()
        torch.cuda.synchronize(device)
        sub = dict(case, q=q_new, seqlens=torch.tensor(new_lens, dtype=torch.int32))
        ref_out, ref_lse = oracle_of(sub)
        check(out, lse, ref_out, ref_lse, new_lens)
        assert read_status(device) == 0
    del graph


def test_empty_batch(device):
    q = torch.zeros(0, 128, 576, dtype=torch.bfloat16, device=device)
    kv = torch.zeros(4, 64, 576, dtype=torch.bfloat16, device=device)
    out, lse = mla_decode(q, kv, torch.zeros(0, dtype=torch.int32, device=device),
                          torch.zeros(0, 3, dtype=torch.int32, device=device), return_lse=True)
    assert out.shape == (0, 128, 512) and lse.shape == (0, 128)


def test_bad_page_id_is_flagged_not_faulted(device):
    case = recipes.paged_case([200, 50], 16, 64, seed=41)
    c = to_dev(case, device)
    bt = c["block_table"].clone()
    bt[0, 1] = 10_000_000  # outside the pool
    read_status(device)
    with pytest.raises(RuntimeError, match="status"):
        mla_decode(c["q"], c["kv"], c["seqlens"], bt, num_splits=1, kernel="generic")
    assert read_status(device) == 0  # the failing call cleared it
    # The good request is unaffected.
    out = mla_decode(c["q"][1:], c["kv"], c["seqlens"][1:], c["block_table"][1:], softmax_scale=c["scale"])
    ref_out, _ = oracle_of(dict(case, q=case["q"][1:], seqlens=case["seqlens"][1:],
                                block_table=case["block_table"][1:]))
    assert np.abs(out.float().cpu().numpy() - ref_out).max() <= OUT_TOL


def _oracle_without_pages(case, bad):
    """The oracle over each request's tokens minus those in the block-table slots ``bad[b]``
    (the masked tokens of a block table whose entries there lie outside the pool)."""
    q = case["q"].float().numpy()
    kv = case["kv"].float().numpy()
    page = kv.shape[1]
    outs, lses, lens = [], [], []
    for b in range(q.shape[0]):
        n = int(case["seqlens"][b])
        rows = []
        for slot in range(-(-n // page)):
            take = min(page, n - slot * page)
            if slot not in bad.get(b, ()):
                rows.append(kv[int(case["block_table"][b, slot])][:take])
        rows = np.concatenate(rows) if rows else np.zeros((0, kv.shape[-1]), np.float32)
        o, l = orc.mla_decode_ref(q[b:b + 1], rows[None], np.array([rows.shape[0]]), None,
                                  softmax_scale=case["scale"])
        outs.append(o)
        lses.append(l)
        lens.append(rows.shape[0])
    return np.concatenate(outs), np.concatenate(lses), lens


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("page_size", [16, 64])
@pytest.mark.parametrize("num_splits", [1, 2])
def test_bad_page_ids_are_masked_on_both_kernels(device, monkeypatch, kernel, page_size, num_splits):
    """A block-table entry outside the pool (too large or negative) masks its page's tokens
    and sets the status bit, on the tcgen05 kernel as on the CUDA-core kernel; with 16-token
    pages a bad page masks part of a 64-token tile, and a whole tile of bad pages leaves the
    request with fewer tokens (or none)."""
    import triton_mla.kernel as tk
    monkeypatch.setattr(tk, "_CHECK", False)
    case = recipes.paged_case([300, 130, 200, 64], 128, page_size, seed=43)
    per_tile = 64 // page_size
    bad = {0: {1, 3}, 1: {0}, 3: set(range(per_tile))}  # request 3: its only tile is all bad
    bt = case["block_table"].clone()
    for b, slots in bad.items():
        for k, slot in enumerate(sorted(slots)):
            bt[b, slot] = 10_000_000 if k % 2 == 0 else -5
    case = dict(case, block_table=bt)
    c = to_dev(case, device)
    read_status(device)
    out, lse = mla_decode(c["q"], c["kv"], c["seqlens"], c["block_table"], softmax_scale=c["scale"],
                          num_splits=num_splits, return_lse=True, kernel=kernel)
    torch.cuda.synchronize()
    if kernel == "auto":
        assert selected_kernel(c["q"], c["kv"], c["block_table"], num_splits=num_splits) == "sm100"
    assert read_status(device) & _lib.STATUS_BAD_PAGE
    ref_out, ref_lse, lens = _oracle_without_pages(case, bad)
    check(out, lse, ref_out, ref_lse, lens)


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("scale", [-0.1, 0.0, -(192 ** -0.5), 0.5])
@pytest.mark.parametrize("num_splits", [1, 3])
def test_softmax_scale_of_any_sign(device, kernel, scale, num_splits):
    """The reference takes any softmax_scale (kernel.py:247-248): zero gives the mean of the
    rows, a negative scale weights the smallest scores most."""
    case = dict(recipes.paged_case([0, 1, 513, 1000], 128, 64, seed=44), scale=scale)
    out, lse = run(case, device, num_splits=num_splits, kernel=kernel)
    ref_out, ref_lse = oracle_of(case)
    check(out, lse, ref_out, ref_lse, case["seqlens"])


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("num_splits", [1, 3])
def test_nan_softmax_scale_gives_nan(device, kernel, num_splits):
    """A NaN scale makes every score NaN: the reference returns NaN rows (and NaN LSE) for
    requests with tokens, and 0 / -inf for empty ones."""
    case = dict(recipes.paged_case([0, 1, 513, 1000], 128, 64, seed=45), scale=float("nan"))
    out, lse = run(case, device, num_splits=num_splits, kernel=kernel)
    ref_out, ref_lse = oracle_of(case)
    out, lse = out.float().cpu().numpy(), lse.cpu().numpy()
    assert np.isnan(ref_out[1:]).all() and np.isnan(ref_lse[1:]).all()
    assert np.isnan(out[1:]).all() and np.isnan(lse[1:]).all()
    assert np.all(out[0] == 0) and np.all(np.isneginf(lse[0]))


# ----------------------------------------------------------------------------- properties at full size
def _baseline_case(cfg, device, seed=0):
    """BASELINE configs 2-4 drawn directly on the device (values N(0,1), shuffled pages)."""
    g = torch.Generator(device=device).manual_seed(seed)
    if cfg == "cfg2":
        lens = torch.full((32,), 4096, dtype=torch.int32)
    elif cfg == "cfg3":
        lens = torch.full((4,), 65536, dtype=torch.int32)
    else:
        lens = torch.randint(1, 16385, (256,), generator=torch.Generator().manual_seed(seed), dtype=torch.int32)
    need = (lens + 63) // 64
    num_pages = int(need.sum())
    kv = torch.randn(num_pages, 64, 576, generator=g, device=device, dtype=torch.bfloat16)
    q = torch.randn(len(lens), 128, 576, generator=g, device=device, dtype=torch.bfloat16)
    perm = torch.randperm(num_pages, generator=torch.Generator().manual_seed(seed + 1))
    bt = torch.zeros(len(lens), int(need.max()), dtype=torch.int32)
    at = 0
    for b, k in enumerate(need.tolist()):
        bt[b, :k] = perm[at:at + k].int()
        at += k
    return q, kv, lens.to(device), bt.to(device)


@pytest.mark.parametrize("cfg", ["cfg2", "cfg3", "cfg4"])
def test_baseline_configs_against_oracle(device, cfg):
    """Full-size BASELINE configs against the oracle: every request of configs 2 and 3 (all
    heads), and 32 requests of config 4 (the longest, the shortest and a seeded sample)."""
    q, kv, lens, bt = _baseline_case(cfg, device)
    scale = 192 ** -0.5
    out, lse = mla_decode(q, kv, lens, bt, softmax_scale=scale, return_lse=True)
    if cfg == "cfg4":
        order = torch.argsort(lens.cpu(), descending=True).tolist()
        rng = np.random.default_rng(4)
        sample = sorted(set(order[:8] + order[-8:] + rng.choice(len(order), 16, replace=False).tolist()))
    else:
        sample = range(len(lens))
    for b in sample:
        n = int(lens[b])
        pages = bt[b, : (n + 63) // 64].long()
        rows = kv[pages].reshape(-1, 576)[:n].float().cpu().numpy()
        ref_out, ref_lse = orc.mla_decode_ref(q[b:b + 1].float().cpu().numpy(), rows[None], np.array([n]), None,
                                              softmax_scale=scale, dtype=np.float32)
        check(out[b:b + 1], lse[b:b + 1], ref_out, ref_lse, [n])


def test_split_invariance_and_determinism(device):
    q, kv, lens, bt = _baseline_case("cfg3", device, seed=3)
    scale = 192 ** -0.5
    o1, l1 = mla_decode(q, kv, lens, bt, softmax_scale=scale, num_splits=1, return_lse=True)
    for s in (2, 7, 18, 64):
        o, l = mla_decode(q, kv, lens, bt, softmax_scale=scale, num_splits=s, return_lse=True)
        assert (o.float() - o1.float()).abs().max().item() <= OUT_TOL
        assert (l - l1).abs().max().item() <= LSE_TOL
    o2, l2 = mla_decode(q, kv, lens, bt, softmax_scale=scale, num_splits=18, return_lse=True)
    o3, l3 = mla_decode(q, kv, lens, bt, softmax_scale=scale, num_splits=18, return_lse=True)
    assert torch.equal(o2, o3) and torch.equal(l2, l3), "decode must be deterministic"


def test_page_permutation_invariance(device):
    """Moving pages around the pool (and the block table with them) changes nothing, bit for bit."""
    q, kv, lens, bt = _baseline_case("cfg2", device, seed=5)
    o1, l1 = mla_decode(q, kv, lens, bt, num_splits=2, return_lse=True)
    perm = torch.randperm(kv.shape[0], device=device)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(kv.shape[0], device=device)
    o2, l2 = mla_decode(q, kv[perm], lens, inv[bt.long()].int(), num_splits=2, return_lse=True)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_batch_independence(device):
    """A request's result does not depend on the other requests in the batch."""
    q, kv, lens, bt = _baseline_case("cfg4", device, seed=9)
    o_all, l_all = mla_decode(q, kv, lens, bt, num_splits=3, return_lse=True)
    for b in (0, 17, 200):
        o_b, l_b = mla_decode(q[b:b + 1], kv, lens[b:b + 1], bt[b:b + 1], num_splits=3, return_lse=True)
        assert torch.equal(o_b[0], o_all[b]) and torch.equal(l_b[0], l_all[b])


def test_constant_cache_returns_the_row(device):
    """Every cached row equal => softmax-weighted average equals that row for any query."""
    g = torch.Generator().manual_seed(8)
    row = torch.randn(576, generator=g).bfloat16()
    kv = row.expand(30, 64, 576).contiguous()
    lens = torch.tensor([1, 64, 1000, 1920], dtype=torch.int32)
    bt = torch.arange(30, dtype=torch.int32).repeat(4, 1)
    q = torch.randn(4, 128, 576, generator=g).bfloat16()
    for kernel in KERNELS:
        out, lse = mla_decode(q.to(device), kv.to(device), lens.to(device), bt.to(device), num_splits=4,
                              return_lse=True, kernel=kernel)
        want = row[:512].float().expand(4, 128, 512)
        assert (out.float().cpu() - want).abs().max().item() <= 1e-2
        s = (q.float() @ row.float()) * 576 ** -0.5
        want_lse = s + torch.log(lens.float())[:, None]
        assert (lse.cpu() - want_lse).abs().max().item() <= LSE_TOL


def test_kernel_selection_for_deepseek_shape(device):
    q, kv, lens, bt = _baseline_case("cfg2", device)
    assert selected_kernel(q, kv, bt) == "sm100"
    assert selected_kernel(q, kv, bt, kernel="generic") == "generic"
    # Page sizes whose largest power-of-two factor is below 8 go to the generic kernel.
    kv3 = torch.zeros(10, 3, 576, dtype=torch.bfloat16, device=device)
    bt3 = torch.zeros(2, 4, dtype=torch.int32, device=device)
    assert selected_kernel(q[:2], kv3, bt3) == "generic"
    assert selected_kernel(q[:2].float(), kv3.float(), bt3) == "generic"


# ----------------------------------------------------------------------------- per-request split plans
# num_splits=None on a ragged batch runs the planner's per-request split counts, units
# longest first (tmla_decode_units), with the merge over per-request slot ranges.
@pytest.mark.parametrize("lens,num_heads,page_size,dtype", [
    ([4096, 1000, 0, 65, 3000, 64, 1, 7777], 128, 64, torch.bfloat16),
    ([300, 0, 0, 12000, 5], 20, 16, torch.bfloat16),
    ([2048, 100, 5000, 1, 64, 9000], 129, 64, torch.float16),
    ([65536, 100, 200, 0, 37], 128, 64, torch.bfloat16),
])
def test_ragged_split_plan_matches_reference(device, lens, num_heads, page_size, dtype):
    from triton_mla.kernel import plan_units
    units, _ = plan_units(lens, num_heads)
    case = recipes.paged_case(lens, num_heads, page_size, seed=21, dtype=dtype)
    out, lse = run(case, device)
    ref_out, ref_lse = oracle_of(case)
    check(out, lse, ref_out, ref_lse, lens)
    assert read_status(device) == 0
    if lens[0] == 65536:
        assert units[units[:, 0] == 0][0, 2] > 1, "the long request is split"


def test_ragged_split_plan_dense_cache_and_agreement(device):
    g = torch.Generator().manual_seed(5)
    B, S = 5, 3000
    q = torch.randn(B, 128, 576, generator=g).to(torch.bfloat16)
    kv = torch.randn(B, S, 576, generator=g).to(torch.bfloat16)
    lens = torch.tensor([3000, 17, 0, 2048, 999], dtype=torch.int32)
    case = dict(q=q, kv=kv, seqlens=lens, block_table=None, scale=recipes.SCALE_192)
    c = to_dev(case, device)
    out_p, lse_p = mla_decode(c["q"], c["kv"], c["seqlens"], None, softmax_scale=c["scale"], return_lse=True)
    out_u, lse_u = mla_decode(c["q"], c["kv"], c["seqlens"], None, softmax_scale=c["scale"], return_lse=True,
                              num_splits=3)
    ref_out, ref_lse = oracle_of(case)
    check(out_p, lse_p, ref_out, ref_lse, lens.tolist())
    assert (out_p.float() - out_u.float()).abs().max().item() <= OUT_TOL


def test_ragged_split_plan_many_short_requests(device):
    """A long request among many empty and one-tile ones."""
    lens = [60000] + [0] * 400 + [37] * 1200
    case = recipes.paged_case(lens, 128, 64, seed=8)
    out, lse = run(case, device)
    sel = [0, 1, 400, 401, 1000, 1600]
    sub = dict(q=case["q"][sel], kv=case["kv"], seqlens=case["seqlens"][sel], block_table=case["block_table"][sel],
               scale=case["scale"])
    ref_out, ref_lse = oracle_of(sub)
    check(out[sel], lse[sel], ref_out, ref_lse, [lens[i] for i in sel])
    assert read_status(device) == 0


def test_split_plan_reused_across_lengths_and_in_a_graph(device):
    """A SplitPlan says how many splits each request gets, not where they start, so it stays
    valid when the lengths change, eagerly and inside a captured CUDA graph."""
    from triton_mla import make_split_plan
    lens0 = [4096, 100, 0, 7000, 33]
    case = recipes.paged_case(lens0, 128, 64, seed=3)
    c = to_dev(case, device)
    plan = make_split_plan(c["seqlens"], 128)
    assert plan.num_slots > 0, "the long requests are split"
    lens = c["seqlens"].clone()
    q = c["q"].clone()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        mla_decode(q, c["kv"], lens, c["block_table"], softmax_scale=c["scale"], return_lse=True, plan=plan)
    torch.cuda.current_stream(device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        g_out, g_lse = mla_decode(q, c["kv"], lens, c["block_table"], softmax_scale=c["scale"], return_lse=True,
                                  plan=plan)
    for new in (lens0, [10, 4000, 300, 1, 7040], [7040, 0, 7040, 64, 65]):
        lens.copy_(torch.tensor(new, dtype=torch.int32, device=device))
        e_out, e_lse = mla_decode(q, c["kv"], lens, c["block_table"], softmax_scale=c["scale"], return_lse=True,
                                  plan=plan)
        graph.replay()
        torch.cuda.synchronize(device)
        sub = dict(case, seqlens=torch.tensor(new, dtype=torch.int32))
        ref_out, ref_lse = oracle_of(sub)
        check(e_out, e_lse, ref_out, ref_lse, new)
        check(g_out, g_lse, ref_out, ref_lse, new)
    del graph


# ----------------------------------------------------------------------------- device-side split plans
# tmla_plan_units_device plans on the GPU from the lengths in device memory: a table of fixed
# capacity (padding entries {-1, 0, 0, -1}), so planning and decode can be captured together.
def _device_plan_host_view(plan):
    units = plan.units.cpu().numpy()
    first = plan.req_first.cpu().numpy()
    real = units[units[:, 0] >= 0]
    pad = units[units[:, 0] < 0]
    return units, real, pad, first


def _check_device_plan(lens, plan):
    units, real, pad, first = _device_plan_host_view(plan)
    lens = np.asarray(lens)
    tiles = (np.maximum(lens, 0) + 63) // 64
    assert len(real) + len(pad) == plan.num_units and len(real) >= len(lens)
    assert np.all(units[len(real):, 0] < 0), "padding entries come after the plan's units"
    assert np.all(pad == np.array([-1, 0, 0, -1]))
    seen = {}
    for b, s, ns, slot in real.tolist():
        assert 0 <= b < len(lens) and 1 <= ns <= 64 and 0 <= s < ns and (b, s) not in seen
        seen[(b, s)] = ns
        assert slot == (-1 if ns == 1 else first[b] + s)
    for b in range(len(lens)):
        ns = seen[(b, 0)]
        assert all(seen.get((b, s)) == ns for s in range(ns)), f"request {b} misses a split"
        assert first[b + 1] - first[b] == (ns if ns > 1 else 0)
    assert first[0] == 0 and first[-1] <= plan.num_slots
    # longest first, up to the planner's bucket width (1/127 of the longest unit)
    sizes = []
    for b, s, ns, _ in real.tolist():
        per = -(-int(tiles[b]) // ns)
        sizes.append(max(0, min(int(tiles[b]), (s + 1) * per) - min(int(tiles[b]), s * per)))
    slack = max(sizes) // 127 + 1 if sizes else 0
    assert all(sizes[i] + slack >= sizes[i + 1] for i in range(len(sizes) - 1))
    return real


@pytest.mark.parametrize("lens", [
    [4096] * 32,
    [65536] * 4,
    [60000] + [0] * 300 + [37] * 700,
    [0, 0, 0],
    [1],
])
def test_device_plan_is_a_valid_plan(device, lens):
    from triton_mla import make_device_split_plan
    from triton_mla.kernel import plan_units
    plan = make_device_split_plan(torch.tensor(lens, dtype=torch.int32, device=device), 128)
    real = _check_device_plan(lens, plan)
    if len(set(lens)) == 1 and lens[0] >= 4096:
        host, _ = plan_units(lens, 128)
        assert set(real[:, 2].tolist()) == set(host[:, 2].tolist()), "uniform batches: the host planner's split"
    if lens[0] == 60000:
        assert real[real[:, 0] == 0][0, 2] > 1, "the long request is split"


def test_device_plan_on_ragged_batches(device):
    from triton_mla import make_device_split_plan
    rng = np.random.default_rng(1)
    g = torch.Generator().manual_seed(0)
    batches = [torch.randint(1, 16385, (256,), generator=g).tolist()]
    batches += [rng.integers(0, 20000, size=int(rng.integers(1, 400))).tolist() for _ in range(8)]
    for lens in batches:
        plan = make_device_split_plan(torch.tensor(lens, dtype=torch.int32, device=device), 128)
        _check_device_plan(lens, plan)
        small = make_device_split_plan(torch.tensor(lens, dtype=torch.int32, device=device), 128,
                                       capacity=len(lens), slot_capacity=0)
        real = _check_device_plan(lens, small)
        assert set(real[:, 2].tolist()) == {1}, "no room for splits: one unit per request"


@pytest.mark.parametrize("lens,num_heads", [
    ([4096, 1000, 0, 65, 3000, 64, 1, 7777], 128),
    ([65536, 100, 200, 0, 37], 128),
    ([2048, 100, 5000, 1, 64, 9000], 200),
])
def test_device_plan_decode_matches_reference(device, lens, num_heads):
    from triton_mla import make_device_split_plan
    case = recipes.paged_case(lens, num_heads, 64, seed=23)
    c = to_dev(case, device)
    plan = make_device_split_plan(c["seqlens"], num_heads)
    out, lse = mla_decode(c["q"], c["kv"], c["seqlens"], c["block_table"], softmax_scale=c["scale"],
                          return_lse=True, plan=plan)
    ref_out, ref_lse = oracle_of(case)
    check(out, lse, ref_out, ref_lse, lens)
    assert read_status(device) == 0


def test_device_plan_and_decode_in_one_graph(device):
    """The plan kernel, the split kernel and the merge captured together, replayed while the
    lengths change (each replay re-plans from the lengths then in memory)."""
    from triton_mla import make_device_split_plan
    lens0 = [4096, 100, 0, 7000, 33, 20000]
    case = recipes.paged_case(lens0, 128, 64, seed=31)
    c = to_dev(case, device)
    lens = c["seqlens"].clone()
    plan = make_device_split_plan(lens, 128)
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        plan.refresh(lens)
        mla_decode(c["q"], c["kv"], lens, c["block_table"], softmax_scale=c["scale"], return_lse=True, plan=plan)
    torch.cuda.current_stream(device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        plan.refresh(lens)
        g_out, g_lse = mla_decode(c["q"], c["kv"], lens, c["block_table"], softmax_scale=c["scale"],
                                  return_lse=True, plan=plan)
    for new in (lens0, [20000, 1, 1, 1, 1, 1], [0, 0, 0, 0, 0, 64], [5000, 5000, 5000, 5000, 5000, 5000]):
        lens.copy_(torch.tensor(new, dtype=torch.int32, device=device))
        graph.replay()
        torch.cuda.synchronize(device)
        sub = dict(case, seqlens=torch.tensor(new, dtype=torch.int32))
        ref_out, ref_lse = oracle_of(sub)
        check(g_out, g_lse, ref_out, ref_lse, new)
        _check_device_plan(new, plan)
        assert read_status(device) == 0
    del graph


# ----------------------------------------------------------------------------- several query tokens
# q [batch, q_len, heads, d] (an extension: the reference decodes one token per request).  Token i
# of a request is its (len - q_len + i)-th row, so it attends to the first len - (q_len - 1 - i)
# cache rows; the oracle runs each token as a one-token decode over that many rows.
def _multi_token_ref(case, q4, seqlens):
    q_len = q4.shape[1]
    ref_out, ref_lse, per_token_lens = [], [], []
    for i in range(q_len):
        li = torch.clamp(seqlens - (q_len - 1 - i), min=0).to(torch.int32)
        o, l = oracle_of(dict(case, q=q4[:, i].contiguous(), seqlens=li))
        ref_out.append(o)
        ref_lse.append(l)
        per_token_lens.append(li.numpy())
    return np.stack(ref_out, 1), np.stack(ref_lse, 1), np.stack(per_token_lens, 1)


def _multi_token_case(lens, q_len, heads, seed):
    case = recipes.paged_case(lens, q_len * heads, 64, seed=seed)
    q4 = case["q"].view(len(lens), q_len, heads, case["q"].shape[-1])
    return (case, q4) + _multi_token_ref(case, q4, case["seqlens"])


@pytest.mark.parametrize("q_len,heads,kernel", [
    (2, 128, "auto"), (3, 128, "auto"), (4, 128, "auto"), (2, 128, "generic"), (2, 16, "auto"), (3, 20, "auto"),
])
@pytest.mark.parametrize("num_splits", [None, 1, 3])
def test_multi_token_decode_matches_reference(device, q_len, heads, kernel, num_splits):
    lens = [4096, 1, 0, 700, 2, 65]
    case, q4, ref_out, ref_lse, tok_lens = _multi_token_case(lens, q_len, heads, seed=q_len * 10 + heads)
    c = to_dev(case, device)
    out, lse = mla_decode(q4.to(device), c["kv"], c["seqlens"], c["block_table"], softmax_scale=c["scale"],
                          num_splits=num_splits, return_lse=True, kernel=kernel)
    assert out.shape == (len(lens), q_len, heads, 512) and lse.shape == (len(lens), q_len, heads)
    expect = "sm100" if (heads % 128 == 0 and kernel == "auto") else "generic"
    assert selected_kernel(q4.to(device), c["kv"], c["block_table"], kernel=kernel) == expect
    for i in range(q_len):
        check(out[:, i], lse[:, i], ref_out[:, i], ref_lse[:, i], tok_lens[:, i])
    assert read_status(device) == 0


def test_multi_token_decode_in_a_graph(device):
    """Two query tokens per request, captured with num_splits=None (a device-made plan) and
    replayed with new lengths."""
    lens0 = [3000, 64, 1, 9000]
    case, q4, _, _, _ = _multi_token_case(lens0, 2, 128, seed=77)
    c = to_dev(case, device)
    q = q4.to(device)
    lens = c["seqlens"].clone()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        mla_decode(q, c["kv"], lens, c["block_table"], softmax_scale=c["scale"], return_lse=True, num_splits=2)
    torch.cuda.current_stream(device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        g_out, g_lse = mla_decode(q, c["kv"], lens, c["block_table"], softmax_scale=c["scale"], return_lse=True)
    for new in (lens0, [9000, 2, 0, 65]):
        lens.copy_(torch.tensor(new, dtype=torch.int32, device=device))
        graph.replay()
        torch.cuda.synchronize(device)
        ref_out, ref_lse, tok_lens = _multi_token_ref(case, q4, torch.tensor(new, dtype=torch.int32))
        for i in range(2):
            check(g_out[:, i], g_lse[:, i], ref_out[:, i], ref_lse[:, i], tok_lens[:, i])
    del graph


# ----------------------------------------------------------------------------- FP8 cache rows
# A uint8 cache of 656-byte rows (triton_mla.fp8_cache; an extension).  The oracle attends to
# the dequantised rows, so the comparison measures the kernel, not the quantisation.
# The tcgen05 kernel forms the latent products in fp16: each dequantised value (e4m3 x scale)
# is rounded to fp16 once (relative error <= 2^-12 for round-to-nearest) and so are the
# queries' latent halves.  A score then moves by up to about 1.2e-3 (numpy, 40 seeds of one
# N(0,1) token with 128 heads: median 9.0e-4, max 1.23e-3), which is the LSE error of a
# one-token request; the tcgen05 FP8 tolerance is therefore 2e-3 on the LSE (the output keeps
# 2e-2).  The CUDA-core kernel computes in fp32 and keeps 1e-3.
FP8_LSE_TOL = {"auto": 2e-3, "generic": LSE_TOL}


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("paged", [True, False])
@pytest.mark.parametrize("num_splits", [None, 1, 3])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fp8_cache_matches_reference(device, kernel, paged, num_splits, dtype):
    from triton_mla import fp8_cache
    lens = [1000, 0, 77, 2048, 1]
    if paged:
        case = recipes.paged_case(lens, 128, 64, seed=91, dtype=dtype)
    else:
        g = torch.Generator().manual_seed(91)
        case = dict(q=torch.randn(len(lens), 128, 576, generator=g).to(dtype),
                    kv=torch.randn(len(lens), 2048, 576, generator=g).to(dtype),
                    seqlens=torch.tensor(lens, dtype=torch.int32), block_table=None, scale=recipes.SCALE_192)
    rows = fp8_cache.quantize_kv(case["kv"])
    ref_case = dict(case, kv=fp8_cache.dequantize_kv(rows))
    ref_out, ref_lse = oracle_of(ref_case)
    c = to_dev(dict(case, kv=rows), device)
    want = "sm100" if kernel == "auto" else "generic"
    assert selected_kernel(c["q"], c["kv"], c["block_table"], kernel=kernel) == want
    out, lse = mla_decode(c["q"], c["kv"], c["seqlens"], c["block_table"], softmax_scale=c["scale"],
                          num_splits=num_splits, return_lse=True, kernel=kernel)
    check(out, lse, ref_out, ref_lse, lens, lse_tol=FP8_LSE_TOL[kernel])
    assert read_status(device) == 0


@pytest.mark.parametrize("kernel", KERNELS)
def test_fp8_cache_with_several_query_tokens(device, kernel):
    from triton_mla import fp8_cache
    lens = [700, 3, 1500]
    case, q4, _, _, _ = _multi_token_case(lens, 2, 128, seed=5)
    rows = fp8_cache.quantize_kv(case["kv"])
    ref_case = dict(case, kv=fp8_cache.dequantize_kv(rows))
    ref_out, ref_lse, tok_lens = _multi_token_ref(ref_case, q4, case["seqlens"])
    c = to_dev(dict(case, kv=rows), device)
    out, lse = mla_decode(q4.to(device), c["kv"], c["seqlens"], c["block_table"], softmax_scale=c["scale"],
                          return_lse=True, kernel=kernel)
    for i in range(2):
        check(out[:, i], lse[:, i], ref_out[:, i], ref_lse[:, i], tok_lens[:, i], lse_tol=FP8_LSE_TOL[kernel])


@pytest.mark.parametrize("page_size", [16, 64])
@pytest.mark.parametrize("num_splits", [1, 2])
def test_fp8_cache_bad_pages_are_masked(device, monkeypatch, page_size, num_splits):
    """FP8 rows on the tcgen05 kernel: a bad block-table entry masks its page's tokens (the
    dequantising warps write zeros for sub-boxes that were not loaded), as for 16-bit rows."""
    import triton_mla.kernel as tk
    from triton_mla import fp8_cache
    monkeypatch.setattr(tk, "_CHECK", False)
    case = recipes.paged_case([300, 130, 200, 64], 128, page_size, seed=45)
    per_tile = 64 // page_size
    bad = {0: {1, 3}, 1: {0}, 3: set(range(per_tile))}
    bt = case["block_table"].clone()
    for b, slots in bad.items():
        for k, slot in enumerate(sorted(slots)):
            bt[b, slot] = 10_000_000 if k % 2 == 0 else -5
    rows = fp8_cache.quantize_kv(case["kv"])
    ref_case = dict(case, kv=fp8_cache.dequantize_kv(rows), block_table=bt)
    c = to_dev(dict(case, kv=rows, block_table=bt), device)
    read_status(device)
    assert selected_kernel(c["q"], c["kv"], c["block_table"], num_splits=num_splits) == "sm100"
    out, lse = mla_decode(c["q"], c["kv"], c["seqlens"], c["block_table"], softmax_scale=c["scale"],
                          num_splits=num_splits, return_lse=True)
    torch.cuda.synchronize()
    assert read_status(device) & _lib.STATUS_BAD_PAGE
    ref_out, ref_lse, lens = _oracle_without_pages(ref_case, bad)
    check(out, lse, ref_out, ref_lse, lens, lse_tol=FP8_LSE_TOL["auto"])


def test_fp8_cache_beyond_fp16_range_is_flagged(device, monkeypatch):
    """A row scale that takes e4m3 values past the fp16 range sets STATUS_RANGE on the tcgen05
    kernel; the other requests stay exact, and the CUDA-core kernel (fp32) decodes that row."""
    import triton_mla.kernel as tk
    from triton_mla import fp8_cache
    monkeypatch.setattr(tk, "_CHECK", False)
    case = recipes.paged_case([200, 150], 128, 64, seed=46)
    kv = case["kv"].clone()
    big_page = int(case["block_table"][0, 1])
    kv[big_page, 3, :128] *= 1e6   # request 0, token 67: its first scale group reaches ~4e6
    rows = fp8_cache.quantize_kv(kv)
    ref_case = dict(case, kv=fp8_cache.dequantize_kv(rows))
    ref_out, ref_lse = oracle_of(ref_case)
    c = to_dev(dict(case, kv=rows), device)
    read_status(device)
    out, lse = mla_decode(c["q"], c["kv"], c["seqlens"], c["block_table"], softmax_scale=c["scale"],
                          num_splits=1, return_lse=True)
    torch.cuda.synchronize()
    assert read_status(device) & _lib.STATUS_RANGE
    check(out[1:], lse[1:], ref_out[1:], ref_lse[1:], case["seqlens"][1:], lse_tol=FP8_LSE_TOL["auto"])
    out_g, lse_g = mla_decode(c["q"], c["kv"], c["seqlens"], c["block_table"], softmax_scale=c["scale"],
                              num_splits=1, return_lse=True, kernel="generic")
    torch.cuda.synchronize()
    assert read_status(device) == 0
    rel = np.abs(out_g[0].float().cpu().numpy() - ref_out[0]).max() / np.abs(ref_out[0]).max()
    assert rel <= 1e-2


def test_fp8_cache_ragged_batch_with_a_split_plan(device):
    """FP8 rows through the per-request split plan (num_splits=None in eager mode), with a long
    request cut into several splits merged from partial slots."""
    from triton_mla import fp8_cache
    from triton_mla.kernel import plan_units
    lens = [65536, 1, 300, 0, 4097, 64, 12000]
    units, _ = plan_units(lens, 128)
    assert units[units[:, 0] == 0][0, 2] > 1, "the long request is split"
    case = recipes.paged_case(lens, 128, 64, seed=93)
    rows = fp8_cache.quantize_kv(case["kv"])
    ref_out, ref_lse = oracle_of(dict(case, kv=fp8_cache.dequantize_kv(rows)))
    c = to_dev(dict(case, kv=rows), device)
    out, lse = mla_decode(c["q"], c["kv"], c["seqlens"], c["block_table"], softmax_scale=c["scale"],
                          return_lse=True)
    check(out, lse, ref_out, ref_lse, lens, lse_tol=FP8_LSE_TOL["auto"])
    assert read_status(device) == 0


def test_fp8_cache_device_plan_in_a_graph(device):
    """FP8 rows with the device planner, the split kernel and the merge captured in one CUDA
    graph and replayed as the lengths change."""
    from triton_mla import fp8_cache, make_device_split_plan
    lens0 = [4096, 100, 0, 7000, 33, 20000]
    case = recipes.paged_case(lens0, 128, 64, seed=94)
    rows = fp8_cache.quantize_kv(case["kv"])
    deq = fp8_cache.dequantize_kv(rows)
    c = to_dev(dict(case, kv=rows), device)
    lens = c["seqlens"].clone()
    plan = make_device_split_plan(lens, 128)
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        plan.refresh(lens)
        mla_decode(c["q"], c["kv"], lens, c["block_table"], softmax_scale=c["scale"], return_lse=True, plan=plan)
    torch.cuda.current_stream(device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        plan.refresh(lens)
        g_out, g_lse = mla_decode(c["q"], c["kv"], lens, c["block_table"], softmax_scale=c["scale"],
                                  return_lse=True, plan=plan)
    for new in (lens0, [20000, 1, 1, 1, 1, 1], [5000, 5000, 5000, 5000, 5000, 5000]):
        lens.copy_(torch.tensor(new, dtype=torch.int32, device=device))
        graph.replay()
        torch.cuda.synchronize(device)
        ref_out, ref_lse = oracle_of(dict(case, kv=deq, seqlens=torch.tensor(new, dtype=torch.int32)))
        check(g_out, g_lse, ref_out, ref_lse, new, lse_tol=FP8_LSE_TOL["auto"])
        assert read_status(device) == 0
    del graph


def test_fp8_cache_full_config_against_oracle(device):
    """BASELINE config 2 with FP8 rows (B=32, S=4096, page 64) on the tcgen05 kernel: every
    request against the oracle over its dequantised rows."""
    from triton_mla import fp8_cache
    q, kv, lens, bt = _baseline_case("cfg2", device)
    rows = fp8_cache.quantize_kv(kv)
    del kv
    scale = 192 ** -0.5
    assert selected_kernel(q, rows, bt) == "sm100"
    out, lse = mla_decode(q, rows, lens, bt, softmax_scale=scale, return_lse=True)
    for b in range(len(lens)):
        n = int(lens[b])
        pages = bt[b, : (n + 63) // 64].long()
        kvb = fp8_cache.dequantize_kv(rows[pages]).reshape(-1, 576)[:n].cpu().numpy()
        ref_out, ref_lse = orc.mla_decode_ref(q[b:b + 1].float().cpu().numpy(), kvb[None], np.array([n]), None,
                                              softmax_scale=scale, dtype=np.float32)
        check(out[b:b + 1], lse[b:b + 1], ref_out, ref_lse, [n], lse_tol=FP8_LSE_TOL["auto"])
    assert read_status(device) == 0


def test_torch_compile_fullgraph_through_the_operator(device):
    """mla_decode is one operator (torch.ops.triton_mla.decode), so torch.compile traces a
    function that calls it, with an explicit split count, into one graph without a break;
    the compiled function matches the oracle."""
    import torch._dynamo

    case = recipes.paged_case([0, 1, 513, 1000], 128, 64, seed=46)
    c = to_dev(case, device)
    scale = c["scale"]

    def f(q, kv, lens, bt):
        out, lse = mla_decode(q, kv, lens, bt, softmax_scale=scale, num_splits=3, return_lse=True)
        return out.float() * 2.0, lse

    torch._dynamo.reset()
    explain = torch._dynamo.explain(f)(c["q"], c["kv"], c["seqlens"], c["block_table"])
    assert explain.graph_break_count == 0 and explain.graph_count == 1, explain.break_reasons
    compiled = torch.compile(f, fullgraph=True, backend="aot_eager")
    out2, lse = compiled(c["q"], c["kv"], c["seqlens"], c["block_table"])
    ref_out, ref_lse = oracle_of(case)
    check(out2 / 2.0, lse, ref_out, ref_lse, case["seqlens"])
    torch._dynamo.reset()


@pytest.mark.parametrize("rows", ["bf16", "fp8"])
def test_decode_timed_out_wait_returns_cleanly(device, rows):
    """A bounded wait of the tcgen05 kernel that runs out (TMLA_FLAG_TEST_STALL: the first CTA
    never loads its first tile, a barrier that nothing completes) sets TMLA_STATUS_TIMEOUT, and
    the pair of CTAs stops, lets what it has in flight land and returns: the call succeeds, the
    requests of the other clusters are right, and the next call on the same device is exact.
    With FP8 rows the wait that runs out is the dequantising warps' wait for the first landing
    slot."""
    import ctypes

    from triton_mla import fp8_cache
    from triton_mla.kernel import _status_word

    case = recipes.paged_case([1024, 777, 300, 65], 128, 64, seed=47)
    lse_tol, kv_format = LSE_TOL, _lib.KV_SAME
    if rows == "fp8":
        fp8_rows = fp8_cache.quantize_kv(case["kv"])
        case = dict(case, kv=fp8_rows)
        lse_tol, kv_format = FP8_LSE_TOL["auto"], _lib.KV_FP8_E4M3
    c = to_dev(case, device)
    B, splits = 4, 2
    lib = _lib.load()
    out = torch.empty(B, 128, 512, dtype=torch.bfloat16, device=device)
    lse = torch.empty(B, 128, dtype=torch.float32, device=device)
    ws = torch.empty(lib.tmla_workspace_bytes(B, 128, splits, 512), dtype=torch.uint8, device=device)
    o_bytes = (B * 128 * splits * 512 * 4 + 255) & ~255
    status = _status_word(device)
    read_status(device)
    bt = c["block_table"]
    p = _lib.TmlaDecodeParams(
        c["q"].data_ptr(), c["q"].stride(0), c["q"].stride(1), c["kv"].data_ptr(), c["kv"].stride(0),
        c["kv"].stride(1), c["kv"].shape[0], 64, c["seqlens"].data_ptr(), bt.data_ptr(), bt.stride(0), bt.shape[1],
        out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(), lse.stride(0), ws.data_ptr(),
        ws.data_ptr() + o_bytes, status.data_ptr(), B, 128, 576, 512, splits, _lib.DTYPE_BF16, _lib.KERNEL_SM100,
        _lib.FLAG_TEST_STALL, case["scale"], 1, kv_format, 20_000_000)
    stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    assert lib.tmla_decode(ctypes.byref(p), stream) == 0
    torch.cuda.synchronize()
    assert read_status(device) & _lib.STATUS_TIMEOUT
    ref_out, ref_lse = oracle_of(dict(case, kv=fp8_cache.dequantize_kv(case["kv"])) if rows == "fp8" else case)
    # request 0 held the stalled cluster
    check(out[1:], lse[1:], ref_out[1:], ref_lse[1:], case["seqlens"][1:], lse_tol=lse_tol)
    p.flags, p.wait_ns = 0, 0
    assert lib.tmla_decode(ctypes.byref(p), stream) == 0
    torch.cuda.synchronize()
    assert read_status(device) == 0
    check(out, lse, ref_out, ref_lse, case["seqlens"], lse_tol=lse_tol)


def test_two_stage_c_abi_keeps_the_fp32_partial_layout(device):
    """tmla_decode_partial writes the documented fp32 split partials (ws_o [B, H, S, 512] of
    normalised rows, ws_lse [B, H, S] base-2) and tmla_combine merges them: the merge done here
    in torch from those buffers, tmla_combine's result, tmla_decode's (whose tcgen05 path keeps
    its partials in the q dtype) and the oracle all agree."""
    import ctypes

    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    lens, splits = [4096, 1000, 0, 65], 5
    case = recipes.paged_case(lens, 128, 64, seed=12)
    c = to_dev(case, device)
    B, H = 4, 128
    nbytes = lib.tmla_workspace_bytes(B, H, splits, 512)
    o_bytes = (B * H * splits * 512 * 4 + 255) & ~255
    results = {}
    for name in ("partial", "decode"):
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        out = torch.full((B, H, 512), float("nan"), dtype=torch.bfloat16, device=device)
        lse = torch.full((B, H), float("nan"), dtype=torch.float32, device=device)
        p = _lib.TmlaDecodeParams(
            c["q"].data_ptr(), c["q"].stride(0), c["q"].stride(1), c["kv"].data_ptr(), c["kv"].stride(0),
            c["kv"].stride(1), c["kv"].shape[0], 64, c["seqlens"].data_ptr(), c["block_table"].data_ptr(),
            c["block_table"].stride(0), c["block_table"].shape[1], out.data_ptr(), out.stride(0), out.stride(1),
            lse.data_ptr(), lse.stride(0), ws.data_ptr(), ws.data_ptr() + o_bytes, None, B, H, 576, 512, splits,
            _lib.DTYPE_BF16, _lib.KERNEL_AUTO, 0, case["scale"])
        if name == "partial":
            assert lib.tmla_decode_partial(ctypes.byref(p), stream) == 0
            torch.cuda.synchronize(device)
            ws_o = ws[: B * H * splits * 512 * 4].view(torch.float32).view(B, H, splits, 512).clone()
            ws_lse = ws[o_bytes: o_bytes + B * H * splits * 4].view(torch.float32).view(B, H, splits).clone()
            assert lib.tmla_combine(ctypes.c_void_p(p.ws_o), ctypes.c_void_p(p.ws_lse), ctypes.c_void_p(out.data_ptr()),
                                    out.stride(0), out.stride(1), ctypes.c_void_p(lse.data_ptr()), lse.stride(0),
                                    B, H, splits, 512, _lib.DTYPE_BF16, stream) == 0
            # The same merge in torch from the fp32 buffers.
            m = ws_lse.amax(-1, keepdim=True)
            m = torch.where(torch.isneginf(m), torch.zeros_like(m), m)
            w = torch.exp2(ws_lse - m)
            wsum = w.sum(-1)
            t_out = (w[..., None] * torch.nan_to_num(ws_o)).sum(-2) / wsum.clamp_min(1e-30)[..., None]
            t_lse = torch.where(wsum > 0, (m[..., 0] + torch.log2(wsum)) * math.log(2.0),
                                torch.full_like(wsum, float("-inf")))
            results["torch"] = (t_out, t_lse)
        else:
            assert lib.tmla_decode(ctypes.byref(p), stream) == 0
        torch.cuda.synchronize(device)
        results[name] = (out, lse)
    ref_out, ref_lse = oracle_of(case)
    for name, (o, l) in results.items():
        check(o, l, ref_out, ref_lse, lens)
    assert (results["torch"][0] - results["partial"][0].float()).abs().max().item() <= OUT_TOL
    valid = torch.tensor(lens, device=device) > 0
    assert (results["torch"][1][valid] - results["partial"][1][valid]).abs().max().item() <= 1e-4
