"""The fused MLA layer operations (``tmla_q_absorb_rope``, ``tmla_kv_norm_rope_append``,
``tmla_o_unabsorb``) against the PyTorch ops of the reference layer they replace
(src/triton_mla/model.py:74-94 and 111-123), and the fused layer step against the
PyTorch-op form of the same step."""

import pytest
import torch
import torch.nn.functional as F

import recipes
from triton_mla import MLA, MLAConfig, layer_ops, read_status
from triton_mla.model import apply_rope

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: 2e-2, torch.float16: 5e-3, torch.float32: 1e-5}


def _close(got, ref, dtype):
    scale = max(float(ref.abs().max()), 1.0)
    err = float((got.float() - ref.float()).abs().max())
    assert err <= TOL[dtype] * scale, f"max-abs error {err:.3e} (scale {scale:.2f})"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("batch,heads", [(1, 16), (16, 128), (37, 20), (80, 20)])
@pytest.mark.parametrize("overlap", [False, True])
def test_q_absorb_rope_matches_torch(device, dtype, batch, heads, overlap):
    g = torch.Generator(device=device).manual_seed(batch * 131 + heads)
    dn, dr, dv, r = 128, 64, 128, 512
    q = torch.randn(batch, heads, dn + dr, generator=g, device=device).to(dtype)
    w = (torch.randn(heads * (dn + dv), r, generator=g, device=device) * 0.05).to(dtype)
    pos = torch.randint(0, 20000, (batch,), generator=g, device=device, dtype=torch.int32)
    got = layer_ops.q_absorb_rope(q, w, pos, dn, dv, 10000.0, overlap=overlap)
    w_uk = w.view(heads, dn + dv, r)[:, :dn]
    ref_abs = torch.einsum("bhd,hdc->bhc", q[..., :dn].float(), w_uk.float())
    ref_pe = apply_rope(q[..., dn:].float(), pos[:, None], 10000.0)
    _close(got[..., :r], ref_abs, dtype)
    _close(got[..., r:], ref_pe, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("paged", [True, False])
@pytest.mark.parametrize("overlap", [False, True])
def test_kv_norm_rope_append_matches_torch(device, dtype, paged, overlap):
    g = torch.Generator(device=device).manual_seed(5)
    batch, r, dr, page = 9, 512, 64, 16
    kva = torch.randn(batch, r + dr, generator=g, device=device).to(dtype)
    wn = (1 + 0.1 * torch.randn(r, generator=g, device=device)).to(dtype)
    pos = torch.randint(0, 200, (batch,), generator=g, device=device, dtype=torch.int32)
    if paged:
        width = 16
        bt = torch.randperm(batch * width, device=device).view(batch, width).int()
        cache = torch.randn(batch * width, page, r + dr, generator=g, device=device).to(dtype)
    else:
        bt = None
        cache = torch.randn(batch, 256, r + dr, generator=g, device=device).to(dtype)
    before = cache.clone()
    seq = torch.empty_like(pos)
    layer_ops.kv_norm_rope_append(kva, wn, pos, cache, bt, 1e-6, 10000.0, seqlens_out=seq, overlap=overlap)
    torch.cuda.synchronize()
    assert torch.equal(seq, pos + 1)
    rows = torch.arange(batch, device=device)
    if paged:
        idx = (bt[rows, (pos // page).long()].long(), (pos % page).long())
    else:
        idx = (rows, pos.long())
    ref_c = F.rms_norm(kva[:, :r].float(), (r,), wn.float(), 1e-6)
    ref_pe = apply_rope(kva[:, r:].float(), pos, 10000.0)
    _close(cache[idx][:, :r], ref_c, dtype)
    _close(cache[idx][:, r:], ref_pe, dtype)
    mask = torch.ones(cache.shape[:2], dtype=torch.bool, device=device)
    mask[idx] = False
    assert torch.equal(cache[mask], before[mask]), "only the new rows are written"


def test_kv_append_past_the_cache_is_flagged_and_dropped(device):
    cache = torch.zeros(4, 16, 576, dtype=torch.bfloat16, device=device)
    bt = torch.tensor([[0, 1], [2, 9]], dtype=torch.int32, device=device)  # page 9 is outside the pool
    kva = torch.ones(2, 576, dtype=torch.bfloat16, device=device)
    wn = torch.ones(512, dtype=torch.bfloat16, device=device)
    read_status(device, reset=True)
    pos = torch.tensor([40, 20], dtype=torch.int32, device=device)  # 40 >= 2 pages x 16 tokens
    layer_ops.kv_norm_rope_append(kva, wn, pos, cache, bt, 1e-6, 10000.0)
    torch.cuda.synchronize()
    assert read_status(device, reset=True) != 0
    assert not cache.any(), "nothing may be written for either request"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("batch", [1, 16, 33])
@pytest.mark.parametrize("overlap", [False, True])
def test_o_unabsorb_matches_torch(device, dtype, batch, overlap):
    g = torch.Generator(device=device).manual_seed(batch)
    heads, dn, dv, r = 128, 128, 128, 512
    o = torch.randn(batch, heads, r, generator=g, device=device).to(dtype)
    w = (torch.randn(heads * (dn + dv), r, generator=g, device=device) * 0.05).to(dtype)
    got = layer_ops.o_unabsorb(o, w, dn, dv, overlap=overlap)
    w_uv = w.view(heads, dn + dv, r)[:, dn:]
    ref = torch.einsum("bhc,hdc->bhd", o.float(), w_uv.float()).reshape(batch, heads * dv)
    _close(got, ref, dtype)


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 3e-2), (torch.float32, 1e-4)])
def test_fused_layer_step_equals_the_op_form(device, dtype, tol):
    cfg = recipes.LAYER_CFG
    model = MLA(MLAConfig(**cfg)).to(device, dtype)
    with torch.no_grad():
        for name, t in recipes.layer_weights(cfg).items():
            getattr(model, name).weight.copy_(t)
    inp = recipes.layer_inputs(True, seed=9)
    bt, lens = inp["block_table"].to(device), inp["seqlens"].to(device)
    x = inp["x"].to(device, dtype)
    kv_a = inp["kv"].to(device, dtype)
    kv_b = kv_a.clone()
    with torch.no_grad():
        out_f, seq_f = model._forward_fused(x, kv_a, lens, bt, None)
        out_o, seq_o = model._forward_ops(x, kv_b, lens, bt, None)
    assert torch.equal(seq_f, seq_o)
    torch.testing.assert_close(out_f.float(), out_o.float(), atol=tol, rtol=tol)
    torch.testing.assert_close(kv_a.float(), kv_b.float(), atol=tol, rtol=tol)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_kv_append_with_q_norm_matches_torch(device, dtype):
    """The cache append and the query path's q_norm in one launch, from the two halves of one
    GEMM output (strided rows)."""
    g = torch.Generator(device=device).manual_seed(12)
    batch, r, dr, qr, page = 7, 512, 64, 1536, 16
    both = torch.randn(batch, qr + r + dr, generator=g, device=device).to(dtype)
    qa, kva = both.split([qr, r + dr], dim=-1)
    wn = (1 + 0.1 * torch.randn(r, generator=g, device=device)).to(dtype)
    wq = (1 + 0.1 * torch.randn(qr, generator=g, device=device)).to(dtype)
    pos = torch.randint(0, 100, (batch,), generator=g, device=device, dtype=torch.int32)
    bt = torch.randperm(batch * 8, device=device).view(batch, 8).int()
    cache = torch.zeros(batch * 8, page, r + dr, device=device, dtype=dtype)
    qn = layer_ops.kv_norm_rope_append(kva, wn, pos, cache, bt, 1e-6, 10000.0, overlap=True, q_in=qa,
                                       q_norm_weight=wq, q_eps=1e-6)
    torch.cuda.synchronize()
    _close(qn, F.rms_norm(qa.float(), (qr,), wq.float(), 1e-6), dtype)
    rows = torch.arange(batch, device=device)
    idx = (bt[rows, (pos // page).long()].long(), (pos % page).long())
    _close(cache[idx][:, :r], F.rms_norm(kva[:, :r].float(), (r,), wn.float(), 1e-6), dtype)
