"""The MLA layer's absorbed decode step (which runs ``mla_decode``) against the
reference layer's output (tests/test_model.py:8-35 of the reference): same
weights, inputs and cache, golden vectors from the reference's fp32 layer."""

import numpy as np
import pytest
import torch

import recipes
from conftest import load_golden
from oracle import mla_oracle as orc
from triton_mla import MLA, MLAConfig, MLADecodeGraph

pytestmark = pytest.mark.gpu


def _model(device, dtype):
    cfg = recipes.LAYER_CFG
    model = MLA(MLAConfig(**cfg)).to(device, dtype)
    with torch.no_grad():
        for name, t in recipes.layer_weights(cfg).items():
            getattr(model, name).weight.copy_(t)
    return model


@pytest.mark.parametrize("paged", [False, True])
@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 3e-2), (torch.float32, 1e-4)])
def test_absorbed_decode_matches_reference_layer(device, paged, dtype, tol):
    gold = load_golden(f"layer_{'paged' if paged else 'dense'}")
    inp = recipes.layer_inputs(paged)
    model = _model(device, dtype)
    kv = inp["kv"].to(device, dtype)
    bt = None if inp["block_table"] is None else inp["block_table"].to(device)
    lens = inp["seqlens"].to(device)
    with torch.no_grad():
        out, new_lens = model(inp["x"].to(device, dtype), kv, lens, bt)
    assert torch.equal(new_lens.cpu(), torch.from_numpy(gold["seqlens_after"]).to(new_lens.dtype))
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(gold["out_naive"]), atol=tol, rtol=tol)
    # The cache row written for the new token matches the reference's.
    pos = inp["seqlens"].long()
    rows = torch.arange(len(pos))
    if paged:
        page = kv.shape[1]
        appended = kv[bt[rows, pos // page].long().cpu(), (pos % page)].float().cpu()
    else:
        appended = kv[rows, pos].float().cpu()
    torch.testing.assert_close(appended, torch.from_numpy(gold["appended"]), atol=tol, rtol=tol)


def test_absorbed_equals_naive_on_device(device):
    """MLA.forward (CUDA decode) against MLA.forward_naive (PyTorch) on the same module."""
    inp = recipes.layer_inputs(True, seed=4)
    model = _model(device, torch.bfloat16)
    kv1 = inp["kv"].to(device, torch.bfloat16)
    kv2 = kv1.clone()
    bt, lens, x = inp["block_table"].to(device), inp["seqlens"].to(device), inp["x"].to(device, torch.bfloat16)
    with torch.no_grad():
        a, _ = model(x, kv1, lens, bt)
        b, _ = model.forward_naive(x, kv2, lens, bt)
    torch.testing.assert_close(a.float(), b.float(), atol=3e-2, rtol=3e-2)


def test_deepseek_v3_layer_step_against_oracle(device):
    """Full DeepSeek-V3 dims (BASELINE config 5 layer), 4 requests, checked against the numpy layer oracle."""
    cfg = MLAConfig()
    torch.manual_seed(0)
    model = MLA(cfg).to(device, torch.bfloat16)
    g = torch.Generator(device=device).manual_seed(1)
    with torch.no_grad():
        for p in model.parameters():
            p.copy_(torch.randn(p.shape, generator=g, device=device) * 0.02)
        model.q_norm.weight.fill_(1.0)
        model.kv_norm.weight.fill_(1.0)
    lens = torch.tensor([100, 1, 700, 2047], dtype=torch.int32, device=device)
    pages = 4 * 32
    kv = torch.randn(pages, 64, cfg.kv_cache_dim, generator=g, device=device).bfloat16()
    bt = torch.randperm(pages, device=device).view(4, 32).int()
    x = torch.randn(4, cfg.hidden_size, generator=g, device=device).bfloat16()
    kv_before = kv.float().cpu().numpy()
    with torch.no_grad():
        out, _ = model(x, kv, lens, bt)
    w = {n: getattr(model, n).weight.detach().double().cpu().numpy() for n in recipes.LAYER_PARAM_ORDER}
    c = dict(hidden_size=cfg.hidden_size, num_heads=cfg.num_heads, q_lora_rank=cfg.q_lora_rank,
             kv_lora_rank=cfg.kv_lora_rank, qk_nope_head_dim=cfg.qk_nope_head_dim,
             qk_rope_head_dim=cfg.qk_rope_head_dim, v_head_dim=cfg.v_head_dim, rope_theta=cfg.rope_theta,
             rms_norm_eps=cfg.rms_norm_eps)
    ref, _ = orc.mla_layer_forward_absorbed(w, c, x.float().cpu().numpy(), kv_before, lens.cpu().numpy(),
                                            bt.cpu().numpy())
    got = out.float().cpu().numpy()
    scale = np.abs(ref).max()
    assert np.abs(got - ref).max() <= 3e-2 * max(scale, 1.0)


def test_decode_step_graph_matches_eager(device):
    """MLADecodeGraph replays MLA.forward: same output and appended cache rows as the eager
    step, following the lengths written in place between replays."""
    inp = recipes.layer_inputs(True, seed=6)
    model = _model(device, torch.bfloat16)
    bt = inp["block_table"].to(device)
    lens0 = inp["seqlens"].to(device)
    kv_eager = inp["kv"].to(device, torch.bfloat16)
    kv_graph = kv_eager.clone()
    lens_graph = lens0.clone()  # the length tensor the graph reads at every replay
    step = MLADecodeGraph(model, kv_graph, lens_graph, bt, num_splits=2)
    kv_graph.copy_(kv_eager)  # undo the warm-up step run before the capture
    g = torch.Generator().manual_seed(7)
    for i in range(3):
        x = torch.randn(inp["x"].shape, generator=g).to(device, torch.bfloat16)
        cur = lens0 + i
        with torch.no_grad():
            ref, ref_next = model(x, kv_eager, cur, bt, num_splits=2)
        lens_graph.copy_(cur)
        out = step(x)
        torch.cuda.synchronize(device)
        torch.testing.assert_close(out.float(), ref.float(), atol=3e-2, rtol=3e-2)
        assert torch.equal(step.next_seqlens, ref_next)
        torch.testing.assert_close(kv_graph.float(), kv_eager.float(), atol=1e-2, rtol=1e-2)
