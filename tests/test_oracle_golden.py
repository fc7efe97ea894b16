"""Pin the numpy oracle to the reference: every oracle function against golden
vectors that the reference's own Python code produced (tests/golden/make_golden.py).

CPU only.  The oracle is then trusted as the checker of the CUDA path.
"""

import numpy as np
import pytest
import torch

import recipes
from conftest import load_golden
from oracle import mla_oracle as orc

DECODE_CASES = {
    "ref_grid_h16": lambda: recipes.ref_grid(16, paged=True),
    "ref_grid_h128": lambda: recipes.ref_grid(128, paged=True),
    "cfg1": recipes.cfg1,
    "edge_p16_h20": recipes.edge_p16_h20,
    "flashmla_layout": recipes.flashmla_layout,
}


def _np(t):
    return None if t is None else t.float().numpy() if t.is_floating_point() else t.numpy()


@pytest.mark.parametrize("name", sorted(DECODE_CASES))
def test_oracle_matches_reference_decode(name):
    case = DECODE_CASES[name]()
    gold = load_golden(name)
    assert str(gold["digest"]) == recipes.tensor_digest(case["q"], case["kv"], case["seqlens"], case["block_table"]), \
        "input generator drifted from the one the golden vectors were made with"
    out, lse = orc.mla_decode_ref(_np(case["q"]), _np(case["kv"]), case["seqlens"].numpy(), _np(case["block_table"]),
                                  softmax_scale=case["scale"])
    np.testing.assert_allclose(out, gold["out"], atol=2e-5, rtol=1e-5)
    valid = np.isfinite(gold["lse"])
    assert np.array_equal(valid, np.isfinite(lse))
    np.testing.assert_allclose(lse[valid], gold["lse"][valid], atol=2e-5, rtol=1e-6)
    assert np.all(out[~valid] == 0)


def test_oracle_dense_equals_paged():
    dense, paged = recipes.ref_grid(16, paged=False), recipes.ref_grid(16, paged=True)
    a, la = orc.mla_decode_ref(_np(dense["q"]), _np(dense["kv"]), dense["seqlens"].numpy(), None,
                               softmax_scale=dense["scale"])
    b, lb = orc.mla_decode_ref(_np(paged["q"]), _np(paged["kv"]), paged["seqlens"].numpy(),
                               paged["block_table"].numpy(), softmax_scale=paged["scale"])
    assert np.array_equal(a, b) and np.array_equal(la, lb)


def test_oracle_masked_form_matches_reference_torch_baseline():
    case = recipes.flashmla_layout()
    gold = load_golden("flashmla_layout")
    out = orc.mla_decode_masked(_np(case["q"]), _np(case["kv"]), case["seqlens"].numpy())
    np.testing.assert_allclose(out, gold["out_torch"], atol=2e-5, rtol=1e-5)


def test_oracle_split_heuristic_matches_reference():
    table = load_golden("ref_num_splits")["table"]
    for b, h, s, n, want in table:
        assert orc.get_num_splits_ref(int(b), int(h), int(s), int(n)) == want


@pytest.mark.parametrize("paged", [False, True])
def test_oracle_layer_matches_reference(paged):
    tag = "paged" if paged else "dense"
    gold = load_golden(f"layer_{tag}")
    cfg = recipes.LAYER_CFG
    w_t = recipes.layer_weights(cfg)
    inp = recipes.layer_inputs(paged)
    assert str(gold["digest"]) == recipes.tensor_digest(inp["x"], inp["kv"], inp["seqlens"], inp["block_table"],
                                                       *[w_t[k] for k in recipes.LAYER_PARAM_ORDER])
    w = {k: v.double().numpy() for k, v in w_t.items()}
    bt = None if inp["block_table"] is None else inp["block_table"].numpy()
    kv1 = inp["kv"].double().numpy().copy()
    out_naive, lens = orc.mla_layer_forward_naive(w, cfg, inp["x"].numpy(), kv1, inp["seqlens"].numpy(), bt)
    kv2 = inp["kv"].double().numpy().copy()
    out_abs, _ = orc.mla_layer_forward_absorbed(w, cfg, inp["x"].numpy(), kv2, inp["seqlens"].numpy(), bt)
    np.testing.assert_array_equal(lens, gold["seqlens_after"])
    np.testing.assert_allclose(out_naive, gold["out_naive"], atol=1e-5, rtol=1e-4)
    np.testing.assert_allclose(out_abs, gold["out_absorbed"], atol=1e-5, rtol=1e-4)
    pos = inp["seqlens"].numpy().astype(np.int64)
    rows = np.arange(len(pos))
    if paged:
        page = kv1.shape[1]
        appended = kv1[bt[rows, pos // page], pos % page]
    else:
        appended = kv1[rows, pos]
    np.testing.assert_allclose(appended, gold["appended"], atol=1e-5, rtol=1e-5)


def test_bf16_round_trip():
    x = torch.randn(1000, generator=torch.Generator().manual_seed(3))
    bits = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(orc.f32_to_bf16(x.numpy()), bits)
    np.testing.assert_array_equal(orc.bf16_to_f32(bits), x.to(torch.bfloat16).float().numpy())
