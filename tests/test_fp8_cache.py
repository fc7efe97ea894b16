"""FP8 cache rows (no GPU): the 656-byte layout and the quantisation round trip."""

import torch

from triton_mla import fp8_cache


def test_row_layout_and_round_trip():
    g = torch.Generator().manual_seed(3)
    kv = torch.randn(4, 7, 576, generator=g) * torch.tensor([0.01, 1.0, 30.0, 500.0]).repeat_interleave(144)
    rows = fp8_cache.quantize_kv(kv)
    assert rows.shape == (4, 7, 656) and rows.dtype == torch.uint8
    back = fp8_cache.dequantize_kv(rows)
    # RoPE values are stored as bf16 (bytes 528-655), exactly.
    assert torch.equal(back[..., 512:], kv[..., 512:].bfloat16().float())
    assert torch.equal(rows[..., 528:].contiguous().view(torch.bfloat16), kv[..., 512:].bfloat16())
    # Scales (bytes 512-527): a group's largest magnitude maps to 448, the e4m3 maximum.
    amax = kv[..., :512].abs().reshape(4, 7, 4, 128).amax(-1)
    scales = rows[..., 512:528].contiguous().view(torch.float32)
    torch.testing.assert_close(scales * 448.0, amax, rtol=1e-6, atol=0)
    # e4m3 keeps 3 mantissa bits: error at most half an ulp, 2^-4 of the value, or half the
    # smallest subnormal step (2^-9 of the group's scale) for values far below the group maximum.
    err = (back[..., :512] - kv[..., :512]).abs()
    step = scales.repeat_interleave(128, dim=-1) * 2.0 ** -9
    assert bool((err <= kv[..., :512].abs() * 2.0 ** -4 + step / 2).all())


def test_zero_rows_stay_zero():
    rows = fp8_cache.quantize_kv(torch.zeros(2, 576))
    assert torch.equal(fp8_cache.dequantize_kv(rows), torch.zeros(2, 576))
