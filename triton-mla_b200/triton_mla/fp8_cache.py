"""FP8 latent cache rows for ``mla_decode`` (an extension: the reference caches 16-bit rows).

A row is 656 bytes per token (DeepSeek dims: 512 latent + 64 RoPE):

* bytes 0-511: the 512 latent values as float8 e4m3;
* bytes 512-527: 4 fp32 scales, scale i multiplying latent values 128 i .. 128 i + 127;
* bytes 528-655: the 64 RoPE values as bf16.

This is the public FP8 MLA cache row of FlashMLA (DeepSeek-V3.2).  A ``torch.uint8`` cache
``[num_pages, page_size, 656]`` passed to ``mla_decode`` is read in this format (C ABI:
``TMLA_KV_FP8_E4M3``); it halves the cache's bytes per token against bf16.  These helpers
convert rows with PyTorch ops on any device; they are not on the decode path.
"""

from __future__ import annotations

import torch

ROW_BYTES = 656
LATENT = 512
ROPE = 64
GROUP = 128        # latent values per scale
E4M3_MAX = 448.0   # largest finite float8 e4m3 value


def quantize_kv(kv: torch.Tensor) -> torch.Tensor:
    """``[..., 576]`` (any float dtype) -> ``[..., 656]`` uint8 rows.  Each group of 128 latent
    values is scaled so that its largest magnitude maps to 448, then rounded to e4m3."""
    assert kv.shape[-1] == LATENT + ROPE
    lead = kv.shape[:-1]
    lat = kv[..., :LATENT].float().reshape(*lead, LATENT // GROUP, GROUP)
    scale = (lat.abs().amax(-1, keepdim=True) / E4M3_MAX).clamp_min(torch.finfo(torch.float32).tiny)
    q8 = (lat / scale).to(torch.float8_e4m3fn).reshape(*lead, LATENT)
    out = torch.empty(*lead, ROW_BYTES, dtype=torch.uint8, device=kv.device)
    out[..., :LATENT] = q8.view(torch.uint8)
    out[..., LATENT:LATENT + 16] = scale.reshape(*lead, LATENT // GROUP).contiguous().view(torch.uint8)
    out[..., LATENT + 16:] = kv[..., LATENT:].to(torch.bfloat16).contiguous().view(torch.uint8)
    return out


def dequantize_kv(rows: torch.Tensor) -> torch.Tensor:
    """``[..., 656]`` uint8 rows -> ``[..., 576]`` float32 (the values ``mla_decode`` attends to)."""
    assert rows.dtype == torch.uint8 and rows.shape[-1] == ROW_BYTES
    lead = rows.shape[:-1]
    rows = rows.contiguous()
    lat = rows[..., :LATENT].contiguous().view(torch.float8_e4m3fn).float().reshape(*lead, LATENT // GROUP, GROUP)
    scale = rows[..., LATENT:LATENT + 16].contiguous().view(torch.float32).reshape(*lead, LATENT // GROUP, 1)
    rope = rows[..., LATENT + 16:].contiguous().view(torch.bfloat16).float()
    return torch.cat([(lat * scale).reshape(*lead, LATENT), rope], dim=-1)
