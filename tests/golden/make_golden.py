"""Generate the golden fixtures in this folder by running the REFERENCE's own code.

Run once, in a container that has the reference checkout (it is not needed
afterwards; the fixtures are committed):

    python tests/golden/make_golden.py /path/to/triton-mla

It imports the reference package from ``<ref>/src`` (with ``TRITON_INTERPRET=1``
so its Triton kernel runs on the CPU for the absorbed layer path) and evaluates

* ``triton_mla.reference.mla_decode_ref`` (reference.py:16-31) in fp32 on the
  bf16-valued inputs of each decode recipe,
* ``triton_mla.reference.mla_decode_torch`` (reference.py:34-44) for the 4-D
  FlashMLA-layout case,
* ``triton_mla.model.MLA.forward_naive`` and ``MLA.forward`` (model.py:101-144)
  in fp32 for the small layer recipe.

Each ``.npz`` stores the outputs, a SHA-256 of the generated inputs and the
recipe name; the tests regenerate the inputs from ``recipes.py``.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import recipes  # noqa: E402


def _import_reference(ref_root: Path):
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(ref_root / "src"))
    import triton_mla  # noqa: F401  (the reference package)
    from triton_mla import MLA, MLAConfig, mla_decode, reference
    return reference, MLA, MLAConfig, mla_decode


def _decode_case(reference, name, case, out_dir):
    q, kv, lens, bt = case["q"], case["kv"], case["seqlens"], case["block_table"]
    out, lse = reference.mla_decode_ref(q.float(), kv.float(), lens, bt, softmax_scale=case["scale"])
    np.savez(out_dir / f"{name}.npz", out=out.numpy().astype(np.float32),
             lse=lse.numpy().astype(np.float32), digest=recipes.tensor_digest(q, kv, lens, bt),
             recipe=name)
    print(f"{name}: out {tuple(out.shape)} lse finite {int(torch.isfinite(lse).sum())}")


def main(ref_root: str):
    reference, MLA, MLAConfig, mla_decode = _import_reference(Path(ref_root))
    out_dir = HERE
    torch.set_num_threads(os.cpu_count() or 1)

    for h in (16, 128):
        dense = recipes.ref_grid(h, paged=False)
        paged = recipes.ref_grid(h, paged=True)
        o1, _ = reference.mla_decode_ref(dense["q"].float(), dense["kv"].float(), dense["seqlens"],
                                         None, softmax_scale=dense["scale"])
        o2, _ = reference.mla_decode_ref(paged["q"].float(), paged["kv"].float(), paged["seqlens"],
                                         paged["block_table"], softmax_scale=paged["scale"])
        assert torch.equal(o1, o2), "dense and paged layouts of the same values must agree exactly"
        _decode_case(reference, f"ref_grid_h{h}", paged, out_dir)

    _decode_case(reference, "cfg1", recipes.cfg1(), out_dir)
    _decode_case(reference, "edge_p16_h20", recipes.edge_p16_h20(), out_dir)

    fm = recipes.flashmla_layout()
    ref_t = reference.mla_decode_torch(fm["q"].float(), fm["kv"].float(), fm["seqlens"])
    ref_o, ref_l = reference.mla_decode_ref(fm["q"].float(), fm["kv"].float(), fm["seqlens"])
    np.savez(out_dir / "flashmla_layout.npz", out=ref_o.numpy(), lse=ref_l.numpy(),
             out_torch=ref_t.numpy(), digest=recipes.tensor_digest(fm["q"], fm["kv"], fm["seqlens"]),
             recipe="flashmla_layout")
    print("flashmla_layout: done")

    from triton_mla.kernel import get_num_splits  # the reference's H100 heuristic (kernel.py:190-201)
    grid = [(b, h, s, n) for b in (1, 2, 4, 8, 32, 128, 256) for h in (16, 128) for s in (1, 100, 777, 4096, 65536)
            for n in (132, 148)]
    splits = np.array([[b, h, s, n, get_num_splits(b, h, s, n)] for b, h, s, n in grid], dtype=np.int64)
    np.savez(out_dir / "ref_num_splits.npz", table=splits, recipe="ref_num_splits")
    print(f"ref_num_splits: {len(grid)} entries")

    cfg = recipes.LAYER_CFG
    w = recipes.layer_weights(cfg)
    for paged in (False, True):
        inp = recipes.layer_inputs(paged)
        model = MLA(MLAConfig(**cfg)).float()
        with torch.no_grad():
            for name, t in w.items():
                getattr(model, name).weight.copy_(t)
            kv1 = inp["kv"].clone()
            kv2 = inp["kv"].clone()
            out_naive, lens1 = model.forward_naive(inp["x"], kv1, inp["seqlens"], inp["block_table"])
            out_abs, lens2 = model(inp["x"], kv2, inp["seqlens"], inp["block_table"])
        assert torch.equal(lens1, lens2)
        tag = "paged" if paged else "dense"
        pos = inp["seqlens"].long()
        rows = torch.arange(pos.shape[0])
        if paged:
            page = kv1.shape[1]
            appended = kv1[inp["block_table"][rows, pos // page].long(), pos % page]
        else:
            appended = kv1[rows, pos]
        np.savez(out_dir / f"layer_{tag}.npz", out_naive=out_naive.numpy(), out_absorbed=out_abs.numpy(),
                 appended=appended.numpy(), seqlens_after=lens1.numpy(),
                 digest=recipes.tensor_digest(inp["x"], inp["kv"], inp["seqlens"], inp["block_table"],
                                              *[w[k] for k in recipes.LAYER_PARAM_ORDER]),
                 recipe=f"layer_{tag}")
        err = (out_naive - out_abs).abs().max().item()
        print(f"layer_{tag}: naive vs absorbed max err {err:.2e}")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
