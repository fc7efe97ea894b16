"""triton_mla (B200-native): drop-in replacement for luvadlamudi/triton-mla.

Exports the same names as the reference package (src/triton_mla/__init__.py:1-14).
``mla_decode`` and ``MLA.forward`` run hand-written sm_100a CUDA kernels from
``libtriton_mla_b200.so``; there is no Triton and no CPU implementation.
"""

from . import fp8_cache, layer_ops, sharding
from .kernel import (SplitPlan, get_num_splits, make_device_split_plan, make_split_plan, mla_decode, read_status,
                     selected_kernel)
from .model import MLA, MLAConfig, MLADecodeGraph
from .reference import mla_decode_ref, mla_decode_torch

__version__ = "0.1.1"

__all__ = [
    "MLA",
    "MLAConfig",
    "MLADecodeGraph",
    "SplitPlan",
    "get_num_splits",
    "make_device_split_plan",
    "make_split_plan",
    "mla_decode",
    "mla_decode_ref",
    "mla_decode_torch",
    "read_status",
    "selected_kernel",
]
