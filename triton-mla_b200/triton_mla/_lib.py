"""ctypes binding of the C ABI in ``include/triton_mla_b200.h``.

The shared library ``libtriton_mla_b200.so`` (built by ``triton-mla_b200/build.py``)
holds every CUDA kernel of the package.  There is no other implementation: if
the library is missing, importing the decode path raises, and a non-CUDA
tensor raises before any launch.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_NAME = "libtriton_mla_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

ABI_VERSION = 4

OK = 0
ERR_INVALID_ARG = 1
ERR_UNSUPPORTED = 2
ERR_MISALIGNED = 3
ERR_CUDA = 4
ERR_WORKSPACE = 5
MAX_BATCH = 65535  # requests (and splits) of one decode call
LAYER_FLAG_PDL = 1
LINEAR_FLAG_TEST_STALL = 0x100
LINEAR_MAX_TILES = 65536
W_NK = 0
W_KN = 1
KV_SAME = 0
KV_FP8_E4M3 = 1

STATUS_BAD_PAGE = 0x1
STATUS_TIMEOUT = 0x2
STATUS_RANGE = 0x4      # FP8 rows on the tcgen05 kernel: a value beyond the fp16 range

DTYPE_BF16 = 0
DTYPE_FP16 = 1
DTYPE_FP32 = 2

KERNEL_AUTO = 0
KERNEL_GENERIC = 1
KERNEL_SM100 = 2

FLAG_PARTIAL_ONLY = 0x1
FLAG_TEST_STALL = 0x100

NOALLOC_SCRATCH_BYTES = 32 << 20

# Every symbol the header declares; tests check the library exports all of them.
EXPORTED = (
    "tmla_decode",
    "tmla_decode_noalloc",
    "tmla_decode_partial",
    "tmla_combine",
    "tmla_num_splits",
    "tmla_workspace_bytes",
    "tmla_select_kernel",
    "tmla_error_string",
    "tmla_last_cuda_error",
    "tmla_abi_version",
    "tmla_params_bytes",
    "tmla_q_absorb_rope",
    "tmla_kv_norm_rope_append",
    "tmla_o_unabsorb",
    "tmla_l2_prefetch",
    "tmla_plan_units",
    "tmla_units_workspace_bytes",
    "tmla_decode_units",
    "tmla_plan_units_device",
    "tmla_linear",
    "tmla_linear_workspace_bytes",
)


class TmlaDecodeParams(ctypes.Structure):
    """Mirror of ``TmlaDecodeParams`` (field order and types must match the header)."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("q_stride_b", ctypes.c_int64),
        ("q_stride_h", ctypes.c_int64),
        ("kv", ctypes.c_void_p),
        ("kv_stride_page", ctypes.c_int64),
        ("kv_stride_tok", ctypes.c_int64),
        ("num_pages", ctypes.c_int64),
        ("page_size", ctypes.c_int32),
        ("seqlens", ctypes.c_void_p),
        ("block_table", ctypes.c_void_p),
        ("bt_stride", ctypes.c_int64),
        ("bt_width", ctypes.c_int32),
        ("out", ctypes.c_void_p),
        ("out_stride_b", ctypes.c_int64),
        ("out_stride_h", ctypes.c_int64),
        ("lse", ctypes.c_void_p),
        ("lse_stride_b", ctypes.c_int64),
        ("ws_o", ctypes.c_void_p),
        ("ws_lse", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("batch", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("d_qk", ctypes.c_int32),
        ("d_v", ctypes.c_int32),
        ("num_splits", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("kernel", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("softmax_scale", ctypes.c_float),
        ("q_len", ctypes.c_int32),
        ("kv_format", ctypes.c_int32),
        ("wait_ns", ctypes.c_int64),
    ]


class TmlaQPrepParams(ctypes.Structure):
    """Mirror of ``TmlaQPrepParams``."""

    _fields_ = [
        ("q_in", ctypes.c_void_p),
        ("q_in_stride_b", ctypes.c_int64),
        ("q_in_stride_h", ctypes.c_int64),
        ("w_kv_b", ctypes.c_void_p),
        ("positions", ctypes.c_void_p),
        ("q_out", ctypes.c_void_p),
        ("q_out_stride_b", ctypes.c_int64),
        ("q_out_stride_h", ctypes.c_int64),
        ("batch", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("d_nope", ctypes.c_int32),
        ("d_rope", ctypes.c_int32),
        ("d_v", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("rope_theta", ctypes.c_float),
        ("flags", ctypes.c_int32),
    ]


class TmlaKvAppendParams(ctypes.Structure):
    """Mirror of ``TmlaKvAppendParams``."""

    _fields_ = [
        ("kv_in", ctypes.c_void_p),
        ("kv_in_stride_b", ctypes.c_int64),
        ("norm_weight", ctypes.c_void_p),
        ("positions", ctypes.c_void_p),
        ("seqlens_out", ctypes.c_void_p),
        ("kv_cache", ctypes.c_void_p),
        ("kv_stride_page", ctypes.c_int64),
        ("kv_stride_tok", ctypes.c_int64),
        ("num_pages", ctypes.c_int64),
        ("page_size", ctypes.c_int32),
        ("block_table", ctypes.c_void_p),
        ("bt_stride", ctypes.c_int64),
        ("bt_width", ctypes.c_int32),
        ("status", ctypes.c_void_p),
        ("batch", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("d_rope", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("flags", ctypes.c_int32),
        ("q_in", ctypes.c_void_p),
        ("q_in_stride_b", ctypes.c_int64),
        ("q_norm_weight", ctypes.c_void_p),
        ("q_out", ctypes.c_void_p),
        ("q_out_stride_b", ctypes.c_int64),
        ("q_rank", ctypes.c_int32),
        ("q_eps", ctypes.c_float),
    ]


class TmlaOUnabsorbParams(ctypes.Structure):
    """Mirror of ``TmlaOUnabsorbParams``."""

    _fields_ = [
        ("o", ctypes.c_void_p),
        ("o_stride_b", ctypes.c_int64),
        ("o_stride_h", ctypes.c_int64),
        ("w_kv_b", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("out_stride_b", ctypes.c_int64),
        ("batch", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("d_nope", ctypes.c_int32),
        ("d_v", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("flags", ctypes.c_int32),
    ]


class TmlaLinearParams(ctypes.Structure):
    """Mirror of ``TmlaLinearParams``."""

    _fields_ = [
        ("x", ctypes.c_void_p),
        ("x_stride", ctypes.c_int64),
        ("w", ctypes.c_void_p),
        ("w_stride", ctypes.c_int64),
        ("y", ctypes.c_void_p),
        ("y_stride", ctypes.c_int64),
        ("m", ctypes.c_int32),
        ("n", ctypes.c_int32),
        ("k", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_int64),
        ("num_sms", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("status", ctypes.c_void_p),
        ("groups", ctypes.c_int32),
        ("w_layout", ctypes.c_int32),
        ("x_group_stride", ctypes.c_int64),
        ("w_group_stride", ctypes.c_int64),
        ("y_group_stride", ctypes.c_int64),
        ("wait_ns", ctypes.c_int64),
    ]


class LibraryError(RuntimeError):
    """A non-zero return code from the C ABI."""

    def __init__(self, code: int, what: str, detail: str = ""):
        self.code = code
        msg = f"{what} failed: {error_string(code)}"
        if detail:
            msg += f" ({detail})"
        super().__init__(msg)


_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and type the library; raise loudly if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("TRITON_MLA_LIB", LIB_PATH))
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build the CUDA library with `python triton-mla_b200/build.py` "
            "(there is no non-CUDA implementation of the decode path)")
    lib = ctypes.CDLL(str(path))
    P = ctypes.POINTER(TmlaDecodeParams)
    i32, i64, vp, f32p = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p
    lib.tmla_decode.argtypes = [P, vp]
    lib.tmla_decode.restype = ctypes.c_int
    lib.tmla_decode_noalloc.argtypes = [P, vp]
    lib.tmla_decode_noalloc.restype = ctypes.c_int
    lib.tmla_decode_partial.argtypes = [P, vp]
    lib.tmla_decode_partial.restype = ctypes.c_int
    lib.tmla_combine.argtypes = [f32p, f32p, vp, i64, i64, f32p, i64, i32, i32, i32, i32, i32, vp]
    lib.tmla_combine.restype = ctypes.c_int
    lib.tmla_num_splits.argtypes = [i32, i32, i32, i32]
    lib.tmla_num_splits.restype = i32
    lib.tmla_workspace_bytes.argtypes = [i32, i32, i32, i32]
    lib.tmla_workspace_bytes.restype = ctypes.c_size_t
    lib.tmla_select_kernel.argtypes = [P]
    lib.tmla_select_kernel.restype = ctypes.c_int
    lib.tmla_error_string.argtypes = [ctypes.c_int]
    lib.tmla_error_string.restype = ctypes.c_char_p
    lib.tmla_last_cuda_error.argtypes = []
    lib.tmla_last_cuda_error.restype = ctypes.c_char_p
    lib.tmla_abi_version.argtypes = []
    lib.tmla_abi_version.restype = ctypes.c_int
    lib.tmla_params_bytes.argtypes = []
    lib.tmla_params_bytes.restype = ctypes.c_size_t
    lib.tmla_plan_units.argtypes = [vp, i32, i32, i32, i32, vp, vp]
    lib.tmla_plan_units.restype = i32
    lib.tmla_units_workspace_bytes.argtypes = [i32, i32, i32]
    lib.tmla_units_workspace_bytes.restype = ctypes.c_size_t
    lib.tmla_decode_units.argtypes = [P, vp, vp, i32, i32, vp]
    lib.tmla_decode_units.restype = ctypes.c_int
    lib.tmla_plan_units_device.argtypes = [vp, i32, i32, i32, i32, i32, vp, vp, vp]
    lib.tmla_plan_units_device.restype = ctypes.c_int
    lib.tmla_linear_workspace_bytes.argtypes = [i32, i32, i32, i32, i32]
    lib.tmla_linear_workspace_bytes.restype = i64
    for name, st in (("tmla_q_absorb_rope", TmlaQPrepParams), ("tmla_kv_norm_rope_append", TmlaKvAppendParams),
                     ("tmla_o_unabsorb", TmlaOUnabsorbParams), ("tmla_linear", TmlaLinearParams)):
        fn = getattr(lib, name)
        fn.argtypes = [ctypes.POINTER(st), vp]
        fn.restype = ctypes.c_int
    lib.tmla_l2_prefetch.argtypes = [vp, i64, i64, i32, i32, vp]
    lib.tmla_l2_prefetch.restype = ctypes.c_int
    if lib.tmla_abi_version() != ABI_VERSION:
        raise ImportError(f"{path}: ABI version {lib.tmla_abi_version()} != {ABI_VERSION}; rebuild it")
    if lib.tmla_params_bytes() != ctypes.sizeof(TmlaDecodeParams):
        raise ImportError("TmlaDecodeParams layout of the library and of the binding differ; rebuild it")
    _lib = lib
    return lib


TORCH_OP_PATH = Path(__file__).resolve().parent / "libtriton_mla_torch.so"
_torch_op_loaded = False


def load_torch_op():
    """Register ``torch.ops.triton_mla.decode`` (the decode as a PyTorch operator, over the C
    ABI); returns the operator.  Raises ImportError when its library is missing."""
    global _torch_op_loaded
    import torch

    if not _torch_op_loaded:
        if not TORCH_OP_PATH.exists():
            raise ImportError(f"{TORCH_OP_PATH} is missing: build it with `python triton-mla_b200/build.py`")
        load()  # the C library first: the operator library links against it
        torch.ops.load_library(str(TORCH_OP_PATH))
        _torch_op_loaded = True
    return torch.ops.triton_mla.decode


def error_string(code: int) -> str:
    return load().tmla_error_string(code).decode()


def check(code: int, what: str) -> None:
    if code == OK:
        return
    detail = load().tmla_last_cuda_error().decode() if code == ERR_CUDA else ""
    raise LibraryError(code, what, detail)
