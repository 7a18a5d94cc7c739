"""ctypes binding of ``libc3b200.so`` (declarations in ``include/c3b200.h``).

The product path has no fallback: if the library is missing or fails to load,
``lib()`` raises.  Structures below mirror the header field for field.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path
from typing import Iterable, List, Optional, Sequence

import numpy as np

_LIB_PATH = Path(__file__).resolve().parent / "libc3b200.so"
_lib: Optional[C.CDLL] = None

MAX_RANK = 8

# dtypes
F32, BF16, F16, I64, I32, U8 = 0, 1, 2, 3, 4, 5
DTYPE_CODE = {"float32": F32, "bfloat16": BF16, "float16": F16, "int64": I64, "int32": I32, "uint8": U8}
DTYPE_SIZE = {F32: 4, BF16: 2, F16: 2, I64: 8, I32: 4, U8: 1}
TENSOR_ARENA = 1

# kernel ids
K_EW, K_COPY, K_IM2COL, K_REDUCE, K_GEMM, K_LAYERNORM, K_SOFTMAX, K_ATTN_SCORES, K_GATHER, K_CONV, \
    K_GEMM_TC, K_CONV_TC, K_FLASH_ATTN, K_EMBED, K_STEM_IM2COL, K_GAP_NHWC, K_STEM_CONV, \
    K_QUANT_E4M3, K_GEMM_FP8, K_QUANT_FP4, K_GEMM_W4A16, K_DEQUANT_FP4, K_WAIT_PROBE, K_GEMM_TF32 = range(1, 25)
KERNEL_NAMES = {
    0: "noop", K_EW: "ew", K_COPY: "copy", K_IM2COL: "im2col", K_REDUCE: "reduce", K_GEMM: "gemm_simt",
    K_LAYERNORM: "layernorm", K_SOFTMAX: "softmax", K_ATTN_SCORES: "attn_scores", K_GATHER: "gather",
    K_CONV: "conv_simt", K_GEMM_TC: "gemm_tc", K_CONV_TC: "conv_tc", K_FLASH_ATTN: "flash_attn",
    K_EMBED: "embed", K_STEM_IM2COL: "stem_im2col", K_GAP_NHWC: "gap_nhwc", K_STEM_CONV: "stem_conv",
    K_QUANT_E4M3: "quant_e4m3", K_GEMM_FP8: "gemm_fp8", K_QUANT_FP4: "quant_fp4", K_GEMM_W4A16: "gemm_w4a16",
    K_DEQUANT_FP4: "dequant_fp4", K_WAIT_PROBE: "wait_probe", K_GEMM_TF32: "gemm_tf32",
}

# ew ops
(OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_RELU, OP_ERF, OP_ERF_AS, OP_SQRT, OP_EXP, OP_RECIP, OP_ADD_IMM,
 OP_MUL_IMM, OP_MAX_IMM, OP_COPY) = range(14)
EW_MAX_OPS, EW_MAX_IN = 12, 6
RED_MEAN, RED_SUM, RED_MAX = 0, 1, 2
ACT_NONE, ACT_RELU, ACT_GELU = 0, 1, 2
BIAS_NONE, BIAS_COL, BIAS_ROW, BIAS_FULL, BIAS_SCALAR = range(5)


class Tensor(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("dtype", C.c_int32), ("ndim", C.c_int32),
                ("shape", C.c_int64 * MAX_RANK), ("flags", C.c_int32), ("_pad", C.c_int32)]


class EwParams(C.Structure):
    _fields_ = [("n_ops", C.c_int32), ("_pad", C.c_int32), ("op", C.c_int32 * EW_MAX_OPS),
                ("a", C.c_int32 * EW_MAX_OPS), ("b", C.c_int32 * EW_MAX_OPS), ("imm", C.c_float * EW_MAX_OPS)]


class CopyParams(C.Structure):
    _fields_ = [("in_offset", C.c_int64), ("in_stride", C.c_int64 * MAX_RANK)]


class ConvGeom(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("kh", "kw", "sh", "sw", "ph0", "pw0", "ph1", "pw1", "dh", "dw")]


class ReduceParams(C.Structure):
    _fields_ = [("outer", C.c_int64), ("reduce", C.c_int64), ("inner", C.c_int64), ("op", C.c_int32),
                ("_pad", C.c_int32)]


class GemmParams(C.Structure):
    _fields_ = [("M", C.c_int64), ("N", C.c_int64), ("K", C.c_int64), ("batch", C.c_int64),
                ("stride_a", C.c_int64), ("stride_b", C.c_int64), ("stride_c", C.c_int64),
                ("trans_a", C.c_int32), ("trans_b", C.c_int32), ("alpha", C.c_float), ("beta", C.c_float),
                ("bias_mode", C.c_int32), ("act", C.c_int32), ("has_residual", C.c_int32), ("_pad", C.c_int32)]


class LayerNormParams(C.Structure):
    _fields_ = [("rows", C.c_int64), ("cols", C.c_int64), ("epsilon", C.c_float), ("has_residual", C.c_int32),
                ("has_bias", C.c_int32), ("write_sum", C.c_int32)]


class SoftmaxParams(C.Structure):
    _fields_ = [("outer", C.c_int64), ("axis", C.c_int64), ("inner", C.c_int64)]


class AttnScoresParams(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("q0", "q1", "k0", "k1", "rows", "cols", "inner", "out0", "out1")] + \
               [("m", C.c_int32 * 4), ("_pad", C.c_int32)]


class GatherParams(C.Structure):
    _fields_ = [("outer", C.c_int64), ("axis_len", C.c_int64), ("n_idx", C.c_int64), ("inner", C.c_int64)]


class ConvParams(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("n", "c", "h", "w", "cout", "ho", "wo", "layout")] + \
               [("g", ConvGeom)] + [(n, C.c_int32) for n in ("has_bias", "has_residual", "act", "_pad")]


class GemmTcParams(C.Structure):
    _fields_ = [("M", C.c_int64), ("N", C.c_int64), ("K", C.c_int64), ("bias_mode", C.c_int32),
                ("act", C.c_int32), ("has_residual", C.c_int32), ("block_n", C.c_int32)]


class ConvTcParams(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("n", "h", "w", "cin", "cout", "ho", "wo", "k", "stride", "pad",
                                         "has_residual", "act", "block_n", "mode", "has_shortcut")]


class FlashParams(C.Structure):
    _fields_ = [("batch", C.c_int32), ("seq", C.c_int32), ("heads", C.c_int32), ("head_dim", C.c_int32),
                ("scale", C.c_float), ("causal", C.c_int32)]


class EmbedParams(C.Structure):
    _fields_ = [("batch", C.c_int64), ("seq", C.c_int64), ("dim", C.c_int64), ("vocab", C.c_int64)]


class StemParams(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("n", "c", "h", "w", "ho", "wo", "kpad", "_pad")] + \
               [("g", ConvGeom), ("_pad2", C.c_int32 * 2)]


class StemConvParams(C.Structure):
    _fields_ = [("geom", StemParams), ("cout", C.c_int32), ("act", C.c_int32)]


class QuantParams(C.Structure):
    _fields_ = [("M", C.c_int64), ("K", C.c_int64)]


class GapParams(C.Structure):
    _fields_ = [("n", C.c_int64), ("hw", C.c_int64), ("c", C.c_int64)]


class WaitProbeParams(C.Structure):
    _fields_ = [("code", C.c_int32)]


EXPORTS = [
    "c3b_version", "c3b_last_error", "c3b_kernel_id", "c3b_launch", "c3b_device_status", "c3b_sm_count",
    "c3b_set_wait_limit_ns",
    "c3b_plan_create", "c3b_plan_destroy", "c3b_plan_arena", "c3b_plan_upload", "c3b_plan_download",
    "c3b_plan_add_input_slot",
    "c3b_plan_add_output_slot", "c3b_plan_slot_ptr", "c3b_plan_add_h2d", "c3b_plan_add_d2h",
    "c3b_plan_add_record", "c3b_plan_add_wait", "c3b_plan_add_kernel", "c3b_plan_finalize",
    "c3b_plan_launch", "c3b_plan_sync", "c3b_plan_run", "c3b_plan_run_timed", "c3b_plan_kernel_count",
    "c3b_plan_origin_stream", "c3b_plan_stream",
]


def lib_path() -> Path:
    return Path(os.environ.get("C3B200_LIB", str(_LIB_PATH)))


def lib() -> C.CDLL:
    """Load the CUDA library; raises if it is missing (no CPU fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not path.exists():
        raise RuntimeError(f"libc3b200.so not found at {path}; build it with `python -m hackathon_b200.build`")
    L = C.CDLL(str(path))
    vp, i32, u64, sz = C.c_void_p, C.c_int, C.c_uint64, C.c_size_t
    T = C.POINTER(Tensor)
    L.c3b_version.restype = i32
    L.c3b_last_error.restype = C.c_char_p
    L.c3b_kernel_id.argtypes = [C.c_char_p]
    L.c3b_launch.argtypes = [i32, T, i32, T, i32, vp, sz, vp]
    L.c3b_device_status.argtypes = [C.POINTER(C.c_int)]
    L.c3b_set_wait_limit_ns.argtypes = [u64]
    L.c3b_plan_create.argtypes = [C.POINTER(vp), u64, i32, i32]
    L.c3b_plan_destroy.argtypes = [vp]
    L.c3b_plan_arena.argtypes = [vp]
    L.c3b_plan_arena.restype = vp
    L.c3b_plan_upload.argtypes = [vp, u64, vp, u64]
    L.c3b_plan_download.argtypes = [vp, u64, vp, u64]
    L.c3b_plan_add_input_slot.argtypes = [vp, u64]
    L.c3b_plan_add_output_slot.argtypes = [vp, u64]
    L.c3b_plan_slot_ptr.argtypes = [vp, i32, i32]
    L.c3b_plan_slot_ptr.restype = vp
    L.c3b_plan_add_h2d.argtypes = [vp, i32, i32, u64, u64, u64]
    L.c3b_plan_add_d2h.argtypes = [vp, i32, i32, u64, u64, u64]
    L.c3b_plan_add_record.argtypes = [vp, i32, i32]
    L.c3b_plan_add_wait.argtypes = [vp, i32, i32]
    L.c3b_plan_add_kernel.argtypes = [vp, i32, i32, T, i32, T, i32, vp, sz]
    L.c3b_plan_finalize.argtypes = [vp, i32]
    L.c3b_plan_launch.argtypes = [vp]
    L.c3b_plan_sync.argtypes = [vp, C.c_double]
    L.c3b_plan_run.argtypes = [vp]
    L.c3b_plan_run_timed.argtypes = [vp, C.POINTER(C.c_float), i32]
    L.c3b_plan_stream.argtypes = [vp, i32, C.POINTER(vp), C.POINTER(vp), C.POINTER(C.c_float)]
    L.c3b_plan_kernel_count.argtypes = [vp]
    L.c3b_plan_origin_stream.argtypes = [vp]
    L.c3b_plan_origin_stream.restype = vp
    _lib = L
    return L


def last_error() -> str:
    return lib().c3b_last_error().decode(errors="replace")


def check(rc: int, what: str) -> int:
    if rc < 0:
        raise RuntimeError(f"{what} failed ({rc}): {last_error()}")
    return rc


def make_tensor(ptr: int, dtype: int, shape: Sequence[int], arena: bool = False) -> Tensor:
    if len(shape) > MAX_RANK:
        raise ValueError(f"rank {len(shape)} exceeds {MAX_RANK}")
    t = Tensor()
    t.ptr = int(ptr)
    t.dtype = int(dtype)
    t.ndim = len(shape)
    for i, d in enumerate(shape):
        t.shape[i] = int(d)
    t.flags = TENSOR_ARENA if arena else 0
    return t


def tensor_array(ts: Sequence[Tensor]):
    arr = (Tensor * max(1, len(ts)))()
    for i, t in enumerate(ts):
        arr[i] = t
    return arr


def launch(kid: int, ins: Sequence[Tensor], outs: Sequence[Tensor], params, stream: int = 0) -> None:
    L = lib()
    ia, oa = tensor_array(ins), tensor_array(outs)
    pp = C.byref(params) if params is not None else None
    plen = C.sizeof(params) if params is not None else 0
    check(L.c3b_launch(kid, ia, len(ins), oa, len(outs), pp, plen, C.c_void_p(stream)), f"{KERNEL_NAMES.get(kid, kid)}")


def kernel_id(name: str) -> int:
    L = lib()
    rc = L.c3b_kernel_id(name.encode())
    if rc < 0:
        raise RuntimeError(last_error())
    return rc


def set_wait_limit_ns(ns: int) -> None:
    check(lib().c3b_set_wait_limit_ns(int(ns)), "set_wait_limit_ns")


def device_status() -> int:
    v = C.c_int(0)
    check(lib().c3b_device_status(C.byref(v)), "device_status")
    return v.value
