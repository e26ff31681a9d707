"""ctypes binding of libw8a8.so (include/w8a8.h).

This is the same C ABI a Rust/C host binds; Python goes through it too, so the
tests exercise exactly the exported entry points.  There is no fallback: if the
library is missing or cannot be loaded, importing this module raises.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("W8A8_LIBRARY", os.path.join(HERE, "libw8a8.so"))
HEADER = os.path.join(os.path.dirname(HERE), "include", "w8a8.h")

OK = 0
ERR_RUNTIME = -1
ERR_OOM = -9
ERR_ACCELERATOR = -10
ERR_VALUE = -20
ERR_INDEX = -21

F32, F16, BF16, S32, S8, E4M3 = 0, 1, 2, 3, 4, 5
MAX_RANKS, PEER_FLAG_WORDS = 8, 32
SCALE_EAGER, SCALE_KITCHEN, SCALE_KITCHEN_CUDA = 0, 1, 2
DQ_EAGER, DQ_SCALE_PRODUCT, DQ_CHAINED, DQ_SEPARATE = 0, 1, 2, 3
ACT_NONE, ACT_GELU_TANH = 0, 1
STEP_DENOISED, STEP_EULER, STEP_ER_SDE, STEP_CHURN = 0, 1, 2, 3


class Epilogue(ctypes.Structure):
    _fields_ = [
        ("ws", ctypes.c_void_p),
        ("ws_numel", ctypes.c_int64),
        ("bias", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("ldr", ctypes.c_int64),
        ("residual_scale", ctypes.c_void_p),
        ("dequant_order", ctypes.c_int32),
        ("activation", ctypes.c_int32),
        ("residual_scale_rows", ctypes.c_int64),
    ]


class SamplerStep(ctypes.Structure):
    _fields_ = [
        ("mode", ctypes.c_int32),
        ("stage", ctypes.c_int32),
        ("last", ctypes.c_int32),
        ("has_noise", ctypes.c_int32),
        ("cfg_scale", ctypes.c_float),
        ("s_noise", ctypes.c_float),
        ("denoised_input", ctypes.c_int32),
    ]


class GemmConfig(ctypes.Structure):
    _fields_ = [
        ("block_n", ctypes.c_int32),
        ("group_m", ctypes.c_int32),
        ("max_ctas", ctypes.c_int32),
        ("cta_group", ctypes.c_int32),
    ]


class W8A8Error(RuntimeError):
    """A failing libw8a8 call that is not a ValueError/IndexError/MemoryError."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


_vp, _i64, _i32, _u64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint64
_EP = ctypes.POINTER(Epilogue)
_CFG = ctypes.POINTER(GemmConfig)

SIGNATURES = {
    "w8a8_last_error": (ctypes.c_char_p, []),
    "w8a8_last_accelerator_code": (_i32, []),
    "w8a8_abi_version": (_i32, []),
    "w8a8_device_error": (_i32, [_vp]),
    "w8a8_quantize_rowwise": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _i32, _i32, _u64, _vp]),
    "w8a8_quantize_rowwise_convrot": (_i32, [_vp, _i32, _i64, _i64, _i64, _i32, _i32, _vp,
                                             ctypes.c_float, _vp, _i64, _vp, _i32, _vp]),
    "w8a8_quantize_rowwise_modulated": (_i32, [_vp, _i32, _i64, _i64, _i64, _i32, _vp,
                                               ctypes.c_float, _vp, _vp, _i64, _i32, _vp, _i64,
                                               _vp, _i32, _vp]),
    "w8a8_row_absmax": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _vp]),
    "w8a8_quantize_rowwise_given_absmax": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _i32, _vp]),
    "w8a8_gemm_dequant": (_i32, [_vp, _i64, _vp, _i64, _vp, _EP, _vp, _i32, _i64, _i64, _i64, _i64, _CFG, _vp]),
    "w8a8_rms_rope": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                             _vp, _i64, _vp, _vp, ctypes.c_float, _vp]),
    "w8a8_gemm_dequant_rms_rope": (_i32, [_vp, _i64, _vp, _i64, _vp, _EP, _vp, _i64, _i64, _i64,
                                          _i64, _i64, _vp, _i32, _vp, ctypes.c_float, _i32, _vp,
                                          _i64, _CFG, _vp]),
    "w8a8_rope_freqs_rows_bytes": (_i64, [_i64]),
    "w8a8_rope_freqs_rows": (_i32, [_vp, _i64, _i64, _vp, _vp]),
    "w8a8_gemm_splitk_workspace_bytes": (_i64, [_i64, _i64]),
    "w8a8_allgather_recv_bytes": (_i64, [_i64, _i64, _i32, _i32]),
    "w8a8_peer_barrier": (_i32, [_vp, _i32, _i32, ctypes.c_uint, _vp]),
    "w8a8_gemm_dequant_allgather": (_i32, [_vp, _i64, _vp, _i64, _vp, _EP, _vp, _i32, _i64, _i64,
                                           _i64, _i64, _vp, _vp, _i32, _i32, ctypes.c_uint,
                                           _CFG, _vp]),
    "w8a8_allgather_finish": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _vp, _i32, _i32,
                                     ctypes.c_uint, _vp]),
    "w8a8_reduce_scatter_rows": (_i64, [_i64, _i32]),
    "w8a8_reduce_scatter_recv_bytes": (_i64, [_i64, _i64, _i32]),
    "w8a8_gemm_s32_reduce_scatter": (_i32, [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _i32,
                                            _i32, ctypes.c_uint, _CFG, _vp]),
    "w8a8_reduce_scatter_finish": (_i32, [_vp, _EP, _vp, _i32, _i64, _i64, _i64, _vp, _vp, _vp,
                                          _i32, _i32, ctypes.c_uint, _vp]),
    "w8a8_gemm_auto_workspace_bytes": (_i64, [_i64, _i64, _i64, _CFG]),
    "w8a8_weight_tiles_bytes": (_i64, [_i64, _i64]),
    "w8a8_pack_weight_tiles": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp]),
    "w8a8_gemm_dequant_tiled": (_i32, [_vp, _i64, _vp, _vp, _EP, _vp, _i32, _i64, _i64, _i64, _i64,
                                       _i32, _vp, _i64, _CFG, _vp]),
    "w8a8_gemm_dequant_splitk": (_i32, [_vp, _i64, _vp, _i64, _vp, _EP, _vp, _i32, _i64, _i64, _i64,
                                        _i64, _i32, _vp, _i64, _CFG, _vp]),
    "w8a8_gemm_dequant_splitk_static": (_i32, [_vp, _i64, _vp, _i64, _vp, _EP, _vp, _i32, _i64,
                                               _i64, _i64, _i64, _i32, _CFG, _vp]),
    "w8a8_gemm_s32": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _CFG, _vp]),
    "w8a8_dequantize_linear": (_i32, [_vp, _vp, _EP, _vp, _i32, _i64, _i64, _vp]),
    "w8a8_gemv_dequant": (_i32, [_vp, _vp, _vp, _EP, _vp, _i32, _i64, _i64, _i64, _vp]),
    "w8a8_linear_small": (_i32, [_vp, _i32, _vp, _EP, _i32, _vp, _vp, _vp, _i32, _i64, _i64, _i64, _vp]),
    "w8a8_quantize_fp8_tensor": (_i32, [_vp, _i32, _i64, _vp, _vp, _vp]),
    "w8a8_fp8_gemm": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i64, _i64, _i64, _CFG, _vp]),
    "w8a8_quantize_mxfp8": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _vp]),
    "w8a8_mxfp8_gemm": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i64, _i64, _i64, _CFG, _vp]),
    "w8a8_sampler_step": (_i32, [_vp, _vp, _vp, _i32, _i64, _vp, ctypes.POINTER(SamplerStep), _vp,
                                 _vp, _vp, _vp, _vp]),
}


def header_symbols(path: str = HEADER) -> list[str]:
    """Function names declared in include/w8a8.h."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(w8a8_[a-z0-9_]+)\s*\(", text)))


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libw8a8.so not found at {LIB_PATH}; build it with `python -m imagine_b200.build`")
    lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_LOCAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


LIB = _load()


def check(rc: int) -> None:
    """Raise the Python exception matching a libw8a8 status code."""
    if rc == OK:
        return
    msg = (LIB.w8a8_last_error() or b"").decode(errors="replace")
    if rc == ERR_VALUE:
        raise ValueError(msg)
    if rc == ERR_INDEX:
        raise IndexError(msg)
    if rc == ERR_OOM:
        raise MemoryError(msg)
    raise W8A8Error(rc, msg)
