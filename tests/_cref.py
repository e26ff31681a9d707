"""ctypes access to the scalar C oracle (oracle/ref_w8a8.c), built on demand
with its Makefile.  Test infrastructure only."""
from __future__ import annotations

import ctypes
import functools
import os
import subprocess

import torch

ORACLE_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle")
DTYPE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
ACT = {None: 0, "gelu_tanh": 1, "swiglu": 2, "rms_norm": 3, "situ": 4}


@functools.lru_cache(maxsize=1)
def lib():
    subprocess.run(["make", "-s", "-C", ORACLE_DIR], check=True)
    so = ctypes.CDLL(os.path.join(ORACLE_DIR, "_build", "libref_w8a8.so"))
    vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
    so.ref_quantize_rowwise_bf16.argtypes = [vp, i64, i64, vp, vp]
    so.ref_int8_gemm.argtypes = [vp, vp, i64, i64, i64, vp]
    so.ref_dequant_eager_bf16.argtypes = [vp, vp, vp, i64, vp, i64, i64, vp]
    so.ref_quantize_fp8_bf16.argtypes = [vp, i64, f32, vp]
    so.ref_quantize_mxfp8_bf16.argtypes = [vp, i64, i64, vp, vp]
    so.ref_fht256.argtypes = [vp]
    so.ref_quantize_act_rot.argtypes = [vp, i32, i64, i64, i64, i32, i32, vp, f32, i32, vp, vp]
    so.ref_quantize_modulated.argtypes = [vp, i32, i64, i64, i32, vp, f32, vp, vp, i64, i32, i32,
                                          vp, vp]
    return so


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def fht256(v: torch.Tensor) -> torch.Tensor:
    """Normalised 256-point Hadamard transform of each 256-group (fp32)."""
    out = v.to(torch.float32).contiguous().clone()
    flat = out.view(-1, 256)
    for i in range(flat.shape[0]):
        lib().ref_fht256(_p(flat[i]))
    return out


def quantize_act_rot(x: torch.Tensor, rotate: bool, act=None, act_w=None, eps=0.0,
                     kitchen=True):
    """The fused activation + ConvRot quantiser restated in C: returns
    (q int8 [M, K], scale fp32 [M])."""
    assert x.dim() == 2
    m, width = x.shape
    k = width // 2 if act in ("swiglu", "situ") else width
    xf = x.to(torch.float32).contiguous()
    w = act_w.to(torch.float32).contiguous() if act_w is not None else None
    q = torch.empty(m, k, dtype=torch.int8)
    s = torch.empty(m, dtype=torch.float32)
    lib().ref_quantize_act_rot(_p(xf), DTYPE[x.dtype], m, k, width, int(rotate), ACT[act], _p(w),
                               float(eps), int(kitchen), _p(q), _p(s))
    return q, s


MOD = {"scale": 0, "rms_scale": 1, "adaln": 2, "rms_adaln": 3}


def quantize_modulated(x: torch.Tensor, mode: str, scale: torch.Tensor, shift=None, norm_w=None,
                       eps=1e-6, rotate=False, kitchen=False):
    """The fused modulation + (ConvRot) + row quantiser restated in C:
    (q int8 [M, K], scale fp32 [M]); scale / shift are [G, K] rows covering
    M / G x rows each."""
    m, k = x.shape
    sc = scale.to(torch.float32).reshape(-1, k).contiguous()
    sh = shift.to(torch.float32).reshape(-1, k).contiguous() if shift is not None else None
    w = norm_w.to(torch.float32).contiguous() if norm_w is not None else None
    xf = x.to(torch.float32).contiguous()  # kept alive across the call
    q = torch.empty(m, k, dtype=torch.int8)
    s = torch.empty(m, dtype=torch.float32)
    lib().ref_quantize_modulated(_p(xf), DTYPE[x.dtype], m, k,
                                 MOD[mode], _p(w), float(eps), _p(sc), _p(sh), m // sc.shape[0],
                                 int(rotate), int(kitchen), _p(q), _p(s))
    return q, s
