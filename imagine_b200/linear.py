"""Host-side mirror of the reference's W8A8 linear-family operators.

The functions keep the names, argument meaning and error behaviour of the
reference's registry operators (inference/src/backend_signatures.rs:445-460,
KSRC comfy_kitchen/__init__.py) so a caller written against them can switch
over unchanged; every numeric step runs in libw8a8 (include/w8a8.h) through the
C ABI -- there is no CPU or PyTorch fallback for the linear itself.  PyTorch is
used for device memory, streams and the ATen steps the reference's own CUDA
route also delegates to ATen for shapes its fused kernels do not take (input
activations and ConvRot rotation when K is not a multiple of 256 up to 16384:
inference/src/cuda_linear.rs:452-475, 586-600).
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _native as N

DTYPE_CODE = {torch.float32: N.F32, torch.float16: N.F16, torch.bfloat16: N.BF16}
DEQUANT = {"eager": N.DQ_EAGER, "scale_product": N.DQ_SCALE_PRODUCT, "chained": N.DQ_CHAINED,
           "separate": N.DQ_SEPARATE}
SCALE_MODE = {"eager": N.SCALE_EAGER, "kitchen": N.SCALE_KITCHEN,
              "kitchen_cuda": N.SCALE_KITCHEN_CUDA}
OUTPUT_ACT = {None: N.ACT_NONE, "none": N.ACT_NONE, "gelu_tanh": N.ACT_GELU_TANH}


def _vp(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _cuda(name: str, t: torch.Tensor, device: Optional[torch.device] = None) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (libw8a8 has no CPU path)")
    if device is not None and t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    return t


def _code(dtype: torch.dtype) -> int:
    if dtype not in DTYPE_CODE:
        raise ValueError(f"unsupported floating dtype {dtype}")
    return DTYPE_CODE[dtype]


def _config(config) -> Optional[N.GemmConfig]:
    if config is None or config == "auto":
        return config
    if isinstance(config, N.GemmConfig):
        return config
    bn, gm, ctas, cg = (tuple(config) + (0, 0, 0, 0))[:4]
    return N.GemmConfig(int(bn), int(gm), int(ctas), int(cg))


def _cfg_ptr(cfg):
    # "auto" outside int8_linear's GEMM: the built-in heuristic
    return ctypes.byref(cfg) if isinstance(cfg, N.GemmConfig) else None


# --------------------------------------------------------------------------
# a1 / a12
# --------------------------------------------------------------------------
def quantize_int8_rowwise(x: torch.Tensor, stochastic_rounding: int = 0, *,
                          scale_mode: str = "eager"):
    """Per-row INT8 quantisation (Kitchen ``quantize_int8_rowwise(x,
    stochastic_rounding)``, inference/src/eager.rs:159-171).

    Returns ``(q int8 [..., K], scale fp32 [..., 1])``.  ``stochastic_rounding > 0``
    selects the reference CUDA kernel's PCG-hash stochastic rounding with that
    seed (native/comfy-port/kitchen/int8_linear.cu:82-95)."""
    _cuda("x", x)
    k = x.shape[-1]
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    m = x2.shape[0]
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    seed = int(stochastic_rounding or 0)
    N.check(N.LIB.w8a8_quantize_rowwise(
        _vp(x2), _code(x2.dtype), m, k, x2.stride(0) if m > 0 else k, _vp(q), k, _vp(s),
        SCALE_MODE[scale_mode], 1 if seed > 0 else 0, max(seed, 0), _stream(x.device)))
    return q.reshape(x.shape), s.reshape(*x.shape[:-1], 1)


def row_absmax(x: torch.Tensor) -> torch.Tensor:
    """max |x| of every row (fp32 [..., 1]): the first half of the K-sharded
    quantiser (all-reduce MAX the result across ranks, then
    ``quantize_int8_rowwise_given_absmax``)."""
    _cuda("x", x)
    k = x.shape[-1]
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    m = x2.shape[0]
    out = torch.empty((m,), dtype=torch.float32, device=x.device)
    N.check(N.LIB.w8a8_row_absmax(_vp(x2), _code(x2.dtype), m, k, x2.stride(0) if m > 0 else k,
                                  _vp(out), _stream(x.device)))
    return out.reshape(*x.shape[:-1], 1)


def quantize_int8_rowwise_given_absmax(x: torch.Tensor, absmax: torch.Tensor, *,
                                       scale_mode: str = "eager"):
    """Quantise x's rows with scales derived from the given per-row absmax (the
    full row's, when x is one K-shard of it).  Returns ``(q, scale [..., 1])``."""
    _cuda("x", x)
    k = x.shape[-1]
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    m = x2.shape[0]
    a = absmax.to(device=x.device, dtype=torch.float32).reshape(-1).contiguous()
    if a.numel() != m:
        raise ValueError(f"absmax has {a.numel()} entries for {m} rows")
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    N.check(N.LIB.w8a8_quantize_rowwise_given_absmax(
        _vp(x2), _code(x2.dtype), m, k, x2.stride(0) if m > 0 else k, _vp(a), _vp(q), k, _vp(s),
        SCALE_MODE[scale_mode], _stream(x.device)))
    return q.reshape(x.shape), s.reshape(*x.shape[:-1], 1)


INPUT_ACT = {None: 0, "none": 0, "gelu_tanh": 1, "swiglu": 2, "rms_norm": 3, "situ": 4}


def quantize_int8_rowwise_convrot(x: torch.Tensor, group: int = 256, input_act: Optional[str] = None,
                                  input_act_weight: Optional[torch.Tensor] = None,
                                  input_act_eps: Optional[float] = None, *,
                                  scale_mode: str = "kitchen"):
    """Input activation + ConvRot + per-row INT8 quantisation in one pass
    (Kitchen ``quantize_int8_rowwise_convrot64``, inference/src/convrot.rs:156-209;
    kernel native/comfy-port/kitchen/int8_linear.cu:1197-1314).

    ``group`` 256 rotates each 256-column group by the normalised Hadamard
    matrix; ``group`` 0 applies only the activation (rounded to x's dtype as
    the reference's ATen activation is).  SwiGLU / SiTU take [..., 2K] rows.
    Returns ``(q int8 [..., K], scale fp32 [..., 1])``."""
    _cuda("x", x)
    if input_act not in INPUT_ACT:
        raise ValueError(f"unknown input_act {input_act!r}")
    code = INPUT_ACT[input_act]
    width = x.shape[-1]
    k = width // 2 if code in (2, 4) else width
    if code in (2, 4) and width % 2:
        raise ValueError("not enough values to unpack (expected 2, got 1)")
    x2 = x.reshape(-1, width)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    m = x2.shape[0]
    w = None
    if code == 3:
        if input_act_weight is None:
            raise ValueError("input_act 'rms_norm' requires act_weight")
        if input_act_eps is None:
            # the reference's fused path refuses an unset epsilon
            # (inference/src/convrot.rs:236-243)
            raise TypeError("float() argument must be a string or a real number, not 'NoneType'")
        w = input_act_weight.to(device=x.device, dtype=x.dtype).reshape(-1).contiguous()
        if w.numel() != k:
            raise ValueError(f"act_weight has {w.numel()} elements for K={k}")
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    N.check(N.LIB.w8a8_quantize_rowwise_convrot(
        _vp(x2), _code(x2.dtype), m, k, x2.stride(0) if m > 0 else width, int(group), code, _vp(w),
        float(input_act_eps or 0.0), _vp(q), k, _vp(s), SCALE_MODE[scale_mode], _stream(x.device)))
    return q.reshape(*x.shape[:-1], k), s.reshape(*x.shape[:-1], 1)


MODULATION = {"scale": 0, "rms_scale": 1, "adaln": 2, "rms_adaln": 3}


def _mod_rows(t: torch.Tensor, rows: int, k: int, name: str, dev, dtype) -> tuple:
    """Modulation tensor as contiguous [G, K] rows plus the number of x rows
    each one covers (a [K] / [1, K] tensor covers all rows; [B, 1, K] or
    [B, K] covers rows / B consecutive rows each)."""
    t = t.to(device=dev, dtype=dtype)
    if t.shape[-1] != k:
        raise ValueError(f"{name} has {t.shape[-1]} features, expected {k}")
    t = t.reshape(-1, k).contiguous()
    g = t.shape[0]
    if g == 0 or rows % g:
        raise ValueError(f"{name} has {g} rows, which do not divide the {rows} activation rows")
    return t, max(rows // g, 1)


def quantize_int8_rowwise_modulated(x: torch.Tensor, mode: str, modulation_scale: torch.Tensor,
                                    shift: Optional[torch.Tensor] = None,
                                    norm_weight: Optional[torch.Tensor] = None, eps: float = 1e-6,
                                    convrot: bool = False, *, scale_mode: str = "eager"):
    """Modulation (``scale``: x(1+s); ``rms_scale``: rms_norm(x, w)(1+s);
    ``adaln``: layer_norm(x)(1+s)+shift; ``rms_adaln``: rms_norm(x)(1+s)+shift),
    optional 256-group ConvRot, and per-row INT8 quantisation in one pass.
    Returns ``(q int8 [..., K], scale fp32 [..., 1])``."""
    _cuda("x", x)
    if mode not in MODULATION:
        raise ValueError(f"unknown modulation {mode!r}")
    k = x.shape[-1]
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    m = x2.shape[0]
    sc, group = _mod_rows(modulation_scale, m, k, "modulation_scale", x.device, x.dtype)
    sh = None
    if mode in ("adaln", "rms_adaln"):
        if shift is None:
            raise ValueError(f"modulation {mode!r} needs a shift")
        sh, g2 = _mod_rows(shift, m, k, "shift", x.device, x.dtype)
        if g2 != group:
            raise ValueError("scale and shift must have the same number of rows")
    w = None
    if mode == "rms_scale":
        if norm_weight is None:
            raise ValueError("modulation 'rms_scale' needs norm_weight")
        w = norm_weight.to(device=x.device, dtype=x.dtype).reshape(-1).contiguous()
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    N.check(N.LIB.w8a8_quantize_rowwise_modulated(
        _vp(x2), _code(x2.dtype), m, k, x2.stride(0) if m > 0 else k, MODULATION[mode], _vp(w),
        float(eps), _vp(sc), _vp(sh), group, 256 if convrot else 0, _vp(q), k, _vp(s),
        SCALE_MODE[scale_mode], _stream(x.device)))
    return q.reshape(x.shape), s.reshape(*x.shape[:-1], 1)


def _modulated_linear(x, mode, modulation_scale, shift, norm_weight, eps, weight, weight_scale,
                      bias, out_dtype, convrot, convrot_groupsize, scale_mode, dequant,
                      output_act, aten_modulate):
    """Shared body of the modulated linears: the fused quantiser when K fits
    it, else the modulation as device ATen ops followed by int8_linear."""
    k = x.shape[-1]
    fused = k % 256 == 0 and 256 <= k <= 16384 and (not convrot or convrot_groupsize == 256)
    if not fused:
        return int8_linear(aten_modulate(x), weight, weight_scale, bias, out_dtype, convrot,
                           convrot_groupsize, scale_mode=scale_mode, dequant=dequant,
                           output_act=output_act)
    _cuda("weight", weight, x.device)
    if weight.dim() != 2 or weight.dtype != torch.int8:
        raise ValueError("weight must be a 2-D int8 tensor [N, K]")
    if k != weight.shape[-1]:
        raise ValueError(f"Input and weight inner dimensions must match, got {k} and {weight.shape[-1]}")
    n = weight.shape[0]
    dev = x.device
    out_dtype = out_dtype or x.dtype
    ws = weight_scale.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
    if ws.numel() not in (1, n):
        raise ValueError(f"INT8 weight scale must be scalar or per-output-channel, got "
                         f"{tuple(weight_scale.shape)} for weight shape {tuple(weight.shape)}")
    q, xs = quantize_int8_rowwise_modulated(x, mode, modulation_scale, shift, norm_weight, eps,
                                            convrot, scale_mode=scale_mode)
    lead = x.shape[:-1]
    q = q.reshape(-1, k)
    xs = xs.reshape(-1)
    m = q.shape[0]
    w = weight if weight.is_contiguous() else weight.contiguous()
    b = bias.to(device=dev, dtype=out_dtype).reshape(-1).contiguous() if bias is not None else None
    out = torch.empty((m, n), dtype=out_dtype, device=dev)
    ep = _epilogue(ws, b, None, None, dequant, output_act, n, n)
    stream = _stream(dev)
    if 1 <= m <= 2:
        N.check(N.LIB.w8a8_gemv_dequant(_vp(q), _vp(w), _vp(xs), ctypes.byref(ep), _vp(out),
                                        _code(out_dtype), m, n, k, stream))
    elif m > 0:
        _gemm_dequant(q, w, xs, ep, out, out_dtype, m, n, k, None, None, stream)
    return out.reshape(*lead, n)


def int8_linear_modulated(x: torch.Tensor, modulation_scale: torch.Tensor, weight: torch.Tensor,
                          weight_scale: torch.Tensor, bias: Optional[torch.Tensor] = None,
                          out_dtype: Optional[torch.dtype] = torch.bfloat16, convrot: bool = False,
                          convrot_groupsize: int = 256, *, scale_mode: str = "eager",
                          dequant: str = "eager", output_act: Optional[str] = None):
    """Registry operator ``int8_linear_modulated`` (inference/src/backend_signatures.rs:
    128-139; eager body inference/src/backend_bindings.rs:329-405):
    ``int8_linear(x * (1 + modulation_scale), ...)`` for one batch-one
    modulation row, with the modulation fused into the quantiser."""
    _cuda("x", x)
    k = x.shape[-1]
    if modulation_scale.numel() != k:
        raise ValueError(f"modulation_scale must contain one batch-one row of {k} values, got "
                         f"{modulation_scale.numel()}")

    def aten(t):
        return t * (modulation_scale.to(device=t.device, dtype=t.dtype).reshape(-1) + 1)
    return _modulated_linear(x, "scale", modulation_scale, None, None, 0.0, weight, weight_scale,
                             bias, out_dtype, convrot, convrot_groupsize, scale_mode, dequant,
                             output_act, aten)


def int8_linear_rms_modulated(x: torch.Tensor, norm_weight: torch.Tensor, norm_eps: float,
                              modulation_scale: torch.Tensor, weight: torch.Tensor,
                              weight_scale: torch.Tensor, bias: Optional[torch.Tensor] = None,
                              out_dtype: Optional[torch.dtype] = torch.bfloat16,
                              convrot: bool = False, convrot_groupsize: int = 256, *,
                              scale_mode: str = "eager", dequant: str = "eager",
                              output_act: Optional[str] = None):
    """Registry operator ``int8_linear_rms_modulated`` (inference/src/backend_signatures.rs:
    140-156): ``int8_linear_modulated(rms_norm(x, norm_weight, norm_eps), ...)``."""
    _cuda("x", x)
    k = x.shape[-1]
    if modulation_scale.numel() != k:
        raise ValueError(f"modulation_scale must contain one batch-one row of {k} values, got "
                         f"{modulation_scale.numel()}")
    eps = float(norm_eps or 0.0)

    def aten(t):
        nrm = torch.nn.functional.rms_norm(t, (k,), norm_weight.to(device=t.device, dtype=t.dtype), eps)
        return nrm * (modulation_scale.to(device=t.device, dtype=t.dtype).reshape(-1) + 1)
    return _modulated_linear(x, "rms_scale", modulation_scale, None, norm_weight, eps, weight,
                             weight_scale, bias, out_dtype, convrot, convrot_groupsize, scale_mode,
                             dequant, output_act, aten)


def adaln_int8_linear(x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor,
                      weight: torch.Tensor, weight_scale: torch.Tensor,
                      bias: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                      eps: float = 1e-6, rms: bool = False, convrot: bool = False,
                      convrot_groupsize: int = 256, *, scale_mode: str = "eager",
                      dequant: str = "eager", output_act: Optional[str] = None):
    """AdaLN modulation (``adaln`` / ``rms_adaln``: norm(x)(1 + scale) + shift,
    inference/src/backend_eager.rs:176-236) followed by the INT8 linear -- the
    pre-QKV / pre-MLP-up step of an MMDiT block -- with the modulation fused
    into the quantiser.  scale / shift: [K], or one row per sample ([B, 1, K]
    for x [B, S, K])."""
    _cuda("x", x)
    k = x.shape[-1]

    def aten(t):
        sc = scale.to(device=t.device, dtype=t.dtype)
        sh = shift.to(device=t.device, dtype=t.dtype)
        if rms:
            nrm = torch.nn.functional.rms_norm(t, (k,), None, eps)
        else:
            nrm = torch.nn.functional.layer_norm(t, (k,), None, None, eps)
        return nrm * (sc + 1) + sh
    return _modulated_linear(x, "rms_adaln" if rms else "adaln", scale, shift, None, eps, weight,
                             weight_scale, bias, out_dtype, convrot, convrot_groupsize, scale_mode,
                             dequant, output_act, aten)


def rms_rope(q: torch.Tensor, k: Optional[torch.Tensor], freqs_cis: torch.Tensor,
             q_scale: torch.Tensor, k_scale: Optional[torch.Tensor] = None,
             epsilon: float = 1e-6):
    """Kitchen op ``rms_rope(q, k, freqs_cis, q_scale, k_scale, epsilon)``
    (inference/src/models/qwen_image21/dit.rs:486-505; eager body
    inference/src/backend_rope.rs:146-223): per-head RMSNorm with weight, then
    the interleaved-pair rotation.  q / k: [..., S, H, D]; freqs_cis: fp32
    [S, D/2, 2, 2] or with leading broadcast dimensions ([B, S, 1, D/2, 2, 2]).
    Returns ``(q_out, k_out)`` (``k_out`` is None without k)."""
    _cuda("q", q)
    d = q.shape[-1]
    heads = q.shape[-2]
    q2 = q.reshape(-1, heads * d)
    if q2.stride(-1) != 1:
        q2 = q2.contiguous()
    rows = q2.shape[0]
    k2 = None
    if k is not None:
        _cuda("k", k, q.device)
        if k.shape != q.shape or k.dtype != q.dtype:
            raise ValueError("q and k must have the same shape and dtype")
        k2 = k.reshape(-1, heads * d)
        if k2.stride(-1) != 1:
            k2 = k2.contiguous()
        if k_scale is None:
            raise ValueError("k needs k_scale")
    f = freqs_cis.to(device=q.device, dtype=torch.float32).reshape(-1, d // 2, 2, 2).contiguous()
    if f.shape[0] == 0 or rows % f.shape[0]:
        raise ValueError(f"freqs_cis has {f.shape[0]} positions for {rows} token rows")
    qs = q_scale.to(device=q.device, dtype=q.dtype).reshape(-1).contiguous()
    ks = (k_scale.to(device=q.device, dtype=q.dtype).reshape(-1).contiguous()
          if k is not None else None)
    if qs.numel() != d or (ks is not None and ks.numel() != d):
        raise ValueError(f"q_scale / k_scale must have head_dim = {d} elements")
    qo = torch.empty_like(q2)
    ko = torch.empty_like(k2) if k2 is not None else None
    N.check(N.LIB.w8a8_rms_rope(
        _vp(q2), _vp(k2), _vp(qo), _vp(ko), _code(q.dtype), rows, heads, d, q2.stride(0),
        k2.stride(0) if k2 is not None else 0, qo.stride(0), ko.stride(0) if ko is not None else 0,
        _vp(f), f.shape[0], _vp(qs), _vp(ks), float(epsilon), _stream(q.device)))
    return qo.reshape(q.shape), (ko.reshape(k.shape) if ko is not None else None)


_FREQS_ROWS: dict = {}


def rope_freqs_rows(freqs_cis: torch.Tensor, rows: int) -> torch.Tensor:
    """The row-blocked rotations the fused RMSNorm + RoPE epilogue reads
    (w8a8_rope_freqs_rows): freqs_cis [S, 64, 2, 2] (or with leading broadcast
    dimensions) for ``rows`` token rows, row r at position r % S.  Built once
    per (freqs_cis, rows) and cached: every block of a forward pass shares
    them."""
    _cuda("freqs_cis", freqs_cis)
    f = freqs_cis.to(dtype=torch.float32).reshape(-1, 64, 2, 2).contiguous()
    if f.shape[0] == 0 or rows % f.shape[0]:
        raise ValueError(f"freqs_cis has {f.shape[0]} positions for {rows} token rows")
    key = (f.device.index, f.data_ptr(), f._version, f.shape[0], rows)
    hit = _FREQS_ROWS.get(key)
    if hit is None:
        if len(_FREQS_ROWS) >= 8:
            _FREQS_ROWS.pop(next(iter(_FREQS_ROWS)))
        n = int(N.LIB.w8a8_rope_freqs_rows_bytes(rows)) // 4
        blocked = torch.empty(n, dtype=torch.float32, device=f.device)
        N.check(N.LIB.w8a8_rope_freqs_rows(_vp(f), f.shape[0], rows, _vp(blocked),
                                           _stream(f.device)))
        # the entry keeps the source alive too: once freed, its address could
        # come back holding other rotations under the same key
        hit = _FREQS_ROWS[key] = (blocked, f)
    return hit[0]


def int8_linear_rms_rope(x: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
                         bias: Optional[torch.Tensor], norm_weight: torch.Tensor,
                         freqs_cis: torch.Tensor, epsilon: float = 1e-6,
                         rope_cols: Optional[int] = None, *, dequant: str = "eager",
                         scale_mode: str = "eager", split_k: Optional[int] = None, config=None,
                         modulation: Optional[tuple] = None):
    """The Q (or K) projection with its RMSNorm + RoPE fused into the GEMM
    epilogue: ``rms_rope(int8_linear(x, weight, ...))`` of the reference's
    attention (inference/src/models/qwen_image21/dit.rs:427-429, 486-505) for
    head_dim 128, with bf16 output.  Columns ``[0, rope_cols)`` (default: all)
    are 128-column heads normalised with ``norm_weight`` -- [128] shared by
    every head, or [rope_cols] per column (q_norm then k_norm for a fused QKV
    weight) -- and rotated by ``freqs_cis`` [S, 64, 2, 2] (row r of x uses
    position r % S); later columns (v) get the plain epilogue.  Returns
    [..., N] bf16.  ``modulation=(scale, shift, eps, rms)`` quantises
    ``norm(x)(1 + scale) + shift`` instead of x (the AdaLN step before an
    MMDiT block's QKV projection), in the same pass as the quantiser."""
    _cuda("x", x)
    dev = x.device
    _cuda("weight", weight, dev)
    if weight.dim() != 2 or weight.dtype != torch.int8:
        raise ValueError("weight must be a 2-D int8 tensor [N, K]")
    n, k = weight.shape
    if x.shape[-1] != k:
        raise ValueError(f"Input and weight inner dimensions must match, got {x.shape[-1]} and {k}")
    rope_cols = n if rope_cols is None else int(rope_cols)
    if n % 128 or rope_cols % 128 or not 0 <= rope_cols <= n:
        raise ValueError(f"N ({n}) and rope_cols ({rope_cols}) must be multiples of the 128-column "
                         "head with rope_cols <= N")
    ws = weight_scale.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
    if ws.numel() not in (1, n):
        raise ValueError(f"INT8 weight scale must be scalar or per-output-channel, got "
                         f"{tuple(weight_scale.shape)} for weight shape {tuple(weight.shape)}")
    nw = norm_weight.to(device=dev, dtype=torch.bfloat16).reshape(-1).contiguous()
    if nw.numel() not in (128, rope_cols):
        raise ValueError(f"norm_weight must have 128 or rope_cols = {rope_cols} elements, got "
                         f"{nw.numel()}")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, k)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    m = x2.shape[0]
    if m == 0:
        return torch.empty((*lead, n), dtype=torch.bfloat16, device=dev)
    stream = _stream(dev)
    if modulation is None:
        q = torch.empty((m, k), dtype=torch.int8, device=dev)
        xs = torch.empty((m,), dtype=torch.float32, device=dev)
        N.check(N.LIB.w8a8_quantize_rowwise(_vp(x2), _code(x2.dtype), m, k, k, _vp(q), k, _vp(xs),
                                            SCALE_MODE[scale_mode], 0, 0, stream))
    else:
        scale, shift, eps_mod, rms = modulation
        q, xs = quantize_int8_rowwise_modulated(x2.reshape(*lead, k), "rms_adaln" if rms else "adaln",
                                                scale, shift, None, eps_mod,
                                                scale_mode=scale_mode)
        q = q.reshape(m, k)
        xs = xs.reshape(m)
    return _rms_rope_gemm(q, xs, lead, weight, ws, bias, nw, freqs_cis, epsilon, rope_cols,
                          dequant, split_k, config, stream)


def _rms_rope_gemm(q, xs, lead, weight, ws, bias, nw, freqs_cis, epsilon, rope_cols, dequant,
                   split_k, config, stream, out=None):
    """The GEMM with the RMSNorm + RoPE epilogue on quantised rows q [M, K];
    ``out``: an [M, N] bf16 view with unit column stride to write into (any
    row stride), else a new tensor."""
    dev = q.device
    m, k = q.shape
    n = weight.shape[0]
    fr = rope_freqs_rows(freqs_cis, m) if rope_cols else None
    w = weight if weight.is_contiguous() else weight.contiguous()
    b = bias.to(device=dev, dtype=torch.bfloat16).reshape(-1).contiguous() if bias is not None else None
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    elif (out.shape != (m, n) or out.dtype != torch.bfloat16 or out.stride(1) != 1
          or out.device != dev):
        raise ValueError(f"out must be a bf16 [{m}, {n}] view with unit column stride")
    ldo = out.stride(0)
    ep = _epilogue(ws, b, None, None, dequant, None, n, n)
    cfg = _config(config)
    cfg = cfg if isinstance(cfg, N.GemmConfig) else None
    if split_k is None:
        nbytes = _auto_workspace_bytes(dev, m, n, k, cfg)
    elif split_k > 1:
        nbytes = int(N.LIB.w8a8_gemm_splitk_workspace_bytes(m, n))
    else:
        nbytes = 0
    scratch = _splitk_scratch(dev, nbytes) if nbytes > 0 else None
    N.check(N.LIB.w8a8_gemm_dequant_rms_rope(
        _vp(q), k, _vp(w), k, _vp(xs), ctypes.byref(ep), _vp(out), ldo, m, n, k, rope_cols,
        _vp(nw), 1 if nw.numel() != 128 else 0, _vp(fr), float(epsilon),
        int(split_k or 0) if scratch is not None else 1, _vp(scratch),
        scratch.numel() if scratch is not None else 0, _cfg_ptr(cfg), stream))
    return out.reshape(*lead, n) if lead is not None else out


def quantize_weight(weight: torch.Tensor, convrot: bool = False, convrot_groupsize: int = 256, *,
                    scale_mode: str = "eager"):
    """Offline per-output-channel weight quantisation
    (inference/src/layout_complete.rs:119-159 TensorWiseINT8Layout.from_float):
    returns ``(w_q int8 [N, K], ws fp32 [N])``.  ``convrot=True`` is the ConvRot
    weight form (``quantize_int8_convrot_weight``, inference/src/convrot.rs:
    378-435): each row rotated by the normalised Hadamard matrix per 256-group
    of K, then quantised -- the fused kernel the reference's CUDA route picks
    for these widths (its ``rowwise64`` path, convrot.rs:345-376)."""
    if not convrot:
        q, s = quantize_int8_rowwise(weight, scale_mode=scale_mode)
        return q, s.reshape(-1)
    if weight.dim() != 2:
        raise ValueError("ConvRot INT8 weight quantization expects a 2D weight tensor")
    if convrot_groupsize != 256:
        raise ValueError("ConvRot weights are supported for group size 256")
    q, s = quantize_int8_rowwise_convrot(weight.contiguous(), 256, scale_mode=scale_mode)
    return q, s.reshape(-1)


# --------------------------------------------------------------------------
# a3 / a4 / a5 / a6
# --------------------------------------------------------------------------
def _residual_scale(scale, lead, n, dtype, dev):
    """The residual scale as the epilogue reads it, with the broadcasting of the
    reference's ``residual.addcmul(out, scale)`` (inference/src/int8_linear.rs:
    99-111) against an output of shape (*lead, n).  Returns (table, rows_per):
    one [N] row for every output row (rows_per 0); a per-sample gate [B, 1, N]
    over an output [B, S, N] as a [B, N] table with rows_per = S (the model's
    gated residual, inference/src/models/qwen_image21/numeric.rs:110-126); any
    other broadcastable shape expanded to one row per output row (rows_per 1)."""
    scale = scale.to(device=dev, dtype=dtype)
    if scale.numel() == n:
        return scale.reshape(-1).contiguous(), 0
    full = (*lead, n)
    try:
        shape = torch.broadcast_shapes(tuple(scale.shape), full)
    except RuntimeError as e:
        raise ValueError(f"residual_scale of shape {tuple(scale.shape)} does not broadcast "
                         f"against the output {full}: {e}") from None
    if shape != full:
        raise ValueError(f"residual_scale of shape {tuple(scale.shape)} broadcasts the output "
                         f"{full} to {shape}")
    s = scale.reshape((1,) * (len(full) - scale.dim()) + tuple(scale.shape))
    if len(lead) >= 2 and s.shape[-2] == 1 and tuple(s.shape[:-2]) == tuple(lead[:-1]):
        return s.reshape(-1, n).contiguous(), lead[-1]
    return scale.expand(full).reshape(-1, n).contiguous(), 1


def _epilogue(weight_scale, bias, residual, residual_scale, dequant, output_act, n, ldr,
              residual_scale_rows=0):
    ep = N.Epilogue()
    ep.ws = weight_scale.data_ptr()
    ep.ws_numel = weight_scale.numel()
    ep.bias = bias.data_ptr() if bias is not None else None
    ep.residual = residual.data_ptr() if residual is not None else None
    ep.ldr = ldr if residual is not None else 0
    ep.residual_scale = residual_scale.data_ptr() if residual_scale is not None else None
    ep.residual_scale_rows = residual_scale_rows if residual is not None else 0
    if dequant not in DEQUANT:
        raise ValueError(f"unknown dequant order {dequant!r}")
    ep.dequant_order = DEQUANT[dequant]
    if output_act not in OUTPUT_ACT:
        raise ValueError(f"unknown output activation {output_act!r}")
    ep.activation = OUTPUT_ACT[output_act]
    return ep


def _apply_input(x, input_act, weight, eps):
    """inference/src/int8_linear.rs:37-97 on the device (ATen, as the reference's
    CUDA route does for activations it does not fuse)."""
    if input_act is None or input_act == "none":
        return x
    if input_act == "gelu_tanh":
        return torch.nn.functional.gelu(x, approximate="tanh")
    if input_act == "swiglu":
        gate, up = x.chunk(2, dim=-1)
        return torch.nn.functional.silu(gate).mul_(up)
    if input_act == "situ":
        a, b = x.chunk(2, dim=-1)
        gated = torch.tanh(b / 4.0) * 4.0 * torch.sigmoid(b)
        return torch.tanh(a / 25.0) * 25.0 * gated
    if input_act == "rms_norm":
        if weight is None:
            raise ValueError("input_act 'rms_norm' requires act_weight")
        return torch.nn.functional.rms_norm(x, (x.shape[-1],), weight.to(x.dtype), eps)
    raise ValueError(f"unknown input_act {input_act!r}")


_HADAMARD: dict = {}


def _hadamard(size: int, device, dtype) -> torch.Tensor:
    """inference/src/int8_utils.rs:21-58 (cached per device/dtype)."""
    key = (size, device, dtype)
    if key not in _HADAMARD:
        if size < 4 or size & (size - 1) or (size.bit_length() - 1) % 2:
            raise ValueError(f"Regular Hadamard size must be a power of 4, got {size}")
        h4 = torch.tensor([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]],
                          dtype=torch.int64).to(dtype)
        h = h4
        while h.shape[0] < size:
            h = torch.kron(h, h4)
        _HADAMARD[key] = (h / (size ** 0.5)).to(device)
    return _HADAMARD[key]


class TiledInt8Weight:
    """An int8 weight [N, K] in the pre-tiled layout of w8a8_pack_weight_tiles
    (128-row x 128-byte tiles, each 16 KB contiguous): what few-row GEMMs
    stream from HBM.  int8_linear takes it in place of the [N, K] tensor."""

    def __init__(self, tiles: torch.Tensor, n: int, k: int):
        self.tiles, self.n, self.k = tiles, n, k

    @property
    def shape(self):
        return torch.Size((self.n, self.k))

    @property
    def device(self):
        return self.tiles.device

    @property
    def dtype(self):
        return torch.int8

    def dim(self):
        return 2

    def is_contiguous(self):
        return True


def pack_weight_tiles(weight: torch.Tensor) -> TiledInt8Weight:
    """Pack an int8 [N, K] weight once (offline) into the pre-tiled layout."""
    _cuda("weight", weight)
    if weight.dim() != 2 or weight.dtype != torch.int8:
        raise ValueError("weight must be a 2-D int8 tensor [N, K]")
    n, k = weight.shape
    if weight.stride(-1) != 1:
        weight = weight.contiguous()
    tiles = torch.empty(int(N.LIB.w8a8_weight_tiles_bytes(n, k)), dtype=torch.int8,
                        device=weight.device)
    N.check(N.LIB.w8a8_pack_weight_tiles(_vp(weight), weight.stride(0) if n else k, n, k,
                                         _vp(tiles), _stream(weight.device)))
    return TiledInt8Weight(tiles, n, k)


_SPLITK_SCRATCH: dict = {}


_AUTO_WS: dict = {}


def _auto_workspace_bytes(dev, m, n, k, cfg) -> int:
    """Scratch bytes the library's automatic split policy uses for this shape
    (few-row split-K, or the tail-wave spread of a large GEMM); 0 for none."""
    c = cfg if isinstance(cfg, N.GemmConfig) else None
    key = (dev.index, m, n, k, None if c is None else (c.block_n, c.group_m, c.max_ctas, c.cta_group))
    v = _AUTO_WS.get(key)
    if v is None:
        with torch.cuda.device(dev):
            v = int(N.LIB.w8a8_gemm_auto_workspace_bytes(m, n, k, _cfg_ptr(c)))
        N.check(0 if v >= 0 else v)
        _AUTO_WS[key] = v
    return v


def _splitk_scratch(dev: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-filled split-K scratch, one per (device, stream): the kernels leave
    it zero-filled after every call, and calls on one stream never overlap."""
    key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
    buf = _SPLITK_SCRATCH.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _SPLITK_SCRATCH[key] = buf
    return buf


def _autotuned_config(q, w, xs, ep, out, out_dtype, m, n, k, stream):
    """config="auto": the tile configuration the autotuner picks for this
    shape and epilogue (timed once per key, then cached), mirroring the
    reference's Int8Autotuner use (inference/src/backend_triton_int8.rs:365-449)."""
    from . import autotune

    key = (m, n, k, "int8", "int8", str(out_dtype), int(ep.ws_numel == 1), int(ep.dequant_order),
           int(ep.activation), ep.residual is not None, ep.bias is not None)

    def run(cfg):
        c = _config(cfg)
        rc = N.LIB.w8a8_gemm_dequant(_vp(q), k, _vp(w), k, _vp(xs), ctypes.byref(ep), _vp(out),
                                     _code(out_dtype), n, m, n, k, ctypes.byref(c), stream)
        if rc == N.ERR_VALUE:
            raise ValueError(N.LIB.w8a8_last_error().decode(errors="replace"))
        N.check(rc)

    return _config(autotune.tune_gemm("int8_dequant", key, run, autotune.CudaBenchmark(out.device)))


def _gemm_dequant(q, w, xs, ep, out, out_dtype, m, n, k, cfg, split_k, stream):
    """w8a8_gemm_dequant, or its split-K form when the 128 x 128 tiles of a
    few-row shape would leave SMs idle (or splits were asked for)."""
    dev = out.device
    if isinstance(w, TiledInt8Weight):
        cfg = None if cfg == "auto" else cfg
        scratch = None
        if split_k != 1 and m > 0 and n % 4 == 0:
            scratch = _splitk_scratch(dev, int(N.LIB.w8a8_gemm_splitk_workspace_bytes(m, n)))
        N.check(N.LIB.w8a8_gemm_dequant_tiled(
            _vp(q), k, _vp(w.tiles), _vp(xs), ctypes.byref(ep), _vp(out), _code(out_dtype), n, m,
            n, k, int(split_k or 0), _vp(scratch), scratch.numel() if scratch is not None else 0,
            _cfg_ptr(cfg), stream))
        return
    if cfg == "auto":
        cfg = _autotuned_config(q, w, xs, ep, out, out_dtype, m, n, k, stream)
        split_k = 1 if split_k is None else split_k
    nbytes = 0
    if split_k is None and m > 0:
        nbytes = _auto_workspace_bytes(dev, m, n, k, cfg)
    elif split_k is not None and split_k > 1:
        nbytes = int(N.LIB.w8a8_gemm_splitk_workspace_bytes(m, n))
    if nbytes > 0:
        scratch = _splitk_scratch(dev, nbytes)
        N.check(N.LIB.w8a8_gemm_dequant_splitk(
            _vp(q), k, _vp(w), k, _vp(xs), ctypes.byref(ep), _vp(out), _code(out_dtype), n, m, n, k,
            int(split_k or 0), _vp(scratch), scratch.numel(), _cfg_ptr(cfg), stream))
    else:
        N.check(N.LIB.w8a8_gemm_dequant(_vp(q), k, _vp(w), k, _vp(xs), ctypes.byref(ep), _vp(out),
                                        _code(out_dtype), n, m, n, k, _cfg_ptr(cfg), stream))


def int8_linear(x: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
                bias: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                convrot: bool = False, convrot_groupsize: int = 256,
                input_act: Optional[str] = None, input_act_weight: Optional[torch.Tensor] = None,
                input_act_eps: float = 0.0, residual: Optional[torch.Tensor] = None,
                residual_scale: Optional[torch.Tensor] = None, *, dequant: str = "eager",
                scale_mode: str = "eager", output_act: Optional[str] = None, config=None,
                split_k: Optional[int] = None):
    """The registry operator ``int8_linear`` (inference/src/backend_signatures.rs:445-460;
    eager body inference/src/int8_linear.rs:198-277; CUDA route
    inference/src/cuda_linear.rs:419-824).

    ``dequant`` / ``scale_mode`` choose which of the reference routes' numerics
    to reproduce (default: the eager route, bit-exact); ``output_act`` applies
    GELU-tanh in the epilogue (the MLP-up fusion).  ``config`` is an optional
    ``(block_n, group_m, max_ctas, cta_group)`` tile configuration, or
    ``"auto"`` to let the autotuner time the candidates once per shape.
    ``split_k``: None lets few-row shapes (whose tiles leave SMs idle) split K
    across CTAs, 1 turns that off, n > 1 asks for n splits; results are the
    same bit for bit either way.
    """
    _cuda("x", x)
    dev = x.device
    tiled = isinstance(weight, TiledInt8Weight)
    _cuda("weight", weight.tiles if tiled else weight, dev)
    if residual is not None and residual_scale is None:
        raise ValueError("int8_linear: residual requires residual_scale")
    out_dtype = out_dtype or x.dtype
    if input_act not in INPUT_ACT:
        raise ValueError(f"unknown input_act {input_act!r}")
    act = INPUT_ACT[input_act]
    k_act = x.shape[-1] // 2 if act in (2, 4) else x.shape[-1]
    # a2 / a6: the activation (and ConvRot over 256-groups) fuse into the
    # quantiser when K is a multiple of 256 up to 16384 -- the shapes the
    # reference's fused kernel takes (inference/src/cuda_linear.rs:400-417).
    # Other shapes run the activation / rotation as device ATen ops first, as
    # the reference's CUDA route does.
    fused = (k_act % 256 == 0 and 256 <= k_act <= 16384
             and ((convrot and convrot_groupsize == 256) or (not convrot and act != 0))
             and not (act == 3 and not convrot and input_act_eps is None))
    if not fused:
        x = _apply_input(x, input_act, input_act_weight, input_act_eps)
    k = k_act if fused else x.shape[-1]
    if weight.dim() != 2 or weight.dtype != torch.int8:
        raise ValueError("weight must be a 2-D int8 tensor [N, K]")
    if k != weight.shape[-1]:
        raise ValueError(f"Input and weight inner dimensions must match, got {k} and {weight.shape[-1]}")
    n = weight.shape[0]
    ws = weight_scale.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
    if ws.numel() not in (1, n):
        raise ValueError(f"INT8 weight scale must be scalar or per-output-channel, got "
                         f"{tuple(weight_scale.shape)} for weight shape {tuple(weight.shape)}")
    if convrot:
        if convrot_groupsize == 0:
            raise ZeroDivisionError("integer modulo by zero")
        if k % convrot_groupsize:
            raise ValueError(f"ConvRot group size {convrot_groupsize} does not divide input "
                             f"features {k}")
    if convrot and not fused:
        h = _hadamard(convrot_groupsize, dev, x.dtype)
        shape = x.shape
        x = torch.matmul(x.reshape(-1, k // convrot_groupsize, convrot_groupsize), h).reshape(shape)
    lead = x.shape[:-1]
    # [B, S, K] whose samples' rows are each contiguous but not adjacent (a
    # slice of a longer sequence): the plain quantiser reads each sample's
    # rows in place instead of a gathered copy
    per_sample = (not fused and x.dim() == 3 and not x.is_contiguous() and x.stride(-1) == 1
                  and x.stride(1) == x.shape[-1] and x.shape[0] * x.shape[1] > 2
                  and x.shape[-1] > 0)
    x2 = x if per_sample else x.reshape(-1, x.shape[-1])
    if not per_sample and not x2.is_contiguous():
        x2 = x2.contiguous()
    m = x.shape[0] * x.shape[1] if per_sample else x2.shape[0]
    w = weight if weight.is_contiguous() else weight.contiguous()
    if tiled and k == 0:
        raise ValueError("pre-tiled weights need K > 0")
    b = bias.to(device=dev, dtype=out_dtype).reshape(-1).contiguous() if bias is not None else None
    r = rs = None
    rs_rows = 0
    if residual is not None:
        r = residual.to(device=dev, dtype=out_dtype).reshape(m, n).contiguous()
        rs, rs_rows = _residual_scale(residual_scale, tuple(lead), n, out_dtype, dev)
    out = torch.empty((m, n), dtype=out_dtype, device=dev)
    ep = _epilogue(ws, b, r, rs, dequant, output_act, n, n, rs_rows)
    stream = _stream(dev)
    if fused:
        q, xs = quantize_int8_rowwise_convrot(x2, 256 if convrot else 0, input_act, input_act_weight,
                                              input_act_eps, scale_mode=scale_mode)
        xs = xs.reshape(-1)
        if 1 <= m <= 2 and not tiled:
            N.check(N.LIB.w8a8_gemv_dequant(_vp(q), _vp(w), _vp(xs), ctypes.byref(ep), _vp(out),
                                            _code(out_dtype), m, n, k, stream))
        else:
            _gemm_dequant(q, w, xs, ep, out, out_dtype, m, n, k, _config(config), split_k, stream)
    elif 1 <= m <= 2 and k > 0 and m * k <= 32768 and not tiled:
        # a5: the AdaLN-modulation shape -- quantise and GEMV in one launch.
        N.check(N.LIB.w8a8_linear_small(_vp(x2), _code(x2.dtype), _vp(w), ctypes.byref(ep),
                                        SCALE_MODE[scale_mode], None, None, _vp(out),
                                        _code(out_dtype), m, n, k, stream))
    else:
        q = torch.empty((m, k), dtype=torch.int8, device=dev)
        xs = (torch.empty if k > 0 else torch.zeros)((m,), dtype=torch.float32, device=dev)
        if per_sample:
            s_rows = x.shape[1]
            for i in range(x.shape[0]):
                N.check(N.LIB.w8a8_quantize_rowwise(
                    _vp(x[i]), _code(x.dtype), s_rows, k, k, _vp(q[i * s_rows:]), k,
                    _vp(xs[i * s_rows:]), SCALE_MODE[scale_mode], 0, 0, stream))
        elif m > 0 and k > 0:
            N.check(N.LIB.w8a8_quantize_rowwise(_vp(x2), _code(x2.dtype), m, k, k, _vp(q), k,
                                                _vp(xs), SCALE_MODE[scale_mode], 0, 0, stream))
        cfg = _config(config)
        _gemm_dequant(q, w, xs, ep, out, out_dtype, m, n, k, cfg, split_k, stream)
    return out.reshape(*lead, n)


class _HostPipeline:
    """Per-device streams and reusable device buffers of int8_linear_host."""

    def __init__(self, dev):
        self.dev = dev
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.bufs: dict = {}

    def buffer(self, name, shape, dtype):
        t = self.bufs.get(name)
        if t is None or t.dtype != dtype or t.numel() < math.prod(shape):
            t = torch.empty(math.prod(shape), dtype=dtype, device=self.dev)
            self.bufs[name] = t
        return t[: math.prod(shape)].view(shape)


_PIPELINES: dict = {}


def int8_linear_host(x: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
                     bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None, *,
                     out_dtype: Optional[torch.dtype] = None, chunks: int = 4,
                     dequant: str = "eager", scale_mode: str = "eager",
                     output_act: Optional[str] = None) -> torch.Tensor:
    """int8_linear on a host-resident activation with a host-resident result:
    x [M, K] and ``out`` [M, N] in pinned host memory, weight / scales / bias on
    the device.  Rows are processed in ``chunks`` blocks on three streams so the
    upload of block i+1, the quantise + GEMM of block i and the download of
    block i-1 overlap (the transfers, not the kernels, bound this call).
    Results equal int8_linear's (plain linear: bias, dequant order, output
    activation) row for row; returns ``out``.  The call returns after the last
    download has completed."""
    if x.is_cuda:
        raise ValueError("int8_linear_host takes a host x; use int8_linear for device tensors")
    dev = weight.device
    _cuda("weight", weight)
    if x.dim() != 2:
        raise ValueError("x must be [M, K]")
    m, k = x.shape
    n = weight.shape[0]
    out_dtype = out_dtype or x.dtype
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, pin_memory=True)
    if out.shape != (m, n) or out.dtype != out_dtype or out.is_cuda:
        raise ValueError("out must be a host [M, N] tensor of the output dtype")
    if weight.dim() != 2 or weight.dtype != torch.int8 or weight.shape[1] != k:
        raise ValueError(f"weight must be an int8 [N, {k}] tensor")
    pipe = _PIPELINES.get(dev.index)
    if pipe is None:
        pipe = _PIPELINES[dev.index] = _HostPipeline(dev)
    compute = torch.cuda.current_stream(dev)
    stream = _stream(dev)
    rows = max(1, -(-m // max(1, chunks)))
    xd = pipe.buffer("x", (2, rows, k), x.dtype)
    yd = pipe.buffer("y", (2, rows, n), out_dtype)
    qd = pipe.buffer("q", (2, rows, k), torch.int8)
    sd = pipe.buffer("s", (2, rows), torch.float32)
    w = weight if weight.is_contiguous() else weight.contiguous()
    ws = weight_scale.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
    if ws.numel() not in (1, n):
        raise ValueError("INT8 weight scale must be scalar or per-output-channel")
    b = bias.to(device=dev, dtype=out_dtype).reshape(-1).contiguous() if bias is not None else None
    ep = _epilogue(ws, b, None, None, dequant, output_act, n, n)
    up_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    down_done = [torch.cuda.Event() for _ in range(2)]
    for i, r0 in enumerate(range(0, m, rows)):
        r1 = min(m, r0 + rows)
        slot = i % 2
        xs, ys = xd[slot, : r1 - r0], yd[slot, : r1 - r0]
        with torch.cuda.stream(pipe.h2d):
            if i >= 2:
                pipe.h2d.wait_event(comp_done[slot])  # slot's previous x consumed
            xs.copy_(x[r0:r1], non_blocking=True)
            up_done[slot].record(pipe.h2d)
        compute.wait_event(up_done[slot])
        if i >= 2:
            compute.wait_event(down_done[slot])  # slot's previous y downloaded
        r = r1 - r0
        qs, ss = qd[slot, :r], sd[slot, :r]
        N.check(N.LIB.w8a8_quantize_rowwise(_vp(xs), _code(x.dtype), r, k, k, _vp(qs), k, _vp(ss),
                                            SCALE_MODE[scale_mode], 0, 0, stream))
        N.check(N.LIB.w8a8_gemm_dequant(_vp(qs), k, _vp(w), k, _vp(ss), ctypes.byref(ep), _vp(ys),
                                        _code(out_dtype), n, r, n, k, None, stream))
        comp_done[slot].record(compute)
        with torch.cuda.stream(pipe.d2h):
            pipe.d2h.wait_event(comp_done[slot])
            out[r0:r1].copy_(ys, non_blocking=True)
            down_done[slot].record(pipe.d2h)
    # work queued on the caller's stream afterwards (and events recorded on
    # it) comes after the last download
    for ev in down_done:
        compute.wait_event(ev)
    pipe.d2h.synchronize()
    return out


def int8_gemm_s32(q: torch.Tensor, w: torch.Tensor, config=None) -> torch.Tensor:
    """``cublas_gemm_int8`` replacement: exact int32 q[M,K] . w[N,K]^T."""
    _cuda("q", q)
    _cuda("w", w, q.device)
    m, k = q.shape
    n = w.shape[0]
    acc = torch.empty((m, n), dtype=torch.int32, device=q.device)
    cfg = _config(config)
    N.check(N.LIB.w8a8_gemm_s32(_vp(q.contiguous()), _vp(w.contiguous()), _vp(acc), m, n, k,
                                _cfg_ptr(cfg), _stream(q.device)))
    return acc


def dequantize_int8_linear(acc, x_scale, weight_scale, bias=None, out_dtype=torch.bfloat16, *,
                           dequant="chained", residual=None, residual_scale=None, lead=None):
    """``dequantize_int8_linear`` replacement (native/comfy-port/kitchen/int8_linear.cu:517-583).

    ``residual`` / ``residual_scale`` add the residual epilogue of
    ``int8_linear`` (``residual + y * residual_scale``, broadcast as there
    against an output of shape ``(*lead, N)``; ``lead`` defaults to (M,)).
    Returns [M, N], or ``(*lead, N)`` when ``lead`` is given."""
    _cuda("acc", acc)
    dev = acc.device
    m, n = acc.shape
    if residual is not None and residual_scale is None:
        raise ValueError("dequantize_int8_linear: residual requires residual_scale")
    lead = tuple(lead) if lead is not None else None
    if lead is not None and math.prod(lead) != m:
        raise ValueError(f"lead {lead} does not hold the {m} accumulator rows")
    ws = weight_scale.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
    xs = x_scale.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
    b = bias.to(device=dev, dtype=out_dtype).reshape(-1).contiguous() if bias is not None else None
    r = rs = None
    rs_rows = 0
    if residual is not None:
        r = residual.to(device=dev, dtype=out_dtype).reshape(m, n).contiguous()
        rs, rs_rows = _residual_scale(residual_scale, lead or (m,), n, out_dtype, dev)
    out = torch.empty((m, n), dtype=out_dtype, device=dev)
    ep = _epilogue(ws, b, r, rs, dequant, None, n, n, rs_rows)
    N.check(N.LIB.w8a8_dequantize_linear(_vp(acc.contiguous()), _vp(xs), ctypes.byref(ep), _vp(out),
                                         _code(out_dtype), m, n, _stream(dev)))
    return out.reshape(*lead, n) if lead is not None else out


def int8_gemv(q, w, x_scale, weight_scale, bias=None, out_dtype=torch.bfloat16, residual=None,
              residual_scale=None, *, dequant="chained"):
    """``int8_gemv_dequant`` replacement (M in {1, 2};
    native/comfy-port/kitchen/int8_linear.cu:585-708)."""
    _cuda("q", q)
    dev = q.device
    m, k = q.shape
    n = w.shape[0]
    ws = weight_scale.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
    xs = x_scale.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
    b = bias.to(device=dev, dtype=out_dtype).reshape(-1).contiguous() if bias is not None else None
    r = residual.to(device=dev, dtype=out_dtype).reshape(m, n).contiguous() if residual is not None else None
    rs, rs_rows = (_residual_scale(residual_scale, (m,), n, out_dtype, dev) if residual is not None
                   else (None, 0))
    out = torch.empty((m, n), dtype=out_dtype, device=dev)
    ep = _epilogue(ws, b, r, rs, dequant, None, n, n, rs_rows)
    N.check(N.LIB.w8a8_gemv_dequant(_vp(q.contiguous()), _vp(w.contiguous()), _vp(xs),
                                    ctypes.byref(ep), _vp(out), _code(out_dtype), m, n, k,
                                    _stream(dev)))
    return out


# --------------------------------------------------------------------------
# a9: FP8 e4m3 per-tensor
# --------------------------------------------------------------------------
def quantize_per_tensor_fp8(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """Kitchen ``quantize_per_tensor_fp8(x, scale)`` with the eager numerics
    (inference/src/eager.rs:74-88).  Returns float8_e4m3fn of x's shape."""
    _cuda("x", x)
    s = scale.to(device=x.device, dtype=torch.float32).reshape(-1)[:1].contiguous()
    xc = x.contiguous()
    out = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    N.check(N.LIB.w8a8_quantize_fp8_tensor(_vp(xc), _code(xc.dtype), xc.numel(), _vp(s),
                                           _vp(out), _stream(x.device)))
    return out


def fp8_linear(a: torch.Tensor, scale_a: torch.Tensor, w: torch.Tensor, scale_w: torch.Tensor,
               bias: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.bfloat16,
               config=None) -> torch.Tensor:
    """Per-tensor FP8 linear: (a . w^T) * (scale_a * scale_w) + bias on tcgen05
    kind::f8f6f4 (replaces ``_scaled_mm`` TensorWise, inference/src/fp8_ops.rs:81-121)."""
    _cuda("a", a)
    dev = a.device
    _cuda("w", w, dev)
    if a.dtype != torch.float8_e4m3fn or w.dtype != torch.float8_e4m3fn:
        raise ValueError("fp8_linear expects float8_e4m3fn operands")
    lead = a.shape[:-1]
    a2 = a.reshape(-1, a.shape[-1]).contiguous()
    m, k = a2.shape
    n = w.shape[0]
    sa = scale_a.to(device=dev, dtype=torch.float32).reshape(-1)[:1].contiguous()
    sw = scale_w.to(device=dev, dtype=torch.float32).reshape(-1)[:1].contiguous()
    b = bias.to(device=dev, dtype=out_dtype).reshape(-1).contiguous() if bias is not None else None
    out = torch.empty((m, n), dtype=out_dtype, device=dev)
    cfg = _config(config)
    N.check(N.LIB.w8a8_fp8_gemm(_vp(a2), _vp(w.contiguous()), _vp(sa), _vp(sw), _vp(b), _vp(out),
                                _code(out_dtype), m, n, k, _cfg_ptr(cfg), _stream(dev)))
    return out.reshape(*lead, n)


# --------------------------------------------------------------------------
# a10: MXFP8
# --------------------------------------------------------------------------
def quantize_mxfp8(x: torch.Tensor):
    """Kitchen ``quantize_mxfp8(x, pad_32x=False)`` (inference/src/eager.rs:176-225):
    returns ``(payload float8_e4m3fn [M, K], scales uint8 [ceil(M/128)*128,
    ceil(K/128)*4])``, the scales in the cuBLAS blocked layout."""
    _cuda("x", x)
    if x.dim() != 2:
        raise ValueError("Input must be 2D")
    m, k = x.shape
    if k % 32:
        raise ValueError("K dimension must be divisible by 32")
    xc = x.contiguous()
    q = torch.empty((m, k), dtype=torch.float8_e4m3fn, device=x.device)
    sf = torch.empty(((m + 127) // 128 * 128, (k // 32 + 3) // 4 * 4), dtype=torch.uint8,
                     device=x.device)
    N.check(N.LIB.w8a8_quantize_mxfp8(_vp(xc), _code(xc.dtype), m, k, k, _vp(q), k, _vp(sf),
                                      _stream(x.device)))
    return q, sf


def mxfp8_linear(a: torch.Tensor, a_scales: torch.Tensor, w: torch.Tensor, w_scales: torch.Tensor,
                 bias: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.bfloat16,
                 config=None) -> torch.Tensor:
    """``scaled_mm_mxfp8`` (inference/src/backend_quant.rs:320-343) on tcgen05
    kind::mxf8f6f4.block_scale: a [M, K] and w [N, K] e4m3 with blocked e8m0
    scales from ``quantize_mxfp8``."""
    _cuda("a", a)
    dev = a.device
    _cuda("w", w, dev)
    m, k = a.shape
    n = w.shape[0]
    b = bias.to(device=dev, dtype=out_dtype).reshape(-1).contiguous() if bias is not None else None
    out = torch.empty((m, n), dtype=out_dtype, device=dev)
    cfg = _config(config)
    N.check(N.LIB.w8a8_mxfp8_gemm(_vp(a.contiguous()), _vp(a_scales.contiguous()),
                                  _vp(w.contiguous()), _vp(w_scales.contiguous()), _vp(b), _vp(out),
                                  _code(out_dtype), m, n, k, _cfg_ptr(cfg), _stream(dev)))
    return out


def device_error(device=None) -> int:
    """Read-and-clear the device-side error word (nonzero: a bounded wait in a
    tcgen05 kernel gave up)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    err = N.LIB.w8a8_device_error(_stream(dev))
    if err:
        # a kernel that gave up may have left split-K partial sums behind
        for (index, _), buf in _SPLITK_SCRATCH.items():
            if index == dev.index:
                buf.zero_()
    return err
