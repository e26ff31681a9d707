"""CPU oracle for the W8A8 linear family -- TEST INFRASTRUCTURE ONLY.

This module restates, operation for operation, the reference's eager (LibTorch)
implementation of the INT8 / FP8 / MXFP8 linear path so that the CUDA kernels in
``imagine_b200`` can be checked against it.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of ``bench.py`` may
import it; the product path never does (it raises if its CUDA library is
missing).

Parity is pinned two ways (see ``tests/test_oracle_golden.py``):
  * against vectors produced by the reference's own Python implementation
    (Kitchen 0.2.37 ``backends/eager/quantization.py``, shipped inside the
    reference's source archive), committed under ``tests/golden/``;
  * against the reference's recorded probe fixture
    (``inference/fixtures/stage-1`` member ``int8-aot/probe.json``): 36 cases of
    quantised codes, row scales and dequantised outputs of its Triton route.

Every function names the reference file:line it follows.  Paths are relative to
the reference repository root; ``KSRC`` is the Kitchen source tree inside
``design/reference-local/native-source-candidates.tar.gz``.
"""
from __future__ import annotations

import math

import numpy as np
import torch

F8_E4M3_MAX = 448.0
E8M0_BIAS = 127
MX_BLOCK = 32

# Output dtype codes used by the reference's CUDA route: 0 f32, 1 f16, 2 bf16
# (inference/src/cuda_linear.rs:488-497).
DTYPE_CODES = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}
CODE_OF = {v: k for k, v in DTYPE_CODES.items()}


# --------------------------------------------------------------------------
# a1 / a12: per-row (per-token, per-output-channel) INT8 quantisation
# --------------------------------------------------------------------------
def _scale_for_math(scale: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """inference/src/eager.rs:94-109 (KSRC eager/quantization.py:816-819):
    cast the fp32 scale to x's dtype, replace exact zeros by finfo.tiny."""
    s = scale.to(x.dtype)
    tiny = torch.finfo(x.dtype).tiny
    return torch.where(s == 0, torch.full_like(s, tiny), s)


def _round_int8(scaled: torch.Tensor) -> torch.Tensor:
    """inference/src/eager.rs:110-121: round half to even in x's dtype, clamp
    to [-128, 127], cast to int8 (the deterministic, seed<=0 branch)."""
    return scaled.round().clamp(-128.0, 127.0).to(torch.int8)


def quantize_int8_rowwise(x: torch.Tensor):
    """inference/src/eager.rs:159-171.

    scale = max(amax_k |x| (as fp32) / 127, 1e-30)   -- IEEE fp32 divide
    q     = clamp(rne(x / dtype(scale)), -128, 127)  -- divide done in x.dtype
    Returns (q int8 [..., K], scale fp32 [..., 1]).
    """
    amax = x.abs().amax(dim=-1, keepdim=True)
    scale = (amax.to(torch.float32) / 127.0).clamp(min=1e-30)
    q = _round_int8(x / _scale_for_math(scale, x))
    return q, scale


def quantize_int8_rowwise_given_absmax(x: torch.Tensor, amax: torch.Tensor):
    """The eager row quantiser (inference/src/eager.rs:159-171) with the row
    absmax supplied instead of computed: what a K-shard of a row must use so
    that its codes equal those of the unsharded row."""
    scale = (amax.reshape(*x.shape[:-1], 1).to(torch.float32) / 127.0).clamp(min=1e-30)
    q = _round_int8(x / _scale_for_math(scale, x))
    return q, scale


def quantize_int8_rowwise_kitchen(x: torch.Tensor):
    """native/comfy-port/kitchen/int8_linear.cu:184-227 (deterministic branch).

    The reference's CUDA quantiser differs from the eager one in the scale:
    scale = max(min(amax, finite_max(T)) * (1/127), 1e-30) (a multiply by the
    fp32 reciprocal, :206-208).  The element step is the same
    (``quant_div_to_float``, :47-51): T(float(x) / float(T(scale))), then
    nearbyint and clamp to [-128, 127].  The divide is the IEEE one.
    """
    finite = {torch.float32: 3.4028234663852886e38, torch.float16: 65504.0,
              torch.bfloat16: 3.3895313892515355e38}[x.dtype]
    amax = x.abs().amax(dim=-1, keepdim=True).to(torch.float32)
    inv127 = torch.tensor(1.0 / 127.0, dtype=torch.float32)
    scale = torch.clamp(torch.minimum(amax, torch.tensor(finite, dtype=torch.float32)) * inv127,
                        min=1e-30)
    scale_t = scale.to(x.dtype).to(torch.float32)
    scaled = (x.to(torch.float32) / scale_t).to(x.dtype).to(torch.float32)
    q = torch.clamp(torch.round(scaled), -128.0, 127.0).to(torch.int8)
    return q, scale


def quantize_int8_tensorwise(x: torch.Tensor):
    """inference/src/eager.rs:135-150 with scale=None: one scale for the whole
    tensor, amax/127 in fp32, then the same element step as the row-wise form."""
    scale = (x.abs().max().to(torch.float32) / 127.0).clamp(min=1e-30)
    q = _round_int8(x / _scale_for_math(scale, x))
    return q, scale


def dequantize_int8(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """inference/src/eager.rs:172-174: float(q) * scale."""
    return q.to(torch.float32) * scale


# --------------------------------------------------------------------------
# a2 / a6: input activations and ConvRot rotation
# --------------------------------------------------------------------------
def apply_input(x: torch.Tensor, act: str | None, weight=None, eps=None) -> torch.Tensor:
    """inference/src/int8_linear.rs:37-97 (KSRC backends/_activations.py:44-68)."""
    if act is None or act == "none":
        return x
    if act == "gelu_tanh":
        return torch.nn.functional.gelu(x, approximate="tanh")
    if act == "swiglu":
        gate, up = x.chunk(2, dim=-1)
        return torch.nn.functional.silu(gate).mul_(up)
    if act == "situ":
        # inference/src/int8_linear.rs:54-74: 25 tanh(a/25) * (4 tanh(b/4) * sigmoid(b))
        a, b = x.chunk(2, dim=-1)
        gated = torch.tanh(b / 4.0).mul_(4.0).mul_(torch.sigmoid(b))
        return torch.tanh(a / 25.0).mul_(25.0).mul_(gated)
    if act == "rms_norm":
        if weight is None:
            raise ValueError("input_act 'rms_norm' requires act_weight")
        return torch.nn.functional.rms_norm(x, (x.shape[-1],), weight.to(x.dtype), eps)
    raise ValueError(f"unknown input_act {act!r}")


def hadamard(size: int, dtype=torch.float32) -> torch.Tensor:
    """inference/src/int8_utils.rs:21-58: regular Hadamard built as a
    Kronecker power of H4, normalised by sqrt(size), in the requested dtype."""
    if size < 4 or (size & (size - 1)) or abs(math.log(size, 4) % 1) > 1e-12:
        raise ValueError(f"Regular Hadamard size must be a power of 4, got {size}")
    h4 = torch.tensor([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]],
                      dtype=torch.int64).to(dtype)
    h = h4
    while h.shape[0] < size:
        h = torch.kron(h, h4)
    return h / math.sqrt(size)


def rotate_activation(x: torch.Tensor, h: torch.Tensor, group: int) -> torch.Tensor:
    """inference/src/int8_utils.rs:97-110: grouped x @ H in x's dtype."""
    shape = x.shape
    if shape[-1] % group:
        raise ValueError(f"features {shape[-1]} not divisible by group_size {group}")
    g = x.reshape(-1, shape[-1] // group, group)
    return torch.matmul(g, h.to(x.dtype)).reshape(shape)


# --------------------------------------------------------------------------
# a3: INT8 accumulation and the three dequant orders found in the reference
# --------------------------------------------------------------------------
def int8_accumulate(a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """inference/src/int8_linear.rs:134-168: exact int32 sum_k a[m,k]*w[n,k].

    The reference pads K and N to multiples of 8 and calls ``_int_mm``; zero
    padding does not change an integer sum, so the result is the exact product
    (|sum| < 2^31 for K < 2^17).  Like the reference, no copy is made when K
    and N are already aligned: ``_int_mm`` then reads the transposed view of W.
    """
    m, k = a.shape
    n = w.shape[0]
    if m == 0 or n == 0 or k == 0:
        return torch.zeros((m, n), dtype=torch.int32)
    if k % 8 == 0 and n % 8 == 0 and m > 16:
        return torch._int_mm(a.contiguous(), w.t())
    pk = (k + 7) // 8 * 8
    pn = (n + 7) // 8 * 8
    a_p = torch.zeros((max(m, 17), pk), dtype=torch.int8)
    a_p[:m, :k] = a
    b_p = torch.zeros((pk, pn), dtype=torch.int8)
    b_p[:k, :n] = w.t()
    return torch._int_mm(a_p, b_p)[:m, :n].contiguous()


def dequant_eager(acc, xs, ws, bias, out_dtype):
    """inference/src/int8_linear.rs:244-268: y = out(float(acc) * (xs * ws)),
    then ``y + bias`` computed in the output dtype (a second rounding)."""
    scale = xs.reshape(-1, 1).to(torch.float32) * ws.reshape(1, -1).to(torch.float32)
    y = (acc.to(torch.float32) * scale).to(out_dtype)
    if bias is not None:
        y = y + bias.to(out_dtype).reshape(1, -1)
    return y


def dequant_scale_product(acc, xs, ws, bias, out_dtype):
    """KSRC backends/triton/quantization.py:861-1018 (the reference's Triton
    route): c = fma(float(acc), xs * ws, float(bias)), rounded once to the
    output dtype.  The single-rounding FMA is what the compiled kernel does
    (the recorded probe outputs of inference/fixtures/stage-1 int8-aot/probe.json
    only match with it); evaluated here in float64, which holds the
    24-bit x 24-bit product exactly."""
    scale = xs.reshape(-1, 1).to(torch.float32) * ws.reshape(1, -1).to(torch.float32)
    y = acc.to(torch.float32).double() * scale.double()
    if bias is not None:
        y = y + bias.to(torch.float32).double().reshape(1, -1)
    return y.to(torch.float32).to(out_dtype)


def dequant_chained(acc, xs, ws, bias, out_dtype):
    """native/comfy-port/kitchen/int8_linear.cu:517-545 and the CUTLASS EVT of
    KSRC backends/cuda/ops/cutlass_gemm_int8.cu:66-120 (the reference's CUDA
    route): fma(float(acc) * xs, ws, float(bias)), rounded once (nvcc contracts
    the last multiply-add).  No recorded output pins this order; tests hold it
    to the output tolerance."""
    y = acc.to(torch.float32) * xs.reshape(-1, 1).to(torch.float32)
    y = y.double() * ws.reshape(1, -1).to(torch.float32).double()
    if bias is not None:
        y = y + bias.to(torch.float32).double().reshape(1, -1)
    return y.to(torch.float32).to(out_dtype)


DEQUANT = {"eager": dequant_eager, "scale_product": dequant_scale_product,
           "chained": dequant_chained}


def apply_residual(out, residual, scale):
    """inference/src/int8_linear.rs:99-112: residual.addcmul(out, scale) in
    the output dtype."""
    if residual is None:
        return out
    if scale is None:
        raise ValueError("residual requires residual_scale")
    return residual.to(out.dtype).addcmul(out, scale.to(out.dtype))


def gelu_tanh(y: torch.Tensor) -> torch.Tensor:
    """GELU-tanh applied to a bf16/f16/f32 tensor in its own dtype (the
    activation the reference folds into the down projection's input,
    inference/src/int8_linear.rs:40, and BASELINE places in MLP-up's epilogue)."""
    return torch.nn.functional.gelu(y, approximate="tanh")


def int8_linear(x, weight, weight_scale, bias=None, out_dtype=torch.bfloat16,
                convrot=False, convrot_groupsize=256, input_act=None,
                input_act_weight=None, input_act_eps=None, residual=None,
                residual_scale=None, dequant="eager", output_act=None):
    """inference/src/int8_linear.rs:198-277 (KSRC eager/quantization.py:985-1087).

    ``dequant`` selects which of the reference's three dequant orders to
    restate (default: the eager one); ``output_act='gelu_tanh'`` applies GELU
    to the linear's output before the residual (the MLP-up epilogue).
    """
    x = apply_input(x, input_act, input_act_weight, input_act_eps)
    if x.shape[-1] != weight.shape[-1]:
        raise ValueError(f"Input and weight inner dimensions must match, got "
                         f"{x.shape[-1]} and {weight.shape[-1]}")
    ws = weight_scale.to(torch.float32).reshape(-1)
    if ws.numel() not in (1, weight.shape[0]):
        raise ValueError("INT8 weight scale must be scalar or per-output-channel")
    if convrot:
        if x.shape[-1] % convrot_groupsize:
            raise ValueError(f"ConvRot group size {convrot_groupsize} does not divide "
                             f"input features {x.shape[-1]}")
        x = rotate_activation(x, hadamard(convrot_groupsize, x.dtype), convrot_groupsize)
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    q, xs = quantize_int8_rowwise(x2)
    acc = int8_accumulate(q, weight)
    y = DEQUANT[dequant](acc, xs, ws, bias, out_dtype)
    if output_act == "gelu_tanh":
        y = gelu_tanh(y)
    y = y.reshape(*shape[:-1], weight.shape[0])
    return apply_residual(y, residual, residual_scale)


# --------------------------------------------------------------------------
# a7: modulation before the linear
# --------------------------------------------------------------------------
def adaln(x, scale, shift, eps=1e-6, rms=False):
    """inference/src/backend_eager.rs:176-197 (KSRC backends/eager/adaln.py:11-20):
    norm(x) * (1 + scale) + shift, every op in x's dtype."""
    k = x.shape[-1]
    if rms:
        nrm = torch.nn.functional.rms_norm(x, (k,), None, eps)
    else:
        nrm = torch.nn.functional.layer_norm(x, (k,), None, None, eps)
    return nrm * (scale.to(x.dtype) + 1) + shift.to(x.dtype)


def int8_linear_modulated(x, modulation_scale, weight, weight_scale, bias=None,
                          out_dtype=torch.bfloat16, convrot=False, convrot_groupsize=256):
    """inference/src/backend_bindings.rs:329-405: int8_linear(x * (1 + s))."""
    k = x.shape[-1]
    if modulation_scale.numel() != k:
        raise ValueError(f"modulation_scale must contain one batch-one row of {k} values, got "
                         f"{modulation_scale.numel()}")
    xm = x * (modulation_scale.to(x.dtype).reshape(-1) + 1)
    return int8_linear(xm, weight, weight_scale, bias, out_dtype, convrot, convrot_groupsize)


def int8_linear_rms_modulated(x, norm_weight, norm_eps, modulation_scale, weight, weight_scale,
                              bias=None, out_dtype=torch.bfloat16, convrot=False,
                              convrot_groupsize=256):
    """inference/src/backend_bindings.rs:352-361: the modulated linear of
    rms_norm(x, norm_weight, norm_eps)."""
    k = x.shape[-1]
    nrm = torch.nn.functional.rms_norm(x, (k,), norm_weight.to(x.dtype), float(norm_eps or 0.0))
    return int8_linear_modulated(nrm, modulation_scale, weight, weight_scale, bias, out_dtype,
                                 convrot, convrot_groupsize)


# --------------------------------------------------------------------------
# a8: Q/K RMSNorm + interleaved RoPE
# --------------------------------------------------------------------------
def rope_interleaved(x: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """inference/src/backend_rope.rs:156-166 (eager_apply, non-split): pairs
    (x[2i], x[2i+1]) rotated by freqs [.., D/2, 2, 2] in the freqs' dtype,
    out_r = f[r][0] x0 + f[r][1] x1, cast back to x's dtype."""
    shape = x.shape
    inp = x.to(freqs.dtype).reshape(*shape[:-1], -1, 1, 2)
    out = freqs[..., 0] * inp[..., 0]
    out.addcmul_(freqs[..., 1], inp[..., 1])
    return out.reshape(shape).to(x.dtype)


def rms_rope(q, k, freqs, q_scale, k_scale, eps):
    """inference/src/backend_rope.rs:203-223 (eager_rms with rot = D):
    rms_norm(x, scale, eps) then the interleaved rotation, for q and k.
    freqs: [S, D/2, 2, 2] broadcast over the leading dimensions of x [.., S, H, D]."""
    d = q.shape[-1]
    f = freqs.reshape(-1, 1, d // 2, 2, 2)  # [S, 1 (heads), D/2, 2, 2]

    def one(x, s):
        nrm = torch.nn.functional.rms_norm(x, (d,), s.to(x.dtype), eps)
        return rope_interleaved(nrm, f)
    return one(q, q_scale), (one(k, k_scale) if k is not None else None)


def quantize_weight(w: torch.Tensor):
    """a12, inference/src/layout_complete.rs:119-159: offline per-output-channel
    weight quantisation = the row-wise quantiser applied to W [N, K]."""
    q, s = quantize_int8_rowwise(w)
    return q, s.reshape(-1)


# --------------------------------------------------------------------------
# a5: M <= 2 GEMV (reference CUDA route) -- integer dot then chained dequant
# --------------------------------------------------------------------------
def int8_gemv(q, w, xs, ws, bias, out_dtype, residual=None, residual_scale=None):
    """native/comfy-port/kitchen/int8_linear.cu:585-708: y[m,n] =
    T(float(sum_k q[m,k] w[n,k]) * xs[m] * ws[n] + b[n]); residual (M=1 only,
    cuda_linear.rs:650-655) is ``addcmul`` in the output dtype."""
    acc = int8_accumulate(q, w)
    y = dequant_chained(acc, xs.reshape(-1), ws.reshape(-1), bias, out_dtype)
    return apply_residual(y, residual, residual_scale)


# --------------------------------------------------------------------------
# a9: FP8 e4m3 per-tensor
# --------------------------------------------------------------------------
def quantize_fp8(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """inference/src/eager.rs:74-88 (KSRC eager/quantization.py:45-58):
    t = x * dtype(1/scale); clamp to +-448 in x.dtype; cast to e4m3fn."""
    recip = (1.0 / scale.to(torch.float32)).to(x.dtype)
    t = x * recip
    t = torch.clamp(t, -F8_E4M3_MAX, F8_E4M3_MAX)
    return t.to(torch.float8_e4m3fn)


def dequantize_fp8(q: torch.Tensor, scale: torch.Tensor, out_dtype=torch.bfloat16):
    """inference/src/eager.rs:89-92: q.to(dtype) * scale.to(dtype)."""
    return q.to(out_dtype) * scale.to(out_dtype)


def fp8_linear(a_q, sa, w_q, sw, bias=None, out_dtype=torch.bfloat16):
    """inference/src/fp8_ops.rs:123-130: the reference's fallback path
    (dequantise both operands to the original dtype, then F.linear).  The fast
    path is cuBLASLt ``_scaled_mm`` with no recorded outputs, so FP8 GEMM parity
    is tolerance-based against this."""
    a = dequantize_fp8(a_q, sa, out_dtype).to(torch.float32)
    w = dequantize_fp8(w_q, sw, out_dtype).to(torch.float32)
    y = a @ w.t()
    if bias is not None:
        y = y + bias.to(torch.float32)
    return y.to(out_dtype)


def fp8_linear_exact(a_q, sa, w_q, sw, bias=None, out_dtype=torch.bfloat16):
    """fp32-accumulated reference of what ``_scaled_mm`` TensorWise computes
    (inference/native/bridge.cpp:401-413): (A_fp8 @ B_fp8^T) * sa * sb + bias."""
    y = (a_q.to(torch.float32) @ w_q.to(torch.float32).t()) * (sa.to(torch.float32) *
                                                                 sw.to(torch.float32))
    if bias is not None:
        y = y + bias.to(torch.float32)
    return y.to(out_dtype)


# --------------------------------------------------------------------------
# a10: MXFP8 (32-element K blocks, e8m0 scales, cuBLAS blocked layout)
# --------------------------------------------------------------------------
def to_blocked(scales: torch.Tensor) -> torch.Tensor:
    """inference/src/block_scales.rs:4-31: pad [rows, cols] to multiples of
    (128, 4) and tile into 128x4 blocks, byte (r, c) of a block at
    (r % 32) * 16 + (r // 32) * 4 + c; blocks in (row_block, col_block) order."""
    rows, cols = scales.shape
    rb, cb = (rows + 127) // 128, (cols + 3) // 4
    padded = torch.zeros((rb * 128, cb * 4), dtype=scales.dtype)
    padded[:rows, :cols] = scales
    t = padded.view(rb, 128, cb, 4).permute(0, 2, 1, 3).reshape(-1, 4, 32, 4)
    return t.transpose(1, 2).reshape(rb * 128, cb * 4)


def from_blocked(blocked: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """inference/src/block_scales.rs:33-47: inverse of ``to_blocked``."""
    rb, cb = (rows + 127) // 128, (cols + 3) // 4
    t = blocked.reshape(-1, 32, 4, 4).transpose(1, 2).reshape(rb, cb, 128, 4)
    return t.permute(0, 2, 1, 3).reshape(rb * 128, cb * 4)[:rows, :cols]


def e8m0_to_f32(e: torch.Tensor) -> torch.Tensor:
    """inference/src/block_scales.rs:49-58: bits e<<23 as fp32, 0 -> 0.0."""
    b = e.to(torch.int32)
    r = torch.bitwise_left_shift(b, 23)
    return torch.where(b == 0, torch.zeros_like(r), r).view(torch.float32)


def quantize_mxfp8(x: torch.Tensor):
    """inference/src/eager.rs:176-225 (KSRC eager/quantization.py:261-328).

    Per 32-element K block: s = max(amax/448, 2^-127) (fp32 IEEE divide);
    e = clamp(ceil(log2 s) + 127, 0, 254); zero blocks get e = 0 and a zero
    payload; payload = e4m3(clamp(x / 2^(e-127), +-448)).  Scales are returned
    in the blocked layout [ceil(M/128)*128, ceil(K/32/4)*4] as uint8.
    """
    rows, cols = x.shape
    if cols % MX_BLOCK:
        raise ValueError("K dimension must be divisible by 32")
    xb = x.reshape(rows, cols // MX_BLOCK, MX_BLOCK)
    amax = xb.abs().amax(dim=-1)
    need = (amax.to(torch.float32) / F8_E4M3_MAX).clamp(min=2.0 ** -127)
    e = (torch.ceil(torch.log2(need)).to(torch.int32) + E8M0_BIAS).clamp(0, 254)
    e_u8 = e.to(torch.uint8)
    sf = e8m0_to_f32(e_u8)
    zero = amax == 0
    sf = torch.where(zero, torch.ones_like(sf), sf)
    scaled = xb.to(torch.float32) / sf.unsqueeze(-1)
    scaled = torch.where(zero.unsqueeze(-1), torch.zeros_like(scaled), scaled)
    payload = scaled.clamp(-F8_E4M3_MAX, F8_E4M3_MAX).reshape(rows, cols).to(torch.float8_e4m3fn)
    e_u8 = torch.where(zero, torch.zeros_like(e_u8), e_u8)
    return payload, to_blocked(e_u8)


def dequantize_mxfp8(payload, blocked, out_dtype=torch.bfloat16):
    """inference/src/eager.rs:227-242."""
    rows, cols = payload.shape
    e = from_blocked(blocked.view(torch.uint8), rows, cols // MX_BLOCK)
    sf = e8m0_to_f32(e)
    y = payload.to(torch.float32).reshape(rows, cols // MX_BLOCK, MX_BLOCK) * sf.unsqueeze(-1)
    return y.reshape(rows, cols).to(out_dtype)


def mxfp8_linear(a_q, a_sf, w_q, w_sf, bias=None, out_dtype=torch.bfloat16):
    """What ``scaled_mm_mxfp8`` (inference/src/backend_quant.rs:320-343)
    computes: sum over K blocks of (a.b) * 2^(ea-127) * 2^(eb-127), in fp32,
    + bias, cast once.  Evaluated by dequantising both operands to fp32 (exact:
    e4m3 x power-of-two fits fp32) and one fp32 matmul."""
    a = dequantize_mxfp8(a_q, a_sf, torch.float32)
    w = dequantize_mxfp8(w_q, w_sf, torch.float32)
    y = a.double() @ w.double().t()
    if bias is not None:
        y = y + bias.to(torch.float64)
    return y.to(torch.float32).to(out_dtype)


# --------------------------------------------------------------------------
# helpers shared by tests and the bench's CPU baseline
# --------------------------------------------------------------------------
def as_bytes(t: torch.Tensor) -> np.ndarray:
    """Raw little-endian bytes of a CPU tensor (for byte-exact comparisons)."""
    t = t.contiguous()
    if t.dtype in (torch.bfloat16, torch.float8_e4m3fn):
        t = t.view(torch.uint8 if t.element_size() == 1 else torch.int16)
    return t.numpy().view(np.uint8).reshape(-1)
