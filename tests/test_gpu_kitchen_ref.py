"""This library's kernels against the reference's own Kitchen CUDA kernels on the
same inputs, on the GPU.

`oracle/_ref/libkitchen_int8_linear.so` is the reference file
native/comfy-port/kitchen/int8_linear.cu compiled in place for sm_100a by
`make -C oracle ref REF=<reference checkout>` (run by `__graft_entry__.build()`
where the checkout is present; the library then travels with the tree).  Its
`extern "C"` launchers (int8_linear.cu:1320-2162) are the kernels the
reference's CUDA route calls through its bridge: the row quantiser with
Kitchen scales (`amax * (1/127)`) and PCG stochastic rounding, the fused input
activation + ConvRot quantiser (`quantize_int8_rowwise_convrot64`), the one-
and two-row GEMV with dequant and the stand-alone dequant.  The library is
built with that file's own flags (--use_fast_math among them), so this pins
the W8A8_SCALE_KITCHEN_CUDA numerics (approximate divide, zero f16 divisor
kept, fast-math activations, the fused kernel's summation order for RMSNorm)
and the dequant order each Kitchen kernel uses (SEPARATE, CHAINED,
SCALE_PRODUCT) -- the forms the bridge library selects -- to the reference's
code itself rather than to a restatement of it.

Bars: every code, scale and output bit bit-exact, in all three input and
output dtypes.  The tests skip when the reference library was not built."""
import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libkitchen_int8_linear.so")
CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
ACT = {None: 0, "gelu_tanh": 1, "swiglu": 2, "rms_norm": 3}


def _ref():
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libkitchen_int8_linear.so was not built (no reference checkout)")
    lib = ctypes.CDLL(REF_LIB)
    vp, i64, i32, b, u64, f32 = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_bool,
                                 ctypes.c_uint64, ctypes.c_float)
    lib.launch_quantize_int8_rowwise_kernel.argtypes = [vp, vp, vp, i64, i64, i32, b, u64, vp]
    lib.launch_quantize_int8_rowwise_convrot64_kernel.argtypes = [vp, vp, vp, i64, i64, i32, i32,
                                                                  b, i32, u64, vp, f32, vp]
    lib.launch_int8_gemv_dequant_kernel.argtypes = [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, b,
                                                    i32, i32, vp]
    lib.launch_dequantize_int8_linear_kernel.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, b, i32,
                                                         i32, vp]
    for f in (lib.launch_quantize_int8_rowwise_kernel,
              lib.launch_quantize_int8_rowwise_convrot64_kernel,
              lib.launch_int8_gemv_dequant_kernel, lib.launch_dequantize_int8_linear_kernel):
        f.restype = None
    return lib


def W():
    import imagine_b200

    return imagine_b200


def cuda():
    return torch.device("cuda", 0)


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream(cuda()).cuda_stream)


def _x(m, k, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g) * 1.5
    x[0] = 0.0                   # an all-zero row
    if m > 2:
        x[2, 5] = 50.0           # an outlier
    return x.to(dtype).to(cuda())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("m,k", [(5600, 3072), (256, 12288), (37, 100), (1, 4096)])
@pytest.mark.parametrize("seed", [0, 12345])
def test_row_quantiser_matches_kitchen_kernel(dtype, m, k, seed):
    """quantize_int8_rowwise (Kitchen scales; seed > 0: stochastic rounding)
    against launch_quantize_int8_rowwise_kernel: every code and scale."""
    lib = _ref()
    x = _x(m, k, dtype, m + k)
    q_ref = torch.empty(m, k, dtype=torch.int8, device=cuda())
    s_ref = torch.empty(m, dtype=torch.float32, device=cuda())
    lib.launch_quantize_int8_rowwise_kernel(_p(x), _p(q_ref), _p(s_ref), m, k, CODE[dtype],
                                            seed > 0, seed, _stream())
    q, s = W().quantize_int8_rowwise(x, seed, scale_mode="kitchen_cuda")
    torch.cuda.synchronize()
    assert torch.equal(s.reshape(-1), s_ref)
    assert torch.equal(q, q_ref)
    if dtype == torch.float16:
        # the all-zero row: its 1e-30 scale is 0 in f16, 0 / 0 codes to -128
        assert bool((q[0] == -128).all())
    assert W().device_error() == 0


def _act_inputs(act, m, k, dtype, seed):
    width = 2 * k if act == "swiglu" else k
    x = _x(m, width, dtype, seed)
    w = None
    if act == "rms_norm":
        g = torch.Generator().manual_seed(seed + 1)
        w = (1 + 0.1 * torch.randn(k, generator=g)).to(dtype).to(cuda())
    return x, w


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("k", [256, 3072, 6144, 12288])
@pytest.mark.parametrize("act", [None, "gelu_tanh", "swiglu", "rms_norm"])
@pytest.mark.parametrize("one_row", [False, True])
def test_convrot_quantiser_matches_kitchen_kernel(dtype, k, act, one_row):
    """quantize_int8_rowwise_convrot (Kitchen CUDA numerics: fp32 activation in
    the fast-math forms, the radix-4 Hadamard in the reference's order, fp32
    absmax, approximate divide) against
    launch_quantize_int8_rowwise_convrot64_kernel.  One row and many rows
    select different block sizes there, so different RMSNorm summation
    orders."""
    lib = _ref()
    m = 1 if one_row else (300 if k <= 3072 else 40)
    x, w = _act_inputs(act, m, k, dtype, k + ACT[act])
    eps = 1e-6
    q_ref = torch.empty(m, k, dtype=torch.int8, device=cuda())
    s_ref = torch.empty(m, dtype=torch.float32, device=cuda())
    lib.launch_quantize_int8_rowwise_convrot64_kernel(_p(x), _p(q_ref), _p(s_ref), m, k, 256,
                                                      CODE[dtype], False, ACT[act], 0, _p(w),
                                                      eps, _stream())
    q, s = W().quantize_int8_rowwise_convrot(x, 256, act, w, eps, scale_mode="kitchen_cuda")
    torch.cuda.synchronize()
    s = s.reshape(-1)
    d = (q.int() - q_ref.int()).abs()
    print(f"{act} {dtype} K={k} M={m}: codes identical {(d == 0).float().mean().item():.6f}, "
          f"scales identical {torch.equal(s, s_ref)}")
    assert torch.equal(s, s_ref)
    assert torch.equal(q, q_ref)
    assert W().device_error() == 0


@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("n,k", [(18432, 3072), (1000, 4096), (64, 160)])
@pytest.mark.parametrize("has_bias", [True, False])
def test_gemv_matches_kitchen_kernel(m, out_dtype, n, k, has_bias):
    """int8_gemv against launch_int8_gemv_dequant_kernel, every output bit:
    one row in the SEPARATE order (that kernel adds the bias in a statement
    of its own), two rows in the CHAINED order (one contracted expression);
    per-channel scales, a bias of the output dtype or none."""
    lib = _ref()
    g = torch.Generator().manual_seed(m + n + k)
    q = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8).to(cuda())
    w = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8).to(cuda())
    xs = (torch.rand(m, generator=g) * 0.05 + 1e-3).to(cuda())
    ws = (torch.rand(n, generator=g) * 0.01 + 1e-4).to(cuda())
    bias = (torch.randn(n, generator=g) * 0.1).to(out_dtype).to(cuda()) if has_bias else None
    out_ref = torch.empty(m, n, dtype=out_dtype, device=cuda())
    lib.launch_int8_gemv_dequant_kernel(_p(q), _p(w), _p(xs), _p(ws), _p(bias), _p(out_ref), m, n,
                                        k, n, has_bias, CODE[out_dtype], CODE[out_dtype], _stream())
    order = "separate" if m == 1 else "chained"
    out = W().int8_gemv(q, w, xs, ws, bias, out_dtype, dequant=order)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.uint8), out_ref.view(torch.uint8))
    assert W().device_error() == 0


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("scalar_ws", [False, True])
@pytest.mark.parametrize("has_bias,n", [(True, 1536), (False, 1536), (False, 1537)])
def test_dequant_matches_kitchen_kernel(out_dtype, scalar_ws, has_bias, n):
    """dequantize_int8_linear against launch_dequantize_int8_linear_kernel on
    int32 accumulators in the range of a K = 3072 product, with the order that kernel's
    dispatch runs: a bias -> SEPARATE; no bias, scalar weight scale and
    N % 4 == 0 (its vec4 kernel) -> SCALE_PRODUCT; otherwise CHAINED."""
    lib = _ref()
    g = torch.Generator().manual_seed(7)
    m = 600
    acc = torch.randint(-(1 << 21), 1 << 21, (m, n), generator=g, dtype=torch.int32).to(cuda())
    xs = (torch.rand(m, generator=g) * 0.05 + 1e-3).to(cuda())
    ws = (torch.rand(1 if scalar_ws else n, generator=g) * 0.01 + 1e-4).to(cuda())
    bias = (torch.randn(n, generator=g) * 0.1).to(out_dtype).to(cuda()) if has_bias else None
    out_ref = torch.empty(m, n, dtype=out_dtype, device=cuda())
    lib.launch_dequantize_int8_linear_kernel(_p(acc), _p(xs), _p(ws), _p(bias), _p(out_ref), m, n,
                                             ws.numel(), has_bias, CODE[out_dtype],
                                             CODE[out_dtype], _stream())
    order = ("separate" if has_bias else
             "scale_product" if scalar_ws and n % 4 == 0 else "chained")
    out = W().dequantize_int8_linear(acc, xs, ws, bias, out_dtype, dequant=order)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.uint8), out_ref.view(torch.uint8))
    assert W().device_error() == 0
