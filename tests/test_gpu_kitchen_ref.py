"""This library's kernels against the reference's own Kitchen CUDA kernels on the
same inputs, on the GPU.

`oracle/_ref/libkitchen_int8_linear.so` is the reference file
native/comfy-port/kitchen/int8_linear.cu compiled in place for sm_100a by
`make -C oracle ref REF=<reference checkout>` (run by `__graft_entry__.build()`
where the checkout is present; the library then travels with the tree).  Its
`extern "C"` launchers (int8_linear.cu:1320-2162) are the kernels the
reference's CUDA route calls through its bridge: the row quantiser with
Kitchen scales (`amax * (1/127)`) and PCG stochastic rounding, the fused input
activation + ConvRot quantiser (`quantize_int8_rowwise_convrot64`), the GEMV
with dequant and the stand-alone dequant (the chained order).  This pins the
Kitchen-numerics forms of this library's kernels to the reference's code
rather than to a restatement of it.

Bars: bit-exact codes, scales and outputs, except where the two sides call a
transcendental in a different form (the activations' tanh / exp / rsqrt):
there codes within one step, 99% identical, scales within one ulp of fp32.
The tests skip when the reference library was not built."""
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
    q, s = W().quantize_int8_rowwise(x, seed, scale_mode="kitchen")
    torch.cuda.synchronize()
    assert torch.equal(s.reshape(-1), s_ref)
    assert torch.equal(q, q_ref)
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
@pytest.mark.parametrize("k", [256, 3072, 12288])
@pytest.mark.parametrize("act", [None, "gelu_tanh", "swiglu", "rms_norm"])
def test_convrot_quantiser_matches_kitchen_kernel(dtype, k, act):
    """quantize_int8_rowwise_convrot (Kitchen numerics: fp32 activation, the
    radix-4 Hadamard in the reference's order, fp32 absmax) against
    launch_quantize_int8_rowwise_convrot64_kernel."""
    lib = _ref()
    m = 300 if k <= 3072 else 40
    x, w = _act_inputs(act, m, k, dtype, k + ACT[act])
    eps = 1e-6
    q_ref = torch.empty(m, k, dtype=torch.int8, device=cuda())
    s_ref = torch.empty(m, dtype=torch.float32, device=cuda())
    lib.launch_quantize_int8_rowwise_convrot64_kernel(_p(x), _p(q_ref), _p(s_ref), m, k, 256,
                                                      CODE[dtype], False, ACT[act], 0, _p(w),
                                                      eps, _stream())
    q, s = W().quantize_int8_rowwise_convrot(x, 256, act, w, eps, scale_mode="kitchen")
    torch.cuda.synchronize()
    s = s.reshape(-1)
    d = (q.int() - q_ref.int()).abs()
    if act is None:
        assert torch.equal(s, s_ref)
        assert torch.equal(q, q_ref)
    else:
        rel = ((s - s_ref).abs() / s_ref.abs().clamp(min=1e-30)).max().item()
        assert rel <= 2.0 ** -23 * 2, f"scale relative difference {rel}"
        assert d.max().item() <= 1
        assert (d == 0).float().mean().item() >= 0.99
    print(f"{act} {dtype} K={k}: codes identical {(d == 0).float().mean().item():.5f}, "
          f"scales identical {torch.equal(s, s_ref)}")
    assert W().device_error() == 0


@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("n,k", [(18432, 3072), (1000, 4096), (64, 160)])
def test_gemv_matches_kitchen_kernel(m, out_dtype, n, k):
    """int8_gemv (the chained dequant order) against
    launch_int8_gemv_dequant_kernel: every output bit, per-channel scales and
    a bias of the output dtype."""
    lib = _ref()
    g = torch.Generator().manual_seed(m + n + k)
    q = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8).to(cuda())
    w = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8).to(cuda())
    xs = (torch.rand(m, generator=g) * 0.05 + 1e-3).to(cuda())
    ws = (torch.rand(n, generator=g) * 0.01 + 1e-4).to(cuda())
    bias = (torch.randn(n, generator=g) * 0.1).to(out_dtype).to(cuda())
    out_ref = torch.empty(m, n, dtype=out_dtype, device=cuda())
    lib.launch_int8_gemv_dequant_kernel(_p(q), _p(w), _p(xs), _p(ws), _p(bias), _p(out_ref), m, n,
                                        k, n, True, CODE[out_dtype], CODE[out_dtype], _stream())
    out = W().int8_gemv(q, w, xs, ws, bias, out_dtype, dequant="chained")
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.uint8), out_ref.view(torch.uint8))
    assert W().device_error() == 0


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("scalar_ws", [False, True])
def test_dequant_matches_kitchen_kernel(out_dtype, scalar_ws):
    """dequantize_int8_linear (chained order) against
    launch_dequantize_int8_linear_kernel on int32 accumulators of a real
    product."""
    lib = _ref()
    g = torch.Generator().manual_seed(7)
    m, k, n = 600, 3072, 1536
    qa = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8).to(cuda())
    wq = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8).to(cuda())
    acc = W().int8_gemm_s32(qa, wq)
    xs = (torch.rand(m, generator=g) * 0.05 + 1e-3).to(cuda())
    ws = (torch.rand(1 if scalar_ws else n, generator=g) * 0.01 + 1e-4).to(cuda())
    bias = (torch.randn(n, generator=g) * 0.1).to(out_dtype).to(cuda())
    out_ref = torch.empty(m, n, dtype=out_dtype, device=cuda())
    lib.launch_dequantize_int8_linear_kernel(_p(acc), _p(xs), _p(ws), _p(bias), _p(out_ref), m, n,
                                             ws.numel(), True, CODE[out_dtype], CODE[out_dtype],
                                             _stream())
    out = W().dequantize_int8_linear(acc, xs, ws, bias, out_dtype, dequant="chained")
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.uint8), out_ref.view(torch.uint8))
    assert W().device_error() == 0
