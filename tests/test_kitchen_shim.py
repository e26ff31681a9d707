"""The imagine_kitchen_call front end (libimagine_kitchen_w8a8.so): the
reference's bridge entry points (inference/native/bridge.hpp:5-6, 14-16, 29)
over libw8a8.  CPU tests cover loading, exports and error mapping; the GPU
tests drive every mapped kernel name with borrowed at::Tensor handles and
compare with the C ABI called directly."""
import ctypes
import os

import pytest
import torch

from oracle import eager as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(ROOT, "imagine_b200", "libimagine_kitchen_w8a8.so")


class KitchenArg(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int64), ("tensor", ctypes.c_void_p),
                ("integer", ctypes.c_int64), ("real", ctypes.c_double)]


def _lib():
    if not os.path.exists(SHIM):
        from imagine_b200 import build as B

        B.build()
        B.build_shim()
    lib = ctypes.CDLL(SHIM)
    lib.imagine_kitchen_call.argtypes = [ctypes.c_char_p, ctypes.POINTER(KitchenArg), ctypes.c_size_t,
                                         ctypes.POINTER(ctypes.c_int64)]
    lib.imagine_kitchen_call.restype = ctypes.c_int
    lib.imagine_last_error.restype = ctypes.c_char_p
    lib.imagine_last_accelerator_code.restype = ctypes.c_int
    lib.imagine_w8a8_tensor_view.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64),
                                             ctypes.POINTER(ctypes.c_int64), ctypes.c_int64,
                                             ctypes.c_int64, ctypes.c_int64,
                                             ctypes.POINTER(ctypes.c_void_p)]
    lib.imagine_w8a8_tensor_free.argtypes = [ctypes.c_void_p]
    return lib


def _call(lib, name, args):
    arr = (KitchenArg * max(len(args), 1))(*args)
    res = ctypes.c_int64(-7)
    rc = lib.imagine_kitchen_call(name.encode(), arr, len(args), ctypes.byref(res))
    return rc, res.value


def test_shim_exports_and_error_mapping():
    lib = _lib()
    rc, _ = _call(lib, "no_such_kernel", [])
    assert rc == -1 and b"Unknown Kitchen kernel" in lib.imagine_last_error()
    rc, _ = _call(lib, "quantize_int8_rowwise", [])  # missing arguments -> IndexError
    assert rc == -21
    rc, _ = _call(lib, "quantize_int8_rowwise", [KitchenArg(2, None, 5, 0.0)])  # not a tensor
    assert rc == -20
    assert lib.imagine_last_accelerator_code() == 0


DT = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.int32: 3, torch.int8: 4}


class Handles:
    """Borrowed at::Tensor* handles for torch tensors (freed on exit)."""

    def __init__(self, lib):
        self.lib, self.ptrs = lib, []

    def t(self, x):
        if x is None:
            return KitchenArg(0, None, 0, 0.0)
        sizes = (ctypes.c_int64 * x.dim())(*x.shape)
        strides = (ctypes.c_int64 * x.dim())(*x.stride())
        out = ctypes.c_void_p()
        assert self.lib.imagine_w8a8_tensor_view(ctypes.c_void_p(x.data_ptr()), sizes, strides,
                                                 x.dim(), DT[x.dtype], x.device.index,
                                                 ctypes.byref(out)) == 0
        self.ptrs.append(out)
        return KitchenArg(1, out.value, 0, 0.0)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        for p in self.ptrs:
            self.lib.imagine_w8a8_tensor_free(p)


def I(v):  # noqa: E743 - the bridge's Int argument
    return KitchenArg(2, None, int(v), 0.0)


def B(v):
    return KitchenArg(4, None, int(bool(v)), 0.0)


def F(v):
    return KitchenArg(3, None, 0, float(v))


@pytest.mark.gpu
def test_shim_linear_routes_match_c_abi():
    import imagine_b200 as W

    lib = _lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    g = torch.Generator().manual_seed(40)
    m, k, n = 300, 3072, 640
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    wq, ws = (t.to(dev) for t in O.quantize_weight(w))
    bias = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    r = torch.randn(m, n, generator=g).to(torch.bfloat16).to(dev)
    rs = torch.rand(n, generator=g).to(torch.bfloat16).to(dev)
    with Handles(lib) as h:
        q = torch.empty(m, k, dtype=torch.int8, device=dev)
        xs = torch.empty(m, 1, dtype=torch.float32, device=dev)
        assert _call(lib, "quantize_int8_rowwise", [h.t(x), h.t(q), h.t(xs), B(0), I(0), I(stream)]) == (0, 0)
        q_ref, xs_ref = W.quantize_int8_rowwise(x, scale_mode="kitchen_cuda")
        assert torch.equal(q, q_ref) and torch.equal(xs, xs_ref)
        out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        rc, res = _call(lib, "cutlass_int8_dequant", [h.t(q), h.t(wq), h.t(xs), h.t(ws), h.t(bias),
                                                       h.t(out), I(2), I(stream)])
        assert rc == 0 and res == 1, lib.imagine_last_error()
        want = W.int8_linear(x, wq, ws, bias, scale_mode="kitchen", dequant="chained")
        assert torch.equal(out, want)
        out2 = torch.empty_like(out)
        rc, res = _call(lib, "cutlass_int8_dequant_residual",
                        [h.t(q), h.t(wq), h.t(xs), h.t(ws), h.t(bias), h.t(rs), h.t(r), h.t(out2),
                         I(2), I(stream)])
        assert rc == 0 and res == 1
        want_r = W.int8_linear(x, wq, ws, bias, residual=r, residual_scale=rs, scale_mode="kitchen",
                               dequant="chained")
        assert torch.equal(out2, want_r)
        acc = torch.empty(m, n, dtype=torch.int32, device=dev)
        ws_buf = torch.empty(1 << 20, dtype=torch.int8, device=dev)
        assert _call(lib, "cublas_gemm_int8", [h.t(q), h.t(wq), h.t(acc), h.t(ws_buf), I(stream)])[0] == 0
        assert torch.equal(acc, W.int8_gemm_s32(q, wq))
        out3 = torch.empty_like(out)
        assert _call(lib, "dequantize_int8_linear", [h.t(acc), h.t(xs), h.t(ws), h.t(bias), h.t(out3),
                                                      I(2), I(stream)])[0] == 0
        # with a bias the Kitchen dequant kernel adds it uncontracted
        assert torch.equal(out3, W.dequantize_int8_linear(acc, xs, ws, bias, torch.bfloat16,
                                                          dequant="separate"))
        # M = 1 / 2 routes
        x1 = x[:2].contiguous()
        q1 = torch.empty(2, k, dtype=torch.int8, device=dev)
        xs1 = torch.empty(2, 1, dtype=torch.float32, device=dev)
        o1 = torch.empty(2, n, dtype=torch.bfloat16, device=dev)
        empty = torch.empty(0, dtype=torch.bfloat16, device=dev)
        assert _call(lib, "int8_linear_m1", [h.t(x1), h.t(q1), h.t(xs1), h.t(wq), h.t(ws), h.t(bias),
                                             h.t(o1), I(2), B(0), I(256), I(0), h.t(empty), F(0.0),
                                             I(stream)])[0] == 0
        assert torch.equal(o1, out[:2])
        o2 = torch.empty_like(o1)
        assert _call(lib, "int8_gemv_dequant", [h.t(q1), h.t(wq), h.t(xs1), h.t(ws), h.t(bias),
                                                h.t(o2), I(2), I(stream)])[0] == 0
        assert torch.equal(o2, o1)
        # fused ConvRot quantiser
        qc = torch.empty(m, k, dtype=torch.int8, device=dev)
        sc = torch.empty(m, 1, dtype=torch.float32, device=dev)
        assert _call(lib, "quantize_int8_rowwise_convrot64",
                     [h.t(x), h.t(qc), h.t(sc), I(256), B(0), I(1), I(0), h.t(empty), F(0.0),
                      I(stream)])[0] == 0
        qr, sr = W.quantize_int8_rowwise_convrot(x, 256, "gelu_tanh", scale_mode="kitchen_cuda")
        assert torch.equal(qc, qr) and torch.equal(sc, sr)
        # an argument error comes back as ValueError (-20) with the message
        rc, _ = _call(lib, "quantize_int8_rowwise_convrot64",
                      [h.t(x), h.t(qc), h.t(sc), I(64), B(0), I(0), I(0), h.t(empty), F(0.0),
                       I(stream)])
        assert rc == -20 and b"group" in lib.imagine_last_error()
    torch.cuda.synchronize()


class _CudaArray:
    """A raw device buffer as a torch tensor (__cuda_array_interface__)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3}


@pytest.mark.gpu
def test_shim_fp8_scaled_mm_matches_c_abi():
    """imagine_fp8_scaled_mm (bridge.cpp:401-413: _scaled_mm_v2 TensorWise) on
    the tcgen05 FP8 GEMM: a [M, K] e4m3, b the column-major [K, N] view of a
    row-major [N, K] weight, scalar fp32 scales, bf16 bias, bf16 output --
    bit-identical to libw8a8's w8a8_fp8_gemm (imagine_b200.fp8_linear)."""
    import imagine_b200 as W

    lib = _lib()
    lib.imagine_fp8_scaled_mm.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64,
                                                                  ctypes.POINTER(ctypes.c_void_p)]
    lib.imagine_w8a8_tensor_info.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
                                             ctypes.POINTER(ctypes.c_int64),
                                             ctypes.POINTER(ctypes.c_int64)]
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(41)
    m, k, n = 520, 3072, 1024
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    sa = (x.abs().amax().float() / 448.0).reshape(1)
    sw = (w.abs().amax().float() / 448.0).reshape(1)
    a8 = W.quantize_per_tensor_fp8(x, sa)
    w8 = W.quantize_per_tensor_fp8(w, sw)
    bias = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    want = W.fp8_linear(a8, sa, w8, sw, bias, torch.bfloat16)

    def view(t, code):
        sizes = (ctypes.c_int64 * t.dim())(*t.shape)
        strides = (ctypes.c_int64 * t.dim())(*t.stride())
        out = ctypes.c_void_p()
        assert lib.imagine_w8a8_tensor_view(ctypes.c_void_p(t.data_ptr()), sizes, strides, t.dim(),
                                            code, dev.index, ctypes.byref(out)) == 0
        return out

    handles = [view(a8, 5), view(w8.t(), 5), view(sa, 0), view(sw, 0), view(bias, 2)]
    out = ctypes.c_void_p()
    try:
        rc = lib.imagine_fp8_scaled_mm(*handles, 15, ctypes.byref(out))  # 15: at::kBFloat16
        assert rc == 0, lib.imagine_last_error()
        ptr, numel, code = ctypes.c_void_p(), ctypes.c_int64(), ctypes.c_int64()
        assert lib.imagine_w8a8_tensor_info(out, ctypes.byref(ptr), ctypes.byref(numel),
                                            ctypes.byref(code)) == 0
        assert numel.value == m * n and code.value == 2
        torch.cuda.synchronize()
        got = torch.as_tensor(_CudaArray(ptr.value, (m, n), "<i2"), device=dev)
        assert torch.equal(got, want.view(torch.int16))
    finally:
        for h in handles + ([out] if out.value else []):
            lib.imagine_w8a8_tensor_free(h)
