"""Split-K GEMM (w8a8_gemm_dequant_splitk) through the C ABI: bit-identical to
the unsplit GEMM and to the eager oracle for every split count, and the
caller's scratch is zero-filled again after every call."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import eager as O

pytestmark = pytest.mark.gpu


def W():
    import imagine_b200

    return imagine_b200


def cuda():
    return torch.device("cuda", 0)


def _case(m, k, n, seed, dt=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dt)
    w = (torch.randn(n, k, generator=g) * 0.02).to(dt)
    b = (torch.randn(n, generator=g) * 0.02).to(dt)
    wq, ws = O.quantize_weight(w)
    return x, wq, ws, b


def _splitk(q, xs, wq, ws, b, out_dtype, split_k, scratch, act=None, residual=None, rscale=None):
    """One w8a8_gemm_dequant_splitk call through the C ABI."""
    from imagine_b200 import _native as N
    from imagine_b200.linear import _epilogue, _stream, _vp, _code

    m, k = q.shape
    n = wq.shape[0]
    out = torch.empty((m, n), dtype=out_dtype, device=cuda())
    ep = _epilogue(ws, b, residual, rscale, "eager", act, n, n)
    rc = N.LIB.w8a8_gemm_dequant_splitk(
        _vp(q), k, _vp(wq), k, _vp(xs), ctypes.byref(ep), _vp(out), _code(out_dtype), n, m, n, k,
        split_k, _vp(scratch), scratch.numel(), None, _stream(cuda()))
    N.check(rc)
    return out


SHAPES = [(256, 12288, 3072), (200, 3072, 3072), (256, 3072, 1000), (130, 4096, 520), (64, 2048, 256)]


@pytest.mark.parametrize("m,k,n", SHAPES)
@pytest.mark.parametrize("split_k", [0, 2, 3, 7])
def test_splitk_bit_identical(m, k, n, split_k):
    from imagine_b200 import _native as N

    x, wq, ws, b = _case(m, k, n, m + k + n)
    xd, wqd, wsd, bd = x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda())
    q, xs = W().quantize_int8_rowwise(xd)
    xs = xs.reshape(-1)
    nbytes = N.LIB.w8a8_gemm_splitk_workspace_bytes(m, n)
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device=cuda())
    ref_dev = W().int8_linear(xd, wqd, wsd, bd, split_k=1)
    for _ in range(2):  # the second call finds the scratch zero-filled again
        y = _splitk(q, xs, wqd, wsd, bd, torch.bfloat16, split_k, scratch)
        assert torch.equal(y.view(torch.int16), ref_dev.view(torch.int16))
        torch.cuda.synchronize()
        assert int(scratch.count_nonzero()) == 0
    ref = O.int8_linear(x, wq, ws, b, out_dtype=torch.bfloat16)
    assert np.array_equal(O.as_bytes(y.cpu()), O.as_bytes(ref))
    assert W().device_error() == 0


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_splitk_epilogues(out_dtype):
    """GELU and the residual epilogue on the split path equal the unsplit GEMM."""
    from imagine_b200 import _native as N

    m, k, n = 256, 6144, 1536
    x, wq, ws, b = _case(m, k, n, 9)
    g = torch.Generator().manual_seed(10)
    r = torch.randn(m, n, generator=g).to(out_dtype).to(cuda())
    rs = torch.rand(n, generator=g).to(out_dtype).to(cuda())
    xd, wqd, wsd, bd = x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(out_dtype).to(cuda())
    q, xs = W().quantize_int8_rowwise(xd)
    xs = xs.reshape(-1)
    scratch = torch.zeros(N.LIB.w8a8_gemm_splitk_workspace_bytes(m, n), dtype=torch.uint8,
                          device=cuda())
    for act, res in [("gelu_tanh", None), (None, (r, rs))]:
        kw = dict(residual=res[0], residual_scale=res[1]) if res else {}
        want = W().int8_linear(xd, wqd, wsd, bd, out_dtype=out_dtype, output_act=act, split_k=1, **kw)
        got = _splitk(q, xs, wqd, wsd, bd, out_dtype, 4, scratch, act,
                      res[0] if res else None, res[1] if res else None)
        assert torch.equal(got, want)
    torch.cuda.synchronize()
    assert int(scratch.count_nonzero()) == 0


def test_splitk_through_int8_linear_default():
    """int8_linear picks split-K by itself for the text-stream shape."""
    m, k, n = 256, 12288, 3072
    x, wq, ws, b = _case(m, k, n, 11)
    y = W().int8_linear(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda()))
    ref = O.int8_linear(x, wq, ws, b, out_dtype=torch.bfloat16)
    assert np.array_equal(O.as_bytes(y.cpu()), O.as_bytes(ref))


def test_splitk_scratch_errors():
    from imagine_b200 import _native as N

    m, k, n = 256, 4096, 512
    x, wq, ws, b = _case(m, k, n, 12)
    q, xs = W().quantize_int8_rowwise(x.to(cuda()))
    need = N.LIB.w8a8_gemm_splitk_workspace_bytes(m, n)
    assert need >= m * n * 4
    small = torch.zeros(need - 256, dtype=torch.uint8, device=cuda())
    with pytest.raises(ValueError, match="scratch"):
        _splitk(q, xs.reshape(-1), wq.to(cuda()), ws.to(cuda()), b.to(cuda()), torch.bfloat16, 4,
                small)


def test_autotuned_config_is_bit_identical():
    """config="auto" times the candidate configurations once per shape (the
    reference's autotuner policy) and the tuned launch gives the same bytes."""
    m, k, n = 384, 3072, 1536
    x, wq, ws, b = _case(m, k, n, 13)
    args = (x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda()))
    want = W().int8_linear(*args)
    got = W().int8_linear(*args, config="auto")
    again = W().int8_linear(*args, config="auto")  # cached choice
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert torch.equal(again.view(torch.int16), want.view(torch.int16))
    from imagine_b200 import autotune

    t = autotune.tuner("int8_dequant")
    assert t.best_config is not None and len(t.last_timings) == len(autotune.GEMM_CONFIGS)


@pytest.mark.parametrize("chunks", [1, 3, 4])
def test_int8_linear_host_matches_device_path(chunks):
    """The pipelined host-buffer linear returns int8_linear's bytes row for row."""
    m, k, n = 1000, 3072, 768
    x, wq, ws, b = _case(m, k, n, 14)
    wd, wsd, bd = wq.to(cuda()), ws.to(cuda()), b.to(cuda())
    want = W().int8_linear(x.to(cuda()), wd, wsd, bd, output_act="gelu_tanh").cpu()
    xp = x.pin_memory()
    for _ in range(2):
        got = W().int8_linear_host(xp, wd, wsd, bd, chunks=chunks, output_act="gelu_tanh")
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("m,k,n", [(256, 12288, 3072), (200, 3008, 1000), (64, 3072, 9216),
                                   (2, 3072, 640)])
@pytest.mark.parametrize("split_k", [None, 1])
def test_pre_tiled_weights_bit_identical(m, k, n, split_k):
    """int8_linear on a pre-tiled weight equals the row-major weight's result
    (K and N tails included: the tiles are zero padded)."""
    x, wq, ws, b = _case(m, k, n, 15 + m)
    xd, wqd, wsd, bd = x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda())
    tw = W().pack_weight_tiles(wqd)
    assert tw.shape == (n, k)
    want = W().int8_linear(xd, wqd, wsd, bd, split_k=1)
    got = W().int8_linear(xd, tw, wsd, bd, split_k=split_k)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert W().device_error() == 0


def test_auto_workspace_bytes():
    """The automatic policy's scratch: the full split's for few-row shapes,
    none for shapes whose tiles fill the SMs (they run every tile whole)."""
    from imagine_b200 import _native as N

    with torch.cuda.device(cuda()):
        assert N.LIB.w8a8_gemm_auto_workspace_bytes(5600, 12288, 3072, None) == 0
        assert N.LIB.w8a8_gemm_auto_workspace_bytes(1400, 3072, 3072, None) == 0
        assert (N.LIB.w8a8_gemm_auto_workspace_bytes(256, 3072, 12288, None)
                == N.LIB.w8a8_gemm_splitk_workspace_bytes(256, 3072))
        assert N.LIB.w8a8_gemm_auto_workspace_bytes(256, 3072, 256, None) == 0  # K too short
