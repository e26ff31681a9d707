"""w8a8_gemm_dequant_splitk_static -- the split-K GEMM on the library's own
fixed scratch, for callers that cannot allocate -- called through the C ABI
and checked bit for bit against the entry points that take caller memory,
on two calls in a row.  A call that splits clears the part of the shared
array it uses before launching, so the second call shows that the clear
makes a used array good again."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(m, k, n, seed):
    import imagine_b200 as W

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    b = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    wq, ws = W.quantize_weight(w)
    q, xs = W.quantize_int8_rowwise(x)
    return q, xs.reshape(-1), wq, ws, b


@pytest.mark.parametrize("m,k,n,split_k", [(256, 12288, 3072, 0), (256, 12288, 3072, 3),
                                           (200, 3072, 1000, 2), (130, 4096, 520, 0)])
def test_static_scratch_matches_caller_scratch(m, k, n, split_k):
    from imagine_b200 import _native as N
    from imagine_b200.linear import _epilogue, _stream, _vp

    q, xs, wq, ws, b = _inputs(m, k, n, m + n)
    dev = q.device
    ep = _epilogue(ws, b, None, None, "eager", None, n, n)
    stream = _stream(dev)
    # existing entry points: caller scratch (split) and the unsplit GEMM
    scratch = torch.zeros(N.LIB.w8a8_gemm_splitk_workspace_bytes(m, n), dtype=torch.uint8,
                          device=dev)
    want = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    N.check(N.LIB.w8a8_gemm_dequant_splitk(_vp(q), k, _vp(wq), k, _vp(xs), ctypes.byref(ep),
                                           _vp(want), N.BF16, n, m, n, k, split_k, _vp(scratch),
                                           scratch.numel(), None, stream))
    plain = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    N.check(N.LIB.w8a8_gemm_dequant(_vp(q), k, _vp(wq), k, _vp(xs), ctypes.byref(ep), _vp(plain),
                                    N.BF16, n, m, n, k, None, stream))
    assert torch.equal(want.view(torch.int16), plain.view(torch.int16))
    for _ in range(2):
        got = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
        N.check(N.LIB.w8a8_gemm_dequant_splitk_static(
            _vp(q), k, _vp(wq), k, _vp(xs), ctypes.byref(ep), _vp(got), N.BF16, n, m, n, k,
            split_k, None, stream))
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    import imagine_b200 as W

    assert W.device_error() == 0


def test_static_scratch_rejects_oversized_splits():
    """A GEMM that would split but whose partial sums do not fit the fixed
    array is refused with a message, and nothing is launched."""
    from imagine_b200 import _native as N
    from imagine_b200.linear import _epilogue, _stream, _vp

    m, k, n = 1024, 2048, 4096  # 16 MiB of partial sums > the 8 MiB scratch
    q, xs, wq, ws, b = _inputs(m, k, n, 7)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=q.device)
    ep = _epilogue(ws, b, None, None, "eager", None, n, n)
    rc = N.LIB.w8a8_gemm_dequant_splitk_static(_vp(q), k, _vp(wq), k, _vp(xs), ctypes.byref(ep),
                                               _vp(out), N.BF16, n, m, n, k, 2, None,
                                               _stream(q.device))
    assert rc == N.ERR_VALUE
    assert b"static scratch" in N.LIB.w8a8_last_error()


@pytest.mark.parametrize("split_k", [0, 1])
def test_static_entry_runs_unsplit_shapes_of_any_size(split_k):
    """Shapes that do not split (the automatic policy runs 1024 x 4096 tiles
    whole; split_k = 1 never splits) need no scratch and run at any size, with
    the plain GEMM's results."""
    from imagine_b200 import _native as N
    from imagine_b200.linear import _epilogue, _stream, _vp

    m, k, n = 1024, 2048, 4096
    q, xs, wq, ws, b = _inputs(m, k, n, 8)
    dev = q.device
    ep = _epilogue(ws, b, None, None, "eager", None, n, n)
    stream = _stream(dev)
    want = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    N.check(N.LIB.w8a8_gemm_dequant(_vp(q), k, _vp(wq), k, _vp(xs), ctypes.byref(ep), _vp(want),
                                    N.BF16, n, m, n, k, None, stream))
    for _ in range(2):
        got = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
        N.check(N.LIB.w8a8_gemm_dequant_splitk_static(
            _vp(q), k, _vp(wq), k, _vp(xs), ctypes.byref(ep), _vp(got), N.BF16, n, m, n, k,
            split_k, None, stream))
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
