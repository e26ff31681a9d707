"""Parity on every BASELINE linear at full size, on the default routes
(no tile configuration given): the MMDiT block's four linears (QKV
3072 -> 9216, out 3072 -> 3072, MLP-up 3072 -> 12288 + GELU-tanh, MLP-down
12288 -> 3072) for the image stream (5600 rows; 11200 at CFG batch 2) and the
text stream (256 rows; 512), the AdaLN modulation GEMV (2 x 3072 -> 18432, and
the 60 blocks' modulation rows as one 2 x 3072 -> 1105920 GEMV), and the FP8
per-tensor and MXFP8 linears on config-3 inputs (N(0, 1) with 1% of entries
x 20) at 5600 x 3072 -> 12288 and -> 3072.

Bars (north star): codes and row scales bit-exact against the oracle on
every row; int32 accumulators bit-exact, as full row checksums
(sum_n acc[m, n] = q[m] . colsum(W)) plus 32 sampled rows compared whole;
outputs of the eager dequant order bit-exact on the sampled rows; GELU, FP8
and MXFP8 outputs within 1% of the output RMS (max over elements of
|y - ref| less half a bf16 ulp of |ref|, the output's own rounding) against
the unrounded reference.  Inputs are seeded synthetic tensors with the
BASELINE distributions (X ~ N(0, 1), W ~ N(0, 0.02))."""
import pytest
import torch

from oracle import eager as O
from tests.test_gpu_parity import assert_rms_close

pytestmark = pytest.mark.gpu

SWEEP = {"qkv": (3072, 9216, None), "out": (3072, 3072, None),
         "mlp_up": (3072, 12288, "gelu_tanh"), "mlp_down": (12288, 3072, None)}
ROWS = [5600, 11200, 256, 512]


def W():
    import imagine_b200

    return imagine_b200


def cuda():
    return torch.device("cuda", 0)


def _weights(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16)
    wq, ws = O.quantize_weight(w)
    return w, wq, ws, b


_WEIGHTS = {}


def _cached_weights(shape):
    if shape not in _WEIGHTS:
        k, n, _ = SWEEP[shape]
        _WEIGHTS[shape] = _weights(n, k, 1000 + k + n)
    return _WEIGHTS[shape]


@pytest.mark.parametrize("rows", ROWS)
@pytest.mark.parametrize("shape", list(SWEEP))
def test_block_linear_default_route(shape, rows):
    k, n, act = SWEEP[shape]
    _, wq, ws, b = _cached_weights(shape)
    g = torch.Generator().manual_seed(rows + k + n)
    x = torch.randn(rows, k, generator=g).to(torch.bfloat16)
    xd = x.to(cuda())
    wqd, wsd, bd = wq.to(cuda()), ws.to(cuda()), b.to(cuda())
    # quantiser: every code and scale
    qd, sd = W().quantize_int8_rowwise(xd)
    qo, so = O.quantize_int8_rowwise(x)
    assert torch.equal(qd.cpu(), qo) and torch.equal(sd.cpu(), so)
    # int32 accumulators of the default route: row checksums of the whole
    # product, and sampled rows compared whole
    acc = W().int8_gemm_s32(qd, wqd)
    colsum = wqd.to(torch.int64).sum(dim=0)
    want = (qd.to(torch.int64) * colsum).sum(dim=1)
    assert torch.equal(acc.to(torch.int64).sum(dim=1), want)
    sample = torch.randperm(rows, generator=g)[:32]
    assert torch.equal(acc[sample.to(cuda())].cpu(), O.int8_accumulate(qo[sample], wq))
    # the linear (quantiser + GEMM + dequant + bias [+ GELU]) on the default route
    y = W().int8_linear(xd, wqd, wsd, bd, output_act=act)
    ref = O.int8_linear(x[sample], wq, ws, b, out_dtype=torch.bfloat16, output_act=act)
    ys = y[sample.to(cuda())]
    if act is None:
        assert torch.equal(ys.cpu().view(torch.int16), ref.view(torch.int16))
    else:
        assert_rms_close(ys, ref)
    assert W().device_error() == 0


@pytest.mark.parametrize("n", [18432, 60 * 18432])
def test_adaln_modulation_gemv(n):
    """SiLU(temb) rows (M = 2, CFG) through the fused quantise + GEMV: one
    block's 3072 -> 18432, and all 60 blocks' modulation weights as one
    matrix (the DiT step's single modulation launch per stream): outputs
    bit-exact against the oracle on sampled output columns."""
    k = 3072
    g = torch.Generator(device=cuda()).manual_seed(n)
    wd = (torch.randn(n, k, generator=g, device=cuda()) * 0.02).to(torch.bfloat16)
    wqd, wsd = W().quantize_weight(wd)
    del wd
    bd = (torch.randn(n, generator=g, device=cuda()) * 0.02).to(torch.bfloat16)
    temb = torch.randn(2, k, generator=g, device=cuda()).to(torch.bfloat16)
    s = torch.nn.functional.silu(temb)
    y = W().int8_linear(s, wqd, wsd, bd)
    cols = torch.randperm(n, generator=torch.Generator().manual_seed(3))[:2048].to(cuda())
    ref = O.int8_linear(s.cpu(), wqd[cols].cpu(), wsd[cols].cpu(), bd[cols].cpu(),
                        out_dtype=torch.bfloat16)
    assert torch.equal(y[:, cols].cpu().view(torch.int16), ref.view(torch.int16))
    assert W().device_error() == 0


def _config3(m, k, seed):
    """Config 3's activations: N(0, 1) with 1% of entries x 20."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    return torch.where(torch.rand(m, k, generator=g) < 0.01, x * 20, x).to(torch.bfloat16)


@pytest.mark.parametrize("n", [12288, 3072])
def test_fp8_per_tensor_full_size(n):
    m, k = 5600, 3072
    x = _config3(m, k, 7 + n)
    w, _, _, b = _weights(n, k, 8 + n)
    sa = (x.abs().max().float() / 448).reshape(1)
    sw = (w.abs().max().float() / 448).reshape(1)
    aq = W().quantize_per_tensor_fp8(x.to(cuda()), sa.to(cuda()))
    wq = W().quantize_per_tensor_fp8(w.to(cuda()), sw.to(cuda()))
    y = W().fp8_linear(aq, sa.to(cuda()), wq, sw.to(cuda()), b.to(cuda()))
    assert W().device_error() == 0
    rows = torch.randperm(m, generator=torch.Generator().manual_seed(n))[:64]
    ref = O.fp8_linear_exact(aq.cpu()[rows], sa, wq.cpu(), sw, b, out_dtype=torch.float32)
    assert_rms_close(y[rows.to(cuda())], ref)


@pytest.mark.parametrize("n", [12288, 3072])
def test_mxfp8_full_size(n):
    m, k = 5600, 3072
    x = _config3(m, k, 9 + n)
    w, _, _, b = _weights(n, k, 10 + n)
    aq, asf = W().quantize_mxfp8(x.to(cuda()))
    wq, wsf = W().quantize_mxfp8(w.to(cuda()))
    y = W().mxfp8_linear(aq, asf, wq, wsf, b.to(cuda()))
    assert W().device_error() == 0
    a_deq = O.dequantize_mxfp8(aq.cpu(), asf.cpu(), out_dtype=torch.float32)
    w_deq = O.dequantize_mxfp8(wq.cpu(), wsf.cpu(), out_dtype=torch.float32)
    rows = torch.randperm(m, generator=torch.Generator().manual_seed(n))[:64]
    ref = a_deq[rows].double() @ w_deq.double().t() + b.double()
    assert_rms_close(y[rows.to(cuda())], ref.float())
