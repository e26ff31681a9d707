"""GPU parity of the fused input-activation + ConvRot quantiser
(w8a8_quantize_rowwise_convrot) against the C restatement of the reference
kernel (oracle/ref_w8a8.c, ref_quantize_act_rot).

Bars: without an activation every code and scale is bit-exact (the FHT is
fp32 additions in the reference's order, the element step is exact).  With
an activation (tanhf / expf / rsqrtf on the device vs libm on the host, and a
different summation order for RMSNorm's mean of squares) codes may move by
one step where the activated value sits on a rounding boundary: at most 1
apart, at least 99% identical, scales within 1e-5 relative; the linear built
on them is held to 1% of output RMS.
"""
import pytest
import torch

from oracle import eager as O
from tests import _cref

pytestmark = pytest.mark.gpu


def W():
    import imagine_b200

    return imagine_b200


def cuda():
    return torch.device("cuda", 0)


def _x(m, width, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, width, generator=g) * 1.5
    x[0] = 0.0                       # an all-zero row
    if m > 2:
        x[2, 7] = 40.0               # an outlier row
    return x.to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("k", [256, 768, 3072, 12288, 16384])
@pytest.mark.parametrize("mode", ["kitchen", "eager"])
def test_convrot_exact(dtype, k, mode):
    m = 37 if k <= 3072 else 9
    x = _x(m, k, dtype, k)
    q, s = W().quantize_int8_rowwise_convrot(x.to(cuda()), 256, scale_mode=mode)
    rq, rs = _cref.quantize_act_rot(x, True, kitchen=(mode == "kitchen"))
    assert torch.equal(s.reshape(-1).cpu(), rs)
    assert torch.equal(q.cpu(), rq)
    assert W().device_error() == 0


ACTS = ["gelu_tanh", "swiglu", "rms_norm", "situ"]


@pytest.mark.parametrize("act", ACTS)
@pytest.mark.parametrize("rotate", [True, False])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_convrot_with_activation(act, rotate, dtype):
    m, k = 65, 3072
    width = 2 * k if act in ("swiglu", "situ") else k
    x = _x(m, width, dtype, 3)
    g = torch.Generator().manual_seed(4)
    aw = (1 + 0.1 * torch.randn(k, generator=g)).to(dtype) if act == "rms_norm" else None
    eps = 1e-6 if act == "rms_norm" else None
    q, s = W().quantize_int8_rowwise_convrot(
        x.to(cuda()), 256 if rotate else 0, act, aw.to(cuda()) if aw is not None else None, eps)
    rq, rs = _cref.quantize_act_rot(x, rotate, act, aw, eps or 0.0)
    s = s.reshape(-1).cpu()
    assert torch.allclose(s, rs, rtol=1e-5, atol=0)
    d = (q.cpu().int() - rq.int()).abs()
    assert d.max().item() <= 1
    assert (d == 0).float().mean().item() >= 0.99


@pytest.mark.parametrize("kw", [
    dict(convrot=True),
    dict(convrot=True, input_act="gelu_tanh"),
    dict(convrot=True, input_act="swiglu"),
    dict(convrot=True, input_act="rms_norm", input_act_eps=1e-6),
    dict(input_act="gelu_tanh"),
    dict(input_act="situ"),
], ids=lambda d: "-".join(f"{k}={v}" for k, v in d.items()))
def test_int8_linear_fused_quantiser_route(kw):
    """int8_linear takes the fused quantiser for these shapes and stays within
    the tolerance bar of the eager oracle (ATen activation, bf16 Hadamard
    matmul, row quantiser, exact GEMM, eager dequant)."""
    m, k, n = 300, 3072, 512
    dt = torch.bfloat16
    act = kw.get("input_act")
    width = 2 * k if act in ("swiglu", "situ") else k
    g = torch.Generator().manual_seed(6)
    x = torch.randn(m, width, generator=g).to(dt)
    w = (torch.randn(n, k, generator=g) * 0.02).to(dt)
    b = (torch.randn(n, generator=g) * 0.02).to(dt)
    wq, ws = O.quantize_weight(w)
    if act == "rms_norm":
        kw = dict(kw, input_act_weight=(1 + 0.1 * torch.randn(k, generator=g)).to(dt))
    dev_kw = {key: (v.to(cuda()) if isinstance(v, torch.Tensor) else v) for key, v in kw.items()}
    y = W().int8_linear(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda()), out_dtype=dt,
                        **dev_kw).float().cpu()
    ref = O.int8_linear(x, wq, ws, b, out_dtype=dt, **kw).float()
    rms = ref.pow(2).mean().sqrt().item()
    half_ulp = torch.pow(2.0, torch.floor(torch.log2(ref.abs().clamp(min=1e-30))) - 8)
    err = ((y - ref).abs() - half_ulp).clamp(min=0).max().item()
    assert err <= 0.01 * rms, (err, rms)


def test_convrot_argument_errors():
    x = torch.zeros(4, 512, dtype=torch.bfloat16, device=cuda())
    with pytest.raises(ValueError):
        W().quantize_int8_rowwise_convrot(x, 64)
    with pytest.raises(ValueError):
        W().quantize_int8_rowwise_convrot(torch.zeros(4, 200, dtype=torch.bfloat16, device=cuda()))
    with pytest.raises(ValueError):
        W().quantize_int8_rowwise_convrot(x, 256, "rms_norm", None, 1e-6)
    with pytest.raises(TypeError):
        W().quantize_int8_rowwise_convrot(x, 256, "rms_norm", torch.ones(512, device=cuda()), None)
    with pytest.raises(ValueError):
        W().quantize_int8_rowwise_convrot(x, 256, "relu")
