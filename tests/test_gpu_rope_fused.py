"""GPU parity of the Q/K projection with its RMSNorm + RoPE fused into the GEMM
epilogue (w8a8_gemm_dequant_rms_rope) against the oracle's
``rms_rope(int8_linear(...))`` (inference/src/int8_linear.rs:198-277 then
inference/src/backend_rope.rs:146-223, restated in oracle/eager.py).

Bar: the projection's bf16 output before the norm is the oracle's bit for bit
(checked through the columns that are not rotated).  The row's fp32 sum of
squares is added in a different order than torch's CPU cascade sum, so the
row's 1/rms can differ in its last bit and move a normalised value across a
bf16 rounding boundary.  A flipped normalised value n moves both outputs of
its pair through the rotation (|f| <= 1), so rotated outputs are held to:
every element within sqrt(2) bf16 ulps of its pair's magnitude (the rotation
preserves it and |n| cannot exceed it) plus one ulp of its own rounding,
>= 99% bit-identical, and the RMS of the error <= 1% of the output RMS.  (A max-abs bound of 1% of RMS cannot hold
for a normalised bf16 output: one ulp at |y| >= 2 RMS is 1.56% of RMS; the
reference's own Triton and eager routes differ by such flips too.)"""
import pytest
import torch

from oracle import eager as O

pytestmark = pytest.mark.gpu


def W():
    import imagine_b200

    return imagine_b200


def cuda():
    return torch.device("cuda", 0)


def _freqs(s, g):
    ang = torch.rand(s, 64, generator=g, dtype=torch.float64) * 6.283
    c, sn = torch.cos(ang), torch.sin(ang)
    return torch.stack([torch.stack([c, -sn], -1), torch.stack([sn, c], -1)], -2).float()


def _case(m, k, n, seed, bias=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = torch.randn(n, k, generator=g) * 0.05
    wq, ws = O.quantize_weight(w)
    b = (torch.randn(n, generator=g) * 0.5).to(torch.bfloat16) if bias else None
    return g, x, wq, ws, b


def _bf16_ulp(v):
    _, e = torch.frexp(v)  # |v| = m 2^e, m in [0.5, 1)
    return torch.ldexp(torch.ones_like(v), e - 8)


def _pair_bound(ref):
    """sqrt(2) ulp of the pair magnitude (a flipped input through the
    rotation) plus one ulp of the element (its own rounding)"""
    p = ref.reshape(*ref.shape[:-1], -1, 2)
    r = p.pow(2).sum(-1, keepdim=True).sqrt().expand_as(p).reshape(ref.shape)
    return 1.4143 * _bf16_ulp(r) + _bf16_ulp(ref)


def _check_roped(got, ref):
    got = got.float().cpu()
    ref = ref.float().cpu()
    d = (got - ref).abs()
    assert bool((d <= _pair_bound(ref)).all()), d.max().item()
    assert (d == 0).float().mean().item() >= 0.99
    assert d.pow(2).mean().sqrt().item() <= 0.01 * ref.pow(2).mean().sqrt().item()


def _reference(x, wq, ws, b, nw, f, eps, dequant, heads_roped):
    """oracle: the projection, then rms_rope over its first heads_roped heads"""
    y = O.int8_linear(x, wq, ws, b, out_dtype=torch.bfloat16, dequant=dequant)
    m, n = y.shape
    s = f.shape[0]
    yr = y[:, : heads_roped * 128].reshape(m // s, s, heads_roped, 128)
    rq, _ = O.rms_rope(yr, None, f, nw, None, eps)
    return y, rq.reshape(m, heads_roped * 128)


@pytest.mark.parametrize("dequant", ["eager", "scale_product", "chained"])
@pytest.mark.parametrize("shape", [(600, 512, 768), (300, 1024, 384), (1000, 256, 128)])
def test_fused_rms_rope_matches_oracle(dequant, shape):
    m, k, n = shape
    g, x, wq, ws, b = _case(m, k, n, sum(shape))
    s = 100 if m % 100 == 0 else m
    f = _freqs(s, g)
    nw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    got = W().int8_linear_rms_rope(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda()),
                                   nw.to(cuda()), f.to(cuda()), 1e-6, dequant=dequant)
    _, ref = _reference(x, wq, ws, b, nw, f, 1e-6, dequant, n // 128)
    assert got.dtype == torch.bfloat16 and got.shape == (m, n)
    _check_roped(got, ref)
    assert W().device_error() == 0


def test_fused_rms_rope_equals_gemm_then_rms_rope():
    """The fused epilogue against the library's own two-kernel form."""
    m, k, n = 512, 768, 1024
    g, x, wq, ws, b = _case(m, k, n, 7)
    f = _freqs(256, g)
    nw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    xd, wd, wsd, bd, nwd, fd = (t.to(cuda()) for t in (x, wq, ws, b, nw, f))
    got = W().int8_linear_rms_rope(xd, wd, wsd, bd, nwd, fd, 1e-5)
    y = W().int8_linear(xd, wd, wsd, bd)
    two, _ = W().rms_rope(y.view(2, 256, n // 128, 128), None, fd, nwd, None, 1e-5)
    _check_roped(got, two.reshape(m, n))


def test_fused_qkv_per_column_norm_and_plain_v():
    """One GEMM for q, k and v: q_norm on the q heads, k_norm on the k heads
    (a per-column norm weight), v columns stored as the plain GEMM stores them."""
    h = 3
    m, k, n = 400, 512, 3 * h * 128
    g, x, wq, ws, b = _case(m, k, n, 11)
    f = _freqs(200, g)
    qn = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    nw = torch.cat([qn.repeat(h), kn.repeat(h)])
    got = W().int8_linear_rms_rope(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda()),
                                   nw.to(cuda()), f.to(cuda()), 1e-6, rope_cols=2 * h * 128)
    y = O.int8_linear(x, wq, ws, b, out_dtype=torch.bfloat16)
    qr, kr = O.rms_rope(y[:, : h * 128].reshape(2, 200, h, 128),
                        y[:, h * 128: 2 * h * 128].reshape(2, 200, h, 128), f, qn, kn, 1e-6)
    got = got.cpu()
    _check_roped(got[:, : h * 128], qr.reshape(m, -1))
    _check_roped(got[:, h * 128: 2 * h * 128], kr.reshape(m, -1))
    assert torch.equal(got[:, 2 * h * 128:], y[:, 2 * h * 128:])  # v: bit-exact
    assert W().device_error() == 0


@pytest.mark.parametrize("config", [(128, 8, 0, 1), (256, 8, 0, 1), (256, 4, 37, 1)])
def test_fused_rms_rope_tile_configs(config):
    m, k, n = 700, 640, 512
    g, x, wq, ws, b = _case(m, k, n, 13, bias=False)
    f = _freqs(700, g)
    nw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    got = W().int8_linear_rms_rope(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), None,
                                   nw.to(cuda()), f.to(cuda()), 1e-6, config=config)
    _, ref = _reference(x, wq, ws, None, nw, f, 1e-6, "eager", n // 128)
    _check_roped(got, ref)


@pytest.mark.parametrize("split_k", [None, 3])
def test_fused_rms_rope_split_k(split_k):
    """Few-row shape: K is split across CTAs (None: chosen from the SM count);
    the last split to arrive runs the norm and rotation."""
    m, k, n = 256, 3072, 768
    g, x, wq, ws, b = _case(m, k, n, 17)
    f = _freqs(256, g)
    nw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    args = (x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda()), nw.to(cuda()), f.to(cuda()))
    got = W().int8_linear_rms_rope(*args, 1e-6, split_k=split_k)
    unsplit = W().int8_linear_rms_rope(*args, 1e-6, split_k=1)
    _, ref = _reference(x, wq, ws, b, nw, f, 1e-6, "eager", n // 128)
    _check_roped(got, ref)
    assert torch.equal(got, unsplit)  # the summed int32 accumulators are exact
    again = W().int8_linear_rms_rope(*args, 1e-6, split_k=split_k)  # scratch left zeroed
    assert torch.equal(again, got)
    assert W().device_error() == 0


def test_fused_rms_rope_ragged_rows_and_empty():
    m, k, n = 131, 256, 256
    g, x, wq, ws, b = _case(m, k, n, 19)
    f = _freqs(131, g)
    nw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    got = W().int8_linear_rms_rope(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda()),
                                   nw.to(cuda()), f.to(cuda()), 1e-6)
    _, ref = _reference(x, wq, ws, b, nw, f, 1e-6, "eager", n // 128)
    _check_roped(got, ref)
    empty = W().int8_linear_rms_rope(torch.zeros(0, k, dtype=torch.bfloat16, device=cuda()),
                                     wq.to(cuda()), ws.to(cuda()), None, nw.to(cuda()),
                                     f.to(cuda()), 1e-6)
    assert empty.shape == (0, n)


def test_fused_rms_rope_errors():
    g, x, wq, ws, b = _case(64, 256, 384, 23)
    xd, wd, wsd = x.to(cuda()), wq.to(cuda()), ws.to(cuda())
    f = _freqs(64, g).to(cuda())
    nw = torch.ones(128, dtype=torch.bfloat16, device=cuda())
    with pytest.raises(ValueError):  # rope_cols not a multiple of the head
        W().int8_linear_rms_rope(xd, wd, wsd, None, nw, f, rope_cols=200)
    with pytest.raises(ValueError):  # norm weight of neither 128 nor rope_cols values
        W().int8_linear_rms_rope(xd, wd, wsd, None, torch.ones(100, device=cuda()), f)
    with pytest.raises(ValueError):  # 64 rows cannot take 48 positions
        W().int8_linear_rms_rope(xd, wd, wsd, None, nw, f[:48])
    w2 = torch.zeros(200, 256, dtype=torch.int8, device=cuda())
    with pytest.raises(ValueError):  # N not a multiple of 128
        W().int8_linear_rms_rope(xd, w2, torch.ones(200, device=cuda()), None, nw, f)


def test_fused_rms_rope_full_size():
    """The Q projection of a 5600-token image stream (two sequences of 2800
    positions), 3072 -> 3072 = 24 heads: against the two-kernel form on every
    row and the oracle on the last 200 rows."""
    m, k, n = 5600, 3072, 3072
    g, x, wq, ws, b = _case(m, k, n, 29)
    f = _freqs(2800, g)
    nw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    args = (x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda()), nw.to(cuda()), f.to(cuda()))
    got = W().int8_linear_rms_rope(*args, 1e-6)
    y = W().int8_linear(*args[:4])
    two, _ = W().rms_rope(y.view(2, 2800, 24, 128), None, args[5], args[4], None, 1e-6)
    _check_roped(got, two.reshape(m, n))
    rows = slice(m - 200, m)
    _, ref = _reference(x[rows], wq, ws, b, nw, f[-200:], 1e-6, "eager", n // 128)
    _check_roped(got[rows], ref)
    assert W().device_error() == 0


def test_rope_freqs_rows_layout():
    """w8a8_rope_freqs_rows: out[((r / 32) * 64 + p) * 32 + r % 32] = the
    rotation of pair p at position r % S, over rows padded to 128."""
    g = torch.Generator().manual_seed(31)
    s, rows = 90, 270
    f = _freqs(s, g)
    fr = W().rope_freqs_rows(f.to(cuda()), rows).cpu().view(-1, 64, 32, 4)
    pad = -(-rows // 128) * 128
    assert fr.shape[0] * 32 == pad
    r = torch.arange(pad)
    want = f.reshape(s, 64, 4)[r % s]                       # [pad, 64, 4]
    got = fr.permute(0, 2, 1, 3).reshape(pad, 64, 4)        # row-major again
    assert torch.equal(got, want)
    with pytest.raises(ValueError):
        W().rope_freqs_rows(f.to(cuda()), 100)  # 100 rows cannot take 90 positions
