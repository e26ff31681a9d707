"""GPU parity of rms_rope (w8a8_rms_rope) against the eager oracle
(inference/src/backend_rope.rs:146-223 restated in oracle/eager.py).

Bar: the head's fp32 sum of squares is added in a different order than
torch's CPU cascade sum, so 1/rms can differ in its last bit.  fp32 outputs
are held to max-abs-error <= 1% of output RMS; 16-bit outputs only move where
the fp32 value sits on a rounding boundary: a flipped normalised value moves
both outputs of its pair through the rotation (|f| <= 1).  They are held to
sqrt(2) ulps of the pair's magnitude plus one ulp of the element, >= 99%
identical, and an error RMS <= 1% of the output RMS (a max-abs bound of 1% of
RMS cannot hold for a normalised 16-bit output: one bf16 ulp at |y| >= 2 RMS
is 1.56% of RMS)."""
import pytest
import torch

from oracle import eager as O

pytestmark = pytest.mark.gpu


def W():
    import imagine_b200

    return imagine_b200


def cuda():
    return torch.device("cuda", 0)


def _freqs(s, d, g):
    """Rotation matrices of the reference's RoPE (cos, -sin; sin, cos) at
    seeded angles: [S, D/2, 2, 2] fp32."""
    ang = torch.rand(s, d // 2, generator=g, dtype=torch.float64) * 6.283
    c, sn = torch.cos(ang), torch.sin(ang)
    return torch.stack([torch.stack([c, -sn], -1), torch.stack([sn, c], -1)], -2).float()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("with_k", [True, False])
def test_rms_rope_matches_eager(dtype, d, with_k):
    g = torch.Generator().manual_seed(d)
    b, s, h = 2, 37, 5
    q = (torch.randn(b, s, h, d, generator=g) * 2).to(dtype)
    k = (torch.randn(b, s, h, d, generator=g) * 2).to(dtype)
    qs = (1 + 0.1 * torch.randn(d, generator=g)).to(dtype)
    ks = (1 + 0.1 * torch.randn(d, generator=g)).to(dtype)
    f = _freqs(s, d, g)
    qo, ko = W().rms_rope(q.to(cuda()), k.to(cuda()) if with_k else None, f.to(cuda()),
                          qs.to(cuda()), ks.to(cuda()) if with_k else None, 1e-6)
    rq, rk = O.rms_rope(q, k if with_k else None, f, qs, ks, 1e-6)
    pairs = [(qo, rq)] + ([(ko, rk)] if with_k else [])
    assert (ko is None) == (not with_k)
    for got, ref in pairs:
        got = got.float().cpu()
        ref = ref.float()
        rms = ref.pow(2).mean().sqrt().item()
        d = (got - ref).abs()
        if dtype == torch.float32:
            assert d.max().item() <= 0.01 * rms
        else:
            bits = 8 if dtype == torch.bfloat16 else 11

            def ulp(v):
                _, e = torch.frexp(v)
                return torch.ldexp(torch.ones_like(v), e - bits)
            p = ref.reshape(*ref.shape[:-1], -1, 2)
            r = p.pow(2).sum(-1, keepdim=True).sqrt().expand_as(p).reshape(ref.shape)
            assert bool((d <= 1.4143 * ulp(r) + ulp(ref)).all()), d.max().item()
            assert (d == 0).float().mean().item() >= 0.99
            assert d.pow(2).mean().sqrt().item() <= 0.01 * rms
    assert W().device_error() == 0


def test_rms_rope_in_qkv_layout():
    """q and k as column slices of one QKV projection output (row stride 3 H D),
    freqs per token of a batch-two sequence."""
    g = torch.Generator().manual_seed(5)
    b, s, h, d = 2, 50, 24, 128
    qkv = torch.randn(b * s, 3 * h * d, generator=g).to(torch.bfloat16).to(cuda())
    q = qkv[:, : h * d].view(b, s, h, d)
    k = qkv[:, h * d: 2 * h * d].view(b, s, h, d)
    qs = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    ks = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    f = _freqs(s, d, g)
    rq, rk = O.rms_rope(q.cpu(), k.cpu(), f, qs, ks, 1e-6)
    qo, ko = W().rms_rope(q, k, f.to(cuda()), qs.to(cuda()), ks.to(cuda()), 1e-6)
    for got, ref in [(qo, rq), (ko, rk)]:
        d_ = (got.float().cpu() - ref.float()).abs()
        assert (d_ == 0).float().mean().item() >= 0.99
        assert d_.max().item() <= 2 ** -6 * max(ref.float().abs().max().item(), 1.0)


def test_rms_rope_errors():
    q = torch.zeros(2, 3, 4, 96, dtype=torch.bfloat16, device=cuda())
    f = torch.zeros(3, 48, 2, 2, device=cuda())
    with pytest.raises(ValueError):
        W().rms_rope(q, None, f, torch.ones(96, device=cuda()))
    q = torch.zeros(2, 3, 4, 128, dtype=torch.bfloat16, device=cuda())
    with pytest.raises(ValueError):
        W().rms_rope(q, None, torch.zeros(4, 64, 2, 2, device=cuda()), torch.ones(128, device=cuda()))
