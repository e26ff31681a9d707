"""GPU parity of libw8a8 (called through its C ABI) against the CPU oracle and
the reference's golden vectors.

Bars: int8 codes, row scales and int32 accumulators are
bit-exact; bf16/f16/f32 outputs of the dequant orders that the oracle restates
exactly are bit-exact too, and everything involving transcendental functions
or a different summation order is held to max-abs-error <= 1% of output RMS.
"""
import numpy as np
import pytest
import torch

from oracle import eager as O
from tests import _golden as G

pytestmark = pytest.mark.gpu

RMS_TOL = 0.01  # max |y - ref| <= 1% of rms(ref)


def W():
    import imagine_b200

    return imagine_b200


def cuda():
    return torch.device("cuda", 0)


def _b(t):
    return O.as_bytes(t.cpu())


def _half_ulp(ref: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Half a unit in the last place of `dtype` at |ref| (0 for fp32)."""
    if dtype == torch.float32:
        return torch.zeros_like(ref)
    mant = {torch.bfloat16: 8, torch.float16: 11}[dtype]
    e = torch.floor(torch.log2(ref.abs().clamp(min=1e-30)))
    return torch.pow(2.0, e - mant)


def assert_rms_close(y, ref, tol=RMS_TOL):
    """max |y - ref| <= tol * rms(ref), after discounting the output dtype's own
    rounding of each element (half an ulp of y's dtype at |ref|): a bf16 output
    cannot represent a large element of a heavy-tailed result closer than that,
    whatever the arithmetic before the final rounding."""
    dtype = y.dtype
    y = y.float().cpu()
    ref = ref.float().cpu()
    rms = ref.pow(2).mean().sqrt().item()
    err = ((y - ref).abs() - _half_ulp(ref, dtype)).clamp(min=0).max().item()
    assert err <= tol * max(rms, 1e-12), f"max abs err {err} > {tol} * rms {rms}"


def no_device_error():
    assert W().device_error() == 0


# ---------------------------------------------------------------- quantiser
KE = G.load("kitchen_eager")
MAN = G.manifest()


@pytest.mark.parametrize("name", [n for n in MAN["kitchen_eager"] if n.startswith("quant/")])
def test_quantize_rowwise_golden(name):
    dt = G.DT[name.split("/")[-1]]
    x = G.tensor(KE[name + "/x"], dt).to(cuda())
    q, s = W().quantize_int8_rowwise(x)
    assert np.array_equal(_b(q), KE[name + "/q"].view(np.uint8).reshape(-1))
    assert np.array_equal(_b(s), KE[name + "/s"].view(np.uint8).reshape(-1))


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(5600, 3072), (256, 12288), (3, 40000), (7, 1001), (1, 8), (130, 24)])
def test_quantize_rowwise_random(dt, shape):
    g = torch.Generator().manual_seed(sum(shape))
    x = (torch.randn(*shape, generator=g) * 4).to(dt)
    x[0, : min(5, shape[1])] = 0
    if shape[0] > 2:
        x[1] = 0
    qg, sg = W().quantize_int8_rowwise(x.to(cuda()))
    qo, so = O.quantize_int8_rowwise(x)
    assert torch.equal(qg.cpu(), qo)
    assert torch.equal(sg.cpu(), so)
    qk, sk = W().quantize_int8_rowwise(x.to(cuda()), scale_mode="kitchen")
    qko, sko = O.quantize_int8_rowwise_kitchen(x)
    assert torch.equal(qk.cpu(), qko)
    assert torch.equal(sk.cpu(), sko)


def test_quantize_3d_input_and_strided_rows():
    x = torch.randn(2, 37, 512, dtype=torch.bfloat16)
    q, s = W().quantize_int8_rowwise(x.to(cuda()))
    qo, so = O.quantize_int8_rowwise(x)
    assert q.shape == (2, 37, 512) and s.shape == (2, 37, 1)
    assert torch.equal(q.cpu(), qo) and torch.equal(s.cpu(), so)


# ---------------------------------------------------------------- int8 GEMM
GEMM_SHAPES = [
    (128, 128, 256),     # one tile
    (300, 3072, 1024),   # M tail, several K blocks
    (130, 160, 264),     # N tail (not a multiple of 256 or 128), K tail inside a block
    (17, 48, 40),        # tiny
    (5600, 3072, 512),   # the image-stream M
    (33, 100, 24),       # K % 16 != 0 -> CUDA-core path
    (4, 0, 16),          # K == 0
]


def _rand_i8(g, *shape):
    return torch.randint(-128, 128, shape, generator=g, dtype=torch.int8)


# (block_n, cta_group): heuristic, 64- and 128-column tiles, 256-column 1-CTA
# tiles, 256x256 tiles on CTA pairs (2-SM MMA)
TILE_CONFIGS = [(0, 0), (64, 1), (128, 1), (256, 1), (256, 2)]


@pytest.mark.parametrize("m,k,n", GEMM_SHAPES)
@pytest.mark.parametrize("bn,cg", TILE_CONFIGS)
def test_gemm_s32_exact(m, k, n, bn, cg):
    g = torch.Generator().manual_seed(m * 7 + k * 3 + n)
    q = _rand_i8(g, m, k)
    w = _rand_i8(g, n, k)
    acc = W().int8_gemm_s32(q.to(cuda()), w.to(cuda()), config=(bn, 8, 0, cg))
    torch.cuda.synchronize()
    no_device_error()
    assert torch.equal(acc.cpu(), O.int8_accumulate(q, w))


@pytest.mark.parametrize("m,k,n", GEMM_SHAPES[:-1])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("cg", [1, 2])
def test_int8_linear_eager_order_bit_exact(m, k, n, out_dtype, cg):
    g = torch.Generator().manual_seed(m + k + n)
    x = torch.randn(m, k, generator=g).to(out_dtype)
    w = (torch.randn(n, k, generator=g) * 0.02).to(out_dtype)
    wq, ws = O.quantize_weight(w)
    b = (torch.randn(n, generator=g) * 0.02).to(out_dtype)
    y = W().int8_linear(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda()), out_dtype=out_dtype,
                        config=(256, 8, 0, cg))
    ref = O.int8_linear(x, wq, ws, b, out_dtype=out_dtype)
    no_device_error()
    assert np.array_equal(_b(y), _b(ref))


@pytest.mark.parametrize("m,k,n", [(256, 3072, 3072), (200, 1024, 520), (64, 512, 96)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_few_row_64_column_tiles_bit_exact(m, k, n, out_dtype):
    """Few-row shapes whose 128-column tiles would leave most SMs idle run on
    64-column tiles (the default there, and asked for explicitly here too):
    bit-exact against the oracle, with GELU and an N tail."""
    g = torch.Generator().manual_seed(m + k + n + 1)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    wq, ws = O.quantize_weight(w)
    b = (torch.randn(n, generator=g) * 0.02).to(out_dtype)
    ref = O.int8_linear(x, wq, ws, b, out_dtype=out_dtype)
    for cfg in (None, (64, 8, 0, 1)):
        y = W().int8_linear(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda()),
                            out_dtype=out_dtype, config=cfg)
        assert np.array_equal(_b(y), _b(ref))
    yg = W().int8_linear(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda()),
                         out_dtype=out_dtype, output_act="gelu_tanh", config=(64, 8, 0, 1))
    assert_rms_close(yg, O.int8_linear(x, wq, ws, b, out_dtype=out_dtype, output_act="gelu_tanh"))
    no_device_error()


@pytest.mark.parametrize("name", [n for n in MAN["kitchen_eager"] if n.startswith("linear/")
                                  and "input_act" not in n and "convrot" not in n])
def test_int8_linear_golden(name):
    dn = [p for p in name.split("_") if p in G.DT][0]
    dt = G.DT[dn]
    x = G.tensor(KE[name + "/x"], dt).to(cuda())
    wq = G.tensor(KE[name + "/wq"], torch.int8).to(cuda())
    ws = G.tensor(KE[name + "/ws"], torch.float32).to(cuda())
    b = G.tensor(KE[name + "/bias"], dt).to(cuda()) if name + "/bias" in KE else None
    kw = {}
    if name + "/residual" in KE:
        kw.update(residual=G.tensor(KE[name + "/residual"], dt).to(cuda()),
                  residual_scale=G.tensor(KE[name + "/residual_scale"], dt).to(cuda()))
    y = W().int8_linear(x, wq, ws, b, out_dtype=dt, **kw)
    ref = G.tensor(KE[name + "/y"], dt)
    if "residual" in name:
        assert_rms_close(y, ref)  # addcmul on the CPU vs one fma on the GPU
        # the linear part before the residual is bit-exact
        y0 = W().int8_linear(x, wq, ws, b, out_dtype=dt)
        r0 = O.int8_linear(x.cpu(), wq.cpu(), ws.cpu(), b.cpu() if b is not None else None, out_dtype=dt)
        assert np.array_equal(_b(y0), _b(r0))
    else:
        assert np.array_equal(_b(y), KE[name + "/y"].view(np.uint8).reshape(-1))
    acc = W().int8_gemm_s32(G.tensor(KE[name + "/xq"], torch.int8).to(cuda()), wq)
    assert np.array_equal(acc.cpu().numpy(), KE[name + "/acc"])


@pytest.mark.parametrize("name", [n for n in MAN["kitchen_eager"] if n.startswith("linear/")
                                  and ("input_act" in n or "convrot" in n)])
def test_int8_linear_golden_input_act_and_convrot(name):
    """Input activations / ConvRot run as device ATen ops before the quantiser
    (as the reference's CUDA route does when it does not fuse them); their
    results may differ from the CPU by an ulp, so the output is held to the
    tolerance bar."""
    dn = [p for p in name.split("_") if p in G.DT][0]
    dt = G.DT[dn]
    x = G.tensor(KE[name + "/x"], dt).to(cuda())
    wq = G.tensor(KE[name + "/wq"], torch.int8).to(cuda())
    ws = G.tensor(KE[name + "/ws"], torch.float32).to(cuda())
    b = G.tensor(KE[name + "/bias"], dt).to(cuda()) if name + "/bias" in KE else None
    kw = {}
    k = wq.shape[1]
    if "input_act" in name:
        if name + "/act_w" in KE:
            kw.update(input_act="rms_norm", input_act_weight=G.tensor(KE[name + "/act_w"], dt).to(cuda()),
                      input_act_eps=1e-6)
        elif x.shape[1] == 2 * k:
            kw.update(input_act="swiglu")
        else:
            kw.update(input_act="gelu_tanh")
    if "convrot" in name:
        kw.update(convrot=True, convrot_groupsize=256)
    y = W().int8_linear(x, wq, ws, b, out_dtype=dt, **kw)
    assert_rms_close(y, G.tensor(KE[name + "/y"], dt))


PROBE = G.load("triton_probe")


@pytest.mark.parametrize("case", MAN["triton_probe"], ids=lambda c: c["name"])
def test_triton_probe_bytes(case):
    """The reference's recorded Triton-route outputs, reproduced by the tcgen05
    GEMM (or the M<=2 GEMV) with kitchen scales and the scale-product epilogue."""
    x, w, ws, b, dt = G.probe_inputs(case)
    y = W().int8_linear(x.to(cuda()), w.to(cuda()), ws.to(cuda()), b.to(cuda()) if b is not None else None,
                        out_dtype=dt, dequant="scale_product", scale_mode="kitchen")
    q, s = W().quantize_int8_rowwise(x.to(cuda()), scale_mode="kitchen")
    assert np.array_equal(_b(q), PROBE[case["name"] + "/q"])
    assert np.array_equal(_b(s), PROBE[case["name"] + "/s"])
    assert np.array_equal(_b(y), PROBE[case["name"] + "/y"])


@pytest.mark.parametrize("order", ["scale_product", "chained"])
@pytest.mark.parametrize("m,k,n", [(300, 3072, 1024), (130, 160, 264), (1, 256, 72), (2, 3072, 520)])
def test_dequant_orders_bit_exact(order, m, k, n):
    g = torch.Generator().manual_seed(11 + m)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    wq = _rand_i8(g, n, k)
    ws = torch.rand(n, generator=g) * 1e-3 + 1e-4
    b = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16)
    y = W().int8_linear(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda()), dequant=order)
    ref = O.int8_linear(x, wq, ws, b, out_dtype=torch.bfloat16, dequant=order)
    assert np.array_equal(_b(y), _b(ref))


@pytest.mark.parametrize("m,k,n", [(300, 3072, 1024), (5600, 3072, 256)])
def test_gelu_epilogue(m, k, n):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    wq, ws = O.quantize_weight(w)
    b = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16)
    y = W().int8_linear(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda()), output_act="gelu_tanh")
    ref = O.int8_linear(x, wq, ws, b, out_dtype=torch.bfloat16, output_act="gelu_tanh")
    assert_rms_close(y, ref)


def test_residual_epilogue():
    g = torch.Generator().manual_seed(9)
    m, k, n = 257, 512, 384
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    wq = _rand_i8(g, n, k)
    ws = torch.rand(n, generator=g) * 1e-3
    r = torch.randn(m, n, generator=g).to(torch.bfloat16)
    rs = torch.rand(n, generator=g).to(torch.bfloat16)
    y = W().int8_linear(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), None, residual=r.to(cuda()),
                        residual_scale=rs.to(cuda()))
    ref = O.int8_linear(x, wq, ws, None, out_dtype=torch.bfloat16, residual=r, residual_scale=rs)
    assert_rms_close(y, ref)


@pytest.mark.parametrize("k", [512, 520, 12288])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_gated_residual_epilogue(k, out_dtype):
    """The model's gated residual (inference/src/models/qwen_image21/numeric.rs:
    110-126) fused into the linear: x [2, S, K], residual [2, S, N] and a
    per-sample gate [2, 1, N] that the reference's addcmul broadcasts
    (inference/src/int8_linear.rs:99-111).  K = 520 takes the CUDA-core path;
    S = 300 puts the sample boundary inside a warp's 32 rows; S = 128 at
    K = 12288 is a few-row shape that takes split-K."""
    g = torch.Generator().manual_seed(k)
    b_, n = 2, 384
    s_ = 128 if k == 12288 else 300
    x = torch.randn(b_, s_, k, generator=g).to(torch.bfloat16)
    wq = _rand_i8(g, n, k)
    ws = torch.rand(n, generator=g) * 1e-3
    bias = (torch.randn(n, generator=g) * 0.1).to(out_dtype)
    r = torch.randn(b_, s_, n, generator=g).to(out_dtype)
    for gate in (torch.randn(b_, 1, n, generator=g).to(out_dtype),      # per sample
                 torch.randn(b_, s_, n, generator=g).to(out_dtype)):    # per row
        y = W().int8_linear(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), bias.to(cuda()),
                            out_dtype=out_dtype, residual=r.to(cuda()), residual_scale=gate.to(cuda()))
        ref = O.int8_linear(x, wq, ws, bias, out_dtype=out_dtype, residual=r, residual_scale=gate)
        assert y.shape == (b_, s_, n)
        assert_rms_close(y, ref)
    no_device_error()


def test_gated_residual_small_m():
    """Two rows (the fused quantise + GEMV launch), one per sample."""
    g = torch.Generator().manual_seed(77)
    k, n = 3072, 1024
    x = torch.randn(2, 1, k, generator=g).to(torch.bfloat16)
    wq = _rand_i8(g, n, k)
    ws = torch.rand(n, generator=g) * 1e-3
    r = torch.randn(2, 1, n, generator=g).to(torch.bfloat16)
    gate = torch.randn(2, 1, n, generator=g).to(torch.bfloat16)
    y = W().int8_linear(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), None, residual=r.to(cuda()),
                        residual_scale=gate.to(cuda()), scale_mode="kitchen", dequant="chained")
    ref = O.int8_linear(x, wq, ws, None, out_dtype=torch.bfloat16, residual=r, residual_scale=gate,
                        dequant="chained")
    assert_rms_close(y, ref, tol=0.02)
    no_device_error()


def test_headline_shape_properties():
    """5600 x 3072 -> 12288 (the MLP-up headline): exact int32 row checksums over
    the whole output, exact rows on a random sample, and the GELU epilogue on
    the sampled rows."""
    g = torch.Generator().manual_seed(0)
    m, k, n = 5600, 3072, 12288
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    wq, ws = O.quantize_weight(w)
    xd = x.to(cuda())
    qd, sd = W().quantize_int8_rowwise(xd)
    acc = W().int8_gemm_s32(qd, wq.to(cuda()))
    q = qd.cpu()
    # checksum of checksums: sum_n acc[m, n] == q[m, :] . colsum(w)
    colsum = wq.to(torch.int64).sum(dim=0)
    want = (q.to(torch.int64) * colsum).sum(dim=1)
    got = acc.to(torch.int64).sum(dim=1).cpu()
    assert torch.equal(got, want)
    rows = torch.randperm(m, generator=g)[:48]
    assert torch.equal(acc[rows.to(cuda())].cpu(), O.int8_accumulate(q[rows], wq))
    y = W().int8_linear(xd, wq.to(cuda()), ws.to(cuda()), None, output_act="gelu_tanh")
    ref = O.int8_linear(x[rows], wq, ws, None, out_dtype=torch.bfloat16, output_act="gelu_tanh")
    assert_rms_close(y[rows.to(cuda())], ref)
    no_device_error()


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_half_width_tail_units(out_dtype):
    """1280 x 512 -> 4096: 160 tiles of 128 x 256 on 148 SMs, so the last 12
    run as 24 half-width units.  Against the same GEMM on 160 CTAs (every tile
    whole, one wave): bit-identical for int32 and every output dtype; the
    oracle on the rows of the half-width tiles."""
    sms = torch.cuda.get_device_properties(cuda()).multi_processor_count
    if sms != 148:
        pytest.skip("tile counts chosen for 148 SMs")
    g = torch.Generator().manual_seed(41)
    m, k, n = 1280, 512, 4096
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n, generator=g) * 0.02).to(out_dtype)
    wq, ws = O.quantize_weight(w)
    xd, wqd, wsd, bd = x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda())
    whole_cfg = (256, 8, 160, 1)
    for act in (None, "gelu_tanh"):
        y = W().int8_linear(xd, wqd, wsd, bd, out_dtype=out_dtype, output_act=act)
        y_whole = W().int8_linear(xd, wqd, wsd, bd, out_dtype=out_dtype, output_act=act,
                                  config=whole_cfg)
        assert torch.equal(y.view(torch.uint8), y_whole.view(torch.uint8))
    qd, _ = W().quantize_int8_rowwise(xd)
    assert torch.equal(W().int8_gemm_s32(qd, wqd), W().int8_gemm_s32(qd, wqd, config=whole_cfg))
    # tile order is grouped by 8 row blocks: the last 12 tiles lie in rows 1024..1279
    rows = torch.arange(1024, 1280, 8)
    y = W().int8_linear(xd, wqd, wsd, bd, out_dtype=out_dtype)
    ref = O.int8_linear(x[rows], wq, ws, b, out_dtype=out_dtype)
    assert np.array_equal(_b(y[rows.to(cuda())]), _b(ref))
    no_device_error()


def test_half_width_tail_units_fp8():
    sms = torch.cuda.get_device_properties(cuda()).multi_processor_count
    if sms != 148:
        pytest.skip("tile counts chosen for 148 SMs")
    g = torch.Generator().manual_seed(43)
    m, k, n = 1280, 512, 4096
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    sa = (x.abs().max().float() / 448).reshape(1)
    sw = (w.abs().max().float() / 448).reshape(1)
    aq = W().quantize_per_tensor_fp8(x.to(cuda()), sa.to(cuda()))
    wq = W().quantize_per_tensor_fp8(w.to(cuda()), sw.to(cuda()))
    y = W().fp8_linear(aq, sa.to(cuda()), wq, sw.to(cuda()), None)
    rows = torch.arange(1024, 1280, 4)
    assert_rms_close(y[rows.to(cuda())],
                     O.fp8_linear_exact(aq.cpu()[rows], sa, wq.cpu(), sw, None, out_dtype=torch.float32))
    no_device_error()


# ---------------------------------------------------------------- GEMV (M <= 2)
@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("k,n", [(3072, 18432), (64, 24), (48, 40), (100, 36)])
def test_gemv_exact(m, k, n):
    g = torch.Generator().manual_seed(m * 1000 + k + n)
    q = _rand_i8(g, m, k)
    wq = _rand_i8(g, n, k)
    xs = torch.rand(m, generator=g) * 0.01
    ws = torch.rand(n, generator=g) * 1e-3
    b = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16)
    y = W().int8_gemv(q.to(cuda()), wq.to(cuda()), xs.to(cuda()), ws.to(cuda()), b.to(cuda()))
    ref = O.int8_gemv(q, wq, xs, ws, b, torch.bfloat16)
    assert np.array_equal(_b(y), _b(ref))


@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("k,n", [(3072, 18432), (64, 24), (100, 36)])
def test_fused_small_linear_matches_eager(m, dt, k, n):
    """a5: SiLU(temb) [2, 3072] -> 18432 through one fused quantise+GEMV launch."""
    g = torch.Generator().manual_seed(m + k + n)
    x = torch.nn.functional.silu(torch.randn(m, k, generator=g)).to(dt)
    w = (torch.randn(n, k, generator=g) * 0.02).to(dt)
    wq, ws = O.quantize_weight(w)
    b = (torch.randn(n, generator=g) * 0.02).to(dt)
    y = W().int8_linear(x.to(cuda()), wq.to(cuda()), ws.to(cuda()), b.to(cuda()), out_dtype=dt)
    ref = O.int8_linear(x, wq, ws, b, out_dtype=dt)
    assert np.array_equal(_b(y), _b(ref))


# ---------------------------------------------------------------- FP8
@pytest.mark.parametrize("name", [n for n in MAN["kitchen_eager"] if n.startswith("fp8")])
def test_fp8_quantize_golden(name):
    dt = G.DT[name.split("/")[-1]]
    x = G.tensor(KE[name + "/x"], dt).to(cuda())
    s = G.tensor(KE[name + "/scale"], torch.float32).to(cuda())
    q = W().quantize_per_tensor_fp8(x, s)
    assert np.array_equal(_b(q), KE[name + "/q"].reshape(-1))


@pytest.mark.parametrize("m,k,n", [(300, 3072, 1024), (5600, 3072, 512), (130, 160, 264), (33, 100, 24)])
@pytest.mark.parametrize("cg", [1, 2])
def test_fp8_linear(m, k, n, cg):
    g = torch.Generator().manual_seed(m + n)
    x = torch.randn(m, k, generator=g)
    x = torch.where(torch.rand(m, k, generator=g) < 0.01, x * 20, x).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    sa = (x.abs().max().float() / 448).reshape(1)
    sw = (w.abs().max().float() / 448).reshape(1)
    b = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16)
    aq = W().quantize_per_tensor_fp8(x.to(cuda()), sa.to(cuda()))
    wq = W().quantize_per_tensor_fp8(w.to(cuda()), sw.to(cuda()))
    assert np.array_equal(_b(aq), _b(O.quantize_fp8(x, sa)))
    y = W().fp8_linear(aq, sa.to(cuda()), wq, sw.to(cuda()), b.to(cuda()), config=(256, 8, 0, cg))
    no_device_error()
    # against the unrounded fp32 result (a bf16 rounding flip on a large element
    # is up to one ulp, which two independently rounded outputs can double)
    assert_rms_close(y, O.fp8_linear_exact(aq.cpu(), sa, wq.cpu(), sw, b, out_dtype=torch.float32))
    # and against the reference's own fallback (bf16-dequantised operands)
    assert_rms_close(y, O.fp8_linear(aq.cpu(), sa, wq.cpu(), sw, b), tol=0.03)


# ---------------------------------------------------------------- MXFP8
@pytest.mark.parametrize("name", [n for n in MAN["kitchen_eager"] if n.startswith("mxfp8/")])
def test_mxfp8_quantize_golden(name):
    dt = G.DT[name.split("/")[-1]]
    x = G.tensor(KE[name + "/x"], dt).to(cuda())
    p, sf = W().quantize_mxfp8(x)
    assert np.array_equal(_b(p), KE[name + "/q"].reshape(-1))
    assert np.array_equal(_b(sf), KE[name + "/sf"].reshape(-1))


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("m,k", [(5600, 3072), (130, 160), (1, 32), (257, 4096)])
def test_mxfp8_quantize_random(dt, m, k):
    g = torch.Generator().manual_seed(m + k)
    x = torch.randn(m, k, generator=g)
    x = torch.where(torch.rand(m, k, generator=g) < 0.01, x * 20, x).to(dt)
    x[0, :32] = 0
    p, sf = W().quantize_mxfp8(x.to(cuda()))
    po, sfo = O.quantize_mxfp8(x)
    assert np.array_equal(_b(sf), _b(sfo))
    assert np.array_equal(_b(p), _b(po))


@pytest.mark.parametrize("cta_group", [1, 2])
@pytest.mark.parametrize("m,k,n", [(300, 3072, 256), (130, 160, 264), (128, 256, 128),
                                   (1000, 1024, 640)])
def test_mxfp8_linear(m, k, n, cta_group):
    """One CTA per 128 x 128 tile, and CTA pairs (256 x 128 tiles; rows of the
    last pair past M, columns past N)."""
    g = torch.Generator().manual_seed(m + k + n)
    x = torch.randn(m, k, generator=g)
    x = torch.where(torch.rand(m, k, generator=g) < 0.01, x * 20, x).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16)
    aq, asf = W().quantize_mxfp8(x.to(cuda()))
    wq, wsf = W().quantize_mxfp8(w.to(cuda()))
    y = W().mxfp8_linear(aq, asf, wq, wsf, b.to(cuda()), config=(0, 8, 0, cta_group))
    no_device_error()
    ref = O.mxfp8_linear(aq.cpu(), asf.cpu(), wq.cpu(), wsf.cpu(), b, out_dtype=torch.float32)
    assert_rms_close(y, ref)


@pytest.mark.parametrize("max_ctas", [0, 3])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("m,k,n", [(300, 3072, 1024), (130, 160, 520), (1000, 1024, 640),
                                   (777, 512, 2304)])
def test_mxfp8_linear_256_columns(m, k, n, out_dtype, max_ctas):
    """256-column MXFP8 tiles on three 128-column TMEM regions (even tiles in
    regions 0-1, odd tiles in 1-2, the shared region handed back first).
    max_ctas = 3 makes every CTA run many tiles, so both placements and every
    barrier phase occur; N tails included."""
    g = torch.Generator().manual_seed(m + k + n + max_ctas)
    x = torch.randn(m, k, generator=g)
    x = torch.where(torch.rand(m, k, generator=g) < 0.01, x * 20, x).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n, generator=g) * 0.02).to(out_dtype)
    aq, asf = W().quantize_mxfp8(x.to(cuda()))
    wq, wsf = W().quantize_mxfp8(w.to(cuda()))
    y = W().mxfp8_linear(aq, asf, wq, wsf, b.to(cuda()), out_dtype=out_dtype,
                         config=(256, 8, max_ctas, 1))
    no_device_error()
    ref = O.mxfp8_linear(aq.cpu(), asf.cpu(), wq.cpu(), wsf.cpu(), b, out_dtype=torch.float32)
    assert_rms_close(y, ref)
    # the 128-column tiles give the same values (fp32 sums of the same MMAs;
    # only the tile shape differs)
    y128 = W().mxfp8_linear(aq, asf, wq, wsf, b.to(cuda()), out_dtype=out_dtype,
                            config=(128, 8, 0, 1))
    assert torch.equal(y.view(torch.int16 if out_dtype == torch.bfloat16 else torch.int32),
                       y128.view(torch.int16 if out_dtype == torch.bfloat16 else torch.int32))
