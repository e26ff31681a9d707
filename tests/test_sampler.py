"""Sampler step loop: host logic on CPU (schedule, CFG = 1 shortcut, C-ABI
argument checks) and the fused CUDA step against the oracle's replay of the
reference's ATen operations (GPU tests, bit-exact).

Reference: inference/src/models/qwen_image21/sampling.rs (schedule, flow
parameterisation, cfg_combine, Euler), cfg.rs:136-207 (full-area CFG),
er_sde.rs (ER-SDE), server/qwen.rs:170-230 (how the server drives them)."""
import ctypes
import math

import pytest
import torch

from oracle import sampler as O


def S():
    from imagine_b200 import sampler

    return sampler


def N():
    from imagine_b200 import _native

    return _native


# ------------------------------------------------------------------ CPU
def test_schedule_matches_oracle():
    fs, fo = S().FluxSampling(), O.FluxSampling()
    assert torch.equal(fs.sigmas, fo.sigmas)
    for steps in (1, 8, 20, 50):
        assert torch.equal(fs.simple(steps), fo.simple(steps))
    assert fs.percent_to_sigma(1e-4) == fo.percent_to_sigma(1e-4)
    assert fs.percent_to_sigma(0.0) == 1.0 and fs.percent_to_sigma(1.0) == 0.0
    # normal / sgm_uniform end on 0 and decrease from sigma(1) = 1
    for sgm in (False, True):
        s = fs.normal(10, sgm)
        assert s[-1] == 0 and float(s[0]) == pytest.approx(1.0, abs=1e-6)
        assert bool((s[1:] <= s[:-1]).all())


@pytest.mark.parametrize("scale,disabled,want", [
    (1.0, False, True), (1.0 + 1e-10, False, True), (1.0, True, False), (2.5, False, False),
    (float("nan"), False, False), (float("inf"), False, False)])
def test_cfg1_shortcut(scale, disabled, want):
    assert S().cfg1_shortcut(scale, disabled) is want
    assert O.cfg1_shortcut(scale, disabled) is want


def test_sampler_step_argument_errors():
    n = N()
    lib = n.LIB
    st = n.SamplerStep(n.STEP_EULER, 1, 0, 0, 2.5, 1.0)
    # unknown mode, ER-SDE stage out of range, missing buffers: refused before any launch
    bad = n.SamplerStep(7, 1, 0, 0, 1.0, 1.0)
    assert lib.w8a8_sampler_step(0x1000, 0x2000, None, n.BF16, 16, 0x3000, ctypes.byref(bad),
                                 None, None, None, None, None) == n.ERR_VALUE
    er = n.SamplerStep(n.STEP_ER_SDE, 4, 0, 0, 1.0, 1.0)
    assert lib.w8a8_sampler_step(0x1000, 0x2000, None, n.BF16, 16, 0x3000, ctypes.byref(er),
                                 None, 0x4000, 0x5000, None, None) == n.ERR_VALUE
    er2 = n.SamplerStep(n.STEP_ER_SDE, 2, 0, 0, 1.0, 1.0)
    assert lib.w8a8_sampler_step(0x1000, 0x2000, None, n.BF16, 16, 0x3000, ctypes.byref(er2),
                                 None, 0x4000, None, None, None) == n.ERR_VALUE
    assert b"old_derivative" in lib.w8a8_last_error()
    er3 = n.SamplerStep(n.STEP_ER_SDE, 1, 0, 1, 1.0, 1.0)
    assert lib.w8a8_sampler_step(0x1000, 0x2000, None, n.BF16, 16, 0x3000, ctypes.byref(er3),
                                 None, 0x4000, None, None, None) == n.ERR_VALUE  # noise missing
    assert lib.w8a8_sampler_step(0x1000, None, None, n.BF16, 16, 0x3000, ctypes.byref(st),
                                 None, None, None, None, None) == n.ERR_VALUE  # model output
    assert lib.w8a8_sampler_step(0x1000, 0x2000, None, n.S8, 16, 0x3000, ctypes.byref(st),
                                 None, None, None, None, None) == n.ERR_VALUE  # int dtype
    assert lib.w8a8_sampler_step(0x1000, 0x2000, None, n.BF16, -1, 0x3000, ctypes.byref(st),
                                 None, None, None, None, None) == n.ERR_VALUE
    # an empty latent is a no-op
    assert lib.w8a8_sampler_step(None, None, None, n.BF16, 0, None, ctypes.byref(st),
                                 None, None, None, None, None) == n.OK


# ------------------------------------------------------------------ GPU
def _model(dtype, a=0.61, b=-0.23):
    """A stand-in for the DiT: branch outputs that are the same function of
    (x, timestep) on the CPU and the GPU, bit for bit (one fp32 multiply, one
    add, one rounding to the output dtype)."""
    def model(x, ts, with_uncond):
        t = ts.reshape(-1, *([1] * (x.dim() - 1)))
        c = x.mul(a).add(t.mul(0.5)).to(dtype)
        u = x.mul(b).sub(t).to(dtype) if with_uncond else None
        return c, u
    return model


def _latent(seed=0, shape=(2, 16, 28, 50)):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g)


def _noises(shape, count, seed=7):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(shape, generator=g) for _ in range(count)]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("cfg", [2.5, 1.0])
@pytest.mark.parametrize("churn", [0.0, 0.4])
def test_euler_bit_exact(dtype, cfg, churn):
    dev = torch.device("cuda", 0)
    sigmas = S().FluxSampling().simple(8)
    x0 = _latent()
    noises = _noises(x0.shape, 8)
    it_o, it_g = iter(noises), iter(noises)
    dens_o, dens_g = [], []
    ref = O.sample_euler(x0.clone(), sigmas, O.cfg_denoiser(_model(dtype), cfg),
                         O.EulerSettings(churn=churn),
                         noise_like=lambda x: next(it_o),
                         callback=lambda i, d: dens_o.append(d.clone()))
    got = S().sample_euler(x0.to(dev), sigmas, _model(dtype), cfg,
                           S().EulerSettings(churn=churn),
                           noise_like=lambda x: next(it_g).to(dev),
                           callback=lambda i, d: dens_g.append(d.cpu()))
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), ref)
    assert len(dens_o) == len(dens_g) == 8
    for a, b in zip(dens_o, dens_g):
        assert torch.equal(a, b)


@pytest.mark.gpu
@pytest.mark.parametrize("cfg", [2.5, 1.0])
@pytest.mark.parametrize("noise", [1.0, 0.0])
@pytest.mark.parametrize("steps", [8, 2])
def test_er_sde_bit_exact(cfg, noise, steps):
    """Scalars on the CPU (as the oracle computes them): the latent trajectory
    equals the reference's operations bit for bit, stages 1-3 included."""
    dev = torch.device("cuda", 0)
    fs = S().FluxSampling()
    sigmas = fs.simple(steps)
    x0 = _latent(1)
    noises = _noises(x0.shape, steps)
    it_o, it_g = iter(noises), iter(noises)
    ref = O.sample_er_sde(x0.clone(), sigmas, O.FluxSampling(),
                          O.cfg_denoiser(_model(torch.bfloat16), cfg),
                          O.ErSdeSettings(noise=noise), noise_like=lambda x: next(it_o))
    got = S().sample_er_sde(x0.to(dev), sigmas, fs, _model(torch.bfloat16), cfg,
                            S().ErSdeSettings(noise=noise), noise_like=lambda x: next(it_g).to(dev))
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), ref)


@pytest.mark.gpu
def test_er_sde_device_sigmas_close():
    """Sigmas on the GPU (the server's placement): the scalars come from ATen's
    CUDA exp / pow / logit / sum, which may differ from the CPU's in the last
    bit, so the latent agrees to fp32 rounding level rather than bit for bit.
    (An fp32 stand-in model: with bf16 outputs one flipped rounding of an
    output element moves it by 2^-8 of itself, which the CFG scale amplifies.)"""
    dev = torch.device("cuda", 0)
    fs = S().FluxSampling()
    sigmas = fs.simple(10)
    x0 = _latent(2)
    noises = _noises(x0.shape, 10)
    it_o, it_g = iter(noises), iter(noises)
    ref = O.sample_er_sde(x0.clone(), sigmas, O.FluxSampling(),
                          O.cfg_denoiser(_model(torch.float32), 3.0),
                          noise_like=lambda x: next(it_o))
    got = S().sample_er_sde(x0.to(dev), sigmas.to(dev), fs, _model(torch.float32), 3.0,
                            noise_like=lambda x: next(it_g).to(dev))
    err = (got.cpu() - ref).abs().max().item()
    assert err <= 1e-5 * ref.abs().max().item()


@pytest.mark.gpu
def test_denoised_mode_and_empty():
    dev = torch.device("cuda", 0)
    n = N()
    x = _latent(3).to(dev)
    oc = torch.randn(x.shape, device=dev).to(torch.bfloat16)
    ou = torch.randn(x.shape, device=dev).to(torch.bfloat16)
    sigma = torch.tensor([0.73], device=dev)
    den = torch.empty_like(x)
    S().sampler_step(x, oc, ou, sigma, n.STEP_DENOISED, cfg_scale=4.0, denoised=den)
    ts = sigma.expand(x.shape[0])
    ref = O.full_area_cfg(x.cpu(), ts.cpu(), lambda *_: (oc.cpu(), ou.cpu()), 4.0)
    assert torch.equal(den.cpu(), ref)
    # negative zero: 0 - 0 * sigma with cond only -> +0 after the aggregation
    z = torch.full((4,), -0.0, device=dev)
    d2 = torch.empty_like(z)
    S().sampler_step(z, torch.zeros(4, device=dev), None, sigma, n.STEP_DENOISED, denoised=d2)
    assert not torch.signbit(d2).any()
    e = torch.empty(0, device=dev)
    S().sampler_step(e, e, None, sigma, n.STEP_EULER)


# ------------------------------------------- the reference's recorded runs
def _fixture():
    from tests import test_oracle_sampler as F

    return F


def _gen(dev_case, seed):
    d = "cuda" if dev_case.startswith("cuda") else "cpu"
    return d, torch.Generator(device=d).manual_seed(seed)


def _fx_cases(key):
    F = _fixture()
    return [c for c in F.FIX[key] if c["dtype"] == "torch.float32"]


@pytest.mark.gpu
@pytest.mark.parametrize("case", _fx_cases("euler"), ids=lambda c: f"{c['device']}-churn{c['churn']}")
def test_euler_matches_recorded_runs(case):
    """The reference's Euler solver runs (qwen_sampling.rs:290-327): flow
    parameterisation of the stand-in model, churn with seeded noise; final
    latent and every step's denoised equal the recorded digests."""
    F = _fixture()
    dev = torch.device("cuda", 0)
    gdev, g = _gen(case["device"], 17)
    sigmas = S().FluxSampling().simple(4).to(gdev)
    dens = []
    got = S().sample_euler(
        F.data(torch.float32, 3).to(dev), sigmas, lambda x, ts, wu: (F.stand_in(x, ts), None), 1.0,
        S().EulerSettings(churn=case["churn"], tmin=0.2, tmax=0.95, noise=0.875),
        noise_like=lambda x: torch.randn(x.shape, generator=g, device=gdev).to(dev),
        callback=lambda i, d: dens.append(d.clone()))
    F.check(got, case["output"], "Euler final")
    assert len(dens) == len(case["denoised"])
    for d, want in zip(dens, case["denoised"]):
        F.check(d, want, "Euler denoised")


@pytest.mark.gpu
@pytest.mark.parametrize("case", _fx_cases("er_sde"),
                         ids=lambda c: f"{c['device']}-st{c['max_stage']}-n{c['noise']}-"
                                       f"{'err' if c['error'] else c['steps']}")
def test_er_sde_matches_recorded_runs(case):
    """The reference's ER-SDE runs (qwen_sampling.rs:155-215): stages 0-4,
    noise scales 0 / 0.875 / 1, the interior-zero-sigma error; the execution
    returns the denoised prediction itself."""
    F = _fixture()
    dev = torch.device("cuda", 0)
    gdev, g = _gen(case["device"], 18 if case["device"] == "cpu" else 17)
    noises, dens = [], []

    def noise_like(x):
        n = torch.randn(x.shape, generator=g, device=gdev)
        noises.append(n)
        return n.to(dev)

    run = lambda: S().sample_er_sde(
        F.data(torch.float32, 3).to(dev), F.er_sde_sigmas(case, gdev), S().FluxSampling(),
        lambda x, ts, wu: (F.stand_in(x, ts), None), 1.0,
        S().ErSdeSettings(noise=case["noise"], max_stage=case["max_stage"]),
        noise_like=noise_like, callback=lambda i, d: dens.append(d.clone()), prediction="denoised")
    if case["error"]:
        with pytest.raises(TypeError, match="unsupported operand"):
            run()
    else:
        F.check(run(), case["output"], "ER-SDE final")
    assert len(noises) == len(case["noises"])
    for n, want in zip(noises, case["noises"]):
        F.check(n, want, "ER-SDE noise")
    for d, want in zip(dens, case["denoised"]):
        F.check(d, want, "ER-SDE denoised")
