"""The sampler oracle pinned to the reference's golden vectors.

tests/golden/sampler_fixture.json holds the SHA-256 digests the reference's
sampler tests check (inference/tests/support/qwen_sampling.rs, fixtures
qwen-image21-sampling.json and qwen-image21-er-sde.json, recorded from the
original ComfyUI sampler); tests/golden/make_sampler_golden.py extracted them.
Each case is rebuilt here exactly as that harness builds it (its `data`
inputs, its stand-in model x * 0.125 + sigma * 0.25, its seeded generators)
and the oracle's outputs must hash to the recorded digests.  The GPU tests in
test_sampler.py run the same cases through the CUDA sampler step."""
import hashlib
import json
import os

import pytest
import torch

from oracle import sampler as O

FIX = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "sampler_fixture.json")))
DT = {"torch.float32": torch.float32, "torch.bfloat16": torch.bfloat16,
      "torch.float16": torch.float16}


def sha(t: torch.Tensor) -> str:
    t = t.detach().cpu().contiguous()
    if t.element_size() == 2:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def check(t, want, note=""):
    assert list(t.shape) == want["shape"], note
    assert str(t.dtype) == want["dtype"], note
    assert sha(t) == want["sha256"], note


def data(dtype, offset, dev="cpu"):
    """qwen_sampling.rs:10-22."""
    return (torch.arange(2 * 64 * 2 * 3, dtype=torch.float32, device=dev).add(offset)
            .remainder(29).mul(0.03125).sub(0.40625).reshape(2, 64, 2, 3).to(dtype))


def randn_like(x, g):
    """The harness's noise draw, ``at::randn(shape, generator, dtype)``
    (inference/native/bridge.cpp:574-577).  For 16-bit dtypes on the CPU the
    torch that recorded the fixtures drew fp32 normals and rounded them (the
    recorded digests match that); the torch here draws 16-bit normals
    differently, so the draw is written out as fp32 then a cast."""
    if x.dtype in (torch.bfloat16, torch.float16) and x.device.type == "cpu":
        return torch.randn(x.shape, generator=g).to(x.dtype)
    return torch.randn(x.shape, dtype=x.dtype, generator=g, device=x.device)


def stand_in(x, sigma):
    """The harness's model output (qwen_sampling.rs:45-47)."""
    return x.mul(0.125).add(sigma.view(2, 1, 1, 1).mul(0.25))


def test_schedules():
    for g in FIX["schedules"]:
        fs = O.FluxSampling(g["shift"], 10000)
        check(fs.sigmas, g["sigmas"], f"sigmas {g['shift']}")
        for c in g["cases"]:
            y = fs.simple(c["steps"]) if c["method"] == "simple" else \
                fs.normal(c["steps"], c["method"] == "sgm_uniform")
            check(y, c["output"], f"{g['shift']}/{c['method']}/{c['steps']}")


@pytest.mark.parametrize("case", [c for c in FIX["algebra"] if c["device"] == "cpu"],
                         ids=lambda c: f"{c['dtype']}-{c['scale']}")
def test_flow_algebra(case):
    dt = DT[case["dtype"]]
    x, noise, out = data(dt, 3), data(dt, 5), data(dt, 7)
    sigma = torch.tensor([0.85, 0.35], dtype=torch.float32)
    check(O.flow_denoised(sigma, out, x), case["denoised"])
    check(O.flow_noise_scaling(sigma, noise, x, 1.0), case["noise"])
    check(O.flow_inverse_noise_scaling(sigma, x), case["inverse"])
    check(O.cfg_combine(out, noise, case["scale"]), case["cfg"])


def test_seeded_noise():
    for c in FIX["noises"]:
        g = torch.Generator().manual_seed(c["seed"])
        check(torch.randn(2, 64, 2, 3, generator=g).to(DT[c["dtype"]]), c["output"])


@pytest.mark.parametrize("case", [c for c in FIX["euler"] if c["device"] == "cpu"],
                         ids=lambda c: f"{c['dtype']}-churn{c['churn']}")
def test_euler(case):
    dt = DT[case["dtype"]]
    g = torch.Generator().manual_seed(17)
    dens = []
    y = O.sample_euler(
        data(dt, 3), O.FluxSampling().simple(4),
        lambda x, s: O.flow_denoised(s, stand_in(x, s), x),
        O.EulerSettings(churn=case["churn"], tmin=0.2, tmax=0.95, noise=0.875),
        noise_like=lambda x: randn_like(x, g),
        callback=lambda i, d: dens.append(d))
    check(y, case["output"], "Euler final")
    assert len(dens) == len(case["denoised"])
    for d, want in zip(dens, case["denoised"]):
        check(d, want, "Euler denoised")


def er_sde_sigmas(case, dev="cpu"):
    if case["explicit_sigmas"] is not None:
        s = torch.tensor([float(v) for v in case["explicit_sigmas"]], dtype=torch.float32)
    else:
        s = O.FluxSampling().simple(case["steps"])
    s = s.to(dev)
    s[0].fill_(case["first"])
    return s


@pytest.mark.parametrize("case", [c for c in FIX["er_sde"] if c["device"] == "cpu"],
                         ids=lambda c: f"{c['dtype']}-st{c['max_stage']}-n{c['noise']}-"
                                       f"{'err' if c['error'] else c['steps']}")
def test_er_sde(case):
    dt = DT[case["dtype"]]
    g = torch.Generator().manual_seed(18)
    noises, dens = [], []

    def noise_like(x):
        n = randn_like(x, g)
        noises.append(n)
        return n

    def denoise(x, s):
        out = stand_in(x, s)
        return out.to(torch.float32) if case["float_output"] else out

    run = lambda: O.sample_er_sde(
        data(dt, 3), er_sde_sigmas(case), O.FluxSampling(), denoise,
        O.ErSdeSettings(noise=case["noise"], max_stage=case["max_stage"]),
        noise_like=noise_like, callback=lambda i, d: dens.append(d))
    if case["error"]:
        with pytest.raises(TypeError, match=case["error"]["message"].replace("(", r"\(")
                           .replace(")", r"\)")):
            run()
    else:
        check(run(), case["output"], "ER-SDE final")
    assert len(noises) == len(case["noises"])
    for n, want in zip(noises, case["noises"]):
        check(n, want, "ER-SDE noise")
    for d, want in zip(dens, case["denoised"]):
        check(d, want, "ER-SDE denoised")
