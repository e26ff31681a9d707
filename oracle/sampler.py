"""CPU oracle for the sampler step loop -- TEST INFRASTRUCTURE ONLY.

Restates, tensor operation for tensor operation, the reference's Qwen-Image
sampling loop: the FLUX/CONST schedule, the flow parameterisation of the
model output, the full-area CFG aggregation and combine, and the Euler and
ER-SDE samplers.  The reference issues these operations through tch, i.e.
the same ATen library torch exposes, so replaying them here in the same order
reproduces its arithmetic (the reference pins torch 2.13.0,
native/comfy-port/reference-lock.json:21; the elementwise and 0-dim
operations used are unchanged across those versions).  Only ``tests/`` may
import this module.

File references are relative to the reference repository root,
``Q = inference/src/models/qwen_image21``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional, Tuple

import torch


# ---------------------------------------------------------------- schedule
class FluxSampling:
    """Q/sampling.rs:5-50 (shift_time, sigma, percent_to_sigma) and :51-62
    (simple)."""

    def __init__(self, shift: float = 0.69, timesteps: int = 10000):
        self.shift = shift
        t = torch.arange(1, timesteps + 1, dtype=torch.int64).div(timesteps)
        self.sigmas = self.shift_time(shift, t)

    @staticmethod
    def shift_time(mu: float, t: torch.Tensor) -> torch.Tensor:
        e = math.exp(mu)
        return t.reciprocal().mul(1).sub(1).pow(1.0).add(e).reciprocal().mul(e)

    def percent_to_sigma(self, percent: float) -> float:
        if percent <= 0.0:
            return 1.0
        if percent >= 1.0:
            return 0.0
        t = 1.0 - percent
        e = math.exp(self.shift)
        return e / (e + (1.0 / t - 1.0) ** 1.0)

    def sigma(self, t: torch.Tensor) -> torch.Tensor:
        return self.shift_time(self.shift, t)

    def simple(self, steps: int) -> torch.Tensor:
        size = self.sigmas.shape[0]
        ss = size / steps
        values = [float(self.sigmas[size - (1 + int(i * ss))]) for i in range(steps)]
        values.append(0.0)
        return torch.tensor(values, dtype=torch.float32)

    def normal(self, steps: int, sgm: bool) -> torch.Tensor:
        """Q/sampling.rs:121-158 (``normal`` and ``sgm_uniform``)."""
        size = self.sigmas.shape[0]
        start = float(self.sigmas[size - 1])
        end = float(self.sigmas[0])
        append = sgm or abs(float(self.sigma(torch.tensor([end], dtype=torch.float32))[0])) > 0.00001
        if not append:
            steps += 1
        t = torch.linspace(start, end, steps + int(sgm), dtype=torch.float32)
        if sgm:
            t = t.narrow(0, 0, steps)
        values = [float(self.sigma(t[i])) for i in range(t.shape[0])]
        if append:
            values.append(0.0)
        return torch.tensor(values, dtype=torch.float32)


# ------------------------------------------------------- denoise and CFG
def append_sigma(sigma: torch.Tensor, rank: int) -> torch.Tensor:
    """Q/sampling.rs:160-164."""
    shape = list(sigma.shape)
    shape += [1] * (rank - len(shape))
    return sigma.reshape(shape)


def flow_denoised(sigma: torch.Tensor, output: torch.Tensor, inp: torch.Tensor) -> torch.Tensor:
    """Q/sampling.rs:165-167 (the model output cast to float first,
    Q/denoiser.rs:131-135)."""
    return inp.sub(output.mul(append_sigma(sigma, output.dim())))


def cfg_combine(cond: torch.Tensor, uncond: torch.Tensor, scale: float) -> torch.Tensor:
    """Q/sampling.rs:178-180."""
    return uncond.add(cond.sub(uncond).mul(scale))


def flow_noise_scaling(sigma: torch.Tensor, noise: torch.Tensor, latent: torch.Tensor,
                       noise_scale: float) -> torch.Tensor:
    """Q/sampling.rs:168-176."""
    s = append_sigma(sigma, noise.dim())
    return s.mul(noise.mul(noise_scale)).add(s.neg().add(1).mul(latent))


def flow_inverse_noise_scaling(sigma: torch.Tensor, latent: torch.Tensor) -> torch.Tensor:
    """Q/sampling.rs:177-183."""
    return latent.div(append_sigma(sigma, latent.dim()).neg().add(1))


def cfg1_shortcut(scale: float, disabled: bool) -> bool:
    """Q/sampling.rs:195-200."""
    return (not disabled and math.isfinite(scale)
            and (scale == 1.0 or abs(scale - 1.0) <= 1e-9 * max(abs(scale), 1.0)))


Model = Callable[[torch.Tensor, torch.Tensor, bool], Tuple[torch.Tensor, Optional[torch.Tensor]]]
Denoise = Callable[[torch.Tensor, torch.Tensor], torch.Tensor]


def full_area_cfg(x: torch.Tensor, timestep: torch.Tensor, model: Model, scale: float,
                  disable_cfg1_optimization: bool = False) -> torch.Tensor:
    """Q/cfg.rs:136-207 for one full-area positive and negative condition that
    are evaluated in one batch: outputs and counts aggregated with the
    reference's operations (zeros, + out * 1, / (1e-37 + 1)), then
    cfg_combine.  ``model(x, timestep, with_uncond)`` returns the raw model
    outputs of the two branches (uncond None without the negative)."""
    with_uncond = not cfg1_shortcut(scale, disable_cfg1_optimization)
    out_c, out_u = model(x, timestep, with_uncond)
    outputs = [torch.zeros_like(x), torch.zeros_like(x)]
    counts = [torch.ones_like(x).mul(1e-37), torch.ones_like(x).mul(1e-37)]
    mult = torch.ones_like(x).mul(1.0)
    branches = [(0, out_c)] + ([(1, out_u)] if with_uncond else [])
    for b, out in branches:
        den = flow_denoised(timestep, out.to(torch.float32), x)
        outputs[b].add_(den.mul(mult))
        counts[b].add_(mult)
    outputs[0].div_(counts[0])
    outputs[1].div_(counts[1])
    return cfg_combine(outputs[0], outputs[1], scale)


def cfg_denoiser(model: Model, scale: float, disable_cfg1_optimization: bool = False) -> Denoise:
    """The Qwen denoiser's ``denoise`` (Q/denoiser.rs:139-157): full_area_cfg
    over the model's two branches."""
    return lambda x, sigma: full_area_cfg(x, sigma, model, scale, disable_cfg1_optimization)


# ------------------------------------------------------------------ Euler
@dataclass
class EulerSettings:
    """Q/sampling.rs:201-217."""
    churn: float = 0.0
    tmin: float = 0.0
    tmax: float = math.inf
    noise: float = 1.0


def sample_euler(x: torch.Tensor, sigmas: torch.Tensor, denoise: Denoise,
                 settings: EulerSettings = EulerSettings(),
                 noise_like: Optional[Callable[[torch.Tensor], torch.Tensor]] = None,
                 callback=None) -> torch.Tensor:
    """Q/sampling.rs:231-277; ``denoise(x, sigma)`` is the execution's
    (e.g. ``cfg_denoiser``)."""
    s_in = torch.ones(x.shape[0], dtype=x.dtype, device=x.device)
    steps = sigmas.shape[0] - 1
    for i in range(steps):
        s = sigmas[i]
        if settings.churn > 0.0 and settings.tmin <= float(s) <= settings.tmax:
            gamma = min(settings.churn / steps, math.sqrt(2.0) - 1.0)
        else:
            gamma = 0.0
        hat = s.mul(gamma + 1.0) if settings.churn > 0.0 else s
        if gamma > 0.0:
            eps = noise_like(x).mul(settings.noise)
            x = x.add(eps.mul(hat.pow(2).sub(s.pow(2)).pow(0.5)))
        denoised = denoise(x, hat.mul(s_in))
        d = x.sub(denoised).div(append_sigma(hat, x.dim()))
        if callback is not None:
            callback(i, denoised)
        dt = sigmas[i + 1].sub(hat)
        x = x.add(d.mul(dt))
    return x


# ----------------------------------------------------------------- ER-SDE
@dataclass
class ErSdeSettings:
    """Q/er_sde.rs:6-17."""
    noise: float = 1.0
    max_stage: int = 3


def noise_scaler(x: torch.Tensor) -> torch.Tensor:
    """Q/er_sde.rs:18-20."""
    return x.mul(x.pow(0.3).exp().add(10.0))


def _previous(value: Optional[torch.Tensor]) -> torch.Tensor:
    """Q/er_sde.rs:21-26."""
    if value is None:
        raise TypeError("unsupported operand type(s) for -: 'Tensor' and 'NoneType'")
    return value


def sample_er_sde(x: torch.Tensor, sigmas: torch.Tensor, sampling: FluxSampling, denoise: Denoise,
                  settings: ErSdeSettings = ErSdeSettings(),
                  noise_like: Optional[Callable[[torch.Tensor], torch.Tensor]] = None,
                  callback=None) -> torch.Tensor:
    """Q/er_sde.rs:29-137; ``denoise(x, sigma)`` is the execution's."""
    noise_template = x
    s_in = torch.ones(x.shape[0], dtype=x.dtype, device=x.device)
    points = torch.arange(0.0, 200.0, dtype=torch.float32, device=x.device)
    if sigmas.shape[0] > 1 and float(sigmas[0]) >= 1.0:
        sigmas = sigmas.clone()
        sigmas[0].fill_(sampling.percent_to_sigma(1e-4))
    half_log_snrs = sigmas.logit().neg()
    lambdas = half_log_snrs.neg().exp()
    old_denoised = None
    old_derivative = None
    for i in range(sigmas.shape[0] - 1):
        sigma = sigmas[i]
        next_sigma = sigmas[i + 1]
        denoised = denoise(x, sigma.mul(s_in))
        if callback is not None:
            callback(i, denoised)
        stage = min(settings.max_stage, i + 1)
        if float(next_sigma) == 0.0:
            x = denoised
        else:
            s = lambdas[i]
            t = lambdas[i + 1]
            alpha_s = sigma.div(s)
            alpha_t = next_sigma.div(t)
            r_alpha = alpha_t.div(alpha_s)
            r = noise_scaler(t).div(noise_scaler(s))
            x = r_alpha.mul(r).mul(x).add(alpha_t.mul(torch.rsub(r, 1.0)).mul(denoised))
            if stage >= 2:
                dt = t.sub(s)
                step = dt.neg().div(200.0)
                positions = t.add(points.mul(step))
                scaled = noise_scaler(positions)
                integral = scaled.reciprocal().mul(1.0).sum().mul(step)
                derivative = denoised.sub(_previous(old_denoised)).div(s.sub(lambdas[i - 1]))
                x = x.add(alpha_t.mul(dt.add(integral.mul(noise_scaler(t)))).mul(derivative))
                if stage >= 3:
                    integral_u = positions.sub(s).div(scaled).sum().mul(step)
                    second = derivative.sub(_previous(old_derivative)).div(s.sub(lambdas[i - 2]).div(2))
                    x = x.add(alpha_t.mul(dt.pow(2).div(2).add(integral_u.mul(noise_scaler(t))))
                              .mul(second))
                old_derivative = derivative
            if settings.noise > 0.0:
                deviation = t.pow(2).sub(s.pow(2).mul(r.pow(2))).sqrt().nan_to_num(0.0)
                x = x.add(alpha_t.mul(noise_like(noise_template)).mul(settings.noise)
                          .mul(deviation))
        old_denoised = denoised
    return x
