"""The Qwen-Image sampling loop around the denoiser, with one fused CUDA pass per step.

The reference's loop (inference/src/models/qwen_image21/sampling.rs:231-277 for
Euler, er_sde.rs:29-137 for ER-SDE; the server picks one,
inference/src/server/qwen.rs:226-230) runs, per step, the model on both CFG
branches, the flow parameterisation of each output (sampling.rs:165-167),
the full-area aggregation and ``cfg_combine`` (cfg.rs:136-207,
sampling.rs:178-180) and the sampler's update of the latent, as a chain of
ATen elementwise operations.  Here everything after the model is ONE kernel
(``w8a8_sampler_step``): it reads the latent and the two model outputs once and
writes the new latent (and the ER-SDE multistep state).

The per-step scalars (sigma_hat, dt, the ER-SDE coefficients) do not depend on
the latent: they are computed once, before the loop, with the reference's own
0-dim tensor operations in its order, on the device the sigmas live on (the
server moves them to the GPU, qwen.rs:188), and handed to the kernel as one
fp32 row per step.  With the same model outputs the latents equal the
reference's bit for bit (every fp32 operation in the kernel rounds once, in
ATen's order).

The model interface: ``model(x, timestep, with_uncond)`` returns the raw
outputs of the conditional and unconditional branches (any float dtype, x's
shape; the second is None when ``with_uncond`` is False, the CFG = 1 shortcut
of sampling.rs:195-200).  With ``prediction="denoised"`` the model instead
returns the denoised prediction itself (an execution whose ``denoise`` already
applied its parameterisation and CFG) and None.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Callable, Optional, Tuple

import torch

from . import _native as N
from .linear import _code, _cuda, _stream, _vp

Model = Callable[[torch.Tensor, torch.Tensor, bool], Tuple[torch.Tensor, Optional[torch.Tensor]]]


class FluxSampling:
    """The FLUX/CONST schedule of Qwen-Image 2.1 (sampling.rs:5-62, :121-158):
    10000 shifted sigmas (shift 0.69) and the ``simple`` / ``normal`` /
    ``sgm_uniform`` step lists."""

    def __init__(self, shift: float = 0.69, timesteps: int = 10000):
        self.shift = shift
        self.sigmas = self.sigma(torch.arange(1, timesteps + 1, dtype=torch.int64).div(timesteps))

    def sigma(self, t: torch.Tensor) -> torch.Tensor:
        e = math.exp(self.shift)
        return t.reciprocal().mul(1).sub(1).pow(1.0).add(e).reciprocal().mul(e)

    def percent_to_sigma(self, percent: float) -> float:
        if percent <= 0.0:
            return 1.0
        if percent >= 1.0:
            return 0.0
        e = math.exp(self.shift)
        return e / (e + (1.0 / (1.0 - percent) - 1.0) ** 1.0)

    def simple(self, steps: int) -> torch.Tensor:
        size = self.sigmas.shape[0]
        ss = size / steps
        vals = [float(self.sigmas[size - (1 + int(i * ss))]) for i in range(steps)] + [0.0]
        return torch.tensor(vals, dtype=torch.float32)

    def normal(self, steps: int, sgm: bool = False) -> torch.Tensor:
        size = self.sigmas.shape[0]
        start, end = float(self.sigmas[size - 1]), float(self.sigmas[0])
        append = sgm or abs(float(self.sigma(torch.tensor([end], dtype=torch.float32))[0])) > 0.00001
        if not append:
            steps += 1
        t = torch.linspace(start, end, steps + int(sgm), dtype=torch.float32)
        if sgm:
            t = t[:steps]
        vals = [float(self.sigma(t[i])) for i in range(t.shape[0])]
        if append:
            vals.append(0.0)
        return torch.tensor(vals, dtype=torch.float32)


def cfg1_shortcut(scale: float, disabled: bool = False) -> bool:
    """sampling.rs:195-200 (math.isclose with rel_tol 1e-9)."""
    return (not disabled and math.isfinite(scale)
            and (scale == 1.0 or abs(scale - 1.0) <= 1e-9 * max(abs(scale), 1.0)))


def sampler_step(x: torch.Tensor, out_cond: Optional[torch.Tensor], out_uncond: Optional[torch.Tensor],
                 coef: torch.Tensor, mode: int, *, cfg_scale: float = 1.0, stage: int = 1,
                 last: bool = False, s_noise: float = 1.0, denoised: Optional[torch.Tensor] = None,
                 old_denoised: Optional[torch.Tensor] = None,
                 old_derivative: Optional[torch.Tensor] = None,
                 noise: Optional[torch.Tensor] = None, denoised_input: bool = False) -> None:
    """One ``w8a8_sampler_step`` launch on x (fp32, updated in place)."""
    _cuda("x", x)
    dev = x.device
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise ValueError("the latent must be a contiguous float32 tensor")
    n = x.numel()

    def same(name, t, dtype=None):
        if t is None:
            return None
        _cuda(name, t, dev)
        if t.numel() != n or not t.is_contiguous() or (dtype is not None and t.dtype != dtype):
            raise ValueError(f"{name} must be a contiguous tensor of {n} elements"
                             + (f" ({dtype})" if dtype is not None else ""))
        return t

    oc = same("out_cond", out_cond)
    ou = same("out_uncond", out_uncond)
    if oc is not None and ou is not None and ou.dtype != oc.dtype:
        raise ValueError("the two branches' outputs must share a dtype")
    step = N.SamplerStep(mode, stage, int(last), int(noise is not None and mode == N.STEP_ER_SDE),
                         float(cfg_scale), float(s_noise), int(denoised_input))
    code = _code(oc.dtype) if oc is not None else N.F32
    N.check(N.LIB.w8a8_sampler_step(
        _vp(x), _vp(oc), _vp(ou), code, n, _vp(coef), ctypes.byref(step),
        _vp(same("denoised", denoised, torch.float32)),
        _vp(same("old_denoised", old_denoised, torch.float32)),
        _vp(same("old_derivative", old_derivative, torch.float32)),
        _vp(same("noise", noise, torch.float32)), _stream(dev)))


def cfg_parallel_model(branch_model: Callable[[torch.Tensor, torch.Tensor, int], torch.Tensor],
                       group=None) -> Model:
    """A ``Model`` whose two CFG branches run on the two ranks of ``group``:
    rank 0 evaluates the conditional branch, rank 1 the unconditional one
    (``branch_model(x, timestep, branch)``), and one all-gather of the outputs
    gives every rank both, so each rank's sampler step computes the same latent.
    The reference batches the two branches on one device instead
    (cfg.rs:170-200); the combine that follows is the same.  Under the CFG = 1
    shortcut both ranks evaluate the conditional branch and nothing is
    exchanged."""
    import torch.distributed as dist

    def model(x, timestep, with_uncond):
        if not with_uncond:
            return branch_model(x, timestep, 0), None
        if dist.get_world_size(group) != 2:
            raise ValueError("CFG-parallel sampling runs on a group of two ranks")
        mine = branch_model(x, timestep, dist.get_rank(group)).contiguous()
        both = [torch.empty_like(mine), torch.empty_like(mine)]
        dist.all_gather(both, mine, group=group)
        return both[0], both[1]

    return model


# ---------------------------------------------------------------- Euler
@dataclass
class EulerSettings:
    """sampling.rs:201-217."""
    churn: float = 0.0
    tmin: float = 0.0
    tmax: float = math.inf
    noise: float = 1.0


def euler_coefficients(sigmas: torch.Tensor, settings: EulerSettings = EulerSettings()):
    """Per step i: (gamma, churn row [1] or None, step row [sigma_hat, sigma_hat,
    sigma_next - sigma_hat]) with sampling.rs:236-270's operations on the
    sigmas' device."""
    steps = sigmas.shape[0] - 1
    out = []
    for i in range(steps):
        s = sigmas[i]
        gamma = (min(settings.churn / steps, math.sqrt(2.0) - 1.0)
                 if settings.churn > 0.0 and settings.tmin <= float(s) <= settings.tmax else 0.0)
        hat = s.mul(gamma + 1.0) if settings.churn > 0.0 else s
        churn = hat.pow(2).sub(s.pow(2)).pow(0.5).reshape(1) if gamma > 0.0 else None
        row = torch.stack([hat, hat, sigmas[i + 1].sub(hat)])
        out.append((gamma, churn, row))
    return out


def _branches(prediction: str, cfg_scale: float, disable_cfg1_optimization: bool) -> bool:
    if prediction not in ("flow", "denoised"):
        raise ValueError(f"prediction must be 'flow' or 'denoised', got {prediction!r}")
    return prediction == "flow" and not cfg1_shortcut(cfg_scale, disable_cfg1_optimization)


def sample_euler(x: torch.Tensor, sigmas: torch.Tensor, model: Model, cfg_scale: float = 1.0,
                 settings: EulerSettings = EulerSettings(),
                 noise_like: Optional[Callable[[torch.Tensor], torch.Tensor]] = None,
                 callback=None, disable_cfg1_optimization: bool = False,
                 prediction: str = "flow") -> torch.Tensor:
    """sampling.rs:231-277 with the denoiser of denoiser.rs:139-157; returns the
    final latent (a new fp32 tensor).  ``callback(i, denoised)`` sees each
    step's CFG-combined prediction."""
    x = _cuda("x", x).to(torch.float32).contiguous().clone()
    coefs = [(g, c.to(x.device) if c is not None else None, r.to(x.device))
             for g, c, r in euler_coefficients(sigmas, settings)]
    with_uncond = _branches(prediction, cfg_scale, disable_cfg1_optimization)
    raw = prediction == "denoised"
    den = torch.empty_like(x) if callback is not None else None
    s_in = torch.ones(x.shape[0], dtype=torch.float32, device=x.device)
    for i, (gamma, churn, row) in enumerate(coefs):
        if gamma > 0.0:
            sampler_step(x, None, None, churn, N.STEP_CHURN, s_noise=settings.noise,
                         noise=noise_like(x).to(torch.float32).contiguous())
        out_c, out_u = model(x, row[0].mul(s_in), with_uncond)
        sampler_step(x, out_c.contiguous(), out_u.contiguous() if with_uncond else None, row,
                     N.STEP_EULER, cfg_scale=cfg_scale, denoised=den, denoised_input=raw)
        if callback is not None:
            callback(i, den)
    return x


# ---------------------------------------------------------------- ER-SDE
@dataclass
class ErSdeSettings:
    """er_sde.rs:6-17."""
    noise: float = 1.0
    max_stage: int = 3


def _noise_scaler(v: torch.Tensor) -> torch.Tensor:
    return v.mul(v.pow(0.3).exp().add(10.0))


def er_sde_coefficients(sigmas: torch.Tensor, sampling: FluxSampling,
                        settings: ErSdeSettings = ErSdeSettings()):
    """Per step i: (stage, last, row of the 9 scalars w8a8_sampler_step reads)
    with er_sde.rs:45-134's 0-dim operations on the sigmas' device."""
    points = torch.arange(0.0, 200.0, dtype=torch.float32, device=sigmas.device)
    if sigmas.shape[0] > 1 and float(sigmas[0]) >= 1.0:
        sigmas = sigmas.clone()
        sigmas[0].fill_(sampling.percent_to_sigma(1e-4))
    lambdas = sigmas.logit().neg().neg().exp()
    zero = torch.zeros((), dtype=torch.float32, device=sigmas.device)
    out = []
    for i in range(sigmas.shape[0] - 1):
        sigma, nxt = sigmas[i], sigmas[i + 1]
        stage = min(settings.max_stage, i + 1)
        last = float(nxt) == 0.0
        row = [sigma] + [zero] * 8
        if not last:
            s, t = lambdas[i], lambdas[i + 1]
            alpha_t = nxt.div(t)
            r_alpha = alpha_t.div(sigma.div(s))
            ns_t = _noise_scaler(t)
            r = ns_t.div(_noise_scaler(s))
            row[1] = r_alpha.mul(r)
            row[2] = alpha_t.mul(torch.rsub(r, 1.0))
            if stage >= 2:
                dt = t.sub(s)
                step = dt.neg().div(200.0)
                positions = t.add(points.mul(step))
                scaled = _noise_scaler(positions)
                integral = scaled.reciprocal().mul(1.0).sum().mul(step)
                row[3] = alpha_t.mul(dt.add(integral.mul(_noise_scaler(t))))
                row[4] = s.sub(lambdas[i - 1])
                if stage >= 3:
                    integral_u = positions.sub(s).div(scaled).sum().mul(step)
                    row[5] = alpha_t.mul(dt.pow(2).div(2).add(integral_u.mul(_noise_scaler(t))))
                    row[6] = s.sub(lambdas[i - 2]).div(2)
            row[7] = alpha_t
            if settings.noise > 0.0:
                row[8] = t.pow(2).sub(s.pow(2).mul(r.pow(2))).sqrt().nan_to_num(0.0)
        out.append((stage, last, torch.stack(row)))
    return out


def sample_er_sde(x: torch.Tensor, sigmas: torch.Tensor, sampling: FluxSampling, model: Model,
                  cfg_scale: float = 1.0, settings: ErSdeSettings = ErSdeSettings(),
                  noise_like: Optional[Callable[[torch.Tensor], torch.Tensor]] = None,
                  callback=None, disable_cfg1_optimization: bool = False,
                  prediction: str = "flow") -> torch.Tensor:
    """er_sde.rs:29-137 (``sample_er_sde``, CONST/FLUX path); returns the final
    latent.  ``noise_like(x)`` must draw the reference's noise stream (its
    seeded generator); it is called once per non-final step when
    ``settings.noise > 0``.  Raises the reference's TypeError when a stage-3
    step finds no previous derivative (an interior zero sigma,
    er_sde.rs:21-26)."""
    x = _cuda("x", x).to(torch.float32).contiguous().clone()
    rows = [(st, last, r.to(x.device)) for st, last, r in er_sde_coefficients(sigmas, sampling, settings)]
    with_uncond = _branches(prediction, cfg_scale, disable_cfg1_optimization)
    raw = prediction == "denoised"
    old_den = torch.empty_like(x)
    old_der = torch.empty_like(x)
    have_der = False
    den = torch.empty_like(x) if callback is not None else None
    s_in = torch.ones(x.shape[0], dtype=torch.float32, device=x.device)
    for i, (stage, last, row) in enumerate(rows):
        out_c, out_u = model(x, row[0].mul(s_in), with_uncond)
        if not last and stage >= 3 and not have_der:
            if callback is not None:
                sampler_step(x, out_c.contiguous(), out_u.contiguous() if with_uncond else None,
                             row, N.STEP_DENOISED, cfg_scale=cfg_scale, denoised=den,
                             denoised_input=raw)
                callback(i, den)
            raise TypeError("unsupported operand type(s) for -: 'Tensor' and 'NoneType'")
        noise = None
        if not last and settings.noise > 0.0:
            # the reference draws in the shape and dtype of the initial latent
            noise = noise_like(x).to(torch.float32).contiguous()
        # stages 0 and 1 take the same update, as do 3 and above
        sampler_step(x, out_c.contiguous(), out_u.contiguous() if with_uncond else None, row,
                     N.STEP_ER_SDE, cfg_scale=cfg_scale, stage=max(1, min(3, stage)), last=last,
                     s_noise=settings.noise, denoised=den, old_denoised=old_den,
                     old_derivative=old_der, noise=noise, denoised_input=raw)
        have_der = have_der or (not last and stage >= 2)
        if callback is not None:
            callback(i, den)
    return x
