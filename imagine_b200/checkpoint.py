"""Quantised linear layers from a checkpoint's state dict.

The reference's loader (inference/src/checkpoint/quantized.rs:111-300, extra
keys :430-445) reads, for each quantised linear with key prefix ``P``:

* ``P.weight``       the payload: int8 [N, K], float8_e4m3fn [N, K], or the
                     MXFP8 e4m3 payload;
* ``P.weight_scale`` the weight scale (int8: per output channel or one value;
                     fp8: one value; mxfp8: the blocked e8m0 scales);
* ``P.comfy_quant``  a uint8 tensor holding JSON metadata: ``format``
                     (``int8_tensorwise`` / ``float8_e4m3fn`` / ``mxfp8`` here),
                     ``convrot`` and ``convrot_groupsize`` (also accepted under
                     ``params``), ``full_precision_matrix_mult``;
* ``P.input_scale``  (fp8 / mxfp8, optional) the static activation scale;
* ``P.bias``         (optional).

Each layer becomes a :class:`QuantizedLinear` whose call runs the matching
operator of this package, as the reference's ``Linear::forward``
(inference/src/models/qwen_image21/layers.rs:78-160) does: INT8 layouts
quantise the activation inside ``int8_linear`` (per token, ConvRot when the
weight was rotated); FP8 quantises it per tensor with ``input_scale`` (1 when
absent); MXFP8 quantises it in 32-element blocks.  A layer whose metadata asks
for full-precision matrix multiplication keeps its payload and is reported as
such; running it is outside this package (the W8A8 path only).
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from typing import Dict, Optional

import torch

FORMATS = ("int8_tensorwise", "float8_e4m3fn", "mxfp8")


def read_quant_config(conf: torch.Tensor) -> dict:
    """The JSON held by a ``comfy_quant`` tensor (its bytes, any integer dtype)."""
    if conf.device.type != "cpu":
        # the reference decodes the bytes on the host and refuses device tensors
        raise TypeError("can't convert cuda:0 device type tensor to numpy. Use Tensor.cpu() to "
                        "copy the tensor to host memory first.")
    raw = conf.contiguous().reshape(-1).view(torch.uint8).numpy().tobytes()
    try:
        meta = json.loads(raw)
    except ValueError as e:
        raise ValueError(f"comfy_quant metadata is not JSON: {e}") from None
    if not isinstance(meta, dict):
        raise ValueError("comfy_quant metadata must be a JSON object")
    return meta


def quant_config_tensor(meta: dict) -> torch.Tensor:
    """A ``comfy_quant`` tensor (uint8 bytes of the JSON) for ``meta``."""
    raw = json.dumps(meta).encode()
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).clone()


def _truth(v) -> bool:
    if isinstance(v, str):
        return v.strip().lower() in ("1", "true", "yes")
    return bool(v)


@dataclass
class QuantizedLinear:
    name: str
    format: str
    weight: torch.Tensor
    weight_scale: torch.Tensor
    bias: Optional[torch.Tensor] = None
    convrot: bool = False
    convrot_groupsize: int = 256
    input_scale: Optional[torch.Tensor] = None
    full_precision: bool = False

    @property
    def out_features(self) -> int:
        return int(self.weight.shape[0])

    def __call__(self, x: torch.Tensor, out_dtype: Optional[torch.dtype] = None, **kw) -> torch.Tensor:
        from . import linear as L

        if self.full_precision:
            raise ValueError(f"layer {self.name} asks for full-precision matrix multiplication, "
                             "which is outside the W8A8 path")
        out_dtype = out_dtype or x.dtype
        if self.format == "int8_tensorwise":
            return L.int8_linear(x, self.weight, self.weight_scale, self.bias, out_dtype,
                                 self.convrot, self.convrot_groupsize, **kw)
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if self.format == "float8_e4m3fn":
            sa = self.input_scale if self.input_scale is not None else \
                torch.ones((), dtype=torch.float32, device=x.device)
            sa = sa.to(device=x.device, dtype=torch.float32).reshape(1)
            aq = L.quantize_per_tensor_fp8(x2, sa)
            y = L.fp8_linear(aq, sa, self.weight, self.weight_scale, self.bias, out_dtype=out_dtype)
        else:  # mxfp8
            aq, asf = L.quantize_mxfp8(x2)
            y = L.mxfp8_linear(aq, asf, self.weight, self.weight_scale, self.bias,
                               out_dtype=out_dtype)
        return y.reshape(*lead, self.out_features)


def load_quantized_linear(state: Dict[str, torch.Tensor], prefix: str,
                          device: Optional[torch.device] = None) -> Optional[QuantizedLinear]:
    """The layer at ``prefix`` (e.g. ``"transformer_blocks.0.attn.to_q."``), its
    keys removed from ``state``; None when the prefix has no weight.  Raises
    the reference's errors: an unknown format, or an INT8 / MXFP8 layer
    without ``weight_scale``."""
    weight = state.pop(f"{prefix}weight", None)
    if weight is None:
        return None
    name = prefix.rstrip(".")
    conf = state.pop(f"{prefix}comfy_quant", None)
    if conf is None:
        raise ValueError(f"layer {name} has no comfy_quant metadata (not a quantised layer)")
    meta = read_quant_config(conf)
    fmt = meta.get("format")
    if not isinstance(fmt, str):
        raise ValueError(f"Unknown quantization format for layer {name}")
    params = meta.get("params") if isinstance(meta.get("params"), dict) else {}

    def option(key, default=None):
        return meta.get(key, params.get(key, default))

    if fmt not in FORMATS:
        raise ValueError(f"Unknown quantization format for layer {name}: {fmt!r} (this package "
                         f"runs {', '.join(FORMATS)})")
    scale = state.pop(f"{prefix}weight_scale", None)
    if scale is None:
        what = {"int8_tensorwise": "INT8 weight scale", "mxfp8": "MXFP8 block scales",
                "float8_e4m3fn": "FP8 weight scale"}[fmt]
        raise ValueError(f"Missing {what} for layer {name}")
    bias = state.pop(f"{prefix}bias", None)
    input_scale = state.pop(f"{prefix}input_scale", None)
    dev = device or weight.device
    dtype = {"int8_tensorwise": torch.int8, "float8_e4m3fn": torch.float8_e4m3fn,
             "mxfp8": torch.float8_e4m3fn}[fmt]
    if weight.dtype != dtype:
        raise ValueError(f"layer {name}: {fmt} payload must be {dtype}, got {weight.dtype}")
    convrot = fmt == "int8_tensorwise" and _truth(option("convrot", False))
    group = int(option("convrot_groupsize", 256)) if convrot else 256
    sdt = torch.uint8 if fmt == "mxfp8" else torch.float32
    return QuantizedLinear(
        name=name, format=fmt, weight=weight.to(dev),
        weight_scale=scale.to(device=dev, dtype=sdt) if fmt != "mxfp8" else scale.to(dev),
        bias=bias.to(dev) if bias is not None else None, convrot=convrot,
        convrot_groupsize=group,
        input_scale=input_scale.to(dev) if input_scale is not None else None,
        full_precision=_truth(option("full_precision_matrix_mult", False)))


def load_quantized_linears(state: Dict[str, torch.Tensor],
                           device: Optional[torch.device] = None) -> Dict[str, QuantizedLinear]:
    """Every quantised linear of a state dict (the prefixes that carry a
    ``comfy_quant`` key), removed from ``state``; returns {name: layer}."""
    prefixes = sorted(k[: -len("comfy_quant")] for k in state if k.endswith(".comfy_quant"))
    out = {}
    for p in prefixes:
        layer = load_quantized_linear(state, p, device)
        if layer is not None:
            out[layer.name] = layer
    return out


def load_file(path: str, device: Optional[torch.device] = None) -> Dict[str, QuantizedLinear]:
    """Every quantised linear of a safetensors checkpoint."""
    from safetensors.torch import load_file as _load

    return load_quantized_linears(_load(path), device)


def quantize_linear_state(prefix: str, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                          *, convrot: bool = False, convrot_groupsize: int = 256,
                          scale_mode: str = "eager") -> Dict[str, torch.Tensor]:
    """The state-dict entries of one INT8 layer in the reference's format, from a
    float weight on the GPU: per-output-channel codes and scales (ConvRot-rotated
    first when ``convrot``; inference/src/layout_complete.rs:119-159,
    inference/src/convrot.rs:378-435) and the ``comfy_quant`` metadata."""
    from . import linear as L

    q, s = L.quantize_weight(weight, convrot=convrot, convrot_groupsize=convrot_groupsize,
                             scale_mode=scale_mode)
    meta = {"format": "int8_tensorwise"}
    if convrot:
        meta.update(convrot=True, convrot_groupsize=convrot_groupsize)
    out = {f"{prefix}weight": q, f"{prefix}weight_scale": s,
           f"{prefix}comfy_quant": quant_config_tensor(meta)}
    if bias is not None:
        out[f"{prefix}bias"] = bias
    return out
