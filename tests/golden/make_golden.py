"""Regenerate the golden fixtures under tests/golden/ from the reference itself.

Run in a container that has the reference checkout (it is not needed at test
time):

    python tests/golden/make_golden.py --reference /path/to/imagine

Two sources, both the reference's own:

1. ``kitchen_eager.npz`` -- the reference's Python implementation of the path,
   Kitchen 0.2.37 ``comfy_kitchen/backends/eager/quantization.py``, which the
   Rust crate's eager route restates op for op (inference/src/eager.rs,
   inference/src/int8_linear.rs).  It ships as source inside the reference's
   archive ``design/reference-local/native-source-candidates.tar.gz``; this
   script extracts it to a temporary directory, imports it on the CPU and
   records inputs and outputs (as raw bytes) for seeded cases.
2. ``triton_probe.npz`` -- the reference's recorded regression fixture
   ``inference/fixtures/stage-1`` member ``int8-aot/probe.json`` (36 cases of the
   Triton INT8 route: codes, row scales and dequantised outputs; inputs are the
   closed forms of inference/tests/primitives.rs:2268-2290).  Only that JSON
   member is read from the archive.
3. ``autotuning_policy.json`` -- the reference's recorded autotuner fixture
   (member ``runtime/autotuning-policy.json``): the do_bench device trace and
   quantiles, and the candidate-selection trace with ties and failures.
"""
from __future__ import annotations

import argparse
import io
import json
import os
import subprocess
import sys
import tarfile
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def raw(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    elif t.dtype in (torch.float8_e4m3fn, getattr(torch, "float8_e8m0fnu", None)):
        t = t.view(torch.uint8)
    return t.numpy().copy()


def load_kitchen(reference: str, tmp: str):
    arc = os.path.join(reference, "design/reference-local/native-source-candidates.tar.gz")
    with tarfile.open(arc) as tf:
        members = [m for m in tf.getmembers()
                   if m.name.startswith("comfy-kitchen/comfy_kitchen/") and m.isfile()
                   and m.name.endswith(".py")]
        tf.extractall(tmp, members=members, filter="data")
    sys.path.insert(0, os.path.join(tmp, "comfy-kitchen"))
    from comfy_kitchen.backends.eager import quantization as q  # noqa: E402
    return q


def kitchen_cases(q):
    out = {}
    meta = []
    g = torch.Generator().manual_seed(1234)

    def add(name, **arrays):
        for k, v in arrays.items():
            out[f"{name}/{k}"] = v
        meta.append(name)

    # --- a1: row-wise quantiser ------------------------------------------
    special = []
    # the reference's own primitive inputs (inference/tests/primitives.rs:1697-1745)
    x = torch.arange(64, dtype=torch.float32) * 0.125 - 4
    x = x.reshape(4, 16)
    x[0] = 0
    special.append(("prim4x16", x))
    special.append(("prim4x64", (torch.arange(256, dtype=torch.float32) * 0.03125 - 4).reshape(4, 64)))
    # ties and extremes: exact .5 after division, a zero row, a row with one huge value
    t = torch.zeros(5, 96)
    t[0] = torch.linspace(-127.5, 127.5, 96)
    t[1] = 0
    t[2, 3] = 3.0e4
    t[2, 4:] = torch.linspace(-1, 1, 92)
    t[3] = torch.arange(96) % 7 - 3.5
    t[4] = -torch.arange(96) * 1e-3
    special.append(("ties", t))
    for dn, dt in DT.items():
        for name, base in special:
            xx = base.to(dt)
            qq, ss = q.quantize_int8_rowwise(xx)
            add(f"quant/{name}/{dn}", x=raw(xx), q=raw(qq), s=raw(ss))
        for (m, k) in [(1, 16), (2, 48), (7, 1040), (5, 3072), (70, 272), (2, 12288)]:
            xx = (torch.randn(m, k, generator=g) * 3).to(dt)
            if m > 2:
                xx[1] = 0
            qq, ss = q.quantize_int8_rowwise(xx)
            add(f"quant/rand{m}x{k}/{dn}", x=raw(xx), q=raw(qq), s=raw(ss))

    # --- a3/a4/a6: int8_linear (eager order) ------------------------------
    lin = [
        # (m, k, n, dtype, bias, ws_mode, extra)
        (1, 64, 24, "bf16", True, "channel", {}),
        (2, 3072, 16, "bf16", True, "channel", {}),
        (37, 160, 40, "bf16", False, "tensor", {}),
        (130, 256, 136, "bf16", True, "channel", {}),
        (136, 64, 136, "bf16", True, "channel", {}),
        (64, 256, 128, "f16", True, "channel", {}),
        (48, 192, 136, "f32", True, "tensor", {}),
        (96, 256, 128, "bf16", True, "channel", {"residual": True}),
        (64, 256, 96, "bf16", True, "channel", {"input_act": "gelu_tanh"}),
        (32, 256, 96, "bf16", True, "channel", {"input_act": "swiglu"}),
        (64, 256, 96, "bf16", False, "channel", {"input_act": "rms_norm"}),
        (64, 512, 80, "bf16", True, "channel", {"convrot": True}),
    ]
    for i, (m, k, n, dn, has_b, wsm, extra) in enumerate(lin):
        dt = DT[dn]
        kin = k * (2 if extra.get("input_act") == "swiglu" else 1)
        x = torch.randn(m, kin, generator=g).to(dt)
        w = (torch.randn(n, k, generator=g) * 0.02).to(dt)
        if wsm == "channel":
            wq, ws = q.quantize_int8_rowwise(w)
            ws = ws.reshape(-1)
        else:
            wq, ws = q.quantize_int8_tensorwise(w)
            ws = ws.reshape(1)
        b = (torch.randn(n, generator=g) * 0.02).to(dt) if has_b else None
        kw = {}
        arrays = dict(x=raw(x), wq=raw(wq), ws=raw(ws))
        if b is not None:
            arrays["bias"] = raw(b)
        if extra.get("residual"):
            r = torch.randn(m, n, generator=g).to(dt)
            rs = (torch.rand(n, generator=g)).to(dt)
            kw.update(residual=r, residual_scale=rs)
            arrays.update(residual=raw(r), residual_scale=raw(rs))
        if extra.get("input_act"):
            kw["input_act"] = extra["input_act"]
            if extra["input_act"] == "rms_norm":
                aw = (1 + 0.1 * torch.randn(k, generator=g)).to(dt)
                kw.update(input_act_weight=aw, input_act_eps=1e-6)
                arrays["act_w"] = raw(aw)
        if extra.get("convrot"):
            kw.update(convrot=True, convrot_groupsize=256)
        y = q.int8_linear(x, wq, ws, b, out_dtype=dt, **kw)
        # intermediate codes/scales of the activation the linear quantised
        xa = q._apply_input_act(x, kw.get("input_act"), kw.get("input_act_weight"),
                                kw.get("input_act_eps", 0.0)) if kw.get("input_act") else x
        if extra.get("convrot"):
            xa = q._rotate_activation(xa, q._build_hadamard(256, device=xa.device, dtype=xa.dtype), 256)
        xq, xs = q.quantize_int8_rowwise(xa.reshape(-1, k))
        acc = q._int8_matmul_accumulate(xq, wq.T.contiguous())
        arrays.update(xq=raw(xq), xs=raw(xs), acc=raw(acc), y=raw(y))
        name = f"linear/{i}_{m}x{k}x{n}_{dn}" + "".join(f"_{k2}" for k2 in sorted(extra))
        add(name, **arrays)

    # --- a9: fp8 per-tensor quantiser --------------------------------------
    for dn in ("bf16", "f16", "f32"):
        dt = DT[dn]
        x = torch.randn(67, 96, generator=g)
        mask = torch.rand(67, 96, generator=g) < 0.01
        x = torch.where(mask, x * 20, x).to(dt)
        scale = (x.abs().max().float() / 448.0).reshape(1)
        f = q.quantize_per_tensor_fp8(x, scale)
        d = q.dequantize_per_tensor_fp8(f, scale, torch.bfloat16)
        add(f"fp8/{dn}", x=raw(x), scale=raw(scale), q=raw(f), dq=raw(d))
        # a non-power scale with saturation
        s2 = torch.tensor([0.01], dtype=torch.float32)
        f2 = q.quantize_per_tensor_fp8(x, s2)
        add(f"fp8sat/{dn}", x=raw(x), scale=raw(s2), q=raw(f2))

    # --- a10: mxfp8 quantiser (payload + blocked e8m0 scales) ---------------
    for dn in ("bf16", "f16", "f32"):
        dt = DT[dn]
        for (m, k) in [(3, 64), (130, 96), (65, 256)]:
            x = torch.randn(m, k, generator=g)
            mask = torch.rand(m, k, generator=g) < 0.01
            x = torch.where(mask, x * 20, x)
            x[0, :32] = 0  # a zero block
            x = x.to(dt)
            p, s = q.quantize_mxfp8(x)
            d = q.dequantize_mxfp8(p, s, torch.bfloat16)
            add(f"mxfp8/{m}x{k}/{dn}", x=raw(x), q=raw(p), sf=raw(s), dq=raw(d))
    return out, meta


def fixture_member(reference: str, member: str) -> bytes:
    """One JSON member of the split fixture archive (nothing else is extracted)."""
    parts = sorted(os.path.join(reference, "inference/fixtures/stage-1", p)
                   for p in os.listdir(os.path.join(reference, "inference/fixtures/stage-1"))
                   if p.startswith("oracles.tar.gz.part-"))
    cat = subprocess.Popen(["cat", *parts], stdout=subprocess.PIPE)
    tar = subprocess.run(["tar", "-xzOf", "-", member], stdin=cat.stdout,
                         capture_output=True, check=True)
    cat.wait()
    return tar.stdout


def probe_cases(reference: str):
    d = json.load(io.BytesIO(fixture_member(reference, "int8-aot/probe.json")))

    def lst(v):
        return np.asarray(v if isinstance(v, list) else json.loads(v), dtype=np.uint8)

    out = {}
    meta = []
    for i, c in enumerate(d["cases"]):
        name = f"probe/{i}"
        out[f"{name}/q"] = lst(c["quantized"])
        out[f"{name}/s"] = lst(c["scale"])
        out[f"{name}/y"] = lst(c["output"])
        meta.append(dict(name=name, dtype=c["dtype"].strip("'").replace("torch.", ""),
                         m=int(c["m"]), n=int(c["n"]), k=int(c["k"]),
                         has_bias=str(c["has_bias"]) == "True",
                         weight_scale=str(c["weight_scale"]).strip("'")))
    return out, meta


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    torch.manual_seed(0)
    with tempfile.TemporaryDirectory() as tmp:
        q = load_kitchen(args.reference, tmp)
        arrays, names = kitchen_cases(q)
    np.savez_compressed(os.path.join(HERE, "kitchen_eager.npz"), **arrays)
    policy = json.loads(fixture_member(args.reference, "runtime/autotuning-policy.json"))
    with open(os.path.join(HERE, "autotuning_policy.json"), "w") as f:
        json.dump(policy, f, indent=1)
    parrays, pmeta = probe_cases(args.reference)
    np.savez_compressed(os.path.join(HERE, "triton_probe.npz"), **parrays)
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump({"kitchen_eager": names, "triton_probe": pmeta,
                   "generator": "tests/golden/make_golden.py",
                   "reference_sources": [
                       "design/reference-local/native-source-candidates.tar.gz "
                       "(comfy-kitchen 0.2.37 be003b7, backends/eager/quantization.py)",
                       "inference/fixtures/stage-1/oracles.tar.gz.part-* member int8-aot/probe.json"],
                   "torch": torch.__version__}, f, indent=1)
    print("wrote", len(names), "kitchen cases and", len(pmeta), "probe cases")


if __name__ == "__main__":
    main()
