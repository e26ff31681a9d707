"""Loading helpers for the committed golden fixtures (tests/golden/)."""
import json
import os

import numpy as np
import torch

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
_cache = {}


def load(name):
    if name not in _cache:
        _cache[name] = dict(np.load(os.path.join(HERE, name + ".npz")))
    return _cache[name]


def manifest():
    with open(os.path.join(HERE, "manifest.json")) as f:
        return json.load(f)


def tensor(arr: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    """Rebuild a tensor from the raw array written by make_golden.raw()."""
    t = torch.from_numpy(arr.copy())
    if dtype == torch.bfloat16:
        return t.view(torch.bfloat16)
    if dtype in (torch.float8_e4m3fn,):
        return t.view(torch.float8_e4m3fn)
    return t.to(dtype) if t.dtype != dtype else t


def probe_inputs(case):
    """Closed-form inputs of the reference's probe cases
    (inference/tests/primitives.rs:2268-2290)."""
    m, n, k = case["m"], case["n"], case["k"]
    dt = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[case["dtype"]]
    x = (torch.arange(m * k, dtype=torch.float32) * 0.03125 - 4).reshape(m, k).to(dt)
    w = ((torch.arange(n * k, dtype=torch.int32) % 255) - 127).to(torch.int8).reshape(n, k)
    if case["weight_scale"] == "tensorwise":
        ws = torch.tensor([0.07], dtype=torch.float32)
    else:
        ws = torch.arange(n, dtype=torch.float32) * 0.001 + 0.07
    b = (torch.arange(n, dtype=torch.float32) * 0.013).to(dt) if case["has_bias"] else None
    return x, w, ws, b, dt
