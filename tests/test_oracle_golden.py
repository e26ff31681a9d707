"""Pin the CPU oracle against the reference's own outputs (no GPU needed).

* kitchen_eager.npz: produced by the reference's Python implementation
  (Kitchen eager backend) -- tests/golden/make_golden.py.
* triton_probe.npz: the reference's recorded Triton-route probe fixture
  (inference/fixtures/stage-1 int8-aot/probe.json), 36 cases.
"""
import numpy as np
import pytest
import torch

from oracle import eager as O
from tests import _golden as G

KE = G.load("kitchen_eager")
MAN = G.manifest()


def _b(t):
    return O.as_bytes(t)


@pytest.mark.parametrize("name", [n for n in MAN["kitchen_eager"] if n.startswith("quant/")])
def test_quantize_rowwise_matches_reference(name):
    dt = G.DT[name.split("/")[-1]]
    x = G.tensor(KE[name + "/x"], dt)
    q, s = O.quantize_int8_rowwise(x)
    assert np.array_equal(_b(q), KE[name + "/q"].view(np.uint8).reshape(-1))
    assert np.array_equal(_b(s), KE[name + "/s"].view(np.uint8).reshape(-1))


@pytest.mark.parametrize("name", [n for n in MAN["kitchen_eager"] if n.startswith("linear/")])
def test_int8_linear_matches_reference(name):
    dn = [p for p in name.split("_") if p in G.DT][0]
    dt = G.DT[dn]
    x = G.tensor(KE[name + "/x"], dt)
    wq = G.tensor(KE[name + "/wq"], torch.int8)
    ws = G.tensor(KE[name + "/ws"], torch.float32)
    kw = {}
    b = G.tensor(KE[name + "/bias"], dt) if name + "/bias" in KE else None
    if name + "/residual" in KE:
        kw.update(residual=G.tensor(KE[name + "/residual"], dt),
                  residual_scale=G.tensor(KE[name + "/residual_scale"], dt))
    if "input_act" in name:
        k = wq.shape[1]
        if name + "/act_w" in KE:
            kw.update(input_act="rms_norm", input_act_weight=G.tensor(KE[name + "/act_w"], dt),
                      input_act_eps=1e-6)
        elif x.shape[1] == 2 * k:
            kw.update(input_act="swiglu")
        else:
            kw.update(input_act="gelu_tanh")
    if "convrot" in name:
        kw.update(convrot=True, convrot_groupsize=256)
    y = O.int8_linear(x, wq, ws, b, out_dtype=dt, **kw)
    assert np.array_equal(_b(y), KE[name + "/y"].view(np.uint8).reshape(-1)), name
    # intermediate codes, scales and exact accumulators
    xa = O.apply_input(x, kw.get("input_act"), kw.get("input_act_weight"), kw.get("input_act_eps"))
    if kw.get("convrot"):
        xa = O.rotate_activation(xa, O.hadamard(256, xa.dtype), 256)
    xq, xs = O.quantize_int8_rowwise(xa.reshape(-1, wq.shape[1]))
    assert np.array_equal(_b(xq), KE[name + "/xq"].view(np.uint8).reshape(-1))
    assert np.array_equal(_b(xs), KE[name + "/xs"].view(np.uint8).reshape(-1))
    acc = O.int8_accumulate(xq, wq)
    assert np.array_equal(acc.numpy(), KE[name + "/acc"])


@pytest.mark.parametrize("name", [n for n in MAN["kitchen_eager"] if n.startswith("fp8")])
def test_fp8_quantize_matches_reference(name):
    dt = G.DT[name.split("/")[-1]]
    x = G.tensor(KE[name + "/x"], dt)
    s = G.tensor(KE[name + "/scale"], torch.float32)
    q = O.quantize_fp8(x, s)
    assert np.array_equal(_b(q), KE[name + "/q"].reshape(-1))
    if name + "/dq" in KE:
        d = O.dequantize_fp8(q, s, torch.bfloat16)
        assert np.array_equal(_b(d), KE[name + "/dq"].view(np.uint8).reshape(-1))


@pytest.mark.parametrize("name", [n for n in MAN["kitchen_eager"] if n.startswith("mxfp8/")])
def test_mxfp8_quantize_matches_reference(name):
    dt = G.DT[name.split("/")[-1]]
    x = G.tensor(KE[name + "/x"], dt)
    p, sf = O.quantize_mxfp8(x)
    assert np.array_equal(_b(p), KE[name + "/q"].reshape(-1))
    assert np.array_equal(_b(sf), KE[name + "/sf"].reshape(-1))
    d = O.dequantize_mxfp8(p, sf, torch.bfloat16)
    assert np.array_equal(_b(d), KE[name + "/dq"].view(np.uint8).reshape(-1))


def test_blocked_layout_roundtrip():
    e = torch.randint(0, 255, (300, 13), dtype=torch.uint8)
    assert torch.equal(O.from_blocked(O.to_blocked(e), 300, 13), e)


PROBE = G.load("triton_probe")


@pytest.mark.parametrize("case", MAN["triton_probe"], ids=lambda c: c["name"])
def test_triton_probe_pins_kitchen_scale_and_fma_epilogue(case):
    """The reference's recorded Triton-route bytes are reproduced exactly by the
    Kitchen scale (amax * (1/127)) and the single-rounding FMA epilogue."""
    x, w, ws, b, dt = G.probe_inputs(case)
    q, s = O.quantize_int8_rowwise_kitchen(x)
    assert np.array_equal(_b(q), PROBE[case["name"] + "/q"])
    assert np.array_equal(_b(s), PROBE[case["name"] + "/s"])
    acc = O.int8_accumulate(q, w)
    y = O.dequant_scale_product(acc, s, ws, b, dt)
    assert np.array_equal(_b(y), PROBE[case["name"] + "/y"])
