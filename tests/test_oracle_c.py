"""The scalar C restatement (oracle/ref_w8a8.c) agrees with the torch oracle
and with the reference's golden vectors: two independent CPU restatements."""
import ctypes
import os
import subprocess

import numpy as np
import pytest
import torch

from oracle import eager as O
from tests import _golden as G

ORACLE_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle")


@pytest.fixture(scope="module")
def ref():
    subprocess.run(["make", "-s", "-C", ORACLE_DIR], check=True)
    lib = ctypes.CDLL(os.path.join(ORACLE_DIR, "_build", "libref_w8a8.so"))
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.ref_quantize_rowwise_bf16.argtypes = [vp, i64, i64, vp, vp]
    lib.ref_int8_gemm.argtypes = [vp, vp, i64, i64, i64, vp]
    lib.ref_dequant_eager_bf16.argtypes = [vp, vp, vp, i64, vp, i64, i64, vp]
    lib.ref_quantize_fp8_bf16.argtypes = [vp, i64, ctypes.c_float, vp]
    lib.ref_quantize_mxfp8_bf16.argtypes = [vp, i64, i64, vp, vp]
    return lib


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_c_quantiser_and_linear_match(ref):
    g = torch.Generator().manual_seed(5)
    m, k, n = 37, 160, 72
    x = (torch.randn(m, k, generator=g) * 3).to(torch.bfloat16)
    x[1] = 0
    q = torch.empty(m, k, dtype=torch.int8)
    s = torch.empty(m, dtype=torch.float32)
    ref.ref_quantize_rowwise_bf16(_p(x), m, k, _p(q), _p(s))
    qo, so = O.quantize_int8_rowwise(x)
    assert torch.equal(q, qo) and torch.equal(s, so.reshape(-1))
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    wq, ws = O.quantize_weight(w)
    acc = torch.empty(m, n, dtype=torch.int32)
    ref.ref_int8_gemm(_p(q), _p(wq), m, n, k, _p(acc))
    assert torch.equal(acc, O.int8_accumulate(qo, wq))
    b = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16)
    y = torch.empty(m, n, dtype=torch.bfloat16)
    ref.ref_dequant_eager_bf16(_p(acc), _p(s), _p(ws), n, _p(b), m, n, _p(y))
    yo = O.int8_linear(x, wq, ws, b, out_dtype=torch.bfloat16)
    assert torch.equal(y.view(torch.int16), yo.view(torch.int16))


@pytest.mark.parametrize("name", [n for n in G.manifest()["kitchen_eager"]
                                  if n.startswith("quant/") and n.endswith("/bf16")])
def test_c_quantiser_golden(ref, name):
    ke = G.load("kitchen_eager")
    x = G.tensor(ke[name + "/x"], torch.bfloat16)
    m, k = x.shape
    q = torch.empty(m, k, dtype=torch.int8)
    s = torch.empty(m, dtype=torch.float32)
    ref.ref_quantize_rowwise_bf16(_p(x.contiguous()), m, k, _p(q), _p(s))
    assert np.array_equal(O.as_bytes(q), ke[name + "/q"].view(np.uint8).reshape(-1))


def test_c_fp8_and_mxfp8_golden(ref):
    ke = G.load("kitchen_eager")
    x = G.tensor(ke["fp8/bf16/x"], torch.bfloat16).contiguous()
    sc = float(G.tensor(ke["fp8/bf16/scale"], torch.float32)[0])
    out = torch.empty(x.numel(), dtype=torch.uint8)
    ref.ref_quantize_fp8_bf16(_p(x), x.numel(), sc, _p(out))
    assert np.array_equal(out.numpy(), ke["fp8/bf16/q"].reshape(-1))
    for name in [n for n in G.manifest()["kitchen_eager"] if n.startswith("mxfp8/") and n.endswith("bf16")]:
        x = G.tensor(ke[name + "/x"], torch.bfloat16).contiguous()
        m, k = x.shape
        q = torch.empty(m, k, dtype=torch.uint8)
        sf = torch.empty(((m + 127) // 128 * 128) * ((k // 32 + 3) // 4 * 4), dtype=torch.uint8)
        ref.ref_quantize_mxfp8_bf16(_p(x), m, k, _p(q), _p(sf))
        assert np.array_equal(q.numpy().reshape(-1), ke[name + "/q"].reshape(-1)), name
        assert np.array_equal(sf.numpy(), ke[name + "/sf"].reshape(-1)), name


def test_c_fht_is_the_normalised_hadamard():
    """The C FHT (the reference kernel's radix-4 butterfly order) computes
    x . H_256 of inference/src/int8_utils.rs:21-58."""
    from tests import _cref
    g = torch.Generator().manual_seed(11)
    x = torch.randn(4, 512, generator=g)
    got = _cref.fht256(x).double()
    h = O.hadamard(256, torch.float64)
    want = (x.double().reshape(4, 2, 256) @ h).reshape(4, 512)
    assert (got - want).abs().max().item() < 1e-5


def _golden_linear_kwargs(ke, name, dt):
    kw = {}
    k = ke[name + "/wq"].shape[1]
    x = G.tensor(ke[name + "/x"], dt)
    if "input_act" in name:
        if name + "/act_w" in ke:
            kw.update(act="rms_norm", act_w=G.tensor(ke[name + "/act_w"], dt), eps=1e-6)
        elif x.shape[1] == 2 * k:
            kw.update(act="swiglu")
        else:
            kw.update(act="gelu_tanh")
    return x, kw


@pytest.mark.parametrize("name", [n for n in G.manifest()["kitchen_eager"] if n.startswith("linear/")
                                  and ("input_act" in n or "convrot" in n)])
def test_c_fused_quantiser_against_golden_linear(name):
    """The fused-quantiser restatement, completed with the exact int32 GEMM and
    the eager dequant, lands within the tolerance bar (1% of output RMS) of
    the reference's golden linear outputs for its input-activation and
    ConvRot cases."""
    from tests import _cref
    ke = G.load("kitchen_eager")
    dn = [p for p in name.split("_") if p in G.DT][0]
    dt = G.DT[dn]
    x, kw = _golden_linear_kwargs(ke, name, dt)
    q, s = _cref.quantize_act_rot(x, "convrot" in name, kitchen=False, **kw)
    wq = G.tensor(ke[name + "/wq"], torch.int8)
    ws = G.tensor(ke[name + "/ws"], torch.float32)
    b = G.tensor(ke[name + "/bias"], dt) if name + "/bias" in ke else None
    y = O.dequant_eager(O.int8_accumulate(q, wq), s, ws, b, dt).float()
    ref = G.tensor(ke[name + "/y"], dt).float()
    rms = ref.pow(2).mean().sqrt().item()
    assert (y - ref).abs().max().item() <= 0.01 * rms + 2 ** -7 * ref.abs().max().item()


def test_c_act_only_none_equals_eager_quantiser():
    from tests import _cref
    g = torch.Generator().manual_seed(12)
    x = (torch.randn(9, 512, generator=g) * 2).to(torch.bfloat16)
    q, s = _cref.quantize_act_rot(x, False, kitchen=False)
    qo, so = O.quantize_int8_rowwise(x)
    assert torch.equal(q, qo) and torch.equal(s, so.reshape(-1))


@pytest.mark.parametrize("mode", ["scale", "rms_scale", "adaln", "rms_adaln"])
def test_c_modulated_quantiser_matches_eager_sequence(mode):
    """The C restatement of the fused modulation quantiser (eager numerics)
    reproduces the ATen sequence followed by the row quantiser: codes within
    one step, >= 99.9% identical (the normalisation statistics are summed in
    a different order)."""
    from tests import _cref
    g = torch.Generator().manual_seed(21)
    b, s, k = 2, 40, 512
    x = torch.randn(b, s, k, generator=g).to(torch.bfloat16)
    sc = (0.3 * torch.randn(b, 1, k, generator=g)).to(torch.bfloat16)
    sh = (0.3 * torch.randn(b, 1, k, generator=g)).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
    if mode == "scale":
        sc = sc[:1]
        xm = x * (sc + 1)
    elif mode == "rms_scale":
        sc = sc[:1]
        xm = torch.nn.functional.rms_norm(x, (k,), w, 1e-6) * (sc + 1)
    else:
        xm = O.adaln(x, sc, sh, 1e-6, rms=(mode == "rms_adaln"))
    qo, so = O.quantize_int8_rowwise(xm.reshape(-1, k))
    q, s_ = _cref.quantize_modulated(x.reshape(-1, k), mode, sc, sh if "adaln" in mode else None,
                                     w if mode == "rms_scale" else None)
    d = (q.int() - qo.int()).abs()
    assert d.max().item() <= 1 and (d == 0).float().mean().item() >= 0.999
