"""Quantised-linear checkpoint ingest (imagine_b200/checkpoint.py) in the
reference's state-dict format (inference/src/checkpoint/quantized.rs:111-300):
metadata decoding, layer discovery, errors and the safetensors round trip on
the CPU; the loaded layers against the oracle on the GPU."""
import pytest
import torch

from imagine_b200 import checkpoint as C
from tests.test_gpu_parity import assert_rms_close


def _int8_state(prefix, n=16, k=32, meta=None, scale=True, bias=True):
    g = torch.Generator().manual_seed(len(prefix))
    st = {f"{prefix}weight": torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8),
          f"{prefix}comfy_quant": C.quant_config_tensor(meta or {"format": "int8_tensorwise"})}
    if scale:
        st[f"{prefix}weight_scale"] = torch.rand(n, 1, generator=g)
    if bias:
        st[f"{prefix}bias"] = torch.randn(n, generator=g).to(torch.bfloat16)
    return st


def test_quant_config_round_trip():
    meta = {"format": "int8_tensorwise", "params": {"convrot": True, "convrot_groupsize": 256}}
    assert C.read_quant_config(C.quant_config_tensor(meta)) == meta
    with pytest.raises(ValueError):
        C.read_quant_config(torch.tensor([1, 2, 3], dtype=torch.uint8))


def test_load_layers_and_options():
    st = {}
    st.update(_int8_state("blocks.0.attn.to_q.", meta={"format": "int8_tensorwise"}))
    st.update(_int8_state("blocks.0.ff.up.", meta={"format": "int8_tensorwise",
                                                   "params": {"convrot": "true",
                                                              "convrot_groupsize": 256}}))
    st["blocks.0.norm.weight"] = torch.ones(4)  # not quantised: left in the state dict
    layers = C.load_quantized_linears(st, torch.device("cpu"))
    assert sorted(layers) == ["blocks.0.attn.to_q", "blocks.0.ff.up"]
    q, up = layers["blocks.0.attn.to_q"], layers["blocks.0.ff.up"]
    assert q.format == "int8_tensorwise" and not q.convrot and q.bias is not None
    assert up.convrot and up.convrot_groupsize == 256
    assert q.weight.dtype == torch.int8 and q.weight_scale.dtype == torch.float32
    assert list(st) == ["blocks.0.norm.weight"]


def test_load_errors_follow_the_reference():
    st = _int8_state("a.", meta={"format": "nvfp4"})
    with pytest.raises(ValueError, match="Unknown quantization format for layer a"):
        C.load_quantized_linear(st, "a.")
    st = _int8_state("b.", scale=False)
    with pytest.raises(ValueError, match="Missing INT8 weight scale for layer b"):
        C.load_quantized_linear(st, "b.")
    st = _int8_state("c.", meta={"convrot": True})
    with pytest.raises(ValueError, match="Unknown quantization format for layer c"):
        C.load_quantized_linear(st, "c.")
    assert C.load_quantized_linear({}, "d.") is None


def test_safetensors_round_trip(tmp_path):
    from safetensors.torch import save_file

    st = _int8_state("m.lin.", meta={"format": "int8_tensorwise", "convrot": True})
    save_file(st, str(tmp_path / "m.safetensors"))
    layers = C.load_file(str(tmp_path / "m.safetensors"), torch.device("cpu"))
    lin = layers["m.lin"]
    assert torch.equal(lin.weight, st["m.lin.weight"]) and lin.convrot


@pytest.mark.gpu
@pytest.mark.parametrize("convrot", [False, True])
def test_int8_layer_from_checkpoint_matches_oracle(tmp_path, convrot):
    """Quantise a bf16 weight on the GPU into the reference's format, write it
    as safetensors, load it back and run it: against the eager oracle."""
    from safetensors.torch import save_file

    from oracle import eager as O

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(768, 512, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(768, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(2, 150, 512, generator=g).to(torch.bfloat16)
    st = C.quantize_linear_state("blk.ff.", w.to(dev), b.to(dev), convrot=convrot)
    save_file({k: v.cpu() for k, v in st.items()}, str(tmp_path / "q.safetensors"))
    layer = C.load_file(str(tmp_path / "q.safetensors"), dev)["blk.ff"]
    y = layer(x.to(dev))
    ref = O.int8_linear(x, layer.weight.cpu(), layer.weight_scale.cpu(), b,
                        out_dtype=torch.bfloat16, convrot=convrot)
    assert y.shape == (2, 150, 768)
    assert_rms_close(y, ref)
    import imagine_b200 as W
    assert W.device_error() == 0


@pytest.mark.gpu
def test_fp8_layer_from_checkpoint():
    from oracle import eager as O
    import imagine_b200 as W

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(6)
    w = (torch.randn(512, 256, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(300, 256, generator=g).to(torch.bfloat16)
    sw = (w.abs().max().float() / 448).reshape(())
    sa = (x.abs().max().float() / 448).reshape(())
    st = {"l.weight": W.quantize_per_tensor_fp8(w.to(dev), sw.to(dev)).cpu(),
          "l.weight_scale": sw, "l.input_scale": sa,
          "l.comfy_quant": C.quant_config_tensor({"format": "float8_e4m3fn"})}
    layer = C.load_quantized_linear(st, "l.", dev)
    y = layer(x.to(dev))
    aq = O.quantize_fp8(x, sa.reshape(1))
    ref = O.fp8_linear_exact(aq, sa.reshape(1), layer.weight.cpu(), sw.reshape(1), None,
                             out_dtype=torch.float32)
    assert_rms_close(y, ref)
