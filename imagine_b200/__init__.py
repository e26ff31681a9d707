"""B200-native (sm_100a) W8A8 / FP8 linear family with the reference's
operator interface.

The operators load libw8a8.so on first use and raise if it is missing (there
is no fallback).  Importing the package itself does not load the library, so
`imagine_b200.build` can run on a checkout that has not been built yet.
"""
_OPS = (
    "dequantize_int8_linear",
    "device_error",
    "fp8_linear",
    "int8_gemm_s32",
    "int8_gemv",
    "int8_linear",
    "int8_linear_host",
    "quantize_int8_rowwise",
    "quantize_int8_rowwise_convrot",
    "quantize_int8_rowwise_modulated",
    "int8_linear_modulated",
    "int8_linear_rms_modulated",
    "adaln_int8_linear",
    "rms_rope",
    "int8_linear_rms_rope",
    "rope_freqs_rows",
    "pack_weight_tiles",
    "TiledInt8Weight",
    "quantize_per_tensor_fp8",
    "quantize_weight",
    "row_absmax",
    "quantize_int8_rowwise_given_absmax",
    "quantize_mxfp8",
    "mxfp8_linear",
)

__all__ = list(_OPS)


def __getattr__(name):
    if name in _OPS:
        from . import linear

        return getattr(linear, name)
    raise AttributeError(name)
