"""B200-native (sm_100a) W8A8 / FP8 linear family with the reference's
operator interface.  Importing loads libw8a8.so and raises if it is missing."""
from .linear import (  # noqa: F401
    dequantize_int8_linear,
    device_error,
    fp8_linear,
    int8_gemm_s32,
    int8_gemv,
    int8_linear,
    quantize_int8_rowwise,
    quantize_per_tensor_fp8,
    quantize_weight,
)
