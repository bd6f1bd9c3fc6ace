"""dscquant_b200 -- B200-native (sm_100a) W4A4 quantized-linear path.

Operator API mirrors the reference (core/linear.py QuantLinear,
core/quantization.py functions, kernel/w4a4.cu quantize/matmul); the compute
runs in hand-written CUDA kernels behind the C ABI in include/dscq_b200.h.
"""
from . import ops
from .linear import QuantConfig, QuantLinear
from .quantization import (activation_codes, pack_int4, quantize_activation, quantize_weight, ste_round,
                           unpack_int4, weight_codes)

__all__ = ["ops", "QuantConfig", "QuantLinear", "activation_codes", "pack_int4", "quantize_activation",
           "quantize_weight", "ste_round", "unpack_int4", "weight_codes"]
