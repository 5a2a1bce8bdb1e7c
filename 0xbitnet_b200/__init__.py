"""0xbitnet_b200 — B200-native (sm_100a) ternary BitLinear path of 0xBitNet.

Drop-in for the reference's BitLinear hot path (fused RMSNorm + per-token
absmax int8 quantize feeding a ternary GEMV/GEMM over I2_S weights). The
compute lives in ``libobn.so`` (C ABI: include/obn.h); this package is its host
mirror. Import it with ``importlib.import_module("0xbitnet_b200")``.
"""
from . import i2s
from ._lib import LIB_PATH, ObnError, lib
from .bitlinear import (BitLinear, check_device_errors, lm_head_f16, lm_head_f16_batched,
                        rmsnorm, rmsnorm_quantize)

lib()  # fail loudly at import when the CUDA library has not been built

__all__ = ["BitLinear", "rmsnorm_quantize", "rmsnorm", "lm_head_f16", "lm_head_f16_batched", "check_device_errors", "ObnError",
           "LIB_PATH", "i2s", "lib"]
