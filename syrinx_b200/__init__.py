"""syrinx_b200 — B200-native quantized dual-AR decode (slow AR + fast AR codebook head).

The product is libsyrinx_b200.so (sm_100a kernels + C ABI, include/syrinx_dualar.h);
this package is its Python binding and the host-side mirror of the reference interface.
"""
from ._lib import LIB_PATH, SyrinxError, lib
from .configs import (COSYVOICE2_LM, COSYVOICE3_LM, PRESETS, QWEN3_4B, S1_MINI, SX_DTYPE_BF16, SX_DTYPE_F32,
                      SX_DTYPE_Q4_K, SX_DTYPE_Q8_0, TINY_S2, ModelConfig, Stack, frame_bytes, shrink)
from .dualar import (GREEDY, B200DualAr, Model, Sampler, SamplingParams, SlowStep, drive,
                     synth_blob)

__all__ = [
    "LIB_PATH", "SyrinxError", "lib", "COSYVOICE2_LM", "COSYVOICE3_LM", "PRESETS", "QWEN3_4B", "S1_MINI", "TINY_S2",
    "SX_DTYPE_BF16", "SX_DTYPE_F32", "SX_DTYPE_Q4_K", "SX_DTYPE_Q8_0", "ModelConfig", "Stack", "frame_bytes", "shrink",
    "GREEDY", "B200DualAr", "Model", "Sampler", "SamplingParams", "SlowStep", "drive", "synth_blob",
]
