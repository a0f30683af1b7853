"""ctypes binding of libsyrinx_b200.so (the C ABI in include/syrinx_dualar.h).

The shared library is built in-tree (``make -C syrinx_b200/csrc``). Loading fails loudly
when it is missing: there is no CPU fallback for the product path.
"""
from __future__ import annotations

import ctypes as C
import os

from .configs import SxCodecInfo, SxModelDesc, SxSamplingParams

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libsyrinx_b200.so")

SAMPLE_FN = C.CFUNCTYPE(C.c_uint32, C.c_void_p, C.POINTER(C.c_float), C.c_int32)

# name -> (restype, argtypes); every symbol declared in include/syrinx_dualar.h
_u32p = C.POINTER(C.c_uint32)
_f32p = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int32)
_u8p = C.POINTER(C.c_uint8)
SIGNATURES = {
    "sx_last_error": (C.c_char_p, []),
    "sx_version": (C.c_char_p, []),
    "sx_synth_blob_size": (C.c_int, [C.POINTER(SxModelDesc), C.c_int32, C.POINTER(C.c_size_t)]),
    "sx_synth_blob_write": (C.c_int, [C.POINTER(SxModelDesc), C.c_int32, C.c_uint64, C.c_void_p, C.c_size_t]),
    "sx_model_create": (C.c_int, [C.POINTER(SxModelDesc), C.c_void_p, C.c_size_t, C.c_int32, C.POINTER(C.c_void_p)]),
    "sx_model_create_tp": (C.c_int, [C.POINTER(SxModelDesc), C.c_void_p, C.c_size_t, C.c_int32, C.c_int32, C.c_int32,
                                      C.POINTER(C.c_void_p)]),
    "sx_model_destroy": (C.c_int, [C.c_void_p]),
    "sx_model_weight_bytes": (C.c_int, [C.c_void_p, C.POINTER(C.c_size_t)]),
    "sx_session_create": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.POINTER(C.c_void_p)]),
    "sx_session_create_ex": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.POINTER(C.c_void_p)]),
    "sx_session_tp_handle": (C.c_int, [C.c_void_p, C.c_void_p]),
    "sx_session_tp_connect": (C.c_int, [C.c_void_p, C.c_void_p]),
    "sx_session_tp_disconnect": (C.c_int, [C.c_void_p]),
    "sx_session_tp_set_timeout": (C.c_int, [C.c_void_p, C.c_int64]),
    "sx_session_fill_kv_synthetic": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_uint64]),
    "sx_session_reset": (C.c_int, [C.c_void_p]),
    "sx_session_destroy": (C.c_int, [C.c_void_p]),
    "sx_session_len": (C.c_int, [C.c_void_p, C.c_int32, _i32p]),
    "sx_session_set_stream": (C.c_int, [C.c_void_p, C.c_void_p]),
    "sx_profile_gemv": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32]),
    "sx_profile_stack": (C.c_int, [C.c_void_p, C.c_int32, _f32p]),
    "sx_prefill": (C.c_int, [C.c_void_p, _u32p, C.c_int32, _f32p, _f32p]),
    "sx_slow_step": (C.c_int, [C.c_void_p, _u32p, C.c_int32, _f32p, _f32p]),
    "sx_first_code": (C.c_uint32, [C.c_void_p, C.c_uint32]),
    "sx_fast_expand": (C.c_int, [C.c_void_p, C.c_uint32, SAMPLE_FN, C.c_void_p, _u32p]),
    "sx_fast_expand_greedy": (C.c_int, [C.c_void_p, C.c_uint32, _u32p]),
    "sx_frame_step_greedy": (C.c_int, [C.c_void_p, _u32p, C.c_int32, _u32p, _i32p]),
    "sx_decode_greedy": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, _u32p, _i32p]),
    "sx_sampling_params_default": (None, [C.POINTER(SxSamplingParams)]),
    "sx_drive": (C.c_int, [C.c_void_p, _u32p, C.c_int32, C.c_int32, C.c_uint64, C.POINTER(SxSamplingParams), _u32p, _i32p]),
    "sx_decode_sample": (C.c_int, [C.c_void_p, C.c_int32, C.c_uint64, C.POINTER(SxSamplingParams), _u32p, _i32p]),
    "sx_prefill_batch": (C.c_int, [C.c_void_p, _u32p, _i32p, C.c_int32, _f32p, _f32p]),
    "sx_slow_step_batch": (C.c_int, [C.c_void_p, _u32p, _u8p, C.c_int32, _f32p, _f32p]),
    "sx_fast_expand_batch_greedy": (C.c_int, [C.c_void_p, _u32p, _u8p, C.c_int32, _u32p]),
    "sx_decode_greedy_batch": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, _u32p, _i32p]),
    "sx_lm_step_tokens": (C.c_int, [C.c_void_p, _u32p, C.c_int32, _f32p]),
    "sx_lm_step_embeds": (C.c_int, [C.c_void_p, _f32p, C.c_int32, _f32p]),
    "sx_dequantize": (C.c_int, [C.c_int32, C.c_void_p, C.c_int64, _f32p, C.c_int32]),
    "sx_dequantize_noalloc": (C.c_int, [C.c_int32, C.c_void_p, C.c_int64, _f32p, C.c_int32]),
    # include/syrinx_codec.h
    "sx_codec_create": (C.c_int, [C.c_void_p, C.c_size_t, C.c_int32, C.POINTER(C.c_void_p)]),
    "sx_codec_destroy": (C.c_int, [C.c_void_p]),
    "sx_codec_get_info": (C.c_int, [C.c_void_p, C.POINTER(SxCodecInfo)]),
    "sx_codec_reserve": (C.c_int, [C.c_void_p, C.c_int32]),
    "sx_codec_set_stream": (C.c_int, [C.c_void_p, C.c_void_p]),
    "sx_codec_decode": (C.c_int, [C.c_void_p, _u32p, C.c_int32, C.c_int32, _f32p, C.c_size_t]),
    "sx_codec_decode_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p]),
}

_LIB = None


class SyrinxError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"syrinx status {code}: {msg}")
        self.code = code


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build the CUDA extension first "
                "(python -c 'import __graft_entry__ as g; g.build()' or make -C syrinx_b200/csrc)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(rc: int) -> None:
    if rc != 0:
        raise SyrinxError(rc, lib().sx_last_error().decode(errors="replace"))
