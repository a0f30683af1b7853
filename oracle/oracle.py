"""ctypes wrapper of oracle/liboracle.so — the CPU parity checker.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference arm, never by the product package. Built by `make -C oracle`.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from syrinx_b200.configs import ModelConfig, SxModelDesc, SxSamplingParams

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
_L = None

_u32p = C.POINTER(C.c_uint32)
_f32p = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int32)


def lib() -> C.CDLL:
    global _L
    if _L is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} missing: run `make -C oracle`")
        L = C.CDLL(LIB_PATH)
        sig = {
            "oc_last_error": (C.c_char_p, []),
            "oc_num_threads": (C.c_int, []),
            "oc_set_num_threads": (None, [C.c_int]),
            "oc_set_qmode": (None, [C.c_int32]),
            "oc_get_qmode": (C.c_int32, []),
            "oc_linear_q8_0": (None, [_f32p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, _f32p]),
            "oc_linear_q4_k": (None, [_f32p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, _f32p]),
            "oc_q8_0_quantize": (None, [_f32p, C.c_int64, C.c_void_p]),
            "oc_q8_0_dequantize": (None, [C.c_void_p, C.c_int64, _f32p]),
            "oc_q4_k_dequantize": (None, [C.c_void_p, C.c_int64, _f32p]),
            "oc_f16_to_f32": (C.c_float, [C.c_uint16]),
            "oc_f32_to_f16": (C.c_uint16, [C.c_float]),
            "oc_f32_to_bf16": (C.c_uint16, [C.c_float]),
            "oc_rmsnorm": (None, [_f32p, _f32p, C.c_int32, C.c_int32, C.c_float, _f32p]),
            "oc_softmax": (None, [_f32p, C.c_int32, C.c_int32, _f32p]),
            "oc_silu": (None, [_f32p, C.c_int64, _f32p]),
            "oc_rope": (None, [_f32p, C.c_int32, C.c_int32, C.c_int32, _i32p, C.c_float, C.c_int32]),
            "oc_linear_f32": (None, [_f32p, _f32p, _f32p, C.c_int32, C.c_int32, C.c_int32, _f32p]),
            "oc_model_create": (C.c_int, [C.POINTER(SxModelDesc), C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p)]),
            "oc_model_destroy": (None, [C.c_void_p]),
            "oc_tensor_rows": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int64, C.c_int64, _f32p]),
            "oc_tensor_shape": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_int64), C.POINTER(C.c_int64), _i32p]),
            "oc_session_create": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.POINTER(C.c_void_p)]),
            "oc_session_destroy": (None, [C.c_void_p]),
            "oc_session_reset": (None, [C.c_void_p]),
            "oc_session_len": (C.c_int32, [C.c_void_p]),
            "oc_prefill": (C.c_int, [C.c_void_p, _u32p, C.c_int32, _f32p, _f32p]),
            "oc_slow_step": (C.c_int, [C.c_void_p, _u32p, _f32p, _f32p]),
            "oc_lm_step_tokens": (C.c_int, [C.c_void_p, _u32p, C.c_int32, _f32p]),
            "oc_lm_step_embeds": (C.c_int, [C.c_void_p, _f32p, C.c_int32, _f32p]),
            "oc_fast_expand_greedy": (C.c_int, [C.c_void_p, _f32p, C.c_uint32, _u32p, _f32p]),
            "oc_first_code": (C.c_uint32, [C.c_void_p, C.c_uint32]),
            "oc_greedy_semantic": (C.c_uint32, [C.c_void_p, _f32p, C.c_int32, _f32p]),
            "oc_drive_greedy": (C.c_int, [C.c_void_p, _u32p, C.c_int32, C.c_int32, C.c_int32, _u32p, _i32p, _f32p]),
            "oc_drive": (C.c_int, [C.c_void_p, _u32p, C.c_int32, C.c_int32, C.c_uint64, C.POINTER(SxSamplingParams), _u32p, _i32p]),
            "oc_splitmix64_next": (C.c_uint64, [C.POINTER(C.c_uint64)]),
            "oc_synth_blob_size": (C.c_int, [C.POINTER(SxModelDesc), C.c_int32, C.POINTER(C.c_size_t)]),
            "oc_synth_blob_write": (C.c_int, [C.POINTER(SxModelDesc), C.c_int32, C.c_uint64, C.c_void_p, C.c_size_t]),
            "oc_logits_to_probs": (None, [_f32p, C.c_int32, C.c_float, C.c_float, C.c_int32, _f32p]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _L = L
    return _L


def _p(a, ct):
    return a.ctypes.data_as(C.POINTER(ct))


def _check(rc):
    if rc != 0:
        raise RuntimeError(f"oracle status {rc}: {lib().oc_last_error().decode()}")


def synth_blob(cfg: ModelConfig, wtype: int, seed: int) -> np.ndarray:
    """The seeded synthetic SXW1 blob (byte-identical to syrinx_b200.synth_blob)."""
    desc = cfg.to_c()
    size = C.c_size_t()
    _check(lib().oc_synth_blob_size(C.byref(desc), wtype, C.byref(size)))
    buf = np.empty(size.value, np.uint8)
    _check(lib().oc_synth_blob_write(C.byref(desc), wtype, seed, buf.ctypes.data, size.value))
    return buf


# ---- block formats -----------------------------------------------------------------------
def q8_0_quantize(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    out = np.empty(x.size // 32 * 34, np.uint8)
    lib().oc_q8_0_quantize(_p(x, C.c_float), x.size, out.ctypes.data)
    return out


def q8_0_dequantize(blocks: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1)
    n = b.size // 34
    out = np.empty(n * 32, np.float32)
    lib().oc_q8_0_dequantize(b.ctypes.data, n, _p(out, C.c_float))
    return out


def q4_k_dequantize(blocks: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1)
    n = b.size // 144
    out = np.empty(n * 256, np.float32)
    lib().oc_q4_k_dequantize(b.ctypes.data, n, _p(out, C.c_float))
    return out


# ---- ops -----------------------------------------------------------------------------------
def rmsnorm(x, w, eps):
    x = np.ascontiguousarray(x, np.float32)
    rows = x.size // x.shape[-1]
    y = np.empty_like(x)
    lib().oc_rmsnorm(_p(x, C.c_float), _p(np.ascontiguousarray(w, np.float32), C.c_float), rows, x.shape[-1],
                     eps, _p(y, C.c_float))
    return y


def softmax(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().oc_softmax(_p(x, C.c_float), x.size // x.shape[-1], x.shape[-1], _p(y, C.c_float))
    return y


def silu(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().oc_silu(_p(x, C.c_float), x.size, _p(y, C.c_float))
    return y


def rope(x, positions, theta, interleaved=True):
    """x [T, n_heads, head_dim]."""
    y = np.ascontiguousarray(x, np.float32).copy()
    T, H, hd = y.shape
    pos = np.ascontiguousarray(positions, np.int32)
    lib().oc_rope(_p(y, C.c_float), T, H, hd, _p(pos, C.c_int32), theta, int(interleaved))
    return y


def linear(x, w, b=None):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    M, K = x.reshape(-1, x.shape[-1]).shape
    N = w.shape[0]
    y = np.empty((M, N), np.float32)
    bp = None if b is None else _p(np.ascontiguousarray(b, np.float32), C.c_float)
    lib().oc_linear_f32(_p(x, C.c_float), _p(w, C.c_float), bp, M, N, K, _p(y, C.c_float))
    return y


# ---- model ---------------------------------------------------------------------------------
class OracleModel:
    def __init__(self, cfg: ModelConfig, blob: np.ndarray):
        self.cfg = cfg
        self.blob = blob  # tensors are read in place; keep the blob alive
        self._desc = cfg.to_c()
        self.h = C.c_void_p()
        _check(lib().oc_model_create(C.byref(self._desc), blob.ctypes.data, blob.nbytes, C.byref(self.h)))

    def tensor(self, name: str) -> np.ndarray:
        r, c, dt = C.c_int64(), C.c_int64(), C.c_int32()
        _check(lib().oc_tensor_shape(self.h, name.encode(), C.byref(r), C.byref(c), C.byref(dt)))
        out = np.empty((r.value, c.value), np.float32)
        _check(lib().oc_tensor_rows(self.h, name.encode(), 0, r.value, _p(out, C.c_float)))
        return out

    def first_code(self, tok):
        return int(lib().oc_first_code(self.h, tok))

    def greedy_semantic(self, logits, mask_stop=False):
        logits = np.ascontiguousarray(logits, np.float32)
        margin = C.c_float()
        tok = lib().oc_greedy_semantic(self.h, _p(logits, C.c_float), int(mask_stop), C.byref(margin))
        return int(tok), float(margin.value)

    def __del__(self):
        try:
            lib().oc_model_destroy(self.h)
        except Exception:
            pass


class OracleSession:
    def __init__(self, model: OracleModel, max_ctx: int, kv_bf16: bool = True):
        self.model = model
        self.cfg = model.cfg
        self.max_ctx = max_ctx
        self.h = C.c_void_p()
        _check(lib().oc_session_create(model.h, max_ctx, int(kv_bf16), C.byref(self.h)))

    def reset(self):
        lib().oc_session_reset(self.h)

    def prefill(self, prompt):
        p = np.ascontiguousarray(prompt, np.uint32)
        if p.ndim == 1:
            p = p[None, :]
        logits = np.empty(self.cfg.vocab_size, np.float32)
        hidden = np.empty(self.cfg.slow.dim, np.float32)
        _check(lib().oc_prefill(self.h, _p(p, C.c_uint32), p.shape[1], _p(logits, C.c_float), _p(hidden, C.c_float)))
        return logits, hidden

    def slow_step(self, frame):
        f = np.ascontiguousarray(frame, np.uint32).reshape(-1)
        logits = np.empty(self.cfg.vocab_size, np.float32)
        hidden = np.empty(self.cfg.slow.dim, np.float32)
        _check(lib().oc_slow_step(self.h, _p(f, C.c_uint32), _p(logits, C.c_float), _p(hidden, C.c_float)))
        return logits, hidden

    def lm_step_tokens(self, tokens):
        t = np.ascontiguousarray(tokens, np.uint32).reshape(-1)
        logits = np.empty(self.cfg.vocab_size, np.float32)
        _check(lib().oc_lm_step_tokens(self.h, _p(t, C.c_uint32), t.size, _p(logits, C.c_float)))
        return logits

    def lm_step_embeds(self, embeds):
        e = np.ascontiguousarray(embeds, np.float32).reshape(-1, self.cfg.slow.dim)
        logits = np.empty(self.cfg.vocab_size, np.float32)
        _check(lib().oc_lm_step_embeds(self.h, _p(e, C.c_float), e.shape[0], _p(logits, C.c_float)))
        return logits

    def fast_expand_greedy(self, hidden, first_code):
        C_ = self.cfg.num_codebooks
        h = np.ascontiguousarray(hidden, np.float32)
        codes = np.empty(C_, np.uint32)
        fl = np.empty((C_ - 1, self.cfg.codebook_size), np.float32)
        _check(lib().oc_fast_expand_greedy(self.h, _p(h, C.c_float), first_code, _p(codes, C.c_uint32),
                                           _p(fl, C.c_float)))
        return codes, fl

    def drive_greedy(self, prompt, n_frames, mask_stop=False):
        p = np.ascontiguousarray(prompt, np.uint32)
        if p.ndim == 1:
            p = p[None, :]
        out = np.zeros((n_frames, self.cfg.frame_width), np.uint32)
        margins = np.zeros(n_frames, np.float32)
        n = C.c_int32()
        _check(lib().oc_drive_greedy(self.h, _p(p, C.c_uint32), p.shape[1], n_frames, int(mask_stop),
                                     _p(out, C.c_uint32), C.byref(n), _p(margins, C.c_float)))
        return out[: n.value], margins[: n.value]

    def drive(self, prompt, max_frames, seed, params: SxSamplingParams):
        p = np.ascontiguousarray(prompt, np.uint32)
        codes = np.zeros((max(self.cfg.num_codebooks, 1), max_frames), np.uint32)
        n = C.c_int32()
        _check(lib().oc_drive(self.h, _p(p, C.c_uint32), p.shape[1], max_frames, seed, C.byref(params),
                              _p(codes, C.c_uint32), C.byref(n)))
        return codes[:, : n.value]

    def __del__(self):
        try:
            lib().oc_session_destroy(self.h)
        except Exception:
            pass


def num_threads() -> int:
    return int(lib().oc_num_threads())


def set_num_threads(n: int) -> None:
    lib().oc_set_num_threads(int(n))


def set_qmode(mode: int) -> None:
    """Quantized matmul numerics for Q8_0 and Q4_K weights: 0 = mode A (exact dequant x f32
    activations, the default and what the device computes), 1 = mode B (Candle QMatMul:
    activations quantized to Q8_0 / Q8_K, integer block dots; for analysis)."""
    lib().oc_set_qmode(int(mode))


def get_qmode() -> int:
    return int(lib().oc_get_qmode())


def linear_q4_k(x: np.ndarray, blocks: np.ndarray, n_rows: int) -> np.ndarray:
    """x [M][K] f32 . W^T for Q4_K blocks W [n_rows][K/256 blocks of 144 B], in the current mode."""
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    y = np.empty((M, n_rows), np.float32)
    blocks = np.ascontiguousarray(blocks, np.uint8)
    lib().oc_linear_q4_k(_p(x, C.c_float), blocks.ctypes.data, M, n_rows, K, _p(y, C.c_float))
    return y


def linear_q8_0(x: np.ndarray, blocks: np.ndarray, n_rows: int) -> np.ndarray:
    """x [M][K] f32 . W^T for Q8_0 blocks W [n_rows][K/32 blocks], in the current mode."""
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    y = np.empty((M, n_rows), np.float32)
    blocks = np.ascontiguousarray(blocks, np.uint8)
    lib().oc_linear_q8_0(_p(x, C.c_float), blocks.ctypes.data, M, n_rows, K, _p(y, C.c_float))
    return y
