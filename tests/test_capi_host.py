"""Host-side checks of libsyrinx_b200.so that need no GPU: every symbol declared in
include/*.h is exported, the synthetic blob writer is deterministic and its tensors are
valid GGML blocks (read back through the independent oracle parser), and device calls
fail cleanly with a status code when no GPU is visible."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import syrinx_b200 as sx
from syrinx_b200 import _lib
from syrinx_b200.blob import write_blob
from syrinx_b200.configs import SX_DTYPE_F32, SX_DTYPE_Q4_K, SX_DTYPE_Q8_0, TINY_S2, shrink
from oracle import oracle as oc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    for name in os.listdir(os.path.join(ROOT, "include")):
        if name.endswith(".h"):
            text = open(os.path.join(ROOT, "include", name)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            syms |= set(re.findall(r"\b(sx_[a-z0-9_]+)\s*\(", text))
    return syms


def test_every_declared_symbol_is_exported():
    L = _lib.lib()
    syms = declared_symbols()
    assert len(syms) >= 25
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    assert set(_lib.SIGNATURES) == syms, "ctypes signature table out of sync with the header"


def declared_param_counts():
    """sx_name -> number of parameters, from the prototypes in include/*.h."""
    out = {}
    for name in os.listdir(os.path.join(ROOT, "include")):
        if name.endswith(".h"):
            text = open(os.path.join(ROOT, "include", name)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            for fn, params in re.findall(r"\b(sx_[a-z0-9_]+)\s*\(([^;{)]*)\)\s*;", text, flags=re.S):
                params = params.strip()
                out[fn] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_ctypes_signatures_match_header_parameter_counts():
    counts = declared_param_counts()
    assert len(counts) >= 25
    bad = {fn: (n, len(_lib.SIGNATURES[fn][1])) for fn, n in counts.items()
           if fn in _lib.SIGNATURES and len(_lib.SIGNATURES[fn][1]) != n}
    assert not bad, f"parameter counts differ (header, ctypes): {bad}"


def test_version_and_error_string():
    L = _lib.lib()
    assert b"sm_100a" in L.sx_version()
    assert isinstance(L.sx_last_error(), bytes)


def test_synth_blob_deterministic_and_seeded():
    cfg = shrink(TINY_S2, 1, 1)
    a = sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=3)
    b = sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=3)
    c = sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=4)
    assert np.array_equal(a, b)
    assert not np.array_equal(a, c)


@pytest.mark.parametrize("wtype", [SX_DTYPE_Q8_0, SX_DTYPE_Q4_K, SX_DTYPE_F32])
def test_synth_blob_tensors_valid(wtype):
    cfg = shrink(TINY_S2, 1, 1)
    blob = sx.synth_blob(cfg, wtype, seed=1)
    m = oc.OracleModel(cfg, blob)
    w = m.tensor("layers.0.attention.wqkv.weight")
    assert w.shape == (cfg.slow.qkv_rows, cfg.slow.dim)
    # N(0, 0.02)-distributed before quantization
    assert 0.015 < float(w.std()) < 0.025 and abs(float(w.mean())) < 2e-3
    assert np.all(m.tensor("layers.0.attention_norm.weight") == 1.0)
    if wtype == SX_DTYPE_F32:
        return
    # re-quantizing the dequantized Q8_0 values reproduces the blocks (a valid quantization)
    if wtype == SX_DTYPE_Q8_0:
        blocks = oc.q8_0_quantize(w)
        assert np.array_equal(oc.q8_0_dequantize(blocks), w.reshape(-1))


def test_q4_k_quantizer_error_bound():
    """The writer's Q4_K min/max fit: per-element error within one sub-block step."""
    cfg = shrink(TINY_S2, 1, 1)
    f32 = oc.OracleModel(cfg, sx.synth_blob(cfg, SX_DTYPE_F32, seed=5)).tensor("layers.0.feed_forward.w2.weight")
    q4 = oc.OracleModel(cfg, sx.synth_blob(cfg, SX_DTYPE_Q4_K, seed=5)).tensor("layers.0.feed_forward.w2.weight")
    err = np.abs(f32 - q4)
    assert float(err.max()) < 0.02
    assert float(err.mean()) < 0.004


def test_blob_writer_roundtrip():
    rng = np.random.default_rng(0)
    t = {"a.weight": rng.normal(size=(3, 64)).astype(np.float32), "b": rng.normal(size=64).astype(np.float32)}
    x = rng.normal(0, 0.05, size=(2, 64)).astype(np.float32)
    t["q.weight"] = (SX_DTYPE_Q8_0, (2, 64), oc.q8_0_quantize(x))
    blob = write_blob(t)
    assert bytes(blob[:4]) == b"SXW1"
    from tests.toy_lm import TOY_CFG
    m = oc.OracleModel.__new__(oc.OracleModel)  # parse-only through a tensor query
    m.cfg, m.blob, m._desc = TOY_CFG, blob, TOY_CFG.to_c()
    m.h = C.c_void_p()
    rc = oc.lib().oc_model_create(C.byref(m._desc), blob.ctypes.data, blob.nbytes, C.byref(m.h))
    assert rc != 0  # not a toy LM: binding fails on a missing tensor, with a message
    assert b"missing tensor" in oc.lib().oc_last_error()


def test_model_create_without_gpu_reports_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    cfg = shrink(TINY_S2, 1, 1)
    blob = sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=0)
    with pytest.raises(sx.SyrinxError) as e:
        sx.Model(cfg, blob, device=0)
    assert e.value.code in (-2, -1)


def test_bad_blob_rejected_before_device():
    L = _lib.lib()
    cfg = shrink(TINY_S2, 1, 1)
    desc = cfg.to_c()
    junk = np.zeros(64, np.uint8)
    h = C.c_void_p()
    rc = L.sx_model_create(C.byref(desc), junk.ctypes.data, junk.nbytes, 0, C.byref(h))
    assert rc < 0 and not h.value


def test_frame_bytes_config3():
    """bytes/frame of the Qwen3-4B-shaped Q8_0 config: 8.674 GB of weights at b1 (full head)."""
    fb = sx.frame_bytes(sx.QWEN3_4B, SX_DTYPE_Q8_0, ctx=640, semantic_head=False)
    assert abs(fb["slow"] + fb["head"] + fb["fast"] - 8.674e9) / 8.674e9 < 0.01
    assert abs(fb["kv"] - 147456 * 640) < 1
