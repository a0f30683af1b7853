"""The device sampler (sx_decode_sample) against the host-sampled driver loop (sx_drive, the
restatement of the reference `drive` with `Sampler`) and against the CPU oracle's own
`oc_drive` (the reference `drive` + `Sampler` over the oracle's logits): same prompt, seed
and parameters give the same residual codes, the same frame count and the same stop, over
several parameter sets (top-k / top-p / temperature / RAS window), on the tiny dual-AR and
on a 2-layer Qwen3-4B-width model (4096 + 1 allowed semantic ids, 4096 codes)."""
import ctypes as C

import numpy as np
import pytest

import syrinx_b200 as sx
from syrinx_b200 import _lib
from syrinx_b200.configs import SX_DTYPE_Q8_0, TINY_S2, shrink
from syrinx_b200.workloads import dual_ar_prompt, prompt_for
from oracle import oracle as oc

pytestmark = pytest.mark.gpu

PARAMS = [
    (7, sx.SamplingParams()),
    (123, sx.SamplingParams(temperature=0.7, top_p=0.95, top_k=0)),
    (5, sx.SamplingParams(temperature=1.3, top_p=0.8, top_k=5, ras_win_size=4, ras_high_temp=1.5)),
    (99, sx.SamplingParams(temperature=1.0, top_p=1.0, top_k=0, ras_win_size=1)),
]


def host_drive(be, prompt, n, seed, params):
    cfg = be.cfg
    p = np.ascontiguousarray(prompt, dtype=np.uint32)
    codes = np.zeros((cfg.num_codebooks, n), np.uint32)
    nf = C.c_int32()
    pc = params.to_c()
    _lib.check(_lib.lib().sx_drive(be.handle, p.ctypes.data_as(C.POINTER(C.c_uint32)), p.shape[-1], n, seed,
                                   C.byref(pc), codes.ctypes.data_as(C.POINTER(C.c_uint32)), C.byref(nf)))
    return codes[:, : nf.value]


def check(cfg, blob_seed, prompt, n):
    model = sx.Model(cfg, sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=blob_seed))
    be = sx.B200DualAr(model, max_ctx=prompt.shape[-1] + n + 8)
    for seed, params in PARAMS:
        ref = host_drive(be, prompt, n, seed, params)
        be.reset()
        be.prefill(prompt)
        frames = be.decode_sample(n, seed, params)
        assert frames.shape[0] == ref.shape[1], (seed, frames.shape, ref.shape)
        assert np.array_equal(frames[:, 1:].T, ref), f"seed {seed}: first mismatch {np.argwhere(frames[:, 1:].T != ref)[:1]}"
        assert np.all(frames[:, 1] == np.clip(frames[:, 0].astype(np.int64) - cfg.semantic_begin_id, 0,
                                              cfg.codebook_size - 1))
    be.close()
    model.close()


def test_device_sampler_matches_host_drive_tiny():
    check(TINY_S2, 13, prompt_for(TINY_S2, 20, seed=13), 48)


def test_device_sampler_matches_host_drive_4b_width():
    cfg = shrink(sx.QWEN3_4B, 2, 1, name="qwen3-4b-L2")
    check(cfg, 17, dual_ar_prompt(cfg, 24, 18, seed=17), 32)


def check_oracle(cfg, blob_seed, prompt, n):
    blob = sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=blob_seed)
    model = sx.Model(cfg, blob)
    max_ctx = prompt.shape[-1] + n + 8
    be = sx.B200DualAr(model, max_ctx=max_ctx)
    om = oc.OracleModel(cfg, blob)
    osess = oc.OracleSession(om, max_ctx, kv_bf16=False)
    for seed, params in PARAMS:
        ref = osess.drive(prompt, n, seed, params.to_c())
        be.reset()
        be.prefill(prompt)
        frames = be.decode_sample(n, seed, params)
        assert frames.shape[0] == ref.shape[1], (seed, frames.shape, ref.shape)
        bad = np.argwhere(frames[:, 1:].T != ref)
        assert bad.size == 0, f"seed {seed}: first mismatch (codebook, frame) {bad[0]}"
    be.close()
    model.close()


def test_device_sampler_matches_oracle_drive_tiny():
    check_oracle(TINY_S2, 13, prompt_for(TINY_S2, 20, seed=13), 48)


def test_device_sampler_matches_oracle_drive_4b_width():
    cfg = shrink(sx.QWEN3_4B, 2, 1, name="qwen3-4b-L2")
    check_oracle(cfg, 17, dual_ar_prompt(cfg, 24, 18, seed=17), 32)
