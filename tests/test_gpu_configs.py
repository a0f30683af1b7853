"""Parity at the BASELINE configuration shapes (GPU vs the CPU oracle, through the C ABI),
plus size-independent properties at full size.

  config 1  CosyVoice2-LM-shaped Qwen2, Q8_0, seed 0: prompt 128 ids, 64 greedy steps
            with the stop ids masked (min_len covering the run, cv2/sampling.rs:114-122)
  config 2  s1-mini-shaped dual-AR, Q8_0, seed 1: prompt 256, 128 greedy frames
  config 3  Qwen3-4B-shaped dual-AR, Q8_0, seed 2: the BASELINE 512-token prompt (82 text ids
            + 430 reference-voice positions), step-0 logits and 64 greedy frames against the
            oracle run live on the host cores
  config 4  the same architecture in Q4_K at full depth (36 + 4 layers): 8 utterances of
            prompt lengths in [256, 1024] decoded as one batch of 8 on the paged cache, each
            against its own oracle run (committed fixtures, tests/golden/config4_q4k.npz,
            made by tests/golden/make_oracle_fixtures.py: minutes of CPU oracle time)
"""
import numpy as np
import pytest

import syrinx_b200 as sx
from syrinx_b200.configs import SX_DTYPE_Q4_K, SX_DTYPE_Q8_0, shrink
from syrinx_b200.workloads import dual_ar_prompt, lm_prompt, prompt_for
from oracle import oracle as oc

pytestmark = pytest.mark.gpu


def maxabs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def run_pair(cfg, wtype, seed, prompt, n_frames, max_ctx, mask_stop=True):
    blob = sx.synth_blob(cfg, wtype, seed=seed)
    model = sx.Model(cfg, blob)
    be = sx.B200DualAr(model, max_ctx=max_ctx)
    st = be.prefill(prompt)
    frames = be.decode_greedy(n_frames, mask_stop=mask_stop)
    om = oc.OracleModel(cfg, blob)
    os_ = oc.OracleSession(om, max_ctx, kv_bf16=False)
    ol, _ = os_.prefill(prompt)
    err0 = maxabs(st.semantic_logits, ol)
    os_.reset()
    ofr, margins = os_.drive_greedy(prompt, n_frames, mask_stop=mask_stop)
    be.close()
    model.close()
    return frames, ofr, err0, margins


def assert_identical(frames, ofr, margins):
    assert frames.shape == ofr.shape, (frames.shape, ofr.shape)
    bad = np.argwhere(frames != ofr)
    assert bad.size == 0, f"first mismatch frame {bad[0]}, semantic top-2 margin there {margins[bad[0][0]]:.2e}"


def test_config1_cosyvoice2_qwen2():
    cfg = sx.COSYVOICE2_LM
    prompt = lm_prompt(cfg, 128, seed=0)
    frames, ofr, err0, margins = run_pair(cfg, SX_DTYPE_Q8_0, 0, prompt, 64, 256)
    print(f"config1 step-0 logits max-abs {err0:.3e}, min margin {margins.min():.3e}")
    assert err0 <= 2e-2
    assert_identical(frames, ofr, margins)


def test_config2_s1_mini():
    cfg = sx.S1_MINI
    prompt = dual_ar_prompt(cfg, 256, 200, seed=1)
    frames, ofr, err0, margins = run_pair(cfg, SX_DTYPE_Q8_0, 1, prompt, 128, 512)
    print(f"config2 step-0 logits max-abs {err0:.3e}, min margin {margins.min():.3e}")
    assert err0 <= 2e-2
    assert_identical(frames, ofr, margins)


def test_config3_qwen3_4b_512_prompt_64_frames():
    cfg = sx.QWEN3_4B
    prompt = dual_ar_prompt(cfg, 512, 430, seed=2)
    frames, ofr, err0, margins = run_pair(cfg, SX_DTYPE_Q8_0, 2, prompt, 64, 600)
    print(f"config3 (512-token prompt) step-0 logits max-abs {err0:.3e}, min margin {margins.min():.3e}")
    assert err0 <= 2e-2
    assert_identical(frames, ofr, margins)


def test_config4_q4k_full_depth_batch8_vs_oracle(golden_dir):
    import os
    import sys
    sys.path.insert(0, golden_dir)
    from make_oracle_fixtures import CONFIG4_FRAMES, CONFIG4_SEED, config4_prompts

    fx = np.load(os.path.join(golden_dir, "config4_q4k.npz"))
    cfg = sx.QWEN3_4B
    prompts = config4_prompts(cfg)
    assert [p.shape[1] for p in prompts] == list(fx["lens"])
    blob = sx.synth_blob(cfg, SX_DTYPE_Q4_K, seed=CONFIG4_SEED)
    model = sx.Model(cfg, blob)
    be = sx.B200DualAr(model, max_ctx=max(fx["lens"]) + CONFIG4_FRAMES + 8, max_batch=8)
    st = be.prefill_batch(prompts)
    got = be.decode_greedy_batch(8, CONFIG4_FRAMES, mask_stop=True)
    lo, hi = cfg.semantic_begin_id, cfg.semantic_end_id
    for i in range(8):
        sem = np.concatenate([st.semantic_logits[i, lo:hi + 1], st.semantic_logits[i, cfg.stop_token_id:][:1]])
        err = maxabs(sem, fx["logits0_semantic"][i])
        print(f"config4 utterance {i} (T={fx['lens'][i]}): step-0 semantic logits max-abs {err:.3e}, "
              f"min margin {fx['margins'][i].min():.3e}")
        assert err <= 2e-2
        assert_identical(got[i], fx["frames"][i], fx["margins"][i])
    be.close()
    model.close()


def test_q4k_batched_shallow_vs_oracle():
    cfg = shrink(sx.QWEN3_4B, 6, 4, name="qwen3-4b-L6-q4k")
    blob = sx.synth_blob(cfg, SX_DTYPE_Q4_K, seed=3)
    model = sx.Model(cfg, blob)
    prompts = [dual_ar_prompt(cfg, T, T - 8, seed=30 + i) for i, T in enumerate((40, 25, 57, 33))]
    be = sx.B200DualAr(model, max_ctx=128, max_batch=4)
    be.prefill_batch(prompts)
    got = be.decode_greedy_batch(4, 24, mask_stop=True)
    om = oc.OracleModel(cfg, blob)
    for p, g in zip(prompts, got):
        os_ = oc.OracleSession(om, 128, kv_bf16=False)
        ofr, margins = os_.drive_greedy(p, 24, mask_stop=True)
        assert_identical(g, ofr, margins)
    be.close()
    model.close()


def test_config3_full_prompt_properties():
    """Full 512-token prompt, 64 frames: deterministic, batched == single, codes in range,
    and KV-cache exactness (cached step == recompute of the longer prompt, the invariant of
    tests/real_lm_kvcache.rs:143-240)."""
    cfg = sx.QWEN3_4B
    blob = sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=2)
    model = sx.Model(cfg, blob)
    prompt = dual_ar_prompt(cfg, 512, 430, seed=2)
    be = sx.B200DualAr(model, max_ctx=640, max_batch=2)
    be.prefill(prompt)
    a = be.decode_greedy(64, mask_stop=True)
    be.reset()
    be.prefill(prompt)
    b = be.decode_greedy(64, mask_stop=True)
    assert np.array_equal(a, b)
    assert np.all((a[:, 0] >= cfg.semantic_begin_id) & (a[:, 0] <= cfg.semantic_end_id))
    assert np.all(a[:, 1:] < cfg.codebook_size)
    assert np.all(a[:, 1] == a[:, 0] - cfg.semantic_begin_id)  # first_code
    # batched (two copies of the prompt) == single
    be.prefill_batch([prompt, prompt])
    bb = be.decode_greedy_batch(2, 64, mask_stop=True)
    assert np.array_equal(bb[0], a) and np.array_equal(bb[1], a)
    # cached single-token step == prefill of the extended prompt (last position)
    be.reset()
    be.prefill(prompt)
    frame = a[0]
    step = be.slow_step(frame, 512)
    be.reset()
    ext = np.concatenate([prompt, frame[:, None]], axis=1)
    full = be.prefill(ext)
    assert int(np.argmax(step.semantic_logits)) == int(np.argmax(full.semantic_logits))
    assert maxabs(step.semantic_logits, full.semantic_logits) <= 1e-3
    be.close()
    model.close()
