"""GPU parity of the B200 path against the CPU oracle and the reference's golden vectors,
through the C ABI. Tolerances: dequantization bit-exact; logits max-abs <= 2e-2 against
the oracle (the bound the reference's parity tests use, tests/real_fish_s2_parity.rs:42);
greedy token streams identical. The default device session keeps K/V in f32, as the
reference CPU cache does, and is compared with the oracle in the same mode (kv_bf16=False).
The bf16 KV mode is compared with the oracle rounding K/V to bf16 the same way, within the
logit tolerance (bf16 rounding turns last-ulp f32 differences into 2^-8 steps, so near-tie
argmaxes may differ there)."""
import numpy as np
import pytest

import syrinx_b200 as sx
from syrinx_b200 import _lib
from syrinx_b200.configs import SX_DTYPE_Q4_K, SX_DTYPE_Q8_0, TINY_S2, shrink
from syrinx_b200.workloads import dual_ar_prompt, prompt_for
from oracle import oracle as oc
from tests.toy_lm import TOY_CFG, toy_blob

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2


def maxabs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def test_dequantize_bitexact(quant_golden):
    import ctypes as C
    g = quant_golden
    for dtype, blocks, gold, per, bb in ((SX_DTYPE_Q8_0, g["q8_blocks"], g["q8_deq"], 32, 34),
                                         (SX_DTYPE_Q4_K, g["q4k_blocks"], g["q4k_deq"], 256, 144)):
        out = np.empty(blocks.size // bb * per, np.float32)
        _lib.check(_lib.lib().sx_dequantize(dtype, blocks.ctypes.data, blocks.size // bb,
                                            out.ctypes.data_as(C.POINTER(C.c_float)), 0))
        assert np.array_equal(out.view(np.uint32), gold.view(np.uint32))


def test_toy_lm_matches_reference_golden(kats):
    """The reference's toy LM forward (f32 weights) through the device path."""
    k = kats["lm_forward"]
    ids = k["input"]["token_ids"]
    gold = np.array(k["data"], np.float32).reshape(k["shape"])
    model = sx.Model(TOY_CFG, toy_blob())
    be = sx.B200DualAr(model, max_ctx=16)
    rows = [be.lm_step_tokens([t]) for t in ids]
    err = maxabs(np.stack(rows), gold)
    assert err <= k["tol"], err
    be.reset()
    last = be.lm_step_tokens(ids)  # chunked causal prefill of all five tokens
    assert maxabs(last, gold[-1]) <= k["tol"]
    be.close()
    model.close()


@pytest.fixture(scope="module", params=[SX_DTYPE_Q8_0, SX_DTYPE_Q4_K], ids=["q8_0", "q4_k"])
def tiny(request):
    cfg = TINY_S2
    blob = sx.synth_blob(cfg, request.param, seed=11)
    model = sx.Model(cfg, blob)
    om = oc.OracleModel(cfg, blob)
    yield cfg, model, om
    model.close()


def test_tiny_prefill_and_step_logits(tiny):
    cfg, model, om = tiny
    prompt = prompt_for(cfg, 37, seed=1)
    be = sx.B200DualAr(model, max_ctx=128)
    os_ = oc.OracleSession(om, 128, kv_bf16=False)
    st = be.prefill(prompt)
    ol, oh = os_.prefill(prompt)
    assert maxabs(st.semantic_logits, ol) <= LOGIT_TOL
    assert maxabs(st.hidden, oh) <= 1e-3
    frame = prompt[:, -1].copy()
    for pos in range(37, 41):
        st = be.slow_step(frame, pos)
        ol, oh = os_.slow_step(frame)
        assert maxabs(st.semantic_logits, ol) <= LOGIT_TOL
        frame[0] = cfg.semantic_begin_id + (pos * 7) % cfg.codebook_size
    be.close()


def test_tiny_fast_expand_greedy(tiny):
    cfg, model, om = tiny
    prompt = prompt_for(cfg, 20, seed=2)
    be = sx.B200DualAr(model, max_ctx=64)
    os_ = oc.OracleSession(om, 64, kv_bf16=False)
    st = be.prefill(prompt)
    _, oh = os_.prefill(prompt)
    for first in (0, 5, cfg.codebook_size - 1):
        codes = be.fast_expand_greedy(first)
        ocodes, _ = os_.fast_expand_greedy(oh, first)
        assert codes == [int(c) for c in ocodes]
    be.close()


@pytest.mark.parametrize("mask_stop", [True, False])
def test_tiny_greedy_decode_token_identical(tiny, mask_stop):
    cfg, model, om = tiny
    prompt = prompt_for(cfg, 29, seed=3)
    be = sx.B200DualAr(model, max_ctx=160)
    be.prefill(prompt)
    frames = be.decode_greedy(64, mask_stop=mask_stop)
    os_ = oc.OracleSession(om, 160, kv_bf16=False)
    ofr, margins = os_.drive_greedy(prompt, 64, mask_stop=mask_stop)
    assert frames.shape == ofr.shape
    assert np.array_equal(frames, ofr), f"first mismatch at {np.argwhere(frames != ofr)[:1]}, margins {margins[:8]}"
    be.close()


def test_greedy_decode_repeatable(tiny):
    """Fresh sessions replaying the frame graph give the oracle's frames every time (the
    kernels of the chain overlap under programmatic dependent launch)."""
    cfg, model, om = tiny
    prompt = prompt_for(cfg, 29, seed=3)
    ofr, _ = oc.OracleSession(om, 160, kv_bf16=False).drive_greedy(prompt, 48, mask_stop=False)
    for _ in range(12):
        be = sx.B200DualAr(model, max_ctx=160)
        be.prefill(prompt)
        assert np.array_equal(be.decode_greedy(48, mask_stop=False), ofr)
        be.close()


def bf16_per_step(cfg, model, om, prompt, n):
    """bf16 KV cache against the oracle rounding K/V to bf16 the same way: teacher-forced on
    the oracle's own frames, the slow-step logits at every one of n steps within the
    tolerance; then the free-running greedy token agreement, reported."""
    be = sx.B200DualAr(model, max_ctx=prompt.shape[1] + n + 8, kv_dtype=sx.SX_DTYPE_BF16)
    os_ = oc.OracleSession(om, prompt.shape[1] + n + 8, kv_bf16=True)
    ofr, _ = os_.drive_greedy(prompt, n, mask_stop=True)
    os_.reset()
    st = be.prefill(prompt)
    ol, _ = os_.prefill(prompt)
    errs = [maxabs(st.semantic_logits, ol)]
    pos = prompt.shape[1]
    for f in range(n - 1):
        st = be.slow_step(ofr[f], pos + f)
        ol, _ = os_.slow_step(ofr[f])
        errs.append(maxabs(st.semantic_logits, ol))
    be.reset()
    be.prefill(prompt)
    frames = be.decode_greedy(n, mask_stop=True)
    agree = float(np.mean(frames == ofr))
    print(f"{cfg.name} bf16 KV: per-step logits max-abs {max(errs):.2e} over {len(errs)} steps, "
          f"free-running token agreement {agree:.3f}")
    be.close()
    return max(errs), agree


def test_bf16_kv_per_step_logits(tiny):
    cfg, model, om = tiny
    err, agree = bf16_per_step(cfg, model, om, prompt_for(cfg, 31, seed=9), 64)
    assert err <= LOGIT_TOL


def test_bf16_kv_per_step_logits_4b_shape():
    cfg = shrink(sx.QWEN3_4B, 4, 2, name="qwen3-4b-L4")
    blob = sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=21)
    model = sx.Model(cfg, blob)
    om = oc.OracleModel(cfg, blob)
    err, agree = bf16_per_step(cfg, model, om, dual_ar_prompt(cfg, 96, 80, seed=21), 64)
    model.close()
    assert err <= LOGIT_TOL


def test_frame_step_and_drive_agree_with_graph_loop(tiny):
    cfg, model, _ = tiny
    prompt = prompt_for(cfg, 16, seed=4)
    be = sx.B200DualAr(model, max_ctx=96)
    be.prefill(prompt)
    ref = be.decode_greedy(12, mask_stop=True)
    be.reset()
    be.prefill(prompt)
    frame, out = None, []
    for _ in range(12):
        frame, stopped = be.frame_step_greedy(frame, mask_stop=True)
        assert not stopped
        out.append(frame.copy())
    assert np.array_equal(np.stack(out), ref)
    # the reference driver loop with a top_k = 1 sampler (host sampling of device logits)
    codes = sx.drive(be, prompt, 12, seed=0, sampling=sx.GREEDY)
    if codes.shape[1] == 12:
        assert np.array_equal(codes.T, ref[:, 1:])
    be.close()


def test_frame_step_bad_frame_is_an_error_and_keeps_the_length(tiny):
    """sx_frame_step_greedy reads the device error flag once, after the whole frame: a frame
    with an out-of-range code returns SX_E_INVALID, leaves the cached length where it was, and
    the next call continues as if the bad frame had never been given."""
    cfg, model, _ = tiny
    prompt = prompt_for(cfg, 10, seed=9)
    be = sx.B200DualAr(model, max_ctx=64)
    be.prefill(prompt)
    f0, _ = be.frame_step_greedy(None, mask_stop=True)
    n = be.seq_len()
    bad = f0.copy()
    bad[1] = cfg.codebook_size + 5
    with pytest.raises(sx.SyrinxError) as e:
        be.frame_step_greedy(bad, mask_stop=True)
    assert e.value.code == -1  # code out of range, reported by the embed kernel's bounds check
    assert be.seq_len() == n
    f1, _ = be.frame_step_greedy(f0, mask_stop=True)
    assert be.seq_len() == n + 1
    be.reset()
    be.prefill(prompt)
    g0, _ = be.frame_step_greedy(None, mask_stop=True)
    g1, _ = be.frame_step_greedy(g0, mask_stop=True)
    assert np.array_equal(f0, g0) and np.array_equal(f1, g1)
    be.close()


def test_batched_decode_equals_single(tiny):
    """Sample i of a batch reproduces a batch-1 run (dualar.rs:237-241), with prompts of
    different lengths kept unpadded in the paged cache."""
    cfg, model, _ = tiny
    prompts = [prompt_for(cfg, T, seed=10 + i) for i, T in enumerate((9, 23, 16))]
    be = sx.B200DualAr(model, max_ctx=96, max_batch=4)
    be.prefill_batch(prompts)
    batch = be.decode_greedy_batch(3, 10, mask_stop=True)
    single = sx.B200DualAr(model, max_ctx=96)
    for p, got in zip(prompts, batch):
        single.reset()
        single.prefill(p)
        assert np.array_equal(got, single.decode_greedy(10, mask_stop=True))
    be.close()
    single.close()


def test_batch_step_logits_match_single(tiny):
    cfg, model, _ = tiny
    prompts = [prompt_for(cfg, T, seed=20 + i) for i, T in enumerate((12, 7))]
    be = sx.B200DualAr(model, max_ctx=64, max_batch=2)
    bst = be.prefill_batch(prompts)
    single = sx.B200DualAr(model, max_ctx=64)
    frames = [[cfg.semantic_begin_id + 3] + [1] * cfg.num_codebooks, [cfg.semantic_begin_id + 9] + [2] * cfg.num_codebooks]
    bst2 = be.slow_step_batch(frames)
    for i, p in enumerate(prompts):
        single.reset()
        s0 = single.prefill(p)
        assert maxabs(s0.semantic_logits, bst.semantic_logits[i]) <= 1e-4
        s1 = single.slow_step(frames[i], p.shape[1])
        assert maxabs(s1.semantic_logits, bst2.semantic_logits[i]) <= 1e-4
    be.close()
    single.close()


def test_errors_are_status_codes(tiny):
    cfg, model, _ = tiny
    be = sx.B200DualAr(model, max_ctx=24)
    with pytest.raises(sx.SyrinxError) as e:
        be.slow_step([cfg.semantic_begin_id] + [0] * cfg.num_codebooks, 0)
    assert e.value.code == -5  # before prefill
    bad = prompt_for(cfg, 8, seed=5)
    bad[1, -1] = cfg.codebook_size + 3
    with pytest.raises(sx.SyrinxError) as e:
        be.prefill(bad)
    assert e.value.code == -1  # code out of range, reported by the kernel's bounds check
    be.reset()
    with pytest.raises(sx.SyrinxError) as e:
        be.prefill(prompt_for(cfg, 30, seed=6))
    assert e.value.code == -7  # exceeds max_ctx
    be.reset()
    st = be.prefill(prompt_for(cfg, 8, seed=7))  # the session stays usable
    assert np.all(np.isfinite(st.semantic_logits))
    with pytest.raises(sx.SyrinxError) as e:
        be.slow_step([cfg.semantic_begin_id] + [0] * cfg.num_codebooks, 3)
    assert e.value.code == -5  # pos != cache length
    be.close()


def test_profile_gemv_runs(tiny):
    cfg, model, _ = tiny
    be = sx.B200DualAr(model, max_ctx=16)
    be.prefill(prompt_for(cfg, 4, seed=8))
    for kind in range(4):
        be.profile_gemv(kind, 3)
    be.close()


def test_long_context_token_identical(tiny):
    """A 1200-token prompt in a 2100-position session (attention keys split over an 8-CTA
    cluster of ~150 keys each), then 16 greedy frames against the oracle."""
    cfg, model, om = tiny
    prompt = prompt_for(cfg, 1200, seed=5)
    be = sx.B200DualAr(model, max_ctx=2100)
    st = be.prefill(prompt)
    frames = be.decode_greedy(16, mask_stop=True)
    os_ = oc.OracleSession(om, 2100, kv_bf16=False)
    ol, _ = os_.prefill(prompt)
    assert maxabs(st.semantic_logits, ol) <= LOGIT_TOL
    os_.reset()
    ofr, margins = os_.drive_greedy(prompt, 16, mask_stop=True)
    assert np.array_equal(frames, ofr), f"first mismatch at {np.argwhere(frames != ofr)[:1]}, margins {margins[:8]}"
    be.close()
