"""The persistent decode kernel (stack.cu: every layer of a stack in one cooperative launch,
weights streamed through a shared-memory ring) against the per-kernel chain it replaces and
against the oracle. SYRINX_STACK=1, read when a session is created, selects the persistent
kernel; the chain is the default. The two paths add the same exact block sums in different
orders (and apply the RMSNorm after the GEMV instead of before), so logits agree to f32
rounding and greedy frames are identical."""
import os

import numpy as np
import pytest

import syrinx_b200 as sx
from syrinx_b200.configs import SX_DTYPE_Q8_0, TINY_S2, shrink
from syrinx_b200.workloads import dual_ar_prompt, prompt_for
from oracle import oracle as oc

pytestmark = pytest.mark.gpu


def session(model, max_ctx, stack: bool, **kw):
    old = os.environ.get("SYRINX_STACK")
    os.environ["SYRINX_STACK"] = "1" if stack else "0"
    try:
        return sx.B200DualAr(model, max_ctx=max_ctx, **kw)
    finally:
        if old is None:
            del os.environ["SYRINX_STACK"]
        else:
            os.environ["SYRINX_STACK"] = old


@pytest.mark.parametrize("cfg,seed,T", [(TINY_S2, 31, 24), (shrink(sx.QWEN3_4B, 3, 2, name="qwen3-4b-L3"), 32, 40),
                                        (shrink(sx.COSYVOICE2_LM, 4, name="cv2-L4"), 33, 30)],
                         ids=["tiny", "4b-L3", "cv2-L4"])
def test_stack_matches_chain_and_oracle(cfg, seed, T):
    blob = sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=seed)
    model = sx.Model(cfg, blob)
    prompt = prompt_for(cfg, T, seed=seed)
    a = session(model, T + 48, stack=True)
    b = session(model, T + 48, stack=False)
    sa, sb = a.prefill(prompt), b.prefill(prompt)
    frame = prompt[:, -1].copy()
    for pos in range(T, T + 3):
        sa, sb = a.slow_step(frame, pos), b.slow_step(frame, pos)
        assert np.max(np.abs(sa.semantic_logits - sb.semantic_logits)) <= 1e-3
    a.reset(); b.reset()
    a.prefill(prompt); b.prefill(prompt)
    fa, fb = a.decode_greedy(32, mask_stop=True), b.decode_greedy(32, mask_stop=True)
    om = oc.OracleModel(cfg, blob)
    ofr, margins = oc.OracleSession(om, T + 48, kv_bf16=False).drive_greedy(prompt, 32, mask_stop=True)
    assert np.array_equal(fa, ofr), f"stack vs oracle: first mismatch {np.argwhere(fa != ofr)[:1]}"
    assert np.array_equal(fb, ofr)
    a.close(); b.close(); model.close()


def test_stack_batched_equals_single():
    cfg = TINY_S2
    model = sx.Model(cfg, sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=34))
    prompts = [prompt_for(cfg, T, seed=40 + i) for i, T in enumerate((9, 23, 16, 30, 12))]
    be = session(model, 96, stack=True, max_batch=8)
    be.prefill_batch(prompts)
    batch = be.decode_greedy_batch(5, 12, mask_stop=True)
    single = session(model, 96, stack=True)
    for p, got in zip(prompts, batch):
        single.reset()
        single.prefill(p)
        assert np.array_equal(got, single.decode_greedy(12, mask_stop=True))
    be.close(); single.close(); model.close()


def test_tensor_core_prefill_bit_identical_to_gemv():
    """The tcgen05 prefill GEMM (gemm_tc.cu) writes the same partials as the mma.sync GEMV:
    prefill logits and the following decode are bit-identical with SYRINX_TC=0 and =1."""
    cfg = shrink(sx.QWEN3_4B, 2, 1, name="qwen3-4b-L2")
    model = sx.Model(cfg, sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=35))
    prompt = dual_ar_prompt(cfg, 150, 120, seed=35)  # chunks of 64, 64, 22 tokens
    out = {}
    for tc in ("0", "1"):
        os.environ["SYRINX_TC"] = tc
        be = sx.B200DualAr(model, max_ctx=200)
        st = be.prefill(prompt)
        out[tc] = (st.semantic_logits.copy(), st.hidden.copy(), be.decode_greedy(6, mask_stop=True))
        be.close()
    del os.environ["SYRINX_TC"]
    assert np.array_equal(out["0"][0].view(np.uint32), out["1"][0].view(np.uint32))
    assert np.array_equal(out["0"][1].view(np.uint32), out["1"][1].view(np.uint32))
    assert np.array_equal(out["0"][2], out["1"][2])
    model.close()
