"""The CosyVoice LM boundary on the GPU, against the CPU oracle, through the C ABI.

  CosyVoice2 (config 1 shape, Q8_0, seed 0): the step-0 input is assembled on the host from
  rows of three tables in the manner of `build_lm_input` (crates/syrinx-lm/src/cv2/
  generate.rs:92): an sos row of a separate `llm_embedding`-like table, text rows of an
  `embed_tokens`-like table, a task-id row, then prompt speech rows of the model's own
  speech table. It goes through sx_lm_step_embeds (`Qwen2Lm::step_logits_cached(embeds)`,
  cv2/generate.rs:119-123); 64 greedy speech tokens follow with the stop ids masked
  (min_len covering the run, cv2/sampling.rs:114-122).
  CosyVoice3 (cv3/mod.rs, cv3/lm.rs:143-169): the same body with the bias-free 6761-row
  `llm_decoder` and the 200 control ids 6561..6760 as the stop set; sos / task id are rows
  of the speech table. Greedy with the stop set masked, then unmasked until a control id.
Tolerances: logits max-abs <= 2e-2, greedy tokens identical.
"""
import numpy as np
import pytest

import syrinx_b200 as sx
from syrinx_b200.configs import SX_DTYPE_Q8_0
from oracle import oracle as oc

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2


def maxabs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def oracle_greedy(osess, om, logits, n, mask_stop):
    """The reference generate loop with a greedy pick: stop on a stop id, else feed the
    token's speech-table row (cv2/generate.rs:136-163, cv3/generate.rs:84-93)."""
    out = []
    cfg = om.cfg
    for _ in range(n):
        tok, _ = om.greedy_semantic(logits, mask_stop=mask_stop)
        if tok in cfg.stop_ids():
            break
        out.append(tok)
        logits = osess.lm_step_tokens([tok])
    return np.array(out, np.uint32)


def test_cv2_embeds_from_several_tables():
    cfg = sx.COSYVOICE2_LM
    blob = sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=0)
    om = oc.OracleModel(cfg, blob)
    speech = om.tensor("embeddings.weight")  # the speech_embedding table the model owns
    rng = np.random.default_rng(5)
    llm_embedding = rng.normal(0, 0.02, (2, cfg.slow.dim)).astype(np.float32)  # sos_eos, task_id
    embed_tokens = rng.normal(0, 0.02, (4000, cfg.slow.dim)).astype(np.float32)
    text_ids = rng.integers(0, 4000, 40)
    prompt_speech = rng.integers(0, 6561, 60)
    embeds = np.concatenate([llm_embedding[:1], embed_tokens[text_ids], llm_embedding[1:2],
                             speech[prompt_speech]]).astype(np.float32)

    model = sx.Model(cfg, blob)
    be = sx.B200DualAr(model, max_ctx=256)
    logits = be.lm_step_embeds(embeds)
    toks = be.decode_greedy(64, mask_stop=True)[:, 0]
    osess = oc.OracleSession(om, 256, kv_bf16=False)
    ol = osess.lm_step_embeds(embeds)
    err = maxabs(logits, ol)
    otoks = oracle_greedy(osess, om, ol, 64, mask_stop=True)
    print(f"cv2 embeds: step-0 logits max-abs {err:.3e}")
    assert err <= LOGIT_TOL
    assert np.array_equal(toks, otoks), f"first mismatch {np.argwhere(toks != otoks)[:1]}"
    # the token shortcut (sx_lm_step_tokens) continues the same cache as the oracle's
    be.reset()
    be.lm_step_embeds(embeds)
    for t in toks[:8]:
        step = be.lm_step_tokens([int(t)])
    osess2 = oc.OracleSession(om, 256, kv_bf16=False)
    osess2.lm_step_embeds(embeds)
    for t in toks[:8]:
        ostep = osess2.lm_step_tokens([int(t)])
    assert maxabs(step, ostep) <= LOGIT_TOL
    be.close()
    model.close()


def test_cv3_head_and_stop_set():
    cfg = sx.COSYVOICE3_LM
    blob = sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=6)
    om = oc.OracleModel(cfg, blob)
    speech = om.tensor("embeddings.weight")  # CV3: sos / task id are rows of this table
    rng = np.random.default_rng(6)
    embed_tokens = rng.normal(0, 0.02, (4000, cfg.slow.dim)).astype(np.float32)
    text_ids = rng.integers(0, 4000, 32)
    prompt_speech = rng.integers(0, 6561, 48)
    embeds = np.concatenate([speech[6561:6562], embed_tokens[text_ids], speech[6563:6564],
                             speech[prompt_speech]]).astype(np.float32)
    model = sx.Model(cfg, blob)
    # stop set masked (step < min_len): 48 tokens identical
    be = sx.B200DualAr(model, max_ctx=256)
    logits = be.lm_step_embeds(embeds)
    toks = be.decode_greedy(48, mask_stop=True)[:, 0]
    osess = oc.OracleSession(om, 256, kv_bf16=False)
    ol = osess.lm_step_embeds(embeds)
    assert logits.shape == (6761,)
    err = maxabs(logits, ol)
    otoks = oracle_greedy(osess, om, ol, 48, mask_stop=True)
    assert err <= LOGIT_TOL
    assert np.array_equal(toks, otoks)
    assert np.all(toks < 6561)
    # stop set live: the run ends on the same control id step
    be.reset()
    be.lm_step_embeds(embeds)
    free = be.decode_greedy(160, mask_stop=False)[:, 0]
    osess3 = oc.OracleSession(om, 256, kv_bf16=False)
    ofree = oracle_greedy(osess3, om, osess3.lm_step_embeds(embeds), 160, mask_stop=False)
    print(f"cv3: step-0 logits max-abs {err:.3e}; unmasked run {free.size} tokens before a control id "
          f"(oracle {ofree.size})")
    assert np.array_equal(free, ofree)
    be.close()
    model.close()
