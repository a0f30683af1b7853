"""Oracle outputs at BASELINE sizes that take the CPU oracle minutes, committed as fixtures so
the GPU parity tests compare against them in seconds.

  config4_q4k.npz  BASELINE config 4: the Qwen3-4B-shaped dual-AR in Q4_K (weights seed 2),
                   8 utterances with prompt lengths uniform in [256, 1024] (numpy
                   default_rng(4)), prompt i = dual_ar_prompt(T_i, round(T_i * 430/512),
                   seed 40 + i). Per utterance the oracle (mode A, f32 KV cache) gives the
                   step-0 logits of the semantic range plus the stop id, and 64 greedy frames
                   with the stop id masked, with the top-2 margin of each semantic argmax.

The oracle computes every output element on one thread in a fixed order, so its results do
not depend on the thread count; the synthetic weights come from the library's seeded writer
(sx_synth_blob_write, host code). Regenerate with
    python tests/golden/make_oracle_fixtures.py
"""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

CONFIG4_SEED = 2
CONFIG4_FRAMES = 64
CONFIG4_UTTERANCES = 8


def config4_prompts(cfg):
    from syrinx_b200.workloads import config4_prompts as prompts

    return prompts(cfg, CONFIG4_UTTERANCES)


def config4() -> None:
    import syrinx_b200 as sx
    from oracle import oracle as oc
    from syrinx_b200.configs import SX_DTYPE_Q4_K

    cfg = sx.QWEN3_4B
    blob = sx.synth_blob(cfg, SX_DTYPE_Q4_K, seed=CONFIG4_SEED)
    om = oc.OracleModel(cfg, blob)
    prompts = config4_prompts(cfg)
    lo, hi = cfg.semantic_begin_id, cfg.semantic_end_id
    frames, margins, logits0 = [], [], []
    for i, p in enumerate(prompts):
        t0 = time.time()
        s = oc.OracleSession(om, p.shape[1] + CONFIG4_FRAMES + 8, kv_bf16=False)
        l0, _ = s.prefill(p)
        sem = np.concatenate([l0[lo:hi + 1], l0[cfg.stop_token_id:cfg.stop_token_id + 1]])
        s.reset()
        fr, mg = s.drive_greedy(p, CONFIG4_FRAMES, mask_stop=True)
        assert fr.shape[0] == CONFIG4_FRAMES
        frames.append(fr)
        margins.append(mg)
        logits0.append(sem.astype(np.float32))
        print(f"utterance {i}: T={p.shape[1]} {time.time() - t0:.1f} s, min margin {mg.min():.3e}", flush=True)
    np.savez_compressed(os.path.join(HERE, "config4_q4k.npz"), lens=np.array([p.shape[1] for p in prompts], np.int32),
                        frames=np.stack(frames), margins=np.stack(margins), logits0_semantic=np.stack(logits0))


if __name__ == "__main__":
    config4()
