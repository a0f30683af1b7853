"""The decode chain's folded merges against the separate merge kernels, bit for bit.

In a decode step the attention kernel adds the wqkv GEMV's k-chunk partials itself, and at one
token the w2 GEMV forms silu(gate) * up from the w1|w3 partials; both add the partials in the
merge kernel's order, so nothing may change in the results. SYRINX_QKV_MERGE=1 and
SYRINX_GLU_MERGE=1 (read once per process) restore the separate k_merge_q8 launches. The same
run in two processes, one each way: greedy frames, the logits and hidden of a cached
single-token step, the fast-AR codes, and a batch of two, all bit-identical.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

RUN = r"""
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import syrinx_b200 as sx
from syrinx_b200.configs import SX_DTYPE_Q8_0, TINY_S2
from syrinx_b200.workloads import prompt_for

cfg = TINY_S2
model = sx.Model(cfg, sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=11))
be = sx.B200DualAr(model, max_ctx=96, max_batch=2)
p0, p1 = prompt_for(cfg, 20, seed=11), prompt_for(cfg, 13, seed=12)
be.prefill(p0)
frames = be.decode_greedy(12, mask_stop=True)
step = be.slow_step(frames[-1], be.seq_len())
codes = np.array(be.fast_expand_greedy(be.first_code(int(np.argmax(step.semantic_logits)))), np.uint32)
be.reset()
be.prefill_batch([p0, p1])
bf = be.decode_greedy_batch(2, 6, mask_stop=True)
bstep = be.slow_step_batch([bf[0][-1], bf[1][-1]])
np.savez(sys.argv[2], frames=frames, logits=step.semantic_logits, hidden=step.hidden, codes=codes,
         b0=bf[0], b1=bf[1], blogits=bstep.semantic_logits, bhidden=bstep.hidden)
be.close()
model.close()
"""


def run(tmp_path, name, separate):
    env = dict(os.environ)
    for k in ("SYRINX_QKV_MERGE", "SYRINX_GLU_MERGE"):
        env.pop(k, None)
        if separate:
            env[k] = "1"
    out = str(tmp_path / f"{name}.npz")
    subprocess.run([sys.executable, "-c", RUN, ROOT, out], env=env, check=True, timeout=180)
    return np.load(out)


def test_folded_merges_bit_identical_to_merge_kernels(tmp_path):
    fold = run(tmp_path, "fold", separate=False)
    sep = run(tmp_path, "sep", separate=True)
    assert fold["frames"].shape[0] == 12
    for k in sep.files:
        a, b = fold[k], sep[k]
        assert a.shape == b.shape, k
        if a.dtype == np.float32:
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"{k}: max diff {np.max(np.abs(a - b))}"
        else:
            assert np.array_equal(a, b), k
