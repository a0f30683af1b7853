"""The TMA-fed batch-1 Q8_0 GEMV (opt-in with SYRINX_GEMV_TMA=1, read once per process) against
the CPU oracle: greedy frames token-identical and step-0 logits within 2e-2, at the
Qwen3-4B shapes (K = 2560 / 4096 / 9728, the whole-row stage plans with one and two x units
per lane) and at the small-K tiny model (row groups, extra stop rows in the head).
Runs in a child process so the switch takes effect before the first launch."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

import syrinx_b200 as sx
from syrinx_b200.configs import SX_DTYPE_Q8_0, shrink
from syrinx_b200.workloads import dual_ar_prompt
from oracle import oracle as oc

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, sys
import numpy as np
import syrinx_b200 as sx
from syrinx_b200.configs import SX_DTYPE_Q8_0, shrink
from syrinx_b200.workloads import dual_ar_prompt
name, n_frames = sys.argv[1], int(sys.argv[2])
cfg = shrink(sx.QWEN3_4B, 2, 2) if name == "qwen3" else sx.TINY_S2
prompt = dual_ar_prompt(cfg, 48, 40, seed=5)
model = sx.Model(cfg, sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=5))
be = sx.B200DualAr(model, max_ctx=48 + n_frames + 8)
st = be.prefill(prompt)
frames = be.decode_greedy(n_frames, mask_stop=True)
print(json.dumps({"logits": np.asarray(st.semantic_logits, np.float64).tolist(), "frames": frames.tolist()}))
"""


def run_child(name, n_frames):
    env = dict(os.environ, SYRINX_GEMV_TMA="1")
    out = subprocess.run([sys.executable, "-c", CHILD, name, str(n_frames)], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("name", ["qwen3", "tiny"])
def test_tma_gemv_decode_matches_oracle(name):
    n_frames = 12
    got = run_child(name, n_frames)
    cfg = shrink(sx.QWEN3_4B, 2, 2) if name == "qwen3" else sx.TINY_S2
    prompt = dual_ar_prompt(cfg, 48, 40, seed=5)
    blob = sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=5)
    om = oc.OracleModel(cfg, blob)
    os_ = oc.OracleSession(om, 48 + n_frames + 8, kv_bf16=False)
    ol, _ = os_.prefill(prompt)
    err = float(np.max(np.abs(np.asarray(got["logits"]) - np.asarray(ol, np.float64))))
    assert err <= 2e-2, err
    os_.reset()
    ofr, margins = os_.drive_greedy(prompt, n_frames, mask_stop=True)
    frames = np.asarray(got["frames"], dtype=ofr.dtype)
    bad = np.argwhere(frames != ofr)
    assert bad.size == 0, f"first mismatch frame {bad[0]}, semantic top-2 margin {margins[bad[0][0]]:.2e}"
