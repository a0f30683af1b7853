"""Host-side checks of bench.py that need no GPU: the kernel count it claims per greedy frame
(`gpu_launches`) follows the decode chain's sequence, with and without the folded merges."""
import importlib
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from syrinx_b200 import QWEN3_4B, shrink  # noqa: E402


def kernels_per_frame(cfg, env):
    old = {k: os.environ.get(k) for k in ("SYRINX_QKV_MERGE", "SYRINX_GLU_MERGE")}
    try:
        for k in old:
            os.environ.pop(k, None)
        os.environ.update(env)
        bench = importlib.import_module("bench")
        return bench.kernels_per_frame(cfg, stack=False)
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def test_kernels_per_frame_matches_the_launch_list():
    # 8 slow + 4 fast layers, 10 codebooks: the ncu launch list of that decode lists 369
    # launches per frame (profiles/launches_frames_config3.md: per 4 frames 808 k_gemv_q8<1>,
    # 384 k_merge_q8<1, 1>, 40 k_merge_q8<1, 3>, 192 k_attention, 40 k_take_code and one
    # k_take_semantic, k_advance and k_embed per frame)
    cfg = shrink(QWEN3_4B, 8, 4)
    assert kernels_per_frame(cfg, {}) == (808 + 384 + 40 + 192 + 40 + 3 * 4) // 4 == 369
    # each of the 48 layer steps has 7 launches folded, 9 with both separate merges
    assert kernels_per_frame(cfg, {"SYRINX_QKV_MERGE": "1", "SYRINX_GLU_MERGE": "1"}) == 369 + 2 * 48
    assert kernels_per_frame(cfg, {"SYRINX_QKV_MERGE": "1"}) == 369 + 48
