"""The oracle's two quantized-matmul modes on a small Q8_0 linear.

Mode A (the default, what the device computes): exact dequantized weights x f32 activations.
Mode B (analysis only): Candle's CPU QMatMul / ggml vec_dot_q8_0_q8_0, restated here
independently in numpy (activation rows quantized to Q8_0 blocks with the gguf-pinned
quantizer, exact int32 block dots, f32 sum of sumi * (d_w * d_x) in block order) and
required bit-exact."""
import numpy as np
import pytest

from oracle import oracle as oc


@pytest.fixture
def q8_case():
    rng = np.random.default_rng(7)
    M, N, K = 3, 40, 256
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    x = rng.normal(0, 1.0, (M, K)).astype(np.float32)
    blocks = oc.q8_0_quantize(w.reshape(-1)).reshape(N, -1)
    return x, blocks, N, K


def test_default_mode_is_exact_dequant(q8_case):
    x, blocks, N, K = q8_case
    assert oc.get_qmode() == 0
    y = oc.linear_q8_0(x, blocks, N)
    wd = oc.q8_0_dequantize(blocks.reshape(-1)).reshape(N, K).astype(np.float64)
    ref = x.astype(np.float64) @ wd.T
    assert np.max(np.abs(y - ref)) <= 1e-5 * max(1.0, np.max(np.abs(ref)))


def test_mode_b_matches_ggml_restatement(q8_case):
    x, blocks, N, K = q8_case
    nb = K // 32
    oc.set_qmode(1)
    try:
        y = oc.linear_q8_0(x, blocks, N)
    finally:
        oc.set_qmode(0)
    wb = blocks.reshape(N, nb, 34)
    dw = wb[:, :, :2].copy().view(np.float16).reshape(N, nb).astype(np.float32)
    qw = wb[:, :, 2:].view(np.int8).astype(np.int32)
    for m in range(x.shape[0]):
        xb = oc.q8_0_quantize(x[m]).reshape(nb, 34)
        dx = xb[:, :2].copy().view(np.float16).reshape(nb).astype(np.float32)
        qx = xb[:, 2:].view(np.int8).astype(np.int32)
        for r in range(N):
            sumf = np.float32(0.0)
            for b in range(nb):
                sumi = int(np.dot(qw[r, b], qx[b]))
                sumf = np.float32(sumf + np.float32(np.float32(sumi) * np.float32(dw[r, b] * dx[b])))
            assert y[m, r] == sumf, (m, r, y[m, r], sumf)
