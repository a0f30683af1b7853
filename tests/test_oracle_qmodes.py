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


@pytest.fixture
def q4k_case():
    """Valid Q4_K blocks with random nibbles and 6-bit scales / mins, and small positive f16
    d / dmin (any bytes decode, only the two f16 fields need to stay finite)."""
    rng = np.random.default_rng(11)
    M, N, K = 3, 24, 512
    nb = K // 256
    blocks = rng.integers(0, 256, (N, nb, 144), dtype=np.uint8)
    d = rng.uniform(1e-4, 4e-3, (N, nb)).astype(np.float16)
    dmin = rng.uniform(1e-4, 4e-3, (N, nb)).astype(np.float16)
    blocks[:, :, 0:2] = d.view(np.uint8).reshape(N, nb, 2)
    blocks[:, :, 2:4] = dmin.view(np.uint8).reshape(N, nb, 2)
    x = rng.normal(0, 1.0, (M, K)).astype(np.float32)
    x[1, 256:] = 0.0  # an all-zero super-block of the activation (d = 0 in Q8_K)
    return x, blocks, N, K


def scale_min_k4(j, sc):
    """Q4_K's 6-bit sub-block scale and min j from the 12 packed bytes."""
    if j < 4:
        return int(sc[j] & 63), int(sc[j + 4] & 63)
    return int((sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4)), int((sc[j + 4] >> 4) | ((sc[j] >> 6) << 4))


def test_q4k_default_mode_is_exact_dequant(q4k_case):
    x, blocks, N, K = q4k_case
    y = oc.linear_q4_k(x, blocks, N)
    wd = oc.q4_k_dequantize(blocks.reshape(-1)).reshape(N, K).astype(np.float64)
    ref = x.astype(np.float64) @ wd.T
    assert np.max(np.abs(y - ref)) <= 1e-5 * max(1.0, np.max(np.abs(ref)))


def test_q4k_mode_b_matches_k_quants_restatement(q4k_case):
    """Mode B for Q4_K restated independently: Q8_K activation blocks (iscale = -128 / signed
    max, halves rounded away from zero, clamped to 127, f32 d = 1 / iscale, sums of 16), the
    integer dot per eight-lane group scaled by the 6-bit sub-block scales, the min term from
    the 16-element sums, f32 lane sums across super-blocks, then sumf + sum of the lanes."""
    x, blocks, N, K = q4k_case
    nb = K // 256
    oc.set_qmode(1)
    try:
        y = oc.linear_q4_k(x, blocks, N)
    finally:
        oc.set_qmode(0)
    f32 = np.float32
    for m in range(x.shape[0]):
        q8, d8, bs = [], [], []
        for b in range(nb):
            xb = x[m, 256 * b: 256 * (b + 1)]
            i = int(np.argmax(np.abs(xb)))  # the first element of largest magnitude
            if xb[i] == 0:
                q8.append(np.zeros(256, np.int32))
                d8.append(f32(0))
                bs.append(np.zeros(16, np.int32))
                continue
            iscale = f32(f32(-128.0) / xb[i])
            v = (iscale * xb).astype(np.float32).astype(np.float64)
            q = np.minimum(127.0, np.sign(v) * np.floor(np.abs(v) + 0.5)).astype(np.int32)
            q8.append(q)
            d8.append(f32(f32(1.0) / iscale))
            bs.append(q.reshape(16, 16).sum(axis=1))
        for r in range(N):
            sums = np.zeros(8, np.float32)
            sumf = f32(0)
            for b in range(nb):
                blk = blocks[r, b]
                dw = blk[0:2].copy().view(np.float16)[0].astype(np.float32)
                mw = blk[2:4].copy().view(np.float16)[0].astype(np.float32)
                qs = blk[16:144].astype(np.int32)
                a = np.empty(256, np.int32)
                for j in range(4):
                    a[64 * j: 64 * j + 32] = qs[32 * j: 32 * j + 32] & 0xF
                    a[64 * j + 32: 64 * j + 64] = qs[32 * j: 32 * j + 32] >> 4
                scs = [scale_min_k4(j, blk[4:16]) for j in range(8)]
                sumi = sum(int(bs[b][j]) * scs[j // 2][1] for j in range(16))
                aux = np.zeros(8, np.int64)
                for j in range(8):
                    prod = (q8[b][32 * j: 32 * j + 32] * a[32 * j: 32 * j + 32]).reshape(4, 8)
                    aux += scs[j][0] * prod.sum(axis=0)
                dd = f32(dw * d8[b])
                for l in range(8):
                    sums[l] = f32(sums[l] + f32(dd * f32(aux[l])))
                dm = f32(mw * d8[b])
                sumf = f32(sumf - f32(dm * f32(sumi)))
            tot = f32(0)
            for l in range(8):
                tot = f32(tot + sums[l])
            assert y[m, r] == f32(sumf + tot), (m, r, y[m, r], f32(sumf + tot))
