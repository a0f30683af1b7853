"""CPU checks of the two facts the Q8_0 tensor-core GEMV (syrinx_b200/csrc/gemv_q8.cu) rests on.

1. The tile-record layout (q8_quant_off / q8_scale_off in sx_internal.hpp) places every
   (row, k) quant of a 16 x 32 tile exactly once, at the byte where the A-operand fragment
   of mma.m16n8k32 (row-major, .s8) expects it: lane t = 4g + c holds a0..a3 = {row g,
   k 4c..4c+3}, {row g+8, same k}, {row g, k 16+4c..}, {row g+8, k 16+4c..}, and word w of
   the scale area holds {d[w], d[w+8]}, the two rows lane 4w..4w+3 accumulates.
2. The activation split: x = sx * (l0 + l1/128 + l2/128^2 + l3/128^3) with sx a power of
   two, every limb an integer in [-64, 64] (int8), exact to 2^-27 of the block's largest
   |x|; and the GEMV's arithmetic on it (exact int32 limb dots, S0*128 + S1 and S2*128 + S3
   rounded to f32, f32 fma of d*sx, halves weighted 2^-7 and 2^-21) stays within 1e-6 of
   the exact dot relative to the sum of |terms|. Restated here in numpy in the kernel's
   order of f32 operations, on blocks with mixed magnitudes, zeros and tiny values.
"""
import numpy as np


def q8_quant_off(rr, kk):
    return ((rr & 7) * 4 + ((kk & 15) >> 2)) * 16 + ((kk >> 4) * 2 + (rr >> 3)) * 4 + (kk & 3)


def q8_scale_off(rr):
    return 512 + (rr & 7) * 4 + (rr >> 3) * 2


def test_tile_record_is_the_mma_a_fragment():
    seen = set()
    for rr in range(16):
        for kk in range(32):
            off = q8_quant_off(rr, kk)
            assert 0 <= off < 512
            seen.add(off)
            lane, reg, byte = off // 16, (off % 16) // 4, off % 4
            g, c = lane // 4, lane % 4
            # PTX mma.m16n8k32 .s8 A fragment: a0 row g k 4c+i; a1 row g+8; a2 row g k 16+4c+i; a3 row g+8
            exp_row = g + (8 if reg in (1, 3) else 0)
            exp_k = 4 * c + byte + (16 if reg >= 2 else 0)
            assert (rr, kk) == (exp_row, exp_k), (rr, kk, lane, reg, byte)
    assert len(seen) == 512
    scale_offs = {q8_scale_off(rr) for rr in range(16)}
    assert scale_offs == set(range(512, 544, 2))
    for w in range(8):  # word w = {d[w], d[w+8]}: the rows g = w and w + 8 of lanes 4w..4w+3
        assert q8_scale_off(w) == 512 + 4 * w and q8_scale_off(w + 8) == 512 + 4 * w + 2


def f32(v):
    return np.float32(v)


def split_block(x):
    """The kernel's limb split of one 32-wide block (f32 arithmetic, rintf = round half even)."""
    x = x.astype(np.float32)
    mx = np.float32(np.max(np.abs(x)))
    e = (int(np.array(mx, np.float32).view(np.uint32)) >> 23) & 0xFF
    if e < 6:
        return np.zeros((4, 32), np.int64), np.float32(0.0)
    sc = np.array((259 - e) << 23, np.uint32).view(np.float32)
    sx = np.array((e - 5) << 23, np.uint32).view(np.float32)
    s = (x * sc).astype(np.float32)
    l0 = np.rint(s).astype(np.float32)
    r = ((s - l0) * f32(128)).astype(np.float32)
    l1 = np.rint(r).astype(np.float32)
    r = ((r - l1) * f32(128)).astype(np.float32)
    l2 = np.rint(r).astype(np.float32)
    r = ((r - l2) * f32(128)).astype(np.float32)
    l3 = np.rint(r).astype(np.float32)
    return np.stack([l0, l1, l2, l3]).astype(np.int64), np.float32(sx)


def blocks(rng, n):
    out = []
    for i in range(n):
        kind = i % 5
        if kind == 0:
            x = rng.normal(0, 1, 32)
        elif kind == 1:
            x = rng.normal(0, 1, 32) * np.exp(rng.uniform(-12, 12, 32))  # mixed magnitudes
        elif kind == 2:
            x = np.zeros(32)
            x[rng.integers(0, 32)] = rng.normal(0, 50)
        elif kind == 3:
            x = rng.normal(0, 1e-30, 32)  # tiny block
        else:
            x = rng.normal(0, 1, 32)
            x[::3] = 0.0
        out.append(x.astype(np.float32))
    return out


def test_limb_split_exact_to_2e27_of_block_max():
    rng = np.random.default_rng(5)
    for x in blocks(rng, 400):
        limbs, sx = split_block(x)
        assert np.all(np.abs(limbs) <= 64)
        mx = float(np.max(np.abs(x)))
        if sx == 0:
            assert mx < 2.0 ** -121
            continue
        rec = float(sx) * (limbs[0] + limbs[1] / 128.0 + limbs[2] / 128.0 ** 2 + limbs[3] / 128.0 ** 3)
        assert np.max(np.abs(rec - x.astype(np.float64))) <= 2.0 ** -27 * mx


def test_gemv_arithmetic_within_1e6_of_exact():
    rng = np.random.default_rng(9)
    K, rows = 32 * 40, 24
    xs = np.concatenate(blocks(rng, K // 32))
    q = rng.integers(-128, 128, (rows, K)).astype(np.int64)
    d = rng.uniform(0.0005, 0.004, (rows, K // 32)).astype(np.float16).astype(np.float32)
    exact = np.zeros(rows)
    mag = np.zeros(rows)
    acc_hi = np.zeros(rows, np.float32)
    acc_lo = np.zeros(rows, np.float32)
    for b in range(K // 32):
        xb = xs[b * 32:(b + 1) * 32]
        limbs, sx = split_block(xb)
        for r in range(rows):
            qb = q[r, b * 32:(b + 1) * 32]
            S = limbs @ qb  # exact int32 limb sums (|S| <= 32 * 64 * 128)
            assert np.all(np.abs(S) < 2 ** 31)
            hi, lo = np.float32(S[0] * 128 + S[1]), np.float32(S[2] * 128 + S[3])
            f = np.float32(d[r, b] * sx)
            acc_hi[r] = np.float32(np.float64(f) * np.float64(hi) + np.float64(acc_hi[r]))  # one rounding, as fma
            acc_lo[r] = np.float32(np.float64(f) * np.float64(lo) + np.float64(acc_lo[r]))
            t = d[r, b].astype(np.float64) * qb * xb.astype(np.float64)
            exact[r] += t.sum()
            mag[r] += np.abs(t).sum()
    y = (acc_hi * np.float32(2.0 ** -7)).astype(np.float64) + (acc_lo * np.float32(2.0 ** -21)).astype(np.float64)
    assert np.max(np.abs(y - exact) / (mag + 1e-300)) <= 1e-6
