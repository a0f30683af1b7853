"""sx_dequantize_noalloc (static device scratch, no allocation) against sx_dequantize.

Collected last (file name) and self-contained, so it passes alone and after the rest of
the suite. Two calls in a row with different inputs catch stale scratch; the second one
fills the scratch to its stated capacity. Sizes above the capacity are rejected."""
import ctypes as C

import numpy as np
import pytest

from syrinx_b200 import _lib
from syrinx_b200.configs import SX_DTYPE_Q4_K, SX_DTYPE_Q8_0

pytestmark = pytest.mark.gpu

MAX_BLOCKS = 1024  # SX_DEQUANTIZE_NOALLOC_MAX_BLOCKS
SX_E_RANGE = -7
LAYOUT = {SX_DTYPE_Q8_0: (34, 32, 2), SX_DTYPE_Q4_K: (144, 256, 16)}  # block bytes, values, header bytes


def dequant(fn_name, dtype, blocks):
    bb, per, _ = LAYOUT[dtype]
    n = blocks.size // bb
    out = np.full(n * per, np.nan, np.float32)
    rc = getattr(_lib.lib(), fn_name)(dtype, blocks.ctypes.data, n, out.ctypes.data_as(C.POINTER(C.c_float)), 0)
    _lib.check(rc)
    return out


def full_scratch_blocks(golden_blocks, dtype, seed):
    """MAX_BLOCKS valid blocks: the golden blocks tiled (finite scales kept), quant bytes redrawn."""
    bb, _, hdr = LAYOUT[dtype]
    g = golden_blocks.reshape(-1, bb)
    reps = (MAX_BLOCKS + len(g) - 1) // len(g)
    b = np.tile(g, (reps, 1))[:MAX_BLOCKS].copy()
    b[:, hdr:] = np.random.default_rng(seed).integers(0, 256, size=(MAX_BLOCKS, bb - hdr), dtype=np.uint8)
    return np.ascontiguousarray(b.reshape(-1))


@pytest.mark.parametrize("dtype,key,gold", [(SX_DTYPE_Q8_0, "q8_blocks", "q8_deq"),
                                            (SX_DTYPE_Q4_K, "q4k_blocks", "q4k_deq")])
def test_noalloc_matches_dequantize_two_calls(quant_golden, dtype, key, gold):
    first = np.ascontiguousarray(quant_golden[key])
    second = full_scratch_blocks(first, dtype, seed=11 + dtype)
    for blocks in (first, second):
        ref = dequant("sx_dequantize", dtype, blocks)
        got = dequant("sx_dequantize_noalloc", dtype, blocks)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert np.array_equal(dequant("sx_dequantize_noalloc", dtype, first).view(np.uint32),
                          quant_golden[gold].view(np.uint32))


def test_noalloc_rejects_sizes_beyond_capacity(quant_golden):
    bb = LAYOUT[SX_DTYPE_Q8_0][0]
    blocks = np.zeros((MAX_BLOCKS + 1) * bb, np.uint8)
    out = np.empty((MAX_BLOCKS + 1) * 32, np.float32)
    rc = _lib.lib().sx_dequantize_noalloc(SX_DTYPE_Q8_0, blocks.ctypes.data, MAX_BLOCKS + 1,
                                          out.ctypes.data_as(C.POINTER(C.c_float)), 0)
    assert rc == SX_E_RANGE
    assert "capacity" in _lib.lib().sx_last_error().decode()
    # an empty request is fine and touches nothing
    assert _lib.lib().sx_dequantize_noalloc(SX_DTYPE_Q8_0, blocks.ctypes.data, 0,
                                            out.ctypes.data_as(C.POINTER(C.c_float)), 0) == 0
