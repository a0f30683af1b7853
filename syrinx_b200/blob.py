"""SXW1 weight blobs from named numpy arrays (the container described in
include/syrinx_dualar.h). Quantized tensors are passed as raw GGML block bytes
[rows, n_blocks * block_bytes] together with their logical shape."""
from __future__ import annotations

import struct

import numpy as np

from .configs import SX_DTYPE_F32, SX_DTYPE_Q4_K, SX_DTYPE_Q8_0

_BLOCK = {SX_DTYPE_Q8_0: (32, 34), SX_DTYPE_Q4_K: (256, 144)}


def write_blob(tensors: dict) -> np.ndarray:
    """tensors: name -> f32 ndarray (1-D to 3-D), or (dtype, shape, raw uint8 blocks)."""
    entries = []
    for name, v in tensors.items():
        if isinstance(v, tuple):
            dtype, shape, raw = v
            raw = np.ascontiguousarray(raw, np.uint8).reshape(-1)
            per, bb = _BLOCK[dtype]
            rows, cols = shape
            assert raw.size == rows * cols // per * bb, name
        else:
            a = np.ascontiguousarray(v, np.float32)
            dtype, shape, raw = SX_DTYPE_F32, a.shape, a.view(np.uint8).reshape(-1)
        entries.append((name.encode(), dtype, tuple(int(s) for s in shape), raw))
    header = 24 + sum(4 + len(n) + 8 + 8 * len(s) + 16 for n, _, s, _ in entries)
    header = (header + 63) & ~63
    offs, off = [], 0
    for e in entries:
        offs.append(off)
        off = (off + e[3].size + 63) & ~63
    out = np.zeros(header + off, np.uint8)
    hdr = bytearray(struct.pack("<4sIIIQ", b"SXW1", 1, len(entries), 0, header))
    for (n, dt, s, raw), o in zip(entries, offs):
        hdr += struct.pack("<I", len(n)) + n + struct.pack("<II", dt, len(s))
        hdr += b"".join(struct.pack("<Q", d) for d in s) + struct.pack("<QQ", o, raw.size)
        out[header + o: header + o + raw.size] = raw
    out[: len(hdr)] = np.frombuffer(bytes(hdr), np.uint8)
    return out


def read_blob(blob) -> dict:
    """name -> f32 ndarray, or (dtype, (rows, cols), raw uint8 blocks [rows, bytes per row]),
    from an SXW1 blob (the inverse of write_blob)."""
    b = np.asarray(blob, np.uint8).reshape(-1)
    mv = memoryview(b.tobytes())
    magic, version, n, _, data_off = struct.unpack_from("<4sIIIQ", mv, 0)
    if magic != b"SXW1" or version != 1:
        raise ValueError("not an SXW1 blob")
    pos, out = 24, {}
    for _ in range(n):
        (ln,) = struct.unpack_from("<I", mv, pos)
        name = bytes(mv[pos + 4: pos + 4 + ln]).decode()
        pos += 4 + ln
        dt, nd = struct.unpack_from("<II", mv, pos)
        pos += 8
        shape = struct.unpack_from("<" + "Q" * nd, mv, pos)
        pos += 8 * nd
        off, nbytes = struct.unpack_from("<QQ", mv, pos)
        pos += 16
        raw = b[data_off + off: data_off + off + nbytes]
        if dt == SX_DTYPE_F32:
            out[name] = raw.view(np.float32).reshape(shape).copy()
        else:
            rows = int(shape[0]) if nd == 2 else 1
            out[name] = (dt, tuple(int(s) for s in shape), raw.reshape(rows, -1).copy())
    return out
