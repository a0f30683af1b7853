"""Generates the committed golden fixtures in this directory.

  parity_kat.json   the reference's own known-answer vectors for the op semantics of the
                    path (voldiguarddevelopment/syrinx tests/golden/parity/*.json, specified
                    in its PARITY.md): rope, rmsnorm, softmax, silu, linear, embed, matmul,
                    causal_mask, the FNV-1a/xorshift weight sample and the toy 4-layer LM
                    forward. Re-emitted unchanged (name, input, shape, data, tol).
  quant_golden.npz  GGML Q8_0 quantize/dequantize and Q4_K dequantize vectors produced by
                    gguf-py (gguf.quants, bit-exact with ggml-quants.c) on seeded inputs.

Run in a container that has the reference checkout and gguf installed:
    python tests/golden/make_fixtures.py /path/to/syrinx/tests/golden/parity
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
KATS = ["rope", "rmsnorm", "softmax", "silu", "linear", "embed", "matmul", "add", "mul",
        "causal_mask", "weights_sample", "lm_embed", "lm_forward"]


def parity_kats(src: str) -> None:
    out = {}
    for k in KATS:
        with open(os.path.join(src, k + ".json")) as f:
            d = json.load(f)
        out[k] = {key: d[key] for key in ("name", "input", "shape", "data", "tol")}
    with open(os.path.join(HERE, "parity_kat.json"), "w") as f:
        json.dump(out, f, separators=(",", ":"))


def quant_golden() -> None:
    import gguf.quants as gq
    from gguf import GGMLQuantizationType as T

    rng = np.random.default_rng(20261201)
    # Q8_0: values of several magnitudes, an all-zero block, exact .5 ties after scaling
    x = rng.normal(0.0, 0.02, size=32 * 64).astype(np.float32)
    x[32:64] = 0.0
    x[64:96] = np.linspace(-1.0, 1.0, 32, dtype=np.float32)
    x[96:128] *= 1000.0
    q8 = gq.quantize(x.reshape(1, -1), T.Q8_0).reshape(-1)
    q8_deq = gq.dequantize(q8.reshape(1, -1), T.Q8_0).reshape(-1).astype(np.float32)
    # Q4_K: random valid super-blocks (d, dmin finite f16; all 6-bit scale/min patterns)
    nb = 48
    blocks = rng.integers(0, 256, size=(nb, 144), dtype=np.uint8)
    d = rng.uniform(1e-4, 2e-3, size=nb).astype(np.float16)
    dmin = rng.uniform(0.0, 2e-3, size=nb).astype(np.float16)
    blocks[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    blocks[:, 2:4] = dmin.view(np.uint8).reshape(nb, 2)
    q4k = blocks.reshape(-1)
    q4k_deq = gq.dequantize(q4k.reshape(1, -1), T.Q4_K).reshape(-1).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), q8_src=x, q8_blocks=q8, q8_deq=q8_deq,
                        q4k_blocks=q4k, q4k_deq=q4k_deq)


if __name__ == "__main__":
    src = sys.argv[1] if len(sys.argv) > 1 else None
    if src:
        parity_kats(src)
    quant_golden()
