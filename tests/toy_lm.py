"""The reference's toy parity LM (its PARITY.md sections 2-5): weights are a pure function
of the tensor name (FNV-1a 64 seed -> xorshift64 stream -> (u*2-1)*0.02), vocab 512,
dim 128, 4 layers, 4 heads of 32, SwiGLU 256, RoPE theta 1e4 interleaved, eps 1e-5,
untied output head. Used to pin the oracle and the GPU path to lm_forward.json."""
import numpy as np

from syrinx_b200.blob import write_blob
from syrinx_b200.configs import ModelConfig, Stack

M64 = (1 << 64) - 1


def fnv1a_64(name: str) -> int:
    h = 0xCBF29CE484222325
    for b in name.encode():
        h ^= b
        h = (h * 0x100000001B3) & M64
    return h


def weights(name: str, count: int) -> np.ndarray:
    state = fnv1a_64(name) or 0x9E3779B97F4A7C15
    out = np.empty(count, np.float32)
    for i in range(count):
        x = state
        x ^= (x << 13) & M64
        x ^= x >> 7
        x ^= (x << 17) & M64
        state = x
        u = (x >> 11) * (1.0 / (1 << 53))
        out[i] = np.float32((u * 2.0 - 1.0) * 0.02)
    return out


VOCAB, DIM, LAYERS, HEADS, HD, FFN = 512, 128, 4, 4, 32, 256

TOY_CFG = ModelConfig(
    name="toy-parity-lm",
    slow=Stack(DIM, LAYERS, HEADS, HEADS, HD, FFN, norm_eps=1e-5, rope_base=10000.0),
    fast=Stack(0, 0, 1, 1, 32, 32), vocab_size=VOCAB, num_codebooks=0, codebook_size=0,
    semantic_begin_id=0, semantic_end_id=VOCAB - 1, stop_token_id=VOCAB, num_stop_tokens=0,
    tie_word_embeddings=False)


def toy_blob() -> np.ndarray:
    t = {"embeddings.weight": weights("tok_embeddings", VOCAB * DIM).reshape(VOCAB, DIM)}
    for L in range(LAYERS):
        p = f"layers.{L}."
        t[p + "attention_norm.weight"] = weights(p + "attention_norm.weight", DIM)
        wq = weights(p + "attention.wq.weight", DIM * DIM).reshape(DIM, DIM)
        wk = weights(p + "attention.wk.weight", DIM * DIM).reshape(DIM, DIM)
        wv = weights(p + "attention.wv.weight", DIM * DIM).reshape(DIM, DIM)
        t[p + "attention.wqkv.weight"] = np.concatenate([wq, wk, wv], 0)  # fuse_qkv order q|k|v
        t[p + "attention.wo.weight"] = weights(p + "attention.wo.weight", DIM * DIM).reshape(DIM, DIM)
        t[p + "ffn_norm.weight"] = weights(p + "ffn_norm.weight", DIM)
        t[p + "feed_forward.w1.weight"] = weights(p + "feed_forward.w1.weight", FFN * DIM).reshape(FFN, DIM)
        t[p + "feed_forward.w3.weight"] = weights(p + "feed_forward.w3.weight", FFN * DIM).reshape(FFN, DIM)
        t[p + "feed_forward.w2.weight"] = weights(p + "feed_forward.w2.weight", DIM * FFN).reshape(DIM, FFN)
    t["norm.weight"] = weights("norm.weight", DIM)
    t["output.weight"] = weights("output.weight", VOCAB * DIM).reshape(VOCAB, DIM)
    return write_blob(t)
