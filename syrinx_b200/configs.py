"""Model descriptors (ctypes mirrors of include/syrinx_dualar.h) and the benchmark presets.

The presets are the shapes of the hot-path configurations: the CosyVoice2-LM-shaped Qwen2
decoder, the s1-mini-shaped dual-AR and the Qwen3-4B-shaped (s2-pro) dual-AR, plus small
variants of each for tests. Field meanings follow `TransformerConfig` / `FishConfig`
(crates/syrinx-fish/src/common/config.rs:22-119) and the CosyVoice2 constants
(crates/syrinx-lm/src/cv2/mod.rs:40-56).
"""
from __future__ import annotations

import ctypes as C
import dataclasses

SX_DTYPE_F32 = 0
SX_DTYPE_F16 = 1
SX_DTYPE_Q8_0 = 8
SX_DTYPE_Q4_K = 12
SX_DTYPE_BF16 = 30


class SxTransformerDesc(C.Structure):
    _fields_ = [
        ("dim", C.c_int32),
        ("n_layer", C.c_int32),
        ("n_head", C.c_int32),
        ("n_local_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("intermediate_size", C.c_int32),
        ("norm_eps", C.c_float),
        ("rope_base", C.c_float),
        ("rope_interleaved", C.c_int32),
        ("qk_norm", C.c_int32),
        ("qkv_bias", C.c_int32),
        ("o_bias", C.c_int32),
    ]


class SxModelDesc(C.Structure):
    _fields_ = [
        ("slow", SxTransformerDesc),
        ("fast", SxTransformerDesc),
        ("vocab_size", C.c_int32),
        ("num_codebooks", C.c_int32),
        ("codebook_size", C.c_int32),
        ("semantic_begin_id", C.c_uint32),
        ("semantic_end_id", C.c_uint32),
        ("stop_token_id", C.c_uint32),
        ("num_stop_tokens", C.c_int32),
        ("tie_word_embeddings", C.c_int32),
        ("head_bias", C.c_int32),
        ("scale_codebook_embeddings", C.c_int32),
        ("norm_fastlayer_input", C.c_int32),
    ]


class SxSamplingParams(C.Structure):
    _fields_ = [
        ("temperature", C.c_float),
        ("top_p", C.c_float),
        ("top_k", C.c_int32),
        ("repetition_penalty", C.c_float),
        ("ras_win_size", C.c_int32),
        ("ras_high_temp", C.c_float),
        ("ras_high_top_p", C.c_float),
    ]


class SxCodecInfo(C.Structure):
    """sx_codec_info of include/syrinx_codec.h."""
    _fields_ = [
        ("hop", C.c_int32),
        ("sample_rate", C.c_int32),
        ("num_codebooks", C.c_int32),
        ("semantic_size", C.c_int32),
        ("residual_size", C.c_int32),
        ("codebook_dim", C.c_int32),
        ("latent_dim", C.c_int32),
        ("n_layers", C.c_int32),
    ]


@dataclasses.dataclass(frozen=True)
class Stack:
    dim: int
    n_layer: int
    n_head: int
    n_local_heads: int
    head_dim: int
    intermediate_size: int
    norm_eps: float = 1e-6
    rope_base: float = 1e6
    rope_interleaved: bool = True
    qk_norm: bool = False
    qkv_bias: bool = False
    o_bias: bool = False

    def to_c(self) -> SxTransformerDesc:
        return SxTransformerDesc(
            self.dim, self.n_layer, self.n_head, self.n_local_heads, self.head_dim,
            self.intermediate_size, self.norm_eps, self.rope_base, int(self.rope_interleaved),
            int(self.qk_norm), int(self.qkv_bias), int(self.o_bias))

    @property
    def qkv_rows(self) -> int:
        return (self.n_head + 2 * self.n_local_heads) * self.head_dim

    def layer_params(self) -> int:
        """Matrix parameters of one decoder layer (wqkv + wo + w1 + w3 + w2)."""
        d, F = self.dim, self.intermediate_size
        return self.qkv_rows * d + d * self.n_head * self.head_dim + 3 * F * d


NO_FAST = Stack(0, 0, 1, 1, 32, 32)


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    name: str
    slow: Stack
    fast: Stack
    vocab_size: int
    num_codebooks: int
    codebook_size: int
    semantic_begin_id: int
    semantic_end_id: int
    stop_token_id: int
    num_stop_tokens: int = 1
    tie_word_embeddings: bool = True
    head_bias: bool = False
    scale_codebook_embeddings: bool = False
    norm_fastlayer_input: bool = False

    def to_c(self) -> SxModelDesc:
        return SxModelDesc(
            self.slow.to_c(), self.fast.to_c(), self.vocab_size, self.num_codebooks,
            self.codebook_size, self.semantic_begin_id, self.semantic_end_id, self.stop_token_id,
            self.num_stop_tokens, int(self.tie_word_embeddings), int(self.head_bias),
            int(self.scale_codebook_embeddings), int(self.norm_fastlayer_input))

    @property
    def has_fast(self) -> bool:
        return self.fast.n_layer > 0

    @property
    def frame_width(self) -> int:
        return 1 + self.num_codebooks

    def stop_ids(self) -> range:
        return range(self.stop_token_id, self.stop_token_id + self.num_stop_tokens)

    def n_semantic(self) -> int:
        return self.semantic_end_id - self.semantic_begin_id + 1


def bytes_per_weight(wtype: int) -> float:
    return {SX_DTYPE_Q8_0: 34 / 32, SX_DTYPE_Q4_K: 144 / 256, SX_DTYPE_F32: 4.0}[wtype]


def frame_bytes(cfg: ModelConfig, wtype: int, ctx: float, semantic_head: bool = True,
                kv_elem: int = 2) -> dict:
    """Algorithmic HBM bytes streamed per frame (batch 1):
    slow weights + head rows + C x fast layers + (C-1) x fast_output + KV read
    (2 * L * Hkv * hd * kv_elem B per context position: 2 for bf16, 4 for f32; the fast AR's
    local KV is negligible)."""
    bpw = bytes_per_weight(wtype)
    s = cfg.slow
    slow_w = s.n_layer * s.layer_params() * bpw
    head_rows = (cfg.n_semantic() + cfg.num_stop_tokens) if semantic_head else cfg.vocab_size
    head_w = head_rows * s.dim * bpw
    fast_w = 0.0
    if cfg.has_fast:
        f = cfg.fast
        fast_w = cfg.num_codebooks * f.n_layer * f.layer_params() * bpw
        fast_w += (cfg.num_codebooks - 1) * cfg.codebook_size * f.dim * bpw
    kv = 2 * s.n_layer * s.n_local_heads * s.head_dim * kv_elem * ctx
    return {"slow": slow_w, "head": head_w, "fast": fast_w, "kv": kv,
            "total": slow_w + head_w + fast_w + kv}


# ---- presets ------------------------------------------------------------------------------

# Config 1: CosyVoice2-LM-shaped Qwen2 decoder (cv2/mod.rs:40-56): rotate-half RoPE,
# q/k/v bias, untied `llm_decoder` head with bias, stop ids 6561..6563.
COSYVOICE2_LM = ModelConfig(
    name="cosyvoice2-qwen2-0.5b",
    slow=Stack(896, 24, 14, 2, 64, 4864, 1e-6, 1e6, rope_interleaved=False, qkv_bias=True),
    fast=NO_FAST, vocab_size=6564, num_codebooks=0, codebook_size=0,
    semantic_begin_id=0, semantic_end_id=6560, stop_token_id=6561, num_stop_tokens=3,
    tie_word_embeddings=False, head_bias=True)

# CosyVoice3 LM (cv3/mod.rs:1-69): the same Qwen2 body as CosyVoice2 with a bias-free
# `llm_decoder` of 6761 rows; every id from speech_token_size (6561) up is one of the 200
# control ids that stop decoding (cv3/generate.rs:84-88), masked while step < min_len.
COSYVOICE3_LM = ModelConfig(
    name="cosyvoice3-qwen2-0.5b",
    slow=Stack(896, 24, 14, 2, 64, 4864, 1e-6, 1e6, rope_interleaved=False, qkv_bias=True),
    fast=NO_FAST, vocab_size=6761, num_codebooks=0, codebook_size=0,
    semantic_begin_id=0, semantic_end_id=6560, stop_token_id=6561, num_stop_tokens=200,
    tie_word_embeddings=False, head_bias=False)

# Config 2: s1-mini-shaped dual-AR (Llama slow AR, no QK-norm, pre-norm fast hidden).
S1_MINI = ModelConfig(
    name="s1-mini",
    slow=Stack(1024, 24, 16, 8, 64, 4096),
    fast=Stack(1024, 4, 16, 8, 64, 4096),
    vocab_size=32000 + 1024, num_codebooks=8, codebook_size=1024,
    semantic_begin_id=32000, semantic_end_id=33023, stop_token_id=4,
    tie_word_embeddings=True)

# Config 3: Qwen3-4B-shaped s2-pro dual-AR (QK-norm slow AR, MCF scale, post-norm hidden).
QWEN3_4B = ModelConfig(
    name="s2-pro-qwen3-4b",
    slow=Stack(2560, 36, 32, 8, 128, 9728, qk_norm=True),
    fast=Stack(2560, 4, 32, 8, 128, 9728),
    vocab_size=151936 + 4096, num_codebooks=10, codebook_size=4096,
    semantic_begin_id=151936, semantic_end_id=156031, stop_token_id=151645,
    tie_word_embeddings=True, scale_codebook_embeddings=True, norm_fastlayer_input=True)


def shrink(cfg: ModelConfig, n_layer: int, n_fast_layer: int | None = None, name: str | None = None) -> ModelConfig:
    """Same shapes with fewer layers (tests that must finish on the CPU oracle in seconds)."""
    slow = dataclasses.replace(cfg.slow, n_layer=n_layer)
    fast = cfg.fast if not cfg.has_fast else dataclasses.replace(
        cfg.fast, n_layer=n_fast_layer if n_fast_layer is not None else min(cfg.fast.n_layer, n_layer))
    return dataclasses.replace(cfg, slow=slow, fast=fast, name=name or f"{cfg.name}-L{n_layer}")


# A tiny dual-AR exercising every s2 feature (QK-norm, GQA 4:2, MCF scale, post-norm hidden).
TINY_S2 = ModelConfig(
    name="tiny-s2",
    slow=Stack(256, 2, 4, 2, 64, 512, qk_norm=True),
    fast=Stack(256, 2, 4, 2, 64, 512),
    vocab_size=1024 + 256, num_codebooks=4, codebook_size=256,
    semantic_begin_id=1024, semantic_end_id=1279, stop_token_id=7,
    scale_codebook_embeddings=True, norm_fastlayer_input=True)

PRESETS = {c.name: c for c in (COSYVOICE2_LM, COSYVOICE3_LM, S1_MINI, QWEN3_4B, TINY_S2)}
