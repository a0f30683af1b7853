"""Seeded synthetic inputs with the shapes of the benchmark configurations.

Dual-AR prompts are [(1 + C), T] u32 (row 0 slow-vocab ids, rows 1..C codes, 0 on text
positions; the layout `build_prompt_with_reference` produces, crates/syrinx-fish/src/s2/
mod.rs:202-275): `n_text` text ids uniform below the semantic range, then `n_semantic`
reference-voice positions whose codes are uniform in [0, R) in every codebook row and whose
row-0 id is semantic_begin + code0. Plain-LM prompts (CosyVoice2 shape) are ids uniform
in [0, vocab).
"""
from __future__ import annotations

import numpy as np

from .configs import ModelConfig


def dual_ar_prompt(cfg: ModelConfig, T: int, n_semantic: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    C = cfg.num_codebooks
    p = np.zeros((1 + C, T), np.uint32)
    n_sem = min(n_semantic, T)
    n_text = T - n_sem
    p[0, :n_text] = rng.integers(0, cfg.semantic_begin_id, n_text)
    codes = rng.integers(0, cfg.codebook_size, (C, n_sem))
    p[0, n_text:] = cfg.semantic_begin_id + codes[0]
    p[1:, n_text:] = codes
    return p


def lm_prompt(cfg: ModelConfig, T: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(0, cfg.vocab_size, (1, T)).astype(np.uint32)


def prompt_for(cfg: ModelConfig, T: int, seed: int, semantic_frac: float = 430 / 512) -> np.ndarray:
    if cfg.num_codebooks == 0:
        return lm_prompt(cfg, T, seed)
    return dual_ar_prompt(cfg, T, int(round(T * semantic_frac)), seed)


def config4_prompts(cfg: ModelConfig, n: int = 8) -> list:
    """Config 4's batch: n utterances with prompt lengths uniform in [256, 1024] (seeded),
    each with the config-3 share of reference-voice positions."""
    lens = np.random.default_rng(4).integers(256, 1025, n)
    return [dual_ar_prompt(cfg, int(T), int(round(T * 430 / 512)), seed=40 + i) for i, T in enumerate(lens)]
