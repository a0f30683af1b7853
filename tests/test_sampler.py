"""The host Sampler restated from crates/syrinx-fish/src/common/sampling.rs, checked
against the oracle's independent C restatement and against the reference's own
statistical claims (SplitMix64 uniform, inverse-CDF multinomial unbiased)."""
import ctypes as C

import numpy as np

from oracle import oracle as oc
from syrinx_b200.configs import TINY_S2
from syrinx_b200.dualar import GREEDY, Sampler, SamplingParams, SplitMix64, logits_to_probs


def test_splitmix64_stream_matches_oracle():
    st = C.c_uint64(42)
    r = SplitMix64(42)
    for _ in range(100):
        assert oc.lib().oc_splitmix64_next(C.byref(st)) == r.next_u64()


def test_splitmix64_uniform():
    r = SplitMix64(7)
    u = np.array([r.next_f64() for _ in range(20000)])
    assert 0.0 <= u.min() and u.max() < 1.0
    assert abs(u.mean() - 0.5) < 0.01
    hist, _ = np.histogram(u, bins=10, range=(0, 1))
    assert hist.min() > 1800


def test_logits_to_probs_matches_oracle():
    rng = np.random.default_rng(3)
    for temp, top_p, top_k in [(1.0, 0.9, 30), (0.7, 0.5, 0), (1.3, 1.0, 5), (1.0, 0.9, 1)]:
        logits = rng.normal(size=300).astype(np.float32)
        logits[17] = logits[18] = np.float32(3.0)  # a tie at the top
        a = logits_to_probs(logits, temp, top_p, top_k)
        b = np.empty_like(logits)
        oc.lib().oc_logits_to_probs(logits.ctypes.data_as(C.POINTER(C.c_float)), logits.size, temp, top_p, top_k,
                                    b.ctypes.data_as(C.POINTER(C.c_float)))
        assert np.array_equal(a, b)


def test_greedy_is_argmax_lowest_index():
    """top_k=1 keeps only rank 0 (ties -> lowest index): the greedy draw is the argmax."""
    rng = np.random.default_rng(4)
    s = Sampler(0, GREEDY)
    for _ in range(20):
        logits = rng.normal(size=512).astype(np.float32)
        j = int(rng.integers(0, 511))
        logits[j] = logits[j + 1] = logits.max() + 1
        assert s.sample_codebook(logits, []) == j


def test_semantic_constraint_and_ras():
    cfg = TINY_S2
    logits = np.full(cfg.vocab_size, -1.0, np.float32)
    logits[3] = 100.0  # not allowed: outside the semantic range and not a stop id
    logits[cfg.semantic_begin_id + 5] = 10.0
    s = Sampler(1, GREEDY)
    assert s.sample_semantic(logits, [], cfg) == cfg.semantic_begin_id + 5
    logits[cfg.stop_token_id] = 50.0
    assert s.sample_semantic(logits, [], cfg) == cfg.stop_token_id


def test_multinomial_distribution():
    probs = np.array([0.1, 0.2, 0.3, 0.4], np.float32)
    s = Sampler(9, SamplingParams(temperature=1.0, top_p=1.0, top_k=0))
    logits = np.log(probs)
    draws = np.bincount([s.sample_codebook(logits, []) for _ in range(8000)], minlength=4) / 8000
    assert np.max(np.abs(draws - probs)) < 0.02
