"""Pin the CPU oracle to the reference's own golden vectors (tests/golden/parity_kat.json,
generated from the reference's tests/golden/parity/*.json) and to gguf-py's bit-exact
Q8_0 / Q4_K vectors (tests/golden/quant_golden.npz)."""
import numpy as np
import pytest

from oracle import oracle as oc
from tests.toy_lm import TOY_CFG, toy_blob, weights


def maxabs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def test_rope_interleaved(kats):
    k = kats["rope"]
    x = np.array(k["input"]["x"], np.float32)
    y = oc.rope(x, k["input"]["positions"], k["input"]["theta"], interleaved=True)
    assert maxabs(y.reshape(-1), k["data"]) <= k["tol"]


def test_rope_position_zero_is_identity():
    x = np.random.default_rng(0).normal(size=(1, 3, 64)).astype(np.float32)
    for inter in (True, False):
        assert np.array_equal(oc.rope(x, [0], 1e6, inter), x)


def test_rmsnorm(kats):
    k = kats["rmsnorm"]
    y = oc.rmsnorm(np.array(k["input"]["x"], np.float32), k["input"]["w"], k["input"]["eps"])
    assert maxabs(y.reshape(-1), k["data"]) <= k["tol"]


def test_softmax(kats):
    k = kats["softmax"]
    y = oc.softmax(np.array(k["input"]["x"], np.float32))
    assert maxabs(y.reshape(-1), k["data"]) <= k["tol"]


def test_silu(kats):
    k = kats["silu"]
    y = oc.silu(np.array(k["input"]["x"], np.float32))
    assert maxabs(y.reshape(-1), k["data"]) <= k["tol"]


def test_linear_and_matmul(kats):
    k = kats["linear"]
    inp = k["input"]
    y = oc.linear(np.array(inp["x"], np.float32), np.array(inp["W"], np.float32), np.array(inp["b"], np.float32))
    assert maxabs(y.reshape(-1), k["data"]) <= k["tol"]
    m = kats["matmul"]
    A, B = np.array(m["input"]["A"], np.float32), np.array(m["input"]["B"], np.float32)
    y = oc.linear(A, B.T.copy())  # matmul(A, B) = linear(A, W = B^T)
    assert maxabs(y.reshape(-1), m["data"]) <= m["tol"]


def test_weight_generator_sample(kats):
    k = kats["weights_sample"]
    w = weights(k["input"]["tensor_name"], k["input"]["count"])
    assert maxabs(w, k["data"]) <= k["tol"]


@pytest.fixture(scope="module")
def toy():
    blob = toy_blob()
    return oc.OracleModel(TOY_CFG, blob)


def test_toy_lm_embed(kats, toy):
    k = kats["lm_embed"]
    ids = k["input"]["token_ids"]
    emb = toy.tensor("embeddings.weight")[ids]
    assert maxabs(emb.reshape(-1), k["data"]) <= k["tol"]


def test_toy_lm_forward_incremental(kats, toy):
    """lm_forward row t == the cached single-token step at position t (f32 KV)."""
    k = kats["lm_forward"]
    ids = k["input"]["token_ids"]
    gold = np.array(k["data"], np.float32).reshape(k["shape"])
    s = oc.OracleSession(toy, max_ctx=16, kv_bf16=False)
    rows = [s.lm_step_tokens([ids[0]])] + [s.lm_step_tokens([t]) for t in ids[1:]]
    assert maxabs(np.stack(rows), gold) <= k["tol"]


def test_toy_lm_forward_prefill(kats, toy):
    """Full causal prefill of all tokens == the golden last row; chunked == incremental."""
    k = kats["lm_forward"]
    ids = k["input"]["token_ids"]
    gold = np.array(k["data"], np.float32).reshape(k["shape"])
    s = oc.OracleSession(toy, max_ctx=16, kv_bf16=False)
    last = s.lm_step_tokens(ids)
    assert maxabs(last, gold[-1]) <= k["tol"]
    s2 = oc.OracleSession(toy, max_ctx=16, kv_bf16=False)
    s2.lm_step_tokens(ids[:3])
    assert maxabs(s2.lm_step_tokens(ids[3:]), gold[-1]) <= k["tol"]


def test_q8_0_quantize_matches_gguf(quant_golden):
    g = quant_golden
    blocks = oc.q8_0_quantize(g["q8_src"])
    assert np.array_equal(blocks, g["q8_blocks"]), "Q8_0 quantize differs from ggml/gguf-py"


def test_q8_0_dequantize_bitexact(quant_golden):
    g = quant_golden
    out = oc.q8_0_dequantize(g["q8_blocks"])
    assert np.array_equal(out.view(np.uint32), g["q8_deq"].view(np.uint32))


def test_q4_k_dequantize_bitexact(quant_golden):
    g = quant_golden
    out = oc.q4_k_dequantize(g["q4k_blocks"])
    assert np.array_equal(out.view(np.uint32), g["q4k_deq"].view(np.uint32))


def test_f16_bf16_conversions():
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.normal(0, 1, 2000), rng.normal(0, 1e-5, 500), [0.0, -0.0, 65504.0, 6e-8]]).astype(np.float32)
    for v in x:
        assert oc.lib().oc_f32_to_f16(float(v)) == np.float32(v).astype(np.float16).view(np.uint16)
    bits = np.arange(0, 0x7c00, 7, dtype=np.uint16)
    for b in bits:
        assert oc.lib().oc_f16_to_f32(int(b)) == float(b.view(np.float16))


def test_config4_fixture_matches_its_recipe():
    """tests/golden/config4_q4k.npz holds what make_oracle_fixtures.py describes: 8 prompts of
    lengths in [256, 1024] from its seeded recipe, 64 frames each, semantic ids in range."""
    import os
    import sys

    import numpy as np

    import syrinx_b200 as sx
    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    sys.path.insert(0, here)
    from make_oracle_fixtures import CONFIG4_FRAMES, CONFIG4_UTTERANCES, config4_prompts

    fx = np.load(os.path.join(here, "config4_q4k.npz"))
    cfg = sx.QWEN3_4B
    lens = [p.shape[1] for p in config4_prompts(cfg)]
    assert list(fx["lens"]) == lens and all(256 <= T <= 1024 for T in lens)
    assert fx["frames"].shape == (CONFIG4_UTTERANCES, CONFIG4_FRAMES, cfg.frame_width)
    sem = fx["frames"][:, :, 0]
    assert np.all((sem >= cfg.semantic_begin_id) & (sem <= cfg.semantic_end_id))
    assert np.all(fx["frames"][:, :, 1] == sem - cfg.semantic_begin_id)  # first_code
    assert fx["logits0_semantic"].shape == (CONFIG4_UTTERANCES, cfg.n_semantic() + 1)
