"""Weight ingest (syrinx_b200.ingest) on the CPU: the reference's name remapping and q/k/v
fusion (s2/load.rs:150-310), safetensors and GGUF sources, and prompt assembly
(s2/mod.rs:202-275). The round trips start from a synthetic model's blob, dequantized
exactly and renamed into the HF / s2-pro checkpoint namespaces with split q/k/v; ingesting
that checkpoint must give a model whose oracle logits are bit-identical to the original's
(Q8_0 re-quantization of exactly dequantized blocks reproduces the blocks)."""
import json
import struct

import numpy as np
import pytest

import syrinx_b200 as sx
from syrinx_b200 import ingest as ig
from syrinx_b200.blob import read_blob
from syrinx_b200.configs import SX_DTYPE_F32, SX_DTYPE_Q8_0, TINY_S2
from syrinx_b200.workloads import prompt_for
from oracle import oracle as oc


def test_remap_key_namespaces():
    assert ig.remap_key("text_model.model.layers.3.attention.wqkv.weight") == "layers.3.attention.wqkv.weight"
    assert ig.remap_key("text_model.model.embeddings.weight") == "embeddings.weight"
    assert ig.remap_key("text_model.lm_head.weight") == "output.weight"
    assert ig.remap_key("audio_decoder.layers.1.feed_forward.w2.weight") == "fast_layers.1.feed_forward.w2.weight"
    assert ig.remap_key("audio_decoder.codebook_embeddings.weight") == "codebook_embeddings.weight"
    assert ig.remap_key("audio_decoder.output.weight") == "fast_output.weight"
    assert ig.remap_key("model.layers.0.self_attn.q_proj.weight") == "layers.0.attention.wq.weight"
    assert ig.remap_key("model.layers.5.post_attention_layernorm.weight") == "layers.5.ffn_norm.weight"
    assert ig.remap_key("model.layers.5.mlp.up_proj.weight") == "layers.5.feed_forward.w3.weight"
    assert ig.remap_key("model.layers.5.rotary_emb.inv_freq") is None  # an unknown layer tail is dropped
    assert ig.remap_key("fast_transformer.layers.2.self_attn.o_proj.weight") == "fast_layers.2.attention.wo.weight"
    assert ig.remap_key("model.embed_tokens.weight") == "embeddings.weight"
    assert ig.remap_key("layers.1.attention_norm.weight") == "layers.1.attention_norm.weight"
    assert ig.remap_key("something.else") == "something.else"


def test_fuse_qkv_rows_q_k_v():
    q, k, v = (np.full((r, 4), i, np.float32) for i, r in enumerate((6, 2, 2)))
    out = ig.fuse_qkv({"layers.0.attention.wq.weight": q, "layers.0.attention.wk.weight": k,
                       "layers.0.attention.wv.weight": v, "layers.0.attention.wq.bias": np.zeros(6, np.float32)})
    assert list(out) == ["layers.0.attention.wq.bias", "layers.0.attention.wqkv.weight"]
    assert np.array_equal(out["layers.0.attention.wqkv.weight"], np.concatenate([q, k, v]))


def _dequant(v):
    from gguf import GGMLQuantizationType, quants

    if isinstance(v, tuple):
        return quants.dequantize(v[2], GGMLQuantizationType.Q8_0).reshape(v[1])
    return v


def _hf_checkpoint(cfg, blob):
    """The synthetic model as an HF-named slow AR + s2-pro-named fast AR, q/k/v split."""
    t = read_blob(blob)
    s = cfg.slow
    q_rows, kv_rows = s.n_head * s.head_dim, s.n_local_heads * s.head_dim
    tail = {"attention_norm.weight": "input_layernorm.weight", "ffn_norm.weight": "post_attention_layernorm.weight",
            "attention.wo.weight": "self_attn.o_proj.weight", "attention.q_norm.weight": "self_attn.q_norm.weight",
            "attention.k_norm.weight": "self_attn.k_norm.weight", "feed_forward.w1.weight": "mlp.gate_proj.weight",
            "feed_forward.w3.weight": "mlp.up_proj.weight", "feed_forward.w2.weight": "mlp.down_proj.weight"}
    top = {"embeddings.weight": "model.embed_tokens.weight", "norm.weight": "model.norm.weight",
           "output.weight": "lm_head.weight", "fast_embeddings.weight": "audio_decoder.embeddings.weight",
           "codebook_embeddings.weight": "audio_decoder.codebook_embeddings.weight",
           "fast_norm.weight": "audio_decoder.norm.weight", "fast_output.weight": "audio_decoder.output.weight"}
    out = {}
    for name, v in t.items():
        w = _dequant(v)
        if name.startswith("layers."):
            _, n, rest = name.split(".", 2)
            if rest == "attention.wqkv.weight":
                out[f"model.layers.{n}.self_attn.q_proj.weight"] = w[:q_rows]
                out[f"model.layers.{n}.self_attn.k_proj.weight"] = w[q_rows:q_rows + kv_rows]
                out[f"model.layers.{n}.self_attn.v_proj.weight"] = w[q_rows + kv_rows:]
            else:
                out[f"model.layers.{n}.{tail[rest]}"] = w
        elif name.startswith("fast_layers."):
            out["audio_decoder.layers." + name[len("fast_layers."):]] = w
        else:
            out[top[name]] = w
    return out


def _write_safetensors(path, tensors):
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        raw = np.ascontiguousarray(a, np.float32).tobytes()
        header[name] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))


def _oracle_logits(cfg, blob, prompt):
    om = oc.OracleModel(cfg, blob)
    sess = oc.OracleSession(om, 64, kv_bf16=False)
    logits, hidden = sess.prefill(prompt)
    return logits, hidden


@pytest.fixture(scope="module")
def tiny_case():
    cfg = TINY_S2
    blob = sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=21)
    prompt = prompt_for(cfg, 9, seed=21)
    return cfg, blob, prompt, _oracle_logits(cfg, blob, prompt)


def test_safetensors_roundtrip_bit_identical(tiny_case, tmp_path):
    cfg, blob, prompt, (ref_l, ref_h) = tiny_case
    ck = _hf_checkpoint(cfg, blob)
    half = len(ck) // 2
    names = list(ck)
    _write_safetensors(tmp_path / "a.safetensors", {n: ck[n] for n in names[:half]})
    _write_safetensors(tmp_path / "b.safetensors", {n: ck[n] for n in names[half:]})
    out = ig.ingest_files([str(tmp_path / "a.safetensors"), str(tmp_path / "b.safetensors")], SX_DTYPE_Q8_0)
    orig, got = read_blob(blob), read_blob(out)
    assert set(orig) == set(got)
    for name, v in orig.items():
        g = got[name]
        if isinstance(v, tuple):
            assert g[0] == v[0] and g[1] == v[1] and np.array_equal(g[2], v[2]), name
        else:
            assert np.array_equal(g, v), name
    l, h = _oracle_logits(cfg, out, prompt)
    assert np.array_equal(l, ref_l) and np.array_equal(h, ref_h)


def test_gguf_roundtrip_keeps_blocks(tiny_case, tmp_path):
    import gguf
    from gguf import GGMLQuantizationType as Q

    cfg, blob, prompt, (ref_l, _) = tiny_case
    t = read_blob(blob)
    w = gguf.GGUFWriter(str(tmp_path / "m.gguf"), "syrinx")
    for name, v in t.items():
        key = name.replace("layers.", "text_model.model.layers.", 1) if name.startswith("layers.") else name
        if isinstance(v, tuple):
            w.add_tensor(key, v[2], raw_dtype=Q.Q8_0)
        else:
            w.add_tensor(key, v)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    out = ig.ingest_files([str(tmp_path / "m.gguf")])
    l, _ = _oracle_logits(cfg, out, prompt)
    assert np.array_equal(l, ref_l)


def test_f32_ingest_keeps_values(tiny_case):
    cfg, blob, _, _ = tiny_case
    ck = _hf_checkpoint(cfg, blob)
    got = read_blob(ig.ingest(ck, SX_DTYPE_F32))
    wqkv = got["layers.0.attention.wqkv.weight"]
    assert wqkv.dtype == np.float32
    assert np.array_equal(wqkv, np.concatenate([ck[f"model.layers.0.self_attn.{p}_proj.weight"] for p in "qkv"]))


def test_build_prompt_with_reference_layout():
    codes = np.array([[3, 1, 4], [1, 5, 9]], np.uint32)  # [C=2, T=3]
    p = ig.build_prompt_with_reference([10, 11], codes, [20, 21, 22], semantic_begin_id=1000)
    assert p.shape == (3, 8)
    assert p[0].tolist() == [10, 11, 1003, 1001, 1004, 20, 21, 22]
    assert p[1].tolist() == [0, 0, 3, 1, 4, 0, 0, 0]
    assert p[2].tolist() == [0, 0, 1, 5, 9, 0, 0, 0]
    assert np.array_equal(ig.build_prompt_with_reference([10, 11], codes[None], [20, 21, 22], 1000), p)
