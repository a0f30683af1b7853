"""Weight ingest: checkpoints -> the library's SXW1 weight blob, and prompt assembly.

Restates the reference loader (crates/syrinx-fish/src/s2/load.rs):
  * `remap_key` follows `remap_qwen3_key` / `remap_layer_tail` (load.rs:150-242): the real
    s2-pro namespace (`text_model.model.*` slow AR, `audio_decoder.*` fast AR), the
    fish-native names (passed through) and HF-Qwen3 names (`model.layers.N.self_attn.*`);
    unknown names are kept under their own name;
  * `fuse_qkv` follows `fuse_qkv` (load.rs:271-310): split `<p>.wq/.wk/.wv` weights (and
    biases, when all three ship) become `<p>.wqkv`, rows q | k | v;
  * 2-D weights are quantized to Q8_0 with ggml's rule (gguf-py `quantize`, the same bytes
    as ggml's `quantize_row_q8_0_ref`, as the reference quantizes at load,
    cv2/load.rs:99-105), or kept f32; 1-D tensors (norm gains, biases) stay f32;
    tensors that already hold GGML Q8_0 / Q4_K blocks (a GGUF file) are copied as they are.

Sources: safetensors files (f32 / f16 / bf16) and GGUF files (F32 / F16 / Q8_0 / Q4_K
tensors whose names are in one of the namespaces above).

`build_prompt_with_reference` lays out a voice-cloning prompt from token ids the caller's
tokenizer produced, as the reference does (crates/syrinx-fish/src/s2/mod.rs:202-275).
"""
from __future__ import annotations

import json
import struct

import numpy as np

from .blob import write_blob
from .configs import SX_DTYPE_F32, SX_DTYPE_Q4_K, SX_DTYPE_Q8_0

_LAYER_TAIL = {
    "input_layernorm.weight": "attention_norm.weight",
    "post_attention_layernorm.weight": "ffn_norm.weight",
    "self_attn.q_proj.weight": "attention.wq.weight",
    "self_attn.q_proj.bias": "attention.wq.bias",
    "self_attn.k_proj.weight": "attention.wk.weight",
    "self_attn.k_proj.bias": "attention.wk.bias",
    "self_attn.v_proj.weight": "attention.wv.weight",
    "self_attn.v_proj.bias": "attention.wv.bias",
    "self_attn.o_proj.weight": "attention.wo.weight",
    "self_attn.o_proj.bias": "attention.wo.bias",
    "self_attn.q_norm.weight": "attention.q_norm.weight",
    "self_attn.k_norm.weight": "attention.k_norm.weight",
    "mlp.gate_proj.weight": "feed_forward.w1.weight",
    "mlp.up_proj.weight": "feed_forward.w3.weight",
    "mlp.down_proj.weight": "feed_forward.w2.weight",
}

_EXACT = {
    # real s2-pro namespace
    "text_model.model.embeddings.weight": "embeddings.weight",
    "text_model.model.norm.weight": "norm.weight",
    "text_model.lm_head.weight": "output.weight",
    "audio_decoder.embeddings.weight": "fast_embeddings.weight",
    "audio_decoder.codebook_embeddings.weight": "codebook_embeddings.weight",
    "audio_decoder.norm.weight": "fast_norm.weight",
    "audio_decoder.output.weight": "fast_output.weight",
    # HF top-level
    "model.embed_tokens.weight": "embeddings.weight",
    "model.norm.weight": "norm.weight",
    "lm_head.weight": "output.weight",
    # HF-style audio decoder exports
    "model.audio_decoder.embeddings.weight": "fast_embeddings.weight",
    "model.audio_decoder.norm.weight": "fast_norm.weight",
    "model.audio_decoder.output.weight": "fast_output.weight",
    "model.codebook_embeddings.weight": "codebook_embeddings.weight",
    "model.fast_project_in.weight": "fast_project_in.weight",
    "model.fast_project_in.bias": "fast_project_in.bias",
}

_NATIVE_EXACT = {"embeddings.weight", "codebook_embeddings.weight", "fast_embeddings.weight", "norm.weight",
                 "fast_norm.weight", "fast_output.weight", "output.weight"}


def remap_key(k: str) -> str | None:
    """The reference name of checkpoint tensor `k` (None: a per-layer tail it drops)."""
    if k.startswith("text_model.model.layers."):
        n, tail = k[len("text_model.model.layers."):].split(".", 1)
        return f"layers.{n}.{tail}"
    if k.startswith("audio_decoder.layers."):
        n, tail = k[len("audio_decoder.layers."):].split(".", 1)
        return f"fast_layers.{n}.{tail}"
    if k in _EXACT and (k.startswith("text_model.") or k.startswith("audio_decoder.")):
        return _EXACT[k]
    if k.startswith("layers.") or k.startswith("fast_layers.") or k in _NATIVE_EXACT or k.startswith("fast_project_in."):
        return k
    if k in _EXACT:
        return _EXACT[k]
    if k.startswith("model.layers."):
        n, tail = k[len("model.layers."):].split(".", 1)
        t = _LAYER_TAIL.get(tail)
        return f"layers.{n}.{t}" if t else None
    for pfx in ("model.audio_decoder.layers.", "fast_transformer.layers."):
        if k.startswith(pfx):
            n, tail = k[len(pfx):].split(".", 1)
            t = _LAYER_TAIL.get(tail)
            return f"fast_layers.{n}.{t}" if t else None
    return k


def _concat_rows(parts):
    """Row-concatenate tensors: f32 arrays, or (dtype, (rows, cols), raw blocks) of one dtype."""
    if all(isinstance(p, np.ndarray) for p in parts):
        return np.concatenate(parts, axis=0)
    dts = {p[0] for p in parts if isinstance(p, tuple)}
    if len(dts) != 1 or not all(isinstance(p, tuple) for p in parts):
        raise ValueError("fuse_qkv: q, k and v must share one storage type")
    cols = {p[1][1] for p in parts}
    if len(cols) != 1:
        raise ValueError("fuse_qkv: q, k and v must share the input width")
    raw = np.concatenate([np.asarray(p[2], np.uint8).reshape(p[1][0], -1) for p in parts], axis=0)
    return (parts[0][0], (sum(p[1][0] for p in parts), parts[0][1][1]), raw)


def fuse_qkv(t: dict) -> dict:
    """Fuse `<p>.wq/.wk/.wv` weights (and biases when all three ship) into `<p>.wqkv`, rows
    q | k | v; a `<p>.wqkv` already present is kept."""
    out = dict(t)
    for key in [k for k in t if k.endswith(".wq.weight")]:
        base = key[: -len(".wq.weight")]
        for suffix in ("weight", "bias"):
            q, k_, v = (f"{base}.{n}.{suffix}" for n in ("wq", "wk", "wv"))
            fused = f"{base}.wqkv.{suffix}"
            if fused not in out and q in out and k_ in out and v in out:
                out[fused] = _concat_rows([out[q], out[k_], out[v]])
                for n in (q, k_, v):
                    del out[n]
    return out


def quantize_q8_0(w: np.ndarray) -> tuple:
    """ggml Q8_0 blocks of a 2-D f32 matrix (gguf-py's quantizer, bit-exact with ggml)."""
    from gguf import GGMLQuantizationType, quants

    w = np.ascontiguousarray(w, np.float32)
    if w.ndim != 2 or w.shape[1] % 32:
        raise ValueError(f"Q8_0 needs a 2-D matrix with a multiple of 32 columns, got {w.shape}")
    return (SX_DTYPE_Q8_0, w.shape, quants.quantize(w, GGMLQuantizationType.Q8_0))


# ---- readers ------------------------------------------------------------------------------

_ST_DTYPES = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16, "F64": np.float64}


def read_safetensors(path: str) -> dict:
    """name -> f32 ndarray from a .safetensors file (f32 / f16 / bf16 / f64 tensors)."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
        data = np.frombuffer(f.read(), np.uint8)
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        dt = info["dtype"]
        if dt not in _ST_DTYPES:
            raise ValueError(f"{path}: tensor {name} has unsupported dtype {dt}")
        lo, hi = info["data_offsets"]
        a = data[lo:hi].view(_ST_DTYPES[dt]).reshape(info["shape"])
        if dt == "BF16":
            a = (a.astype(np.uint32) << 16).view(np.float32)
        out[name] = np.ascontiguousarray(a, np.float32)
    return out


def read_gguf(path: str) -> dict:
    """name -> f32 ndarray (F32 / F16 tensors) or (dtype, (rows, cols), raw GGML blocks)
    (Q8_0 / Q4_K tensors) from a GGUF file."""
    from gguf import GGMLQuantizationType as Q
    from gguf import GGUFReader

    out = {}
    for t in GGUFReader(path).tensors:
        dims = [int(d) for d in t.shape][::-1]  # GGUF lists the innermost dimension first
        if t.tensor_type in (Q.F32, Q.F16):
            out[t.name] = np.ascontiguousarray(np.asarray(t.data, np.float32).reshape(dims))
        elif t.tensor_type in (Q.Q8_0, Q.Q4_K):
            if len(dims) != 2:
                raise ValueError(f"{path}: quantized tensor {t.name} is not 2-D")
            dt = SX_DTYPE_Q8_0 if t.tensor_type == Q.Q8_0 else SX_DTYPE_Q4_K
            out[t.name] = (dt, (dims[0], dims[1]), np.ascontiguousarray(t.data, np.uint8).reshape(dims[0], -1))
        else:
            raise ValueError(f"{path}: tensor {t.name} has unsupported type {t.tensor_type.name}")
    return out


# ---- ingest -------------------------------------------------------------------------------

def ingest(tensors: dict, wtype: int = SX_DTYPE_Q8_0) -> np.ndarray:
    """An SXW1 blob from checkpoint tensors (as returned by read_safetensors / read_gguf, or
    merged from several shards): names remapped, q/k/v fused, every f32 2-D weight stored as
    `wtype` (SX_DTYPE_Q8_0 or SX_DTYPE_F32); quantized tensors are kept as they are."""
    if wtype not in (SX_DTYPE_Q8_0, SX_DTYPE_F32):
        raise ValueError("ingest quantizes to Q8_0 or keeps f32 (Q4_K blocks are copied from GGUF only)")
    named = {}
    for k, v in tensors.items():
        name = remap_key(k)
        if name is None:
            continue
        if name in named:
            raise ValueError(f"two checkpoint tensors map to {name}")
        named[name] = v
    named = fuse_qkv(named)
    out = {}
    for name, v in named.items():
        if isinstance(v, tuple):
            out[name] = v
        elif v.ndim == 2 and wtype == SX_DTYPE_Q8_0:
            out[name] = quantize_q8_0(v)
        else:
            out[name] = np.ascontiguousarray(v, np.float32)
    return write_blob(out)


def ingest_files(paths: list[str], wtype: int = SX_DTYPE_Q8_0) -> np.ndarray:
    """ingest() over the tensors of several checkpoint files (.safetensors or .gguf shards)."""
    tensors = {}
    for p in paths:
        part = read_gguf(p) if p.endswith(".gguf") else read_safetensors(p)
        dup = set(part) & set(tensors)
        if dup:
            raise ValueError(f"{p}: tensors already read from another shard: {sorted(dup)[:3]}")
        tensors.update(part)
    return ingest(tensors, wtype)


# ---- prompt assembly ------------------------------------------------------------------------

def build_prompt_with_reference(head_ids, ref_codes, tail_ids, semantic_begin_id: int) -> np.ndarray:
    """The [1 + C, T] prompt of a voice-cloning request (s2/mod.rs:202-275): the tokenized
    head text (system turn up to `Speech:`), the reference audio span, and the tokenized
    tail (end of the system turn, the user turn with the target text, `<|voice|>`). Row 0
    holds the text ids and, on the audio span, semantic_begin_id + code 0; rows 1.. hold
    the reference codes on the audio span and 0 elsewhere. The caller's tokenizer produces
    head_ids / tail_ids from the reference's chat template."""
    head = np.asarray(head_ids, np.uint32).reshape(-1)
    tail = np.asarray(tail_ids, np.uint32).reshape(-1)
    codes = np.asarray(ref_codes, np.uint32)
    if codes.ndim == 3:
        codes = codes.reshape(codes.shape[-2], codes.shape[-1])
    n_cb, t_ref = codes.shape
    total = head.size + t_ref + tail.size
    out = np.zeros((1 + n_cb, total), np.uint32)
    out[0, : head.size] = head
    out[0, head.size: head.size + t_ref] = semantic_begin_id + codes[0]
    out[1:, head.size: head.size + t_ref] = codes
    out[0, head.size + t_ref:] = tail
    return out
