"""CPU restatement of the codec decode, in float64 numpy: the s2 `EvaGanDac::decode`
(crates/syrinx-fish/src/s2/codec.rs:342-379) and the s1 `ModdedDac::decode`
(crates/syrinx-fish/src/s1/codec.rs:262-290), which is the same decoder without the
post_module transformer and with its tensors at the top level of the names.

TEST INFRASTRUCTURE ONLY: imported by tests/ and by nothing on the product path.

Parity status: unpinned. The reference's codec check (tests/real_fish_s2_parity.rs:125-143,
waveform max-abs 1e-3) reads a fixture produced from the real `codec.pth`, which is not in
the reference tree, and the Rust/Candle reference cannot be built here. What is pinned:
the convolution primitives against torch.nn.functional (an independent implementation of
the same conv1d / conv_transpose1d definitions Candle follows) in tests/test_codec_oracle.py,
and RMSNorm / interleaved RoPE / softmax / SiLU through the reference's own known-answer
vectors, which the decode-step oracle's identical formulas already pass.

Weights are a dict name -> array in the reference's shapes (conv [out, in, K], transposed
conv [in, out, K], linear [out, in]); activations are channels-first [C, T].
"""
from __future__ import annotations

import math

import numpy as np
from scipy.special import erf

TF_HEAD_DIM = 64        # codec.rs:58-60
TF_ROPE_BASE = 10000.0  # codec.rs:61-63
TF_NORM_EPS = 1e-5      # codec.rs:64-65
SNAKE_EPS = 1e-9        # codec.rs:66-67
LN_EPS = 1e-6           # codec.rs:205-210
DILATIONS = (1, 3, 9)   # codec.rs:320-322


def _f(w, name):
    return np.asarray(w[name], np.float64)


def causal_conv1d(x, weight, bias, dilation=1, groups=1):
    """CausalConvNet.forward at stride 1 (codec.rs:93-115): left-pad (K-1)*dilation zeros,
    valid convolution (the alignment pad of codec.rs:630-641 is 0 at stride 1)."""
    cout, cin_g, K = weight.shape
    C, L = x.shape
    pad = (K - 1) * dilation
    xp = np.concatenate([np.zeros((C, pad)), x], axis=1)
    y = np.zeros((cout, L))
    if groups == 1:
        for k in range(K):
            y += weight[:, :, k] @ xp[:, k * dilation: k * dilation + L]
    else:
        assert groups == C == cout and cin_g == 1
        for k in range(K):
            y += weight[:, 0, k][:, None] * xp[:, k * dilation: k * dilation + L]
    return y + bias[:, None]


def causal_transpose1d(x, weight, bias, stride):
    """CausalTransConvNet.forward (codec.rs:117-137): ConvTranspose1d (full output
    (L-1)*stride + K), bias, then drop K - stride samples on the right."""
    cin, cout, K = weight.shape
    L = x.shape[1]
    full = np.zeros((cout, (L - 1) * stride + K))
    for k in range(K):
        full[:, k: k + (L - 1) * stride + 1: stride] += weight[:, :, k].T @ x
    full += bias[:, None]
    return full[:, : full.shape[1] - (K - stride)]


def snake(x, alpha):
    """Snake1d (codec.rs:139-149)."""
    a = np.asarray(alpha, np.float64).reshape(-1)[:, None]
    return x + (1.0 / (a + SNAKE_EPS)) * np.sin(a * x) ** 2


def rms_norm_cf(x, w, eps=TF_NORM_EPS):
    """RMSNorm over the channel axis (s2/nn.rs:100-106)."""
    return x / np.sqrt((x * x).mean(axis=0, keepdims=True) + eps) * w[:, None]


def layer_norm_cf(x, w, b, eps=LN_EPS):
    """Channels-last LayerNorm (codec.rs:647-655) applied per time step of [C, T]."""
    mean = x.mean(axis=0, keepdims=True)
    xc = x - mean
    var = (xc * xc).mean(axis=0, keepdims=True)
    return xc / np.sqrt(var + eps) * w[:, None] + b[:, None]


def rope_tables(T, head_dim=TF_HEAD_DIM, base=TF_ROPE_BASE):
    """precompute_rope (s2/nn.rs:117-141): inv_freq and angles in f32, cos/sin of them."""
    half = head_dim // 2
    i = np.arange(half, dtype=np.float32)
    inv = np.float32(1.0) / np.power(np.float32(base), np.float32(2.0) * i / np.float32(head_dim))
    ang = np.arange(T, dtype=np.float32)[:, None] * inv[None, :]  # [T, half] f32
    return np.cos(ang.astype(np.float64)), np.sin(ang.astype(np.float64))


def apply_rope(x, cos, sin):
    """Interleaved RoPE (s2/nn.rs:154-166) on x [T, H, D]."""
    x0, x1 = x[..., 0::2], x[..., 1::2]
    c, s = cos[:, None, :], sin[:, None, :]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x1 * c + x0 * s
    return out


def transformer(w, prefix, x):
    """The full-causal RoPE transformer (codec.rs:559-626); x channels-first [dim, T]."""
    n = 0
    while f"{prefix}.layers.{n}.attention_norm.weight" in w:
        n += 1
    if n == 0:
        return x
    D, T = x.shape
    H = D // TF_HEAD_DIM
    cos, sin = rope_tables(T)
    mask = np.triu(np.full((T, T), -np.inf), k=1)
    h = x
    for layer in range(n):
        p = f"{prefix}.layers.{layer}"
        hn = rms_norm_cf(h, _f(w, f"{p}.attention_norm.weight"))
        qkv = _f(w, f"{p}.attention.wqkv.weight") @ hn  # [3D, T]
        q = qkv[:D].T.reshape(T, H, TF_HEAD_DIM)
        k = qkv[D: 2 * D].T.reshape(T, H, TF_HEAD_DIM)
        v = qkv[2 * D:].T.reshape(T, H, TF_HEAD_DIM)
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        s = np.einsum("thd,shd->hts", q, k) / math.sqrt(TF_HEAD_DIM) + mask[None]
        s = np.exp(s - s.max(axis=-1, keepdims=True))
        pr = s / s.sum(axis=-1, keepdims=True)
        ctx = np.einsum("hts,shd->thd", pr, v).reshape(T, D).T  # [D, T]
        a = _f(w, f"{p}.attention.wo.weight") @ ctx
        h = h + a * _f(w, f"{p}.attention_layer_scale.gamma")[:, None]
        hn = rms_norm_cf(h, _f(w, f"{p}.ffn_norm.weight"))
        g = _f(w, f"{p}.feed_forward.w1.weight") @ hn
        u = _f(w, f"{p}.feed_forward.w3.weight") @ hn
        f = _f(w, f"{p}.feed_forward.w2.weight") @ ((g / (1.0 + np.exp(-g))) * u)
        h = h + f * _f(w, f"{p}.ffn_layer_scale.gamma")[:, None]
    return rms_norm_cf(h, _f(w, f"{prefix}.norm.weight"))


def grn(x, gamma, beta):
    """ConvNeXt-V2 GRN over the time axis (codec.rs:237-257); x is [C, T]."""
    gx = np.sqrt((x * x).sum(axis=1, keepdims=True))  # [C, 1]
    nx = gx / (gx.mean(axis=0, keepdims=True) + 1e-6)
    return x + (x * nx * gamma[:, None] + beta[:, None])


def convnext(w, prefix, x):
    """ConvNeXt block (codec.rs:189-235): depthwise causal k7 conv, LayerNorm, pwconv1,
    GELU (erf), optional GRN, pwconv2, optional layer scale, residual."""
    C = x.shape[0]
    h = causal_conv1d(x, _f(w, f"{prefix}.dwconv.conv.weight"), _f(w, f"{prefix}.dwconv.conv.bias"),
                      groups=C)
    h = layer_norm_cf(h, _f(w, f"{prefix}.norm.weight"), _f(w, f"{prefix}.norm.bias"))
    h = _f(w, f"{prefix}.pwconv1.weight") @ h + _f(w, f"{prefix}.pwconv1.bias")[:, None]
    h = 0.5 * h * (1.0 + erf(h / math.sqrt(2.0)))
    if f"{prefix}.grn.gamma" in w:
        h = grn(h, _f(w, f"{prefix}.grn.gamma").reshape(-1), _f(w, f"{prefix}.grn.beta").reshape(-1))
    h = _f(w, f"{prefix}.pwconv2.weight") @ h + _f(w, f"{prefix}.pwconv2.bias")[:, None]
    if f"{prefix}.gamma" in w:
        h = h * _f(w, f"{prefix}.gamma").reshape(-1)[:, None]
    return x + h


def residual_unit(w, prefix, x, dilation):
    """ResidualUnit (codec.rs:151-186)."""
    y = snake(x, _f(w, f"{prefix}.block.0.alpha"))
    y = causal_conv1d(y, _f(w, f"{prefix}.block.1.conv.weight"), _f(w, f"{prefix}.block.1.conv.bias"),
                      dilation=dilation)
    y = snake(y, _f(w, f"{prefix}.block.2.alpha"))
    y = causal_conv1d(y, _f(w, f"{prefix}.block.3.conv.weight"), _f(w, f"{prefix}.block.3.conv.bias"))
    return x[:, : y.shape[1]] + y


def decode_codebook(w, prefix, codes):
    """One quantizer's from_codes (codec.rs:259-276): codebook rows, then out_proj (k=1)."""
    zp = _f(w, f"{prefix}.codebook.weight")[codes].T  # [cbdim, T]
    return causal_conv1d(zp, _f(w, f"{prefix}.out_proj.weight"), _f(w, f"{prefix}.out_proj.bias"))


def upsample(w, z, qp="quantizer."):
    """codec.rs:278-300: per stage a transposed conv (kernel = stride) then ConvNeXt."""
    s = 0
    while f"{qp}upsample.{s}.0.conv.weight" in w:
        wt = _f(w, f"{qp}upsample.{s}.0.conv.weight")
        z = causal_transpose1d(z, wt, _f(w, f"{qp}upsample.{s}.0.conv.bias"), wt.shape[2])
        z = convnext(w, f"{qp}upsample.{s}.1", z)
        s += 1
    return z


def run_generator(w, z):
    """The DAC decoder (codec.rs:302-340)."""
    x = causal_conv1d(z, _f(w, "decoder.model.0.conv.weight"), _f(w, "decoder.model.0.conv.bias"))
    i = 1
    while f"decoder.model.{i}.block.1.conv.weight" in w:
        p = f"decoder.model.{i}"
        x = snake(x, _f(w, f"{p}.block.0.alpha"))
        wt = _f(w, f"{p}.block.1.conv.weight")
        x = causal_transpose1d(x, wt, _f(w, f"{p}.block.1.conv.bias"), wt.shape[2] // 2)
        for r, d in enumerate(DILATIONS):
            x = residual_unit(w, f"{p}.block.{r + 2}", x, d)
        i += 1
    x = snake(x, _f(w, f"decoder.model.{i}.alpha"))
    x = causal_conv1d(x, _f(w, f"decoder.model.{i + 1}.conv.weight"), _f(w, f"decoder.model.{i + 1}.conv.bias"))
    return np.tanh(x)


def decode(w, codes):
    """codes [n_codebooks, T] -> waveform [T * hop] (float64). The s2 codec
    (`EvaGanDac::decode`) nests the RVQ, upsample and post_module under `quantizer.`; the s1
    modded DAC (`ModdedDac::decode`, crates/syrinx-fish/src/s1/codec.rs:262-290) has them at
    the top level and no post_module."""
    codes = np.asarray(codes)
    if codes.ndim == 3:
        codes = codes[0]
    n_cb, T = codes.shape
    qp = "quantizer." if "quantizer.semantic_quantizer.quantizers.0.codebook.weight" in w else ""
    sem = f"{qp}semantic_quantizer.quantizers.0"
    sem_max = w[f"{sem}.codebook.weight"].shape[0] - 1
    z = decode_codebook(w, sem, np.minimum(codes[0].astype(np.int64), sem_max))
    for i in range(n_cb - 1):
        pre = f"{qp}quantizer.quantizers.{i}"
        res_max = w[f"{pre}.codebook.weight"].shape[0] - 1
        z = z + decode_codebook(w, pre, np.minimum(codes[i + 1].astype(np.int64), res_max))
    z = transformer(w, f"{qp}post_module", z)
    z = upsample(w, z, qp)
    return run_generator(w, z).reshape(-1)
