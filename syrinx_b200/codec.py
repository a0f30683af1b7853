"""The device RVQ codec decode behind include/syrinx_codec.h, with the reference's
`RvqCodec` decode surface (crates/syrinx-fish/src/common/codec.rs:13-34).

`CodecShape` describes one causal-DAC codec (`EvaGanDac`, crates/syrinx-fish/src/s2/
codec.rs); `S2_CODEC` holds the s2 geometry (CodecConfig, common/config.rs: 10 codebooks,
semantic 4096 x 8, residual 1024 x 8, 44.1 kHz, hop 2048, decoder rates [8, 8, 4, 2]; the
post_module transformer 8 x 1024, 16 heads of 64). `synth_codec_weights` builds seeded
random weights of that architecture under the reference's `codec.pth` names (weight-norm
folded, as s2/load.rs leaves them), since no checkpoint is available offline.
"""
from __future__ import annotations

import ctypes as C
import dataclasses

import numpy as np

from . import _lib
from .blob import write_blob
from .configs import SxCodecInfo


@dataclasses.dataclass(frozen=True)
class CodecShape:
    latent: int = 1024            # RVQ latent / transformer width
    n_layers: int = 8             # quantizer.post_module layers
    ffn: int = 3072               # SwiGLU inner width of the post_module
    semantic_size: int = 4096
    residual_size: int = 1024
    n_residual: int = 9
    codebook_dim: int = 8
    up_factors: tuple = (2, 2)    # quantizer.upsample.{0,1} (kernel = stride)
    convnext_mult: int = 4        # pwconv1 width / channels
    grn: tuple = (False, False)   # ConvNeXt-V2 GRN present per upsample stage
    layer_scale: tuple = (True, True)  # ConvNeXt gamma present per upsample stage
    decoder_dim: int = 1536       # decoder.model.0 output channels
    decoder_rates: tuple = (8, 8, 4, 2)
    sample_rate: int = 44100
    variant: str = "s2"           # "s1": modded-DAC names at the top level, no post_module

    @property
    def hop(self) -> int:
        return int(np.prod(self.up_factors)) * int(np.prod(self.decoder_rates))

    @property
    def num_codebooks(self) -> int:
        return 1 + self.n_residual


S2_CODEC = CodecShape()
# The s1 modded DAC (ModdedDac, crates/syrinx-fish/src/s1/codec.rs): the same decoder and
# upsample, the RVQ and upsample at the top level of the names, no post_module transformer.
S1_CODEC = CodecShape(variant="s1", n_layers=0)
# A small codec of the same structure for quick checks: every branch (GRN and no GRN,
# layer scale and none) is present.
TINY_CODEC = CodecShape(latent=128, n_layers=2, ffn=256, semantic_size=64, residual_size=32,
                        n_residual=3, decoder_dim=96, grn=(True, False), layer_scale=(True, False))


def synth_codec_weights(shape: CodecShape = S2_CODEC, seed: int = 0) -> dict:
    """name -> f32 ndarray in the reference's shapes: conv kernels [out, in, K],
    transposed conv kernels [in, out, K], linear weights [out, in], Snake alphas [1, C, 1].
    Scales keep every stage's activations of order one, so that the waveform is neither
    silent nor saturated by the final tanh."""
    rng = np.random.default_rng(seed)
    w = {}

    def normal(shp, std):
        return rng.standard_normal(shp, dtype=np.float32) * np.float32(std)

    def unif(shp, lo, hi):
        return rng.uniform(lo, hi, shp).astype(np.float32)

    D, cbd = shape.latent, shape.codebook_dim
    qp = "quantizer." if shape.variant == "s2" else ""
    for i in range(shape.num_codebooks):
        pre = (f"{qp}semantic_quantizer.quantizers.0" if i == 0
               else f"{qp}quantizer.quantizers.{i - 1}")
        size = shape.semantic_size if i == 0 else shape.residual_size
        w[f"{pre}.codebook.weight"] = normal((size, cbd), 1.0)
        w[f"{pre}.out_proj.weight"] = normal((D, cbd, 1), 0.3 / np.sqrt(cbd))
        w[f"{pre}.out_proj.bias"] = normal((D,), 0.02)
    F = shape.ffn
    for layer in range(shape.n_layers):
        p = f"{qp}post_module.layers.{layer}"
        w[f"{p}.attention_norm.weight"] = unif((D,), 0.8, 1.2)
        w[f"{p}.attention.wqkv.weight"] = normal((3 * D, D), 1.0 / np.sqrt(D))
        w[f"{p}.attention.wo.weight"] = normal((D, D), 1.0 / np.sqrt(D))
        w[f"{p}.attention_layer_scale.gamma"] = unif((D,), 0.05, 0.3)
        w[f"{p}.ffn_norm.weight"] = unif((D,), 0.8, 1.2)
        w[f"{p}.feed_forward.w1.weight"] = normal((F, D), 1.0 / np.sqrt(D))
        w[f"{p}.feed_forward.w3.weight"] = normal((F, D), 1.0 / np.sqrt(D))
        w[f"{p}.feed_forward.w2.weight"] = normal((D, F), 1.0 / np.sqrt(F))
        w[f"{p}.ffn_layer_scale.gamma"] = unif((D,), 0.05, 0.3)
    if shape.n_layers:
        w[f"{qp}post_module.norm.weight"] = unif((D,), 0.8, 1.2)
    C = D
    for s, f in enumerate(reversed(shape.up_factors)):
        p = f"{qp}upsample.{s}"
        w[f"{p}.0.conv.weight"] = normal((C, C, f), 1.0 / np.sqrt(C))
        w[f"{p}.0.conv.bias"] = normal((C,), 0.02)
        b, C4 = f"{p}.1", shape.convnext_mult * C
        w[f"{b}.dwconv.conv.weight"] = normal((C, 1, 7), 1.0 / np.sqrt(7))
        w[f"{b}.dwconv.conv.bias"] = normal((C,), 0.02)
        w[f"{b}.norm.weight"] = unif((C,), 0.8, 1.2)
        w[f"{b}.norm.bias"] = normal((C,), 0.05)
        w[f"{b}.pwconv1.weight"] = normal((C4, C), 1.0 / np.sqrt(C))
        w[f"{b}.pwconv1.bias"] = normal((C4,), 0.02)
        if shape.grn[s]:
            w[f"{b}.grn.gamma"] = normal((C4,), 0.1)
            w[f"{b}.grn.beta"] = normal((C4,), 0.05)
        w[f"{b}.pwconv2.weight"] = normal((C, C4), 1.0 / np.sqrt(C4))
        w[f"{b}.pwconv2.bias"] = normal((C,), 0.02)
        if shape.layer_scale[s]:
            w[f"{b}.gamma"] = unif((C,), 0.1, 0.5)
    Cd = shape.decoder_dim
    w["decoder.model.0.conv.weight"] = normal((Cd, C, 7), 1.0 / np.sqrt(7 * C))
    w["decoder.model.0.conv.bias"] = normal((Cd,), 0.02)
    C = Cd
    for i, s in enumerate(shape.decoder_rates):
        p = f"decoder.model.{i + 1}"
        Co = C // 2
        w[f"{p}.block.0.alpha"] = unif((1, C, 1), 0.5, 1.5)
        w[f"{p}.block.1.conv.weight"] = normal((C, Co, 2 * s), 1.0 / np.sqrt(2 * C))
        w[f"{p}.block.1.conv.bias"] = normal((Co,), 0.02)
        for r in range(3):
            q = f"{p}.block.{r + 2}.block"
            w[f"{q}.0.alpha"] = unif((1, Co, 1), 0.5, 1.5)
            w[f"{q}.1.conv.weight"] = normal((Co, Co, 7), 1.0 / np.sqrt(7 * Co))
            w[f"{q}.1.conv.bias"] = normal((Co,), 0.02)
            w[f"{q}.2.alpha"] = unif((1, Co, 1), 0.5, 1.5)
            w[f"{q}.3.conv.weight"] = normal((Co, Co, 1), 0.5 / np.sqrt(Co))
            w[f"{q}.3.conv.bias"] = normal((Co,), 0.02)
        C = Co
    n = len(shape.decoder_rates)
    w[f"decoder.model.{n + 1}.alpha"] = unif((1, C, 1), 0.5, 1.5)
    w[f"decoder.model.{n + 2}.conv.weight"] = normal((1, C, 7), 0.1 / np.sqrt(7 * C))
    w[f"decoder.model.{n + 2}.conv.bias"] = np.zeros((1,), np.float32)
    return w


def synth_codes(shape: CodecShape, frames: int, seed: int = 0, n_codebooks: int | None = None) -> np.ndarray:
    """Seeded codes [n_codebooks, frames] (u32) inside each codebook's range."""
    rng = np.random.default_rng(seed)
    ncb = shape.num_codebooks if n_codebooks is None else n_codebooks
    codes = np.empty((ncb, frames), np.uint32)
    codes[0] = rng.integers(0, shape.semantic_size, frames)
    if ncb > 1:
        codes[1:] = rng.integers(0, shape.residual_size, (ncb - 1, frames))
    return codes


def decode_flops(shape: CodecShape, frames: int) -> int:
    """Multiply-adds x 2 of one decode of `frames` frames: the matrix products (linear
    layers, convolutions, transposed convolutions at their kept outputs, causal attention);
    element-wise work is not counted."""
    T, D, F = frames, shape.latent, shape.ffn
    fl = 2 * D * shape.codebook_dim * T * shape.num_codebooks
    fl += shape.n_layers * (2 * T * (3 * D * D + D * D + 3 * F * D) + 2 * 2 * D * T * (T + 1) // 2)
    L, C = T, D
    for f in reversed(shape.up_factors):
        L *= f
        C4 = shape.convnext_mult * C
        fl += 2 * C * C * L + 2 * 7 * C * L + 2 * 2 * C * C4 * L
    fl += 2 * shape.decoder_dim * C * 7 * L
    C = shape.decoder_dim
    for s in shape.decoder_rates:
        Co = C // 2
        L *= s
        fl += 2 * Co * C * 2 * L + 3 * (2 * Co * Co * 7 * L + 2 * Co * Co * L)
        C = Co
    fl += 2 * 7 * C * L
    return int(fl)


def decode_launches(shape: CodecShape) -> int:
    """Kernel launches of one device decode (the sequence of Codec::decode_device)."""
    n = 1  # RVQ from_codes
    if shape.n_layers:
        n += 9 * shape.n_layers + 1  # norm, wqkv, rope, attention, wo, norm, w1|w3, SwiGLU, w2; final norm
    n += sum(5 + (3 if g else 0) for g in shape.grn)  # transposed conv, dwconv, LayerNorm, pwconv1, [GRN], pwconv2
    n += 1 + 14 * len(shape.decoder_rates) + 2  # first conv; Snake + transposed conv + 3 units; Snake + last conv
    return n


class RvqCodec:
    """Codes -> waveform on one GPU (`RvqCodec::decode`, common/codec.rs:26; `EvaGanDac::
    decode`, s2/codec.rs:342-379). `weights` is a dict of f32 arrays (reference names) or
    an SXW1 blob (uint8 array)."""

    def __init__(self, weights, device: int = 0):
        blob = weights if isinstance(weights, np.ndarray) and weights.dtype == np.uint8 else write_blob(weights)
        L = _lib.lib()
        h = C.c_void_p()
        _lib.check(L.sx_codec_create(blob.ctypes.data, blob.nbytes, device, C.byref(h)))
        self._h = h
        info = SxCodecInfo()
        _lib.check(L.sx_codec_get_info(h, C.byref(info)))
        self.info = info

    @property
    def sample_rate(self) -> int:
        return int(self.info.sample_rate)

    @property
    def hop(self) -> int:
        return int(self.info.hop)

    def reserve(self, max_frames: int) -> None:
        _lib.check(_lib.lib().sx_codec_reserve(self._h, int(max_frames)))

    def set_stream(self, stream_ptr: int) -> None:
        _lib.check(_lib.lib().sx_codec_set_stream(self._h, C.c_void_p(stream_ptr)))

    def decode(self, codes) -> np.ndarray:
        """codes [n_codebooks, T] or [1, n_codebooks, T] (host) -> f32 waveform [T * hop]."""
        c = np.asarray(codes)
        if c.ndim == 3:
            if c.shape[0] != 1:
                raise ValueError("codes: batch dimension must be 1")
            c = c[0]
        if c.ndim != 2:
            raise ValueError("codes must be [n_codebooks, T]")
        if c.size and (c.min() < 0):
            raise ValueError("codes must be non-negative")
        c = np.ascontiguousarray(c, np.uint32)
        ncb, T = c.shape
        out = np.empty(T * self.hop, np.float32)
        _lib.check(_lib.lib().sx_codec_decode(
            self._h, c.ctypes.data_as(_lib._u32p), ncb, T,
            out.ctypes.data_as(_lib._f32p), out.size))
        return out

    def decode_device(self, codes_ptr: int, n_codebooks: int, frames: int, wav_ptr: int) -> None:
        """Enqueue a decode on device buffers (codes u32 [n_codebooks][frames], wav f32
        [frames * hop]) on the stream set by set_stream."""
        _lib.check(_lib.lib().sx_codec_decode_device(
            self._h, C.c_void_p(codes_ptr), n_codebooks, frames, C.c_void_p(wav_ptr)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.lib().sx_codec_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
