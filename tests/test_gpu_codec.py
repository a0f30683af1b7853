"""Device codec decode (include/syrinx_codec.h) against the float64 oracle
(oracle/codec_oracle.py) on seeded synthetic weights and codes.

Tolerance: waveform max-abs 1e-3, the reference's own codec bound
(tests/real_fish_s2_parity.rs:43, CODEC_WAV_TOL)."""
import numpy as np
import pytest
import torch

from oracle import codec_oracle as co
from syrinx_b200 import _lib
from syrinx_b200.codec import S1_CODEC, S2_CODEC, TINY_CODEC, RvqCodec, synth_codec_weights, synth_codes

pytestmark = pytest.mark.gpu
WAV_TOL = 1e-3


@pytest.fixture(scope="module")
def tiny():
    w = synth_codec_weights(TINY_CODEC, seed=11)
    return w, RvqCodec(w)


@pytest.fixture(scope="module")
def s2():
    w = synth_codec_weights(S2_CODEC, seed=12)
    return w, RvqCodec(w)


def _check(w, codec, codes):
    got = codec.decode(codes)
    ref = co.decode(w, codes)
    assert got.shape == ref.shape
    d = float(np.max(np.abs(got - ref)))
    assert d < WAV_TOL, f"max-abs {d:.3e}"
    return got


def test_info(tiny, s2):
    for shape, (_, c) in ((TINY_CODEC, tiny), (S2_CODEC, s2)):
        i = c.info
        assert (i.hop, i.sample_rate, i.num_codebooks) == (shape.hop, 44100, shape.num_codebooks)
        assert (i.semantic_size, i.residual_size, i.codebook_dim) == (
            shape.semantic_size, shape.residual_size, shape.codebook_dim)
        assert (i.latent_dim, i.n_layers) == (shape.latent, shape.n_layers)


@pytest.mark.parametrize("T", [1, 5, 37])
def test_tiny_matches_oracle(tiny, T):
    w, c = tiny
    _check(w, c, synth_codes(TINY_CODEC, T, seed=T))


@pytest.mark.parametrize("ncb", [1, 2])
def test_fewer_codebooks(tiny, ncb):
    w, c = tiny
    _check(w, c, synth_codes(TINY_CODEC, 9, seed=3, n_codebooks=ncb))


@pytest.mark.parametrize("T", [8, 40])
def test_s2_matches_oracle(s2, T):
    w, c = s2
    _check(w, c, synth_codes(S2_CODEC, T, seed=100 + T))


def test_s1_modded_dac_matches_oracle():
    """The s1 codec (ModdedDac::decode, s1/codec.rs:262-290): no post_module, top-level names."""
    w = synth_codec_weights(S1_CODEC, seed=13)
    c = RvqCodec(w)
    assert c.info.n_layers == 0 and c.info.num_codebooks == 10 and c.hop == 2048
    _check(w, c, synth_codes(S1_CODEC, 8, seed=14))
    _check(w, c, synth_codes(S1_CODEC, 5, seed=15, n_codebooks=8))  # config 2 emits 8 codebooks
    c.close()


def test_clamped_codes(tiny):
    w, c = tiny
    codes = synth_codes(TINY_CODEC, 6, seed=1)
    big = codes.copy()
    big[0, 2] = 4_000_000_000
    big[3, 5] = TINY_CODEC.residual_size
    clamped = codes.copy()
    clamped[0, 2] = TINY_CODEC.semantic_size - 1
    clamped[3, 5] = TINY_CODEC.residual_size - 1
    assert np.array_equal(c.decode(big), c.decode(clamped))
    _check(w, c, big)


def test_s2_long_prefix_is_stable(s2):
    """Without GRN every stage is causal, so a prefix of the codes decodes to the prefix of
    the waveform (a size-independent check at 480 frames, 22 s of audio). The two decodes
    may run a product on different units (tensor cores when it fills the GPU, CUDA cores
    otherwise), so the check is to 1e-4, ten times inside the parity bound."""
    _, c = s2
    codes = synth_codes(S2_CODEC, 480, seed=5)
    full = c.decode(codes)
    assert full.shape == (480 * S2_CODEC.hop,)
    assert np.isfinite(full).all() and 0.05 < full.std() < 0.9
    head = c.decode(codes[:, :100])
    assert float(np.max(np.abs(head - full[: head.size]))) < 1e-4


def test_device_entry_point_matches_host(tiny):
    _, c = tiny
    codes = synth_codes(TINY_CODEC, 13, seed=8)
    ref = c.decode(codes)
    dc = torch.from_numpy(codes.astype(np.int32)).cuda()
    wav = torch.empty(13 * c.hop, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream()
    c.set_stream(s.cuda_stream)
    c.decode_device(dc.data_ptr(), codes.shape[0], 13, wav.data_ptr())
    s.synchronize()
    c.set_stream(0)
    assert np.array_equal(wav.cpu().numpy(), ref)


def test_argument_errors(tiny):
    _, c = tiny
    assert c.decode(np.zeros((4, 0), np.uint32)).size == 0
    with pytest.raises(_lib.SyrinxError) as e:
        c.decode(np.zeros((TINY_CODEC.num_codebooks + 1, 3), np.uint32))
    assert e.value.code == -1
    codes = np.zeros((4, 3), np.uint32)
    out = np.zeros(3 * c.hop - 1, np.float32)
    rc = _lib.lib().sx_codec_decode(c._h, codes.ctypes.data_as(_lib._u32p), 4, 3,
                                    out.ctypes.data_as(_lib._f32p), out.size)
    assert rc == -7
