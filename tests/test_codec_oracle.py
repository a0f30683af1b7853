"""CPU checks of the codec decode: the oracle's primitives against torch.nn.functional and the
reference's known-answer vectors, the device path's index arithmetic (the implicit im2col
and the stride-phase form of the transposed convolution) restated on the CPU, oracle
invariants, and the C ABI's argument and blob checks (no GPU needed)."""
import ctypes as C
import json
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import codec_oracle as co
from syrinx_b200 import _lib
from syrinx_b200.blob import read_blob, write_blob
from syrinx_b200.codec import S1_CODEC, TINY_CODEC, CodecShape, synth_codec_weights, synth_codes

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
RNG = np.random.default_rng(7)


@pytest.mark.parametrize("K,dil,groups", [(7, 1, 1), (7, 3, 1), (7, 9, 1), (1, 1, 1), (7, 1, 6)])
def test_causal_conv_matches_torch(K, dil, groups):
    C_in, C_out, L = 6, (6 if groups > 1 else 5), 40
    x = RNG.standard_normal((C_in, L))
    w = RNG.standard_normal((C_out, C_in // groups, K))
    b = RNG.standard_normal(C_out)
    ref = F.conv1d(F.pad(torch.tensor(x)[None], ((K - 1) * dil, 0)), torch.tensor(w), torch.tensor(b),
                   dilation=dil, groups=groups)[0].numpy()
    assert np.allclose(co.causal_conv1d(x, w, b, dilation=dil, groups=groups), ref, atol=1e-12)


@pytest.mark.parametrize("s,K", [(8, 16), (4, 8), (2, 4), (2, 2)])
def test_causal_transpose_matches_torch(s, K):
    x = RNG.standard_normal((5, 11))
    w = RNG.standard_normal((5, 3, K))
    b = RNG.standard_normal(3)
    ref = F.conv_transpose1d(torch.tensor(x)[None], torch.tensor(w), torch.tensor(b), stride=s)[0].numpy()
    ref = ref[:, : ref.shape[1] - (K - s)]
    got = co.causal_transpose1d(x, w, b, s)
    assert got.shape == (3, 11 * s)
    assert np.allclose(got, ref, atol=1e-12)


def _implicit_gemm(A, x, K, dil, phase=1, cout=None):
    """The device product of syrinx_b200/csrc/codec.cu, element by element: B[r][n] =
    x[r // K][n - (K-1 - r % K) * dil] (zero before 0); row m of a phase product stores to
    y[m % cout][n * phase + m // cout]."""
    M, R = A.shape
    N = x.shape[1]
    B = np.zeros((R, N))
    for r in range(R):
        ci, tap = divmod(r, K)
        sh = (K - 1 - tap) * dil
        B[r, sh:] = x[ci, : N - sh] if sh < N else 0
    Y = A @ B
    if phase == 1:
        return Y
    y = np.zeros((cout, N * phase))
    for m in range(M):
        y[m % cout, (m // cout)::phase] = Y[m]
    return y


@pytest.mark.parametrize("dil", [1, 3, 9])
def test_device_im2col_indexing(dil):
    x = RNG.standard_normal((4, 30))
    w = RNG.standard_normal((3, 4, 7))
    got = _implicit_gemm(w.reshape(3, -1), x, 7, dil)
    assert np.allclose(got, co.causal_conv1d(x, w, np.zeros(3), dilation=dil), atol=1e-12)


@pytest.mark.parametrize("s,per", [(8, 2), (4, 2), (2, 2), (2, 1)])
def test_device_phase_packing_of_transposed_conv(s, per):
    """The repacking done at load (Loader::tconv): row p*cout + co, column ci*taps + j holds
    kernel tap p + (taps-1-j)*s."""
    Ci, Co, Kt = 5, 3, s * per
    w = RNG.standard_normal((Ci, Co, Kt))
    x = RNG.standard_normal((Ci, 13))
    A = np.zeros((s * Co, Ci * per))
    for p in range(s):
        for c in range(Co):
            for ci in range(Ci):
                for j in range(per):
                    A[p * Co + c, ci * per + j] = w[ci, c, p + (per - 1 - j) * s]
    got = _implicit_gemm(A, x, per, 1, phase=s, cout=Co)
    assert np.allclose(got, co.causal_transpose1d(x, w, np.zeros(Co), s), atol=1e-12)


def test_rope_and_rmsnorm_known_answers():
    kats = json.load(open(os.path.join(ROOT, "tests", "golden", "parity_kat.json")))
    k = kats["rope"]
    x = np.array(k["input"]["x"], np.float64)  # [T, H, D]
    cos, sin = co.rope_tables(x.shape[0], head_dim=x.shape[2], base=k["input"]["theta"])
    assert np.max(np.abs(co.apply_rope(x, cos, sin).reshape(-1) - k["data"])) <= k["tol"]
    k = kats["rmsnorm"]
    x = np.array(k["input"]["x"], np.float64).T  # channels-first
    y = co.rms_norm_cf(x, np.array(k["input"]["w"]), k["input"]["eps"])
    assert np.max(np.abs(y.T.reshape(-1) - k["data"])) <= k["tol"]


def test_gelu_and_layer_norm_match_torch():
    x = RNG.standard_normal((16, 9))
    w, b = RNG.standard_normal(16), RNG.standard_normal(16)
    ref = F.layer_norm(torch.tensor(x.T), (16,), torch.tensor(w), torch.tensor(b), eps=1e-6).numpy().T
    assert np.allclose(co.layer_norm_cf(x, w, b), ref, atol=1e-10)


NO_GRN = CodecShape(latent=128, n_layers=2, ffn=256, semantic_size=64, residual_size=32,
                    n_residual=3, decoder_dim=96, grn=(False, False))


def test_oracle_length_and_causality():
    w = synth_codec_weights(NO_GRN, seed=3)
    codes = synth_codes(NO_GRN, 12, seed=4)
    y = co.decode(w, codes)
    assert y.shape == (12 * NO_GRN.hop,)
    assert 0.05 < y.std() < 0.9  # neither silent nor saturated
    c2 = codes.copy()
    c2[:, 7:] = synth_codes(NO_GRN, 5, seed=5)
    y2 = co.decode(w, c2)
    cut = 7 * NO_GRN.hop
    assert np.array_equal(y[:cut], y2[:cut])
    assert not np.allclose(y[cut:], y2[cut:])


def test_oracle_grn_is_sequence_wide():
    """GRN normalises over the whole time axis, so with it a later frame changes earlier
    samples (codec.rs:237-257); the device path reproduces this, it does not stream."""
    w = synth_codec_weights(TINY_CODEC, seed=3)
    codes = synth_codes(TINY_CODEC, 8, seed=4)
    c2 = codes.copy()
    c2[:, 6:] = synth_codes(TINY_CODEC, 2, seed=9)
    cut = 6 * TINY_CODEC.hop
    assert not np.allclose(co.decode(w, codes)[:cut], co.decode(w, c2)[:cut])


def test_oracle_clamps_codes():
    w = synth_codec_weights(NO_GRN, seed=3)
    codes = synth_codes(NO_GRN, 4, seed=4)
    big = codes.copy()
    big[0, 1] = 10**6
    big[2, 3] = 10**6
    ref = codes.copy()
    ref[0, 1] = NO_GRN.semantic_size - 1
    ref[2, 3] = NO_GRN.residual_size - 1
    assert np.array_equal(co.decode(w, big), co.decode(w, ref))


TINY_S1 = CodecShape(variant="s1", latent=128, n_layers=0, semantic_size=64, residual_size=32,
                     n_residual=3, decoder_dim=96)


def test_s1_names_and_oracle():
    """The s1 modded DAC: RVQ and upsample at the top level of the names, no post_module."""
    w = synth_codec_weights(TINY_S1, seed=2)
    assert "semantic_quantizer.quantizers.0.codebook.weight" in w and "upsample.0.0.conv.weight" in w
    assert not any(k.startswith("quantizer.semantic") or "post_module" in k for k in w)
    assert {k for k in synth_codec_weights(S1_CODEC, seed=0) if "post_module" in k} == set()
    y = co.decode(w, synth_codes(TINY_S1, 6, seed=1))
    assert y.shape == (6 * TINY_S1.hop,) and 0.05 < y.std() < 0.9


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device error path")
def test_s1_blob_parses_before_the_device():
    rc, msg = _create(write_blob(synth_codec_weights(TINY_S1, seed=2)))
    assert rc == -2 and "cuda" in msg.lower()


def test_codec_blob_round_trip_keeps_rank3_kernels():
    w = synth_codec_weights(TINY_CODEC, seed=1)
    back = read_blob(write_blob(w))
    assert back.keys() == w.keys()
    for k in w:
        assert back[k].shape == w[k].shape and np.array_equal(back[k], w[k]), k


def _create(blob):
    h = C.c_void_p()
    rc = _lib.lib().sx_codec_create(blob.ctypes.data, blob.nbytes, 0, C.byref(h))
    return rc, _lib.lib().sx_last_error().decode()


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device error path")
def test_codec_create_without_gpu_reports_cuda_error():
    rc, msg = _create(write_blob(synth_codec_weights(TINY_CODEC, seed=1)))
    assert rc == -2 and "cuda" in msg.lower()


def test_codec_blob_errors_name_the_tensor():
    w = synth_codec_weights(TINY_CODEC, seed=1)
    del w["decoder.model.2.block.3.block.1.conv.weight"]
    rc, msg = _create(write_blob(w))
    assert rc == -4 and "decoder.model.2.block.3.block.1.conv.weight" in msg
    w = synth_codec_weights(TINY_CODEC, seed=1)
    w["decoder.model.0.conv.weight"] = w["decoder.model.0.conv.weight"][:, :, :5]
    rc, msg = _create(write_blob(w))
    assert rc == -4 and "decoder.model" in msg
    w = synth_codec_weights(TINY_CODEC, seed=1)
    w["quantizer.post_module.layers.1.attention.wo.weight"] = np.zeros((3, 3), np.float32)
    rc, msg = _create(write_blob(w))
    assert rc == -4 and "layers.1.attention.wo.weight" in msg


def test_codec_null_arguments():
    L = _lib.lib()
    assert L.sx_codec_create(None, 0, 0, None) == -1
    assert L.sx_codec_decode(None, None, 1, 1, None, 0) == -1
    assert L.sx_codec_set_stream(None, None) == -1
