/*
 * syrinx_codec.h — C ABI of the device RVQ codec decode: a [num_codebooks, T] code matrix
 * (the frames the dual-AR decode emits) to a mono 44.1 kHz waveform.
 *
 * Replaces `RvqCodec::decode` (crates/syrinx-fish/src/common/codec.rs:26) as implemented by
 * the s2 causal-DAC `EvaGanDac::decode` (crates/syrinx-fish/src/s2/codec.rs:342-379): RVQ
 * from_codes (semantic codebook + residual codebooks, summed) -> the `post_module`
 * full-causal RoPE transformer -> ConvNeXt upsample -> DAC decoder (Snake, transposed
 * convs, dilated residual units) -> tanh.
 *
 * The weights are an SXW1 blob (include/syrinx_dualar.h) of f32 tensors under the
 * reference's `codec.pth` names with weight-norm already folded (s2/load.rs folds it at
 * load): e.g. `quantizer.semantic_quantizer.quantizers.0.codebook.weight` [4096, 8],
 * `decoder.model.1.block.1.conv.weight` [1536, 768, 16] (transposed: [in, out, K]),
 * `decoder.model.0.conv.weight` [1536, 1024, 7] ([out, in, K]). Layer counts, widths,
 * upsample factors (kernel of `quantizer.upsample.{s}.0.conv`) and decoder strides
 * (half the kernel of `decoder.model.{i}.block.1.conv`) are read from the tensor shapes.
 *
 * Status codes and sx_last_error() are those of include/syrinx_dualar.h.
 */
#ifndef SYRINX_CODEC_H
#define SYRINX_CODEC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct sx_codec sx_codec;

typedef struct sx_codec_info {
  int32_t hop;            /* waveform samples per code frame (s2: 2048) */
  int32_t sample_rate;    /* 44100 (CodecConfig::sample_rate) */
  int32_t num_codebooks;  /* 1 semantic + the residual quantizers in the blob (s2: 10) */
  int32_t semantic_size;  /* semantic codebook rows (s2: 4096) */
  int32_t residual_size;  /* residual codebook rows (s2: 1024) */
  int32_t codebook_dim;   /* factorized code width (s2: 8) */
  int32_t latent_dim;     /* RVQ latent / transformer width (s2: 1024) */
  int32_t n_layers;       /* post_module transformer layers (s2: 8) */
} sx_codec_info;

/* Parse and upload a codec blob to CUDA device `device` (EvaGanDac::new over load_codec,
 * s2/mod.rs:150-157). SX_E_BLOB names the first missing or mis-shaped tensor. */
int sx_codec_create(const void* blob, size_t blob_size, int32_t device, sx_codec** out);
int sx_codec_destroy(sx_codec* codec);
int sx_codec_get_info(const sx_codec* codec, sx_codec_info* out);

/* Size the activation buffers for inputs of up to `max_frames` frames, so that later
 * decodes of that size allocate nothing. Decodes grow the buffers on demand otherwise. */
int sx_codec_reserve(sx_codec* codec, int32_t max_frames);

/* The CUDA stream (a cudaStream_t, or NULL for the legacy default stream) the device
 * entry point enqueues on and the host entry point runs on. */
int sx_codec_set_stream(sx_codec* codec, void* cuda_stream);

/* Decode host codes [n_codebooks][n_frames] (row-major, u32) into host wav_out, which
 * receives n_frames * hop samples. Codes beyond a codebook's size are clamped to its last
 * row, as the reference does (codec.rs:352-364). n_codebooks must be 1 ..
 * info.num_codebooks; n_frames == 0 writes nothing. SX_E_RANGE if wav_capacity (in
 * samples) is too small. Returns after the waveform is in wav_out. */
int sx_codec_decode(sx_codec* codec, const uint32_t* codes, int32_t n_codebooks, int32_t n_frames,
                    float* wav_out, size_t wav_capacity);

/* The same decode on device buffers, enqueued on the codec's stream without a host
 * synchronisation: codes_dev [n_codebooks][n_frames] u32, wav_dev n_frames * hop f32. */
int sx_codec_decode_device(sx_codec* codec, const uint32_t* codes_dev, int32_t n_codebooks,
                           int32_t n_frames, float* wav_dev);

#ifdef __cplusplus
}
#endif

#endif /* SYRINX_CODEC_H */
