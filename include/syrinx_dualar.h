/*
 * syrinx_dualar.h — C ABI of the B200-native quantized dual-AR decode path.
 *
 * This is the drop-in boundary for the hot path of the Syrinx speech engine: the slow
 * semantic AR transformer step followed by the fast AR codebook expansion, over
 * GGUF-style Q8_0 / Q4_K weights. A thin Rust FFI crate implements the reference's
 * `DualArBackend` trait (crates/syrinx-fish/src/common/dualar.rs:65-136) and the
 * `Qwen2Lm` cached-forward API (crates/syrinx-lm/src/cv2/mod.rs:261-286,
 * cv2/generate.rs:119-163) on top of these entry points.
 *
 * ABI rules
 *   - Every call returns an int status: SX_OK (0) or a negative SX_E_* code. The message
 *     of the last failure on the calling thread is returned by sx_last_error().
 *   - The library owns the model/session handles and all device memory. The caller owns
 *     every host buffer it passes in; host pointers are only read/written during the call.
 *   - A session is not thread-safe (mirrors `&mut self` in the reference). A model may be
 *     shared read-only by several sessions on the same device.
 *   - Plain C types only: no torch, no CUDA types cross this boundary.
 */
#ifndef SYRINX_DUALAR_H
#define SYRINX_DUALAR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------------------- */
#define SX_OK 0
#define SX_E_INVALID (-1)     /* bad argument (null pointer, bad size, bad id) */
#define SX_E_CUDA (-2)        /* a CUDA runtime call failed */
#define SX_E_OOM (-3)         /* device or host allocation failed */
#define SX_E_BLOB (-4)        /* weight blob malformed or inconsistent with the desc */
#define SX_E_STATE (-5)       /* call out of order (e.g. slow_step before prefill) */
#define SX_E_UNSUPPORTED (-6) /* shape / dtype combination not supported */
#define SX_E_RANGE (-7)       /* context or batch exceeds the session's capacity */
#define SX_E_DEVICE (-8)      /* a kernel reported an error status (bounds check) */

/* ---- weight element types (values follow the GGML type ids) -------------------------- */
#define SX_DTYPE_F32 0
#define SX_DTYPE_F16 1
#define SX_DTYPE_Q8_0 8  /* 32-element blocks {f16 d; i8 q[32]}, 34 B */
#define SX_DTYPE_Q4_K 12 /* 256-element super-blocks {f16 d, dmin; u8 scales[12]; u8 qs[128]}, 144 B */
#define SX_DTYPE_BF16 30

/*
 * One autoregressive transformer's shape. Mirrors `TransformerConfig`
 * (crates/syrinx-fish/src/common/config.rs:22-64) plus the attention flags that the
 * reference derives from tensor presence (`AttnShape`, s2/nn.rs:266-274).
 */
typedef struct sx_transformer_desc {
  int32_t dim;               /* residual width */
  int32_t n_layer;           /* decoder layers (0 for "no fast AR") */
  int32_t n_head;            /* query heads */
  int32_t n_local_heads;     /* key/value heads (GQA) */
  int32_t head_dim;          /* per-head width (Qwen3: not dim / n_head) */
  int32_t intermediate_size; /* SwiGLU inner width */
  float norm_eps;            /* RMSNorm epsilon */
  float rope_base;           /* RoPE theta */
  int32_t rope_interleaved;  /* 1: Fish interleaved pairs (2i,2i+1) (s2/nn.rs:154-166);
                                0: HF rotate-half pairs (i, i+hd/2) (cv2/attention.rs:82-88) */
  int32_t qk_norm;           /* per-head QK-RMSNorm before RoPE (s2/nn.rs:325-331) */
  int32_t qkv_bias;          /* wqkv carries a bias (Qwen2 / CosyVoice2) */
  int32_t o_bias;            /* wo carries a bias */
} sx_transformer_desc;

/*
 * Whole dual-AR model. Mirrors `FishConfig` (config.rs:103-119). With fast.n_layer == 0
 * and num_codebooks == 0 the model is a plain decoder LM (the CosyVoice2 `Qwen2Lm` body,
 * cv2/mod.rs:72-86): the "frame" is then a single token id.
 */
typedef struct sx_model_desc {
  sx_transformer_desc slow;
  sx_transformer_desc fast;
  int32_t vocab_size;      /* slow vocab (rows of embeddings.weight and of the head) */
  int32_t num_codebooks;   /* C: codes per frame (0 for a plain LM) */
  int32_t codebook_size;   /* R: residual codebook size (rows of fast_output / fast_embeddings) */
  uint32_t semantic_begin_id;  /* first semantic id (config.rs semantic_begin_id) */
  uint32_t semantic_end_id;    /* last semantic id, inclusive */
  uint32_t stop_token_id;      /* first stop id (<|im_end|>; CosyVoice2: 6561) */
  int32_t num_stop_tokens;     /* stop ids are [stop_token_id, stop_token_id + n) (Fish 1, CV2 3) */
  int32_t tie_word_embeddings; /* head = embeddings.weight (s2/slow_ar.rs:216-221) */
  int32_t head_bias;           /* output.bias present (CosyVoice2 llm_decoder.bias) */
  int32_t scale_codebook_embeddings; /* s2 MCF: x *= 1/sqrt(C+1) on semantic positions
                                        (s2/slow_ar.rs:148-158); s1: 0 */
  int32_t norm_fastlayer_input;      /* s2: fast AR conditioned on the post-norm hidden
                                        (s2/slow_ar.rs:228-244); s1: pre-norm (s1/slow_ar.rs:186-193) */
} sx_model_desc;

typedef struct sx_model sx_model;
typedef struct sx_session sx_session;

/* Thread-local message of the last failed call on this thread ("" if none). */
const char* sx_last_error(void);

/* Library version string, e.g. "syrinx-b200 0.1 sm_100a". */
const char* sx_version(void);

/* ---- weight blobs -------------------------------------------------------------------- *
 * A blob ("SXW1") is a named-tensor container in the reference's weight naming
 * (s2/load.rs:150-310: layers.{l}.attention.wqkv.weight with rows q|k|v, ...). Quantized
 * tensors hold GGML blocks along the last (input) dimension; ndim is 1 or 2, or 3 for f32
 * convolution kernels (the codec's [out, in, K] / [in, out, K]). Layout, little-endian:
 *   char magic[4]="SXW1"; u32 version=1; u32 n_tensors; u32 reserved; u64 data_offset;
 *   n_tensors x { u32 name_len; char name[name_len]; u32 dtype; u32 ndim; u64 shape[ndim];
 *                 u64 offset (from data_offset); u64 nbytes }
 *   data (each tensor 64-byte aligned).
 */

/* Size in bytes of the seeded synthetic blob for `desc` with matrices in `wtype`
 * (SX_DTYPE_Q8_0, SX_DTYPE_Q4_K, SX_DTYPE_F32). Norm gains are 1.0 and biases N(0,0.02)
 * in f32; every other tensor is N(0,0.02) quantized to `wtype`. */
int sx_synth_blob_size(const sx_model_desc* desc, int32_t wtype, size_t* size_out);
/* Write the synthetic blob (host memory, multithreaded). Deterministic in (desc, wtype, seed). */
int sx_synth_blob_write(const sx_model_desc* desc, int32_t wtype, uint64_t seed, void* out,
                        size_t size);

/* ---- model / session ----------------------------------------------------------------- */

/* Upload and repack a blob onto CUDA device `device`. Replaces `S2Pro::load_with_dtype`
 * (s2/mod.rs:119-167) and `Qwen2Lm::load_quantized` (cv2/load.rs:68-122). */
int sx_model_create(const sx_model_desc* desc, const void* blob, size_t blob_size, int32_t device,
                    sx_model** out);
/* Tensor-parallel shard (no reference counterpart: the reference decodes on one device).
 * Rank tp_rank of tp_size (<= 8; one process per GPU) uploads query heads
 * [r*H/tp, (r+1)*H/tp) and kv heads [r*Hkv/tp, ...) of every wqkv, FFN rows
 * [r*F/tp, (r+1)*F/tp) of w1 and w3, and the matching input columns of wo and w2; norms,
 * embeddings and heads are replicated. Q8_0 weights; heads, kv heads and F must divide by
 * tp_size into whole 32-column blocks. Every rank loads the same blob and must then make
 * the same calls in the same order (they exchange residual rows after wo and w2). */
int sx_model_create_tp(const sx_model_desc* desc, const void* blob, size_t blob_size, int32_t device,
                       int32_t tp_rank, int32_t tp_size, sx_model** out);
int sx_model_destroy(sx_model* model);
/* Device bytes held by the model's weights. */
int sx_model_weight_bytes(const sx_model* model, size_t* bytes_out);

/* A decoding session: paged KV cache for up to `max_batch` (<= 8) sequences of `max_ctx`
 * positions each, plus activation buffers. Replaces `KvCache` (s2/nn.rs:223-261;
 * cv2/mod.rs:117-170). sx_session_create keeps K/V in f32, like the reference's CPU
 * cache, so greedy output is token-exact; sx_session_create_ex also accepts
 * SX_DTYPE_BF16 (half the KV bytes; logits within the 2e-2 parity tolerance). */
int sx_session_create(sx_model* model, int32_t max_batch, int32_t max_ctx, sx_session** out);
int sx_session_create_ex(sx_model* model, int32_t max_batch, int32_t max_ctx, int32_t kv_dtype,
                         sx_session** out);
/* Tensor-parallel sessions (no reference counterpart). Each rank writes its session's
 * SX_TP_HANDLE_BYTES-byte handle (a CUDA IPC handle of its exchange region, its GPU's UUID,
 * rank and size), the caller gathers all handles in rank order (e.g. an all-gather over
 * torch.distributed), and every rank passes the whole array to sx_session_tp_connect before
 * its first decode call. Ranks on the same GPU are refused. A peer that does not reach a
 * residual exchange within the session's wait limit (5 s unless sx_session_tp_set_timeout)
 * makes the call return SX_E_DEVICE on every rank of the group: the rank that waited pushes
 * poison words that fail its peers' exchanges too. The session then refuses to decode
 * (SX_E_STATE) until the group reconnects: every rank calls sx_session_tp_disconnect, meets
 * the others (a barrier), and runs handle / gather / connect again, which clears the
 * exchange state; then sx_session_reset and prefill. */
#define SX_TP_HANDLE_BYTES 128
int sx_session_tp_handle(sx_session* s, void* handle_out);
int sx_session_tp_connect(sx_session* s, const void* handles);
/* Unmap the peers' regions (after the group's last decode call, before any rank destroys
 * its session: put a barrier between the two). */
int sx_session_tp_disconnect(sx_session* s);
/* Longest wait of a residual exchange for a peer's row, in ns of the GPU's global timer
 * (default 5 s). Set before the session's first decode loop. No reference counterpart. */
int sx_session_tp_set_timeout(sx_session* s, int64_t timeout_ns);
/* Benchmark surface, no reference counterpart: give the empty sequence `seq` a slow-AR KV
 * cache of `len` positions of seeded values in [-1, 1), as if `len` tokens had been
 * prefilled. A following sx_prefill appends after them and decoding attends over all of
 * them, so long-context decode can be timed without a long prefill. */
int sx_session_fill_kv_synthetic(sx_session* s, int32_t seq, int32_t len, uint64_t seed);
/* Clear every sequence (the reference `reset`, dualar.rs:73). */
int sx_session_reset(sx_session* s);
int sx_session_destroy(sx_session* s);
/* Current cache length of sequence `seq` (== the next token's absolute position). */
int sx_session_len(const sx_session* s, int32_t seq, int32_t* len_out);
/* Enqueue the session's device work on `cuda_stream` (a cudaStream_t of the model's
 * device) instead of its own stream; NULL restores the session stream. Lets a caller
 * order the work with its own streams and time it with its own CUDA events. */
int sx_session_set_stream(sx_session* s, void* cuda_stream);

/* ---- single-sequence path (sequence 0), DualArBackend ---------------------------------- */

/* Prefill the prompt [(1+C) rows x T] row-major (row 0 slow-vocab ids, rows 1..C codes)
 * into an empty session. Writes the last position's raw (unmasked) f32 logits [vocab]
 * and the fast-AR hidden [fast.dim] when the pointers are non-null.
 * Replaces `DualArBackend::prefill` (dualar.rs:79; s2/slow_ar.rs:250-255). */
int sx_prefill(sx_session* s, const uint32_t* prompt, int32_t T, float* logits_out,
               float* hidden_out);

/* One slow step on the previous full frame [1+C] at absolute position `pos`
 * (must equal the cache length). Replaces `DualArBackend::slow_step` (dualar.rs:83;
 * s2/slow_ar.rs:259-271). For a plain LM the frame is [token]. */
int sx_slow_step(sx_session* s, const uint32_t* frame, int32_t pos, float* logits_out,
                 float* hidden_out);

/* Codebook-0 from a semantic id: clamp(tok - semantic_begin, 0, R-1)
 * (s2/fast_ar.rs:105-110). Host-only arithmetic, exported for the FFI crate. */
uint32_t sx_first_code(const sx_model* model, uint32_t semantic_token);

/* Sampling callback used by sx_fast_expand: returns the code drawn from `logits[n]`. */
typedef uint32_t (*sx_sample_fn)(void* user, const float* logits, int32_t n);

/* Fast AR for one frame, conditioned on the hidden left by the last prefill/slow_step.
 * Residual codes 1..C-1 are drawn by `sample` (the driver-owned sampler, dualar.rs:25-29).
 * Writes codes_out[C] (codes_out[0] == first_code). Replaces `DualArBackend::fast_expand`
 * (dualar.rs:92; s2/fast_ar.rs:116-154). */
int sx_fast_expand(sx_session* s, uint32_t first_code, sx_sample_fn sample, void* user,
                   uint32_t* codes_out);

/* Greedy fast AR (argmax, ties to the lowest index) kept on the device: no host round
 * trip per codebook. Equivalent to sx_fast_expand with a top_k=1 sampler. */
int sx_fast_expand_greedy(sx_session* s, uint32_t first_code, uint32_t* codes_out);

/* One greedy frame through the host boundary, the unit of the reference driver loop
 * (dualar.rs:188-219) with a top_k=1 sampler: if `frame_in` is non-null, run
 * slow_step(frame_in) first; then sample the semantic token from the current logits
 * (constraint = semantic range + stop ids, stop masked when mask_stop), expand it with
 * the fast AR and write the full frame [1+C] (semantic, code0..code_{C-1}) to frame_out.
 * Returns SX_OK; *stopped_out = 1 if the semantic token was a stop id. With a frame, the
 * device work is one CUDA graph, captured on the session stream by the first such call
 * (per mask_stop value) and replayed afterwards, with one synchronisation per call. A bad
 * frame (an id or code out of range) returns SX_E_INVALID and leaves the cached length
 * unchanged. */
int sx_frame_step_greedy(sx_session* s, const uint32_t* frame_in, int32_t mask_stop,
                         uint32_t* frame_out, int32_t* stopped_out);

/* Device-resident greedy decode loop (one CUDA graph replay per frame, no host round trip):
 * after sx_prefill, generate up to n_frames frames. frames_out is [n_frames x (1+C)]
 * row-major (semantic, code0..). Stops early on a stop id unless mask_stop. */
int sx_decode_greedy(sx_session* s, int32_t n_frames, int32_t mask_stop, uint32_t* frames_out,
                     int32_t* n_frames_out);

/* ---- host-sampled driver (the reference `drive`, dualar.rs:161-230) ------------------ */
typedef struct sx_sampling_params {
  float temperature;        /* SamplingParams::temperature (sampling.rs:45-61) */
  float top_p;
  int32_t top_k;            /* 0 = unbounded */
  float repetition_penalty;
  int32_t ras_win_size;
  float ras_high_temp;
  float ras_high_top_p;
} sx_sampling_params;

/* The defaults of SamplingParams::default (sampling.rs:63-77). */
void sx_sampling_params_default(sx_sampling_params* p);

/* Run `drive` with the reference sampler (SplitMix64 stream seeded `seed`) on the host:
 * prefill, then per frame sample semantic (constraint + RAS), stop check, fast expand,
 * slow step. codes_out is [C x max_frames] row-major ([num_codebooks, T] like the
 * reference's result, with T = *n_frames_out columns valid at stride max_frames). */
int sx_drive(sx_session* s, const uint32_t* prompt, int32_t T, int32_t max_frames, uint64_t seed,
             const sx_sampling_params* params, uint32_t* codes_out, int32_t* n_frames_out);

/* The sampled frame loop kept on the device (the reference `drive` with `Sampler`,
 * dualar.rs:188-219, sampling.rs:132-268), for sequence 0 after sx_prefill: per frame the
 * semantic draw (constraint, top-p / top-k, temperature, RAS with its second draw), the
 * residual-code draws and the slow step run in one CUDA graph with no host round trip. The
 * SplitMix64 stream seeded `seed` is consumed in the reference order, so the draws equal
 * sx_drive's for the same prompt, seed and parameters (up to an f64 exp ulp landing on a
 * comparison). frames_out is [n_frames][1 + C] (semantic id, codes); *n_frames_out counts
 * the frames before a stop id was drawn. ras_win_size must be <= 64. */
int sx_decode_sample(sx_session* s, int32_t n_frames, uint64_t seed, const sx_sampling_params* params,
                     uint32_t* frames_out, int32_t* n_frames_out);

/* ---- batched path (DualArBackend::*_batch, dualar.rs:105-135; drive_batch 246-364) ---- *
 * Sequences keep their own lengths in the paged cache, so no left padding is needed:
 * sample i's real positions are 0..T_i exactly as in a batch-1 run. */

/* Prefill N prompts (N <= max_batch); prompt i is [(1+C) x T_i] row-major and the prompts
 * are concatenated. logits_out [N x vocab], hidden_out [N x fast.dim] (nullable). */
int sx_prefill_batch(sx_session* s, const uint32_t* prompts, const int32_t* lens, int32_t n,
                     float* logits_out, float* hidden_out);

/* One batched slow step: frames [N x (1+C)]; active[i]==0 skips sample i (its cache does
 * not advance). logits_out [N x vocab], hidden_out [N x fast.dim] (nullable). */
int sx_slow_step_batch(sx_session* s, const uint32_t* frames, const uint8_t* active, int32_t n,
                       float* logits_out, float* hidden_out);

/* Greedy batched fast AR: first_codes[N], active[N]; codes_out [N x C]. */
int sx_fast_expand_batch_greedy(sx_session* s, const uint32_t* first_codes, const uint8_t* active,
                                int32_t n, uint32_t* codes_out);

/* Device-resident greedy decode of N prefilled sequences for n_frames frames each.
 * frames_out [N x n_frames x (1+C)]; n_frames_out[N] frames produced per sequence. */
int sx_decode_greedy_batch(sx_session* s, int32_t n, int32_t n_frames, int32_t mask_stop,
                           uint32_t* frames_out, int32_t* n_frames_out);

/* ---- CosyVoice2 Qwen2 LM path (config-1 shape) ---------------------------------------- */

/* Feed t_new token ids of a plain LM (num_codebooks == 0) through the cached forward and
 * return the last position's logits [vocab] (head bias included). Replaces
 * `Qwen2Lm::step_logits_cached` (cv2/generate.rs:119-123) for token inputs. */
int sx_lm_step_tokens(sx_session* s, const uint32_t* tokens, int32_t t_new, float* logits_out);

/* Feed t_new caller-assembled input embeddings [t_new x slow.dim] (f32, row-major) of
 * sequence 0 through the cached forward at the next positions and return the last
 * position's logits [vocab] (head bias included; nullable). Replaces
 * `Qwen2Lm::step_logits_cached(embeds)` (cv2/generate.rs:119-123), whose step-0 input
 * `build_lm_input` (cv2/generate.rs:92) concatenates rows of several tables (sos / task id,
 * text embed_tokens, speech_embedding). Later tokens may follow through sx_lm_step_tokens
 * or sx_decode_greedy, which embed ids from embeddings.weight (the speech table). */
int sx_lm_step_embeds(sx_session* s, const float* embeds, int32_t t_new, float* logits_out);

/* ---- profiling ------------------------------------------------------------------------ */

/* Enqueue n_launches batch-1 decode GEMVs of one slow-layer matrix kind (0 wqkv,
 * 1 wo, 2 w1|w3 with SwiGLU, 3 w2, 4 w1|w3 alone as a one-token step runs it: partials
 * only, the SwiGLU formed by the next w2 GEMV) on the session stream, cycling through the layers so
 * every launch streams its weights from HBM. No host synchronization: bracket with CUDA
 * events on the session stream to time the kernel alone. Requires a prefilled session. */
int sx_profile_gemv(sx_session* s, int32_t kind, int32_t n_launches);

/* One launch of the persistent decode-stack kernel (the slow stack, or the fast one when
 * `fast`) for sequence 0 at its current position, with %globaltimer stamps in every CTA.
 * Writes phase_us_out[28]: [0] total us, [1] setup, [2] the final residual phase; then for
 * each of the five phases p (wqkv, attention, wo, w1|w3, w2), averaged over the layers,
 * [3 + 4p + i]: i = 0 the phase, 1 the slowest CTA's prologue, 2 the slowest CTA's arrival
 * after the phase start, 3 the grid barrier (last arrival to the next phase's start);
 * [23..27] the attention steps of CTA 0 (merge loads, scaling, QK-norm / RoPE / KV append,
 * the key loop, the write-out). The
 * step's K/V slot is written as a decode step would write it; the cache length does not
 * advance. */
int sx_profile_stack(sx_session* s, int32_t fast, float* phase_us_out);

/* ---- exact dequantization (parity surface) ------------------------------------------- */

/* Dequantize n_blocks GGML blocks of `dtype` (Q8_0 / Q4_K) on the device, bit-exact with
 * ggml's dequantize_row_* and gguf-py; host in / host out. */
int sx_dequantize(int32_t dtype, const void* blocks, int64_t n_blocks, float* out, int32_t device);

/* No reference counterpart (the reference dequantizes on the CPU while loading weights).
 * sx_dequantize without any device allocation: blocks and values are staged through static
 * device scratch sized for SX_DEQUANTIZE_NOALLOC_MAX_BLOCKS blocks (144 KB in, 1 MB out per
 * device) instead of a cudaMalloc/cudaFree per call; same kernel, bit-identical values.
 * n_blocks above the maximum returns SX_E_RANGE. The first call on a device resolves the
 * scratch address (cudaGetSymbolAddress) and should come before any stream capture on that
 * device. Nothing in the scratch has to start at zero. Calls that overlap on one device
 * (several host threads) race on the shared scratch: serialize them. */
#define SX_DEQUANTIZE_NOALLOC_MAX_BLOCKS 1024
int sx_dequantize_noalloc(int32_t dtype, const void* blocks, int64_t n_blocks, float* out, int32_t device);

#ifdef __cplusplus
}
#endif
#endif /* SYRINX_DUALAR_H */
