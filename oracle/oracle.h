/*
 * oracle.h — CPU restatement of the reference's quantized dual-AR decode path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the B200 kernels.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may
 * load it; the product path (syrinx_b200) never links, loads or calls it.
 *
 * It restates, with f32 activations and OpenMP over all host cores:
 *   - GGML Q8_0 / Q4_K block formats (dequantize bit-exact with gguf-py / ggml);
 *   - the Fish dual-AR forward: MCF embed (crates/syrinx-fish/src/s2/slow_ar.rs:101-161,
 *     s1/slow_ar.rs:85-127), pre-norm decoder blocks (s2/slow_ar.rs:166-202), attention
 *     with QK-norm + interleaved RoPE + GQA (s2/nn.rs:284-360), SwiGLU (s2/nn.rs:452-457),
 *     the tied head (s2/slow_ar.rs:207-246), the fast AR (s2/fast_ar.rs:67-154);
 *   - the CosyVoice2 Qwen2 body (crates/syrinx-lm/src/cv2/mod.rs:181-286,
 *     cv2/attention.rs:46-119) through the same code with rotate-half RoPE and biases;
 *   - the driver loop and the seeded sampler (common/dualar.rs:161-230,
 *     common/sampling.rs:19-268).
 * Quantized matmul: mode A (default, what the device computes) = exact dequantized weights x
 * f32 activations; mode B (oc_set_qmode(1), Q8_0 only, for analysis) restates Candle's CPU
 * QMatMul / ggml vec_dot_q8_0_q8_0 (activations quantized to Q8_0 blocks, exact int32
 * block dots, f32 scale products).
 */
#ifndef SYRINX_ORACLE_H
#define SYRINX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#include "../include/syrinx_dualar.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct oc_model oc_model;
typedef struct oc_session oc_session;

const char* oc_last_error(void);
int oc_num_threads(void);
/* OpenMP threads of later calls (a launcher may have set OMP_NUM_THREADS=1). */
void oc_set_num_threads(int n);
/* Quantized matmul numerics for Q8_0 weights: 0 = mode A (default), 1 = mode B. */
void oc_set_qmode(int32_t mode);
int32_t oc_get_qmode(void);
/* y[M][N] = x[M][K] . W^T for Q8_0 blocks W [N][K/32 blocks], in the current mode. */
void oc_linear_q8_0(const float* x, const uint8_t* blocks, int32_t M, int32_t N, int32_t K, float* y);
/* y[M][N] = x[M][K] . W^T for Q4_K blocks W[N][K/256], in the current mode (A or B). */
void oc_linear_q4_k(const float* x, const uint8_t* blocks, int32_t M, int32_t N, int32_t K, float* y);

/* ---- block formats ---- */
void oc_q8_0_quantize(const float* x, int64_t n, uint8_t* blocks);       /* n % 32 == 0 */
void oc_q8_0_dequantize(const uint8_t* blocks, int64_t n_blocks, float* out);
void oc_q4_k_dequantize(const uint8_t* blocks, int64_t n_blocks, float* out);
float oc_f16_to_f32(uint16_t h);
uint16_t oc_f32_to_f16(float f);
uint16_t oc_f32_to_bf16(float f);

/* ---- single ops (golden KATs) ---- */
void oc_rmsnorm(const float* x, const float* w, int32_t rows, int32_t n, float eps, float* y);
void oc_softmax(const float* x, int32_t rows, int32_t n, float* y);
void oc_silu(const float* x, int64_t n, float* y);
/* x [T][n_heads][hd], positions[T]; interleaved=1 Fish pairs, 0 rotate-half. In place. */
void oc_rope(float* x, int32_t T, int32_t n_heads, int32_t hd, const int32_t* positions,
             float theta, int32_t interleaved);
/* y[M][N] = x[M][K] . W[N][K]^T (+ b) with W f32 row-major. */
void oc_linear_f32(const float* x, const float* w, const float* b, int32_t M, int32_t N, int32_t K,
                   float* y);

/* ---- model ---- */
/* The blob must outlive the model (tensors are read in place). */
int oc_model_create(const sx_model_desc* desc, const void* blob, size_t blob_size, oc_model** out);
void oc_model_destroy(oc_model* m);
/* Dequantize rows [r0, r0+n) of a named tensor to f32 (n * cols floats). */
int oc_tensor_rows(const oc_model* m, const char* name, int64_t r0, int64_t n, float* out);
int oc_tensor_shape(const oc_model* m, const char* name, int64_t* rows, int64_t* cols,
                    int32_t* dtype);

/* kv_bf16: round appended K/V to bf16, as the device cache stores them. */
int oc_session_create(oc_model* m, int32_t max_ctx, int32_t kv_bf16, oc_session** out);
void oc_session_destroy(oc_session* s);
void oc_session_reset(oc_session* s);
int32_t oc_session_len(const oc_session* s);

/* Prompt [(1+C) x T] row-major; logits [vocab], hidden [fast.dim or slow.dim] nullable. */
int oc_prefill(oc_session* s, const uint32_t* prompt, int32_t T, float* logits, float* hidden);
/* Frame [1+C] (plain LM: [1]) at pos == cache length. */
int oc_slow_step(oc_session* s, const uint32_t* frame, float* logits, float* hidden);
/* Plain-LM convenience: t_new tokens through the cached forward, last-position logits. */
int oc_lm_step_tokens(oc_session* s, const uint32_t* tokens, int32_t t_new, float* logits);
/* Input embeddings [t_new x slow.dim] through the cached forward, last-position logits
 * (Qwen2Lm::step_logits_cached(embeds), cv2/generate.rs:119-123). */
int oc_lm_step_embeds(oc_session* s, const float* embeds, int32_t t_new, float* logits);
/* Greedy fast AR from `hidden`; codes [C]; fast_logits [(C-1) x R] nullable. */
int oc_fast_expand_greedy(oc_session* s, const float* hidden, uint32_t first_code, uint32_t* codes,
                          float* fast_logits);
uint32_t oc_first_code(const oc_model* m, uint32_t semantic_token);
/* Greedy argmax of raw logits under the semantic constraint (ties -> lowest index).
 * margin_out (nullable): best minus second-best allowed logit. */
uint32_t oc_greedy_semantic(const oc_model* m, const float* logits, int32_t mask_stop,
                            float* margin_out);

/* Greedy drive: prefill then n_frames frames (stop masked if mask_stop).
 * frames_out [n_frames x (1+C)] (semantic, code0..); margins_out [n_frames] nullable
 * (top-2 gap of the semantic argmax); returns frames produced in *n_out. */
int oc_drive_greedy(oc_session* s, const uint32_t* prompt, int32_t T, int32_t n_frames,
                    int32_t mask_stop, uint32_t* frames_out, int32_t* n_out, float* margins_out);

/* The reference `drive` with the seeded Sampler. codes_out [C x max_frames]. */
int oc_drive(oc_session* s, const uint32_t* prompt, int32_t T, int32_t max_frames, uint64_t seed,
             const sx_sampling_params* p, uint32_t* codes_out, int32_t* n_out);

/* The seeded synthetic weights of sx_synth_blob_size / sx_synth_blob_write (the same
 * writer source compiled into this library), so CPU-only callers need not load the product. */
int oc_synth_blob_size(const sx_model_desc* desc, int32_t wtype, size_t* size_out);
int oc_synth_blob_write(const sx_model_desc* desc, int32_t wtype, uint64_t seed, void* out, size_t size);

/* Sampler pieces, for unit tests against the reference's own semantics. */
uint64_t oc_splitmix64_next(uint64_t* state);
void oc_logits_to_probs(const float* logits, int32_t n, float temperature, float top_p,
                        int32_t top_k, float* probs);

#ifdef __cplusplus
}
#endif
#endif
