// model.hpp — device model and decoding session of the B200 dual-AR path.
#pragma once
#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "blob.hpp"
#include "sx_internal.hpp"

struct sx_model {
  sx_model_desc d{};
  int device = 0;
  std::vector<sx::DevLayer> slow, fast;
  sx::DevMat emb, cb_emb, out_w, fast_out, fast_emb;
  float* norm = nullptr;
  float* out_b = nullptr;
  float* fast_norm = nullptr;
  float* inv_slow = nullptr;
  float* inv_fast = nullptr;
  std::vector<void*> allocs;
  size_t weight_bytes = 0;
  // tensor parallelism: this model holds rank tp_rank's shard of tp_size; d holds the
  // per-rank geometry (n_head, n_local_heads, intermediate_size divided by tp_size)
  int tp_rank = 0, tp_size = 1;
  // the persistent decode stack's per-layer records (device arrays; null when a stack has a
  // matrix that is not Q8_0, which then runs the per-kernel chain)
  sx::StackLayer* slow_stack = nullptr;
  sx::StackLayer* fast_stack = nullptr;
};

struct GreedyGraph {
  cudaGraphExec_t exec = nullptr;
  int M = 0;
  int mask_stop = 0;
  int sampled = 0;  // 1: the device-sampled frame (sx_decode_sample)
  int frame_step = 0;  // 1: sx_frame_step_greedy's slow step + front (not a decode-loop frame)
};

struct sx_session {
  sx_model* m = nullptr;
  int max_batch = 0, max_ctx = 0;
  cudaStream_t st = nullptr;      // stream all work is enqueued on
  cudaStream_t own_st = nullptr;  // the session's own stream (st unless a caller set one)
  int pages_per_seq = 0, n_pages = 0;
  int kv_f32 = 1;                // KV element type: 1 f32 (exact), 0 bf16
  size_t kv_elem = 4;            // bytes per KV element
  uint8_t* kv = nullptr;         // slow: per layer [2][n_pages][Hkv][PAGE][hd]
  uint8_t* fkv = nullptr;        // fast: per layer [2][max_batch][Hkv][PAGE][hd]
  size_t kv_layer_elems = 0, fkv_layer_elems = 0;
  int* page_table = nullptr;   // [max_batch][pages_per_seq]
  int* fpage_table = nullptr;  // [max_batch][1]
  // token lists: decode (graph state) and prefill chunks
  int* tok_seq = nullptr;
  int* tok_pos = nullptr;
  int* ptok_seq = nullptr;
  int* ptok_pos = nullptr;
  int* seq_len = nullptr;
  int* done = nullptr;
  int* frame_count = nullptr;
  int* err = nullptr;
  uint32_t* frames = nullptr;  // [max_batch][1+C]
  uint32_t* ring = nullptr;    // [ring_frames][max_batch][1+C]
  int ring_frames = 0;
  uint32_t* prompt = nullptr;  // [(1+C) * max_ctx]
  // activations
  float* h = nullptr;     // [max_batch][dim] decode residual (h_last after prefill)
  float* hp = nullptr;    // [kMaxPrefillTok][dim] prefill residual
  float* fx = nullptr;    // [max_batch][fast dim] fast residual
  float* xqkv = nullptr;  // [kMaxPrefillTok][max qkv]
  float* attn = nullptr;  // [kMaxPrefillTok][max H*hd]
  float* act = nullptr;   // [kMaxPrefillTok][max F]
  float* logits = nullptr;       // [max_batch][vocab]
  float* fast_logits = nullptr;  // [max_batch][R]
  float* hidden = nullptr;       // [max_batch][dim]
  unsigned long long* amax = nullptr;  // [max_batch]
  sx::SampleState* sstate = nullptr;    // device sampler state of sequence 0
  sx_sampling_params* dparams = nullptr;  // device copy of the sampling parameters
  float* q8_part = nullptr;  // Q8_0 GEMV partial sums [tile][k-chunk][token][16]
  size_t q8_part_cap = 0;    // floats
  float* q8_part2 = nullptr;  // one-token w1|w3 partials, read by the w2 GEMV that writes q8_part
  size_t q8_part2_cap = 0;    // floats
  // persistent decode stack scratch: the residual's second buffer, attention split partials,
  // per-chunk sums of squares and the grid barrier counter
  uint8_t* tc_scratch = nullptr;  // tensor-core prefill GEMM: B operands of every k block
  size_t tc_scratch_bytes = 0;
  float* stack_xb = nullptr;
  float* stack_attn = nullptr;
  float* stack_ss = nullptr;
  unsigned long long* stack_bar = nullptr;
  bool stack_enabled = false;  // SYRINX_STACK=1 selects the persistent stack kernel
  // tensor parallelism: the receive region (rx [2][kMaxTp][xb_cap] 8-byte words) peers map
  // through CUDA IPC, and the communicator the residual merges use
  void* tp_region = nullptr;
  size_t tp_region_bytes = 0;
  bool tp_connected = false;
  bool tp_failed = false;  // an exchange timed out or saw a poison word: refuse until reconnect
  std::vector<void*> tp_opened;  // peers' regions opened on this device
  sx::TpComm tp;
  std::vector<int> len;  // host mirror of per-sequence cache lengths
  std::vector<int> synthetic_len;  // positions filled by fill_kv_synthetic (a prefill may follow)
  bool device_len_dirty = false;  // device seq_len advanced by a graph loop
  std::vector<GreedyGraph> graphs;
  std::vector<void*> allocs;
};

namespace sx {
int model_create(const sx_model_desc* desc, const void* blob, size_t size, int device, sx_model** out,
                 int tp_rank = 0, int tp_size = 1);
// tensor-parallel exchange setup (see sx_session_tp_handle / sx_session_tp_connect)
int session_tp_handle(sx_session* s, void* out);
int session_tp_connect(sx_session* s, const void* handles);
int session_tp_disconnect(sx_session* s);
int session_tp_set_timeout(sx_session* s, int64_t timeout_ns);
int fill_kv_synthetic(sx_session* s, int seq, int len, uint64_t seed);
// device-sampled frames of sequence 0 (after prefill): the reference drive loop's draws
int decode_sample(sx_session* s, int n_frames, uint64_t seed, const sx_sampling_params* p, uint32_t* frames_out,
                  int* n_frames_out);
void model_destroy(sx_model* m);
int session_create(sx_model* m, int max_batch, int max_ctx, int kv_dtype, sx_session** out);
void session_destroy(sx_session* s);
int session_reset(sx_session* s);
int sync_lengths(sx_session* s);

// prefill one sequence; leaves its last residual in s->h[seq]
int prefill_seq(sx_session* s, int seq, const uint32_t* prompt, int T);
// prefill one sequence from caller-assembled input embeddings [T][dim] (host f32)
int prefill_seq_embeds(sx_session* s, int seq, const float* embeds, int T);
// one slow step for n sequences (frames on the host, [n][1+C]); seqs[i] owns row i of s->h
int slow_step_seqs(sx_session* s, const int* seqs, const uint32_t* frames, int n);
// head over h rows [0, n): full logits to s->logits (if want_logits) and/or the greedy
// argmax over the semantic constraint into s->amax
int run_head(sx_session* s, int n, bool want_logits, bool want_argmax, bool mask_stop);
// fast-AR prefix hidden of rows [0, n) into s->hidden
int make_hidden(sx_session* s, int n);
// greedy fast AR for rows [0, n) with first codes already in frames[seq][1]
int fast_expand_rows(sx_session* s, int n, const int* seqs, bool sampled = false);
int fast_expand_sampled(sx_session* s, uint32_t first_code, sx_sample_fn fn, void* user,
                        uint32_t* codes_out);
int profile_gemv(sx_session* s, int kind, int n_launches);
int profile_stack(sx_session* s, int fast, float* out);
int decode_greedy(sx_session* s, int n, int n_frames, int mask_stop, uint32_t* frames_out,
                  int* n_frames_out);
int frame_step_greedy(sx_session* s, const uint32_t* frame_in, int mask_stop, uint32_t* frame_out,
                      int* stopped);
}  // namespace sx
