// capi.cpp — the extern "C" boundary declared in include/syrinx_dualar.h.
//
// Every entry point validates its arguments, selects the model's device, converts any
// failure into an SX_E_* status with a thread-local message, and never lets a C++
// exception cross the ABI. The host-sampled driver `sx_drive` is the reference's `drive`
// loop (crates/syrinx-fish/src/common/dualar.rs:161-230) over the device slow/fast steps.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include "blob.hpp"
#include "codec.hpp"
#include "model.hpp"
#include "sampling.hpp"

namespace sx {
namespace {
thread_local std::string g_last_error;
}
void set_error(const std::string& msg) { g_last_error = msg; }
}  // namespace sx

using namespace sx;

#define SX_GUARD(...)                                        \
  try {                                                      \
    __VA_ARGS__                                              \
  } catch (const std::bad_alloc&) {                          \
    set_error("host allocation failed");                     \
    return SX_E_OOM;                                         \
  } catch (const std::exception& e) {                        \
    set_error(std::string("internal error: ") + e.what());   \
    return SX_E_INVALID;                                     \
  } catch (...) {                                            \
    set_error("internal error");                             \
    return SX_E_INVALID;                                     \
  }

namespace {

int use_device(const sx_model* m) {
  if (cudaSetDevice(m->device) != cudaSuccess) {
    set_error("cudaSetDevice failed");
    return SX_E_CUDA;
  }
  return SX_OK;
}

int need_session(const sx_session* s) {
  if (!s) {
    set_error("null session");
    return SX_E_INVALID;
  }
  return use_device(s->m);
}

int outputs_single(sx_session* s, float* logits_out, float* hidden_out) {
  const sx_model_desc& d = s->m->d;
  if (logits_out) {
    int rc = run_head(s, 1, true, false, false);
    if (rc) return rc;
    if (cudaMemcpyAsync(logits_out, s->logits, (size_t)d.vocab_size * 4, cudaMemcpyDeviceToHost, s->st) != cudaSuccess) {
      set_error("logits copy failed");
      return SX_E_CUDA;
    }
  }
  if (hidden_out) {
    int rc = make_hidden(s, 1);
    if (rc) return rc;
    if (cudaMemcpyAsync(hidden_out, s->hidden, (size_t)d.slow.dim * 4, cudaMemcpyDeviceToHost, s->st) != cudaSuccess) {
      set_error("hidden copy failed");
      return SX_E_CUDA;
    }
  }
  cudaError_t e = cudaStreamSynchronize(s->st);
  if (e != cudaSuccess) {
    set_error(std::string("stream sync: ") + cudaGetErrorString(e));
    return SX_E_CUDA;
  }
  return SX_OK;
}

uint32_t first_code_of(const sx_model_desc& d, uint32_t tok) {
  const uint32_t raw = tok >= d.semantic_begin_id ? tok - d.semantic_begin_id : 0u;
  const uint32_t mx = d.codebook_size > 0 ? (uint32_t)d.codebook_size - 1 : 0u;
  return std::min(raw, mx);
}

struct HostSampleCtx {
  Sampler* smp;
};
uint32_t host_sample_cb(void* user, const float* logits, int32_t n) {
  return static_cast<HostSampleCtx*>(user)->smp->sample_codebook(logits, n);
}

}  // namespace

extern "C" {

const char* sx_last_error(void) { return g_last_error.c_str(); }
const char* sx_version(void) { return "syrinx-b200 0.1 sm_100a"; }

int sx_synth_blob_size(const sx_model_desc* desc, int32_t wtype, size_t* size_out) {
  SX_GUARD({
    if (!desc || !size_out) {
      set_error("null argument");
      return SX_E_INVALID;
    }
    std::vector<SynthTensor> ts;
    size_t header, total;
    int rc = synth_layout(*desc, wtype, &ts, &header, &total);
    if (rc) {
      set_error("synthetic blob: unsupported weight type or block alignment");
      return rc;
    }
    *size_out = total;
    return SX_OK;
  })
}

int sx_synth_blob_write(const sx_model_desc* desc, int32_t wtype, uint64_t seed, void* out, size_t size) {
  SX_GUARD({
    if (!desc || !out) {
      set_error("null argument");
      return SX_E_INVALID;
    }
    int rc = synth_write(*desc, wtype, seed, out, size);
    if (rc) set_error("synthetic blob: bad size or unsupported weight type");
    return rc;
  })
}

int sx_model_create(const sx_model_desc* desc, const void* blob, size_t blob_size, int32_t device, sx_model** out) {
  SX_GUARD({ return model_create(desc, blob, blob_size, device, out); })
}

int sx_model_create_tp(const sx_model_desc* desc, const void* blob, size_t blob_size, int32_t device,
                       int32_t tp_rank, int32_t tp_size, sx_model** out) {
  SX_GUARD({ return model_create(desc, blob, blob_size, device, out, tp_rank, tp_size); })
}

int sx_session_tp_handle(sx_session* s, void* handle_out) {
  SX_GUARD({ return session_tp_handle(s, handle_out); })
}

int sx_session_tp_connect(sx_session* s, const void* handles) {
  SX_GUARD({ return session_tp_connect(s, handles); })
}

int sx_session_tp_disconnect(sx_session* s) {
  SX_GUARD({ return session_tp_disconnect(s); })
}

int sx_session_tp_set_timeout(sx_session* s, int64_t timeout_ns) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    return session_tp_set_timeout(s, timeout_ns);
  })
}

int sx_decode_sample(sx_session* s, int32_t n_frames, uint64_t seed, const sx_sampling_params* params,
                     uint32_t* frames_out, int32_t* n_frames_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    return decode_sample(s, n_frames, seed, params, frames_out, n_frames_out);
  })
}

int sx_session_fill_kv_synthetic(sx_session* s, int32_t seq, int32_t len, uint64_t seed) {
  SX_GUARD({ return fill_kv_synthetic(s, seq, len, seed); })
}

int sx_model_destroy(sx_model* model) {
  SX_GUARD({
    model_destroy(model);
    return SX_OK;
  })
}

int sx_model_weight_bytes(const sx_model* model, size_t* bytes_out) {
  if (!model || !bytes_out) {
    set_error("null argument");
    return SX_E_INVALID;
  }
  *bytes_out = model->weight_bytes;
  return SX_OK;
}

int sx_session_create(sx_model* model, int32_t max_batch, int32_t max_ctx, sx_session** out) {
  return sx_session_create_ex(model, max_batch, max_ctx, SX_DTYPE_F32, out);
}

int sx_session_create_ex(sx_model* model, int32_t max_batch, int32_t max_ctx, int32_t kv_dtype,
                         sx_session** out) {
  SX_GUARD({
    if (!model) {
      set_error("null model");
      return SX_E_INVALID;
    }
    int rc = use_device(model);
    if (rc) return rc;
    return session_create(model, max_batch, max_ctx, kv_dtype, out);
  })
}

int sx_session_reset(sx_session* s) {
  SX_GUARD({
    if (!s) {
      set_error("null session");
      return SX_E_INVALID;
    }
    return session_reset(s);
  })
}

int sx_session_destroy(sx_session* s) {
  SX_GUARD({
    session_destroy(s);
    return SX_OK;
  })
}

int sx_session_len(const sx_session* s, int32_t seq, int32_t* len_out) {
  if (!s || !len_out || seq < 0 || seq >= s->max_batch) {
    set_error("bad session / sequence");
    return SX_E_INVALID;
  }
  *len_out = s->len[seq];
  return SX_OK;
}

int sx_session_set_stream(sx_session* s, void* cuda_stream) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    cudaStream_t next = cuda_stream ? (cudaStream_t)cuda_stream : s->own_st;
    if (next != s->st) {
      // order the switch: new work waits for everything already queued on the old stream
      cudaEvent_t ev;
      if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess ||
          cudaEventRecord(ev, s->st) != cudaSuccess || cudaStreamWaitEvent(next, ev, 0) != cudaSuccess) {
        set_error("sx_session_set_stream: stream ordering failed");
        return SX_E_CUDA;
      }
      cudaEventDestroy(ev);
      s->st = next;
    }
    return SX_OK;
  })
}

int sx_profile_gemv(sx_session* s, int32_t kind, int32_t n_launches) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    return profile_gemv(s, kind, n_launches);
  })
}

int sx_profile_stack(sx_session* s, int32_t fast, float* phase_us_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    if (!phase_us_out) {
      set_error("null output");
      return SX_E_INVALID;
    }
    return profile_stack(s, fast, phase_us_out);
  })
}

int sx_prefill(sx_session* s, const uint32_t* prompt, int32_t T, float* logits_out, float* hidden_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    if (!prompt) {
      set_error("null prompt");
      return SX_E_INVALID;
    }
    if (s->len[0] != s->synthetic_len[0]) {
      set_error("prefill on a non-empty session (reset first)");
      return SX_E_STATE;
    }
    rc = prefill_seq(s, 0, prompt, T);
    if (rc) return rc;
    return outputs_single(s, logits_out, hidden_out);
  })
}

int sx_slow_step(sx_session* s, const uint32_t* frame, int32_t pos, float* logits_out, float* hidden_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    if (!frame) {
      set_error("null frame");
      return SX_E_INVALID;
    }
    if (pos != s->len[0]) {
      set_error("slow_step pos must equal the current cache length");
      return SX_E_STATE;
    }
    const int seq0 = 0;
    rc = slow_step_seqs(s, &seq0, frame, 1);
    if (rc) return rc;
    return outputs_single(s, logits_out, hidden_out);
  })
}

uint32_t sx_first_code(const sx_model* model, uint32_t semantic_token) {
  return model ? first_code_of(model->d, semantic_token) : 0u;
}

int sx_fast_expand(sx_session* s, uint32_t first_code, sx_sample_fn sample, void* user, uint32_t* codes_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    if (!sample || !codes_out) {
      set_error("null sampler or output");
      return SX_E_INVALID;
    }
    if (s->m->d.fast.n_layer <= 0) {
      set_error("model has no fast AR");
      return SX_E_STATE;
    }
    if (s->len[0] <= 0) {
      set_error("fast_expand before prefill");
      return SX_E_STATE;
    }
    return fast_expand_sampled(s, first_code, sample, user, codes_out);
  })
}

int sx_fast_expand_greedy(sx_session* s, uint32_t first_code, uint32_t* codes_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    const sx_model_desc& d = s->m->d;
    if (!codes_out) {
      set_error("null output");
      return SX_E_INVALID;
    }
    if (d.fast.n_layer <= 0) {
      set_error("model has no fast AR");
      return SX_E_STATE;
    }
    if (s->len[0] <= 0) {
      set_error("fast_expand before prefill");
      return SX_E_STATE;
    }
    if (first_code >= (uint32_t)d.codebook_size) {
      set_error("first_code out of range");
      return SX_E_INVALID;
    }
    const int zero = 0, pos = s->len[0];
    if (cudaMemcpyAsync(s->tok_seq, &zero, 4, cudaMemcpyHostToDevice, s->st) != cudaSuccess ||
        cudaMemcpyAsync(s->tok_pos, &pos, 4, cudaMemcpyHostToDevice, s->st) != cudaSuccess) {
      set_error("token upload failed");
      return SX_E_CUDA;
    }
    rc = make_hidden(s, 1);
    if (rc) return rc;
    if (cudaMemcpyAsync(s->fx, s->hidden, (size_t)d.slow.dim * 4, cudaMemcpyDeviceToDevice, s->st) != cudaSuccess ||
        cudaMemcpyAsync(s->frames + 1, &first_code, 4, cudaMemcpyHostToDevice, s->st) != cudaSuccess) {
      set_error("fast prefix upload failed");
      return SX_E_CUDA;
    }
    rc = fast_expand_rows(s, 1, nullptr);
    if (rc) return rc;
    if (cudaMemcpyAsync(codes_out, s->frames + 1, (size_t)d.num_codebooks * 4, cudaMemcpyDeviceToHost, s->st) != cudaSuccess ||
        cudaStreamSynchronize(s->st) != cudaSuccess) {
      set_error("codes copy failed");
      return SX_E_CUDA;
    }
    return SX_OK;
  })
}

int sx_frame_step_greedy(sx_session* s, const uint32_t* frame_in, int32_t mask_stop, uint32_t* frame_out,
                         int32_t* stopped_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    if (!frame_out) {
      set_error("null output");
      return SX_E_INVALID;
    }
    int stopped = 0;
    rc = frame_step_greedy(s, frame_in, mask_stop, frame_out, &stopped);
    if (stopped_out) *stopped_out = stopped;
    return rc;
  })
}

int sx_decode_greedy(sx_session* s, int32_t n_frames, int32_t mask_stop, uint32_t* frames_out, int32_t* n_frames_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    int n = 0;
    rc = decode_greedy(s, 1, n_frames, mask_stop, frames_out, &n);
    if (n_frames_out) *n_frames_out = n;
    return rc;
  })
}

void sx_sampling_params_default(sx_sampling_params* p) {
  if (!p) return;
  p->temperature = 1.0f;
  p->top_p = 0.9f;
  p->top_k = 30;
  p->repetition_penalty = 1.1f;
  p->ras_win_size = 10;
  p->ras_high_temp = 1.0f;
  p->ras_high_top_p = 0.9f;
}

int sx_drive(sx_session* s, const uint32_t* prompt, int32_t T, int32_t max_frames, uint64_t seed,
             const sx_sampling_params* params, uint32_t* codes_out, int32_t* n_frames_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    if (!prompt || !params || !n_frames_out || max_frames < 0) {
      set_error("null argument");
      return SX_E_INVALID;
    }
    const sx_model_desc& d = s->m->d;
    const int C = d.num_codebooks, V = d.vocab_size;
    if (C > 0 && !codes_out) {
      set_error("null codes_out");
      return SX_E_INVALID;
    }
    session_reset(s);
    SemanticConstraint con{d.semantic_begin_id, d.semantic_end_id, d.stop_token_id,
                           d.stop_token_id + (uint32_t)d.num_stop_tokens};
    Sampler smp{SplitMix64{seed}, *params};
    HostSampleCtx ctx{&smp};
    std::vector<float> logits(V);
    std::vector<uint32_t> window, frame(std::max(C, 1)), full(1 + C);
    const int ras_win = std::max(params->ras_win_size, 1);
    rc = prefill_seq(s, 0, prompt, T);
    if (rc) return rc;
    rc = outputs_single(s, logits.data(), nullptr);
    if (rc) return rc;
    int pos = T, nf = 0;
    for (;;) {
      if (nf >= max_frames) break;
      const uint32_t sem = smp.sample_semantic(logits.data(), V, window, con);
      if (sem >= con.stop_lo && sem < con.stop_hi) break;
      const uint32_t first = first_code_of(d, sem);
      if (C > 0) {
        rc = fast_expand_sampled(s, first, host_sample_cb, &ctx, frame.data());
        if (rc) return rc;
        for (int c = 0; c < C; c++) codes_out[(size_t)c * max_frames + nf] = frame[c];
      }
      nf++;
      window.push_back(sem);
      if ((int)window.size() > ras_win) window.erase(window.begin());
      if (nf >= max_frames) break;
      if (pos + 1 >= s->max_ctx) break;
      full[0] = sem;
      for (int c = 0; c < C; c++) full[1 + c] = frame[c];
      const int seq0 = 0;
      rc = slow_step_seqs(s, &seq0, full.data(), 1);
      if (rc) return rc;
      rc = outputs_single(s, logits.data(), nullptr);
      if (rc) return rc;
      pos++;
    }
    *n_frames_out = nf;
    return SX_OK;
  })
}

int sx_prefill_batch(sx_session* s, const uint32_t* prompts, const int32_t* lens, int32_t n, float* logits_out,
                     float* hidden_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    const sx_model_desc& d = s->m->d;
    if (!prompts || !lens || n < 1 || n > s->max_batch) {
      set_error("bad batch");
      return SX_E_INVALID;
    }
    session_reset(s);
    size_t off = 0;
    for (int i = 0; i < n; i++) {
      rc = prefill_seq(s, i, prompts + off, lens[i]);
      if (rc) return rc;
      off += (size_t)(1 + d.num_codebooks) * lens[i];
    }
    if (logits_out) {
      rc = run_head(s, n, true, false, false);
      if (rc) return rc;
      cudaMemcpyAsync(logits_out, s->logits, (size_t)n * d.vocab_size * 4, cudaMemcpyDeviceToHost, s->st);
    }
    if (hidden_out) {
      rc = make_hidden(s, n);
      if (rc) return rc;
      cudaMemcpyAsync(hidden_out, s->hidden, (size_t)n * d.slow.dim * 4, cudaMemcpyDeviceToHost, s->st);
    }
    if (cudaStreamSynchronize(s->st) != cudaSuccess) {
      set_error("stream sync failed");
      return SX_E_CUDA;
    }
    return SX_OK;
  })
}

int sx_slow_step_batch(sx_session* s, const uint32_t* frames, const uint8_t* active, int32_t n, float* logits_out,
                       float* hidden_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    const sx_model_desc& d = s->m->d;
    if (!frames || n < 1 || n > s->max_batch) {
      set_error("bad batch");
      return SX_E_INVALID;
    }
    std::vector<int> seqs(n), saved(s->len.begin(), s->len.end());
    for (int i = 0; i < n; i++) seqs[i] = i;
    rc = slow_step_seqs(s, seqs.data(), frames, n);
    if (rc) return rc;
    // inactive samples ran through the batch (inert) but their cache does not advance
    if (active)
      for (int i = 0; i < n; i++)
        if (!active[i]) s->len[i] = saved[i];
    if (logits_out) {
      rc = run_head(s, n, true, false, false);
      if (rc) return rc;
      cudaMemcpyAsync(logits_out, s->logits, (size_t)n * d.vocab_size * 4, cudaMemcpyDeviceToHost, s->st);
    }
    if (hidden_out) {
      rc = make_hidden(s, n);
      if (rc) return rc;
      cudaMemcpyAsync(hidden_out, s->hidden, (size_t)n * d.slow.dim * 4, cudaMemcpyDeviceToHost, s->st);
    }
    if (cudaStreamSynchronize(s->st) != cudaSuccess) {
      set_error("stream sync failed");
      return SX_E_CUDA;
    }
    return SX_OK;
  })
}

int sx_fast_expand_batch_greedy(sx_session* s, const uint32_t* first_codes, const uint8_t* active, int32_t n,
                                uint32_t* codes_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    const sx_model_desc& d = s->m->d;
    const int C = d.num_codebooks, width = 1 + C;
    if (!first_codes || !codes_out || n < 1 || n > s->max_batch || d.fast.n_layer <= 0) {
      set_error("bad batch or no fast AR");
      return SX_E_INVALID;
    }
    std::vector<int> ts(n), tp(n);
    std::vector<uint32_t> fr((size_t)n * width, 0);
    for (int i = 0; i < n; i++) {
      if (s->len[i] <= 0) {
        set_error("fast_expand before prefill");
        return SX_E_STATE;
      }
      if (first_codes[i] >= (uint32_t)d.codebook_size) {
        set_error("first_code out of range");
        return SX_E_INVALID;
      }
      ts[i] = i;
      tp[i] = s->len[i];
      fr[(size_t)i * width + 1] = first_codes[i];
    }
    if (cudaMemcpyAsync(s->tok_seq, ts.data(), n * 4, cudaMemcpyHostToDevice, s->st) != cudaSuccess ||
        cudaMemcpyAsync(s->tok_pos, tp.data(), n * 4, cudaMemcpyHostToDevice, s->st) != cudaSuccess ||
        cudaMemcpyAsync(s->frames, fr.data(), fr.size() * 4, cudaMemcpyHostToDevice, s->st) != cudaSuccess) {
      set_error("upload failed");
      return SX_E_CUDA;
    }
    rc = make_hidden(s, n);
    if (rc) return rc;
    cudaMemcpyAsync(s->fx, s->hidden, (size_t)n * d.slow.dim * 4, cudaMemcpyDeviceToDevice, s->st);
    rc = fast_expand_rows(s, n, nullptr);
    if (rc) return rc;
    if (cudaMemcpyAsync(fr.data(), s->frames, fr.size() * 4, cudaMemcpyDeviceToHost, s->st) != cudaSuccess ||
        cudaStreamSynchronize(s->st) != cudaSuccess) {
      set_error("codes copy failed");
      return SX_E_CUDA;
    }
    for (int i = 0; i < n; i++)
      for (int c = 0; c < C; c++)
        codes_out[(size_t)i * C + c] = (active && !active[i]) ? 0u : fr[(size_t)i * width + 1 + c];
    return SX_OK;
  })
}

int sx_decode_greedy_batch(sx_session* s, int32_t n, int32_t n_frames, int32_t mask_stop, uint32_t* frames_out,
                           int32_t* n_frames_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    return decode_greedy(s, n, n_frames, mask_stop, frames_out, n_frames_out);
  })
}

int sx_lm_step_tokens(sx_session* s, const uint32_t* tokens, int32_t t_new, float* logits_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    if (!tokens || t_new <= 0) {
      set_error("empty token list");
      return SX_E_INVALID;
    }
    if (s->m->d.num_codebooks != 0) {
      set_error("sx_lm_step_tokens needs a plain LM (num_codebooks == 0)");
      return SX_E_UNSUPPORTED;
    }
    if (t_new == 1 && s->len[0] > 0) {
      const int seq0 = 0;
      rc = slow_step_seqs(s, &seq0, tokens, 1);
    } else {
      rc = prefill_seq(s, 0, tokens, t_new);
    }
    if (rc) return rc;
    return outputs_single(s, logits_out, nullptr);
  })
}

int sx_lm_step_embeds(sx_session* s, const float* embeds, int32_t t_new, float* logits_out) {
  SX_GUARD({
    int rc = need_session(s);
    if (rc) return rc;
    if (!embeds || t_new <= 0) {
      set_error("empty embedding input");
      return SX_E_INVALID;
    }
    rc = prefill_seq_embeds(s, 0, embeds, t_new);
    if (rc) return rc;
    return outputs_single(s, logits_out, nullptr);
  })
}

int sx_dequantize(int32_t dtype, const void* blocks, int64_t n_blocks, float* out, int32_t device) {
  SX_GUARD({
    if (!blocks || !out || n_blocks < 0 || (dtype != SX_DTYPE_Q8_0 && dtype != SX_DTYPE_Q4_K)) {
      set_error("sx_dequantize: bad arguments");
      return SX_E_INVALID;
    }
    if (n_blocks == 0) return SX_OK;
    if (cudaSetDevice(device) != cudaSuccess) {
      set_error("cudaSetDevice failed");
      return SX_E_CUDA;
    }
    const size_t bb = dtype == SX_DTYPE_Q8_0 ? 34 : 144, per = dtype == SX_DTYPE_Q8_0 ? 32 : 256;
    uint8_t* db = nullptr;
    float* dout = nullptr;
    int rc = SX_OK;
    if (cudaMalloc((void**)&db, (size_t)n_blocks * bb) != cudaSuccess ||
        cudaMalloc((void**)&dout, (size_t)n_blocks * per * 4) != cudaSuccess) {
      set_error("sx_dequantize: device allocation failed");
      rc = SX_E_OOM;
    } else if (cudaMemcpy(db, blocks, (size_t)n_blocks * bb, cudaMemcpyHostToDevice) != cudaSuccess ||
               dequant_blocks(dtype, db, n_blocks, dout, 0) != cudaSuccess ||
               cudaMemcpy(out, dout, (size_t)n_blocks * per * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
      set_error("sx_dequantize: CUDA failure");
      rc = SX_E_CUDA;
    }
    if (db) cudaFree(db);
    if (dout) cudaFree(dout);
    return rc;
  })
}

int sx_dequantize_noalloc(int32_t dtype, const void* blocks, int64_t n_blocks, float* out, int32_t device) {
  SX_GUARD({ return dequantize_noalloc(dtype, blocks, n_blocks, out, device); })
}

// ---- codec decode (include/syrinx_codec.h) --------------------------------------------

int sx_codec_create(const void* blob, size_t blob_size, int32_t device, sx_codec** out) {
  SX_GUARD({
    if (!blob || !out) {
      set_error("null argument");
      return SX_E_INVALID;
    }
    *out = nullptr;
    std::unique_ptr<sx_codec> c(new sx_codec());
    std::string err;
    const int rc = c->load(blob, blob_size, device, &err);
    if (rc) {
      set_error(err);
      return rc;
    }
    *out = c.release();
    return SX_OK;
  })
}

int sx_codec_destroy(sx_codec* codec) {
  SX_GUARD({
    delete codec;
    return SX_OK;
  })
}

int sx_codec_get_info(const sx_codec* codec, sx_codec_info* out) {
  if (!codec || !out) {
    set_error("null argument");
    return SX_E_INVALID;
  }
  out->hop = codec->hop;
  out->sample_rate = 44100;
  out->num_codebooks = 1 + codec->n_res;
  out->semantic_size = codec->sem_size;
  out->residual_size = codec->res_size;
  out->codebook_dim = codec->cb_dim;
  out->latent_dim = codec->latent;
  out->n_layers = codec->n_layers;
  return SX_OK;
}

static int codec_device(const sx_codec* c) {
  if (cudaSetDevice(c->device) != cudaSuccess) {
    set_error("cudaSetDevice failed");
    return SX_E_CUDA;
  }
  return SX_OK;
}

static int codec_check_shape(const sx_codec* c, int32_t n_codebooks, int32_t n_frames) {
  if (n_codebooks < 1 || n_codebooks > 1 + c->n_res || n_frames < 0) {
    set_error("codec decode: n_codebooks must be 1.." + std::to_string(1 + c->n_res) +
              " and n_frames >= 0");
    return SX_E_INVALID;
  }
  return SX_OK;
}

int sx_codec_reserve(sx_codec* codec, int32_t max_frames) {
  SX_GUARD({
    if (!codec || max_frames < 0) {
      set_error("bad argument");
      return SX_E_INVALID;
    }
    int rc = codec_device(codec);
    if (rc) return rc;
    std::string err;
    rc = codec->reserve(max_frames, &err);
    if (rc) set_error(err);
    return rc;
  })
}

int sx_codec_set_stream(sx_codec* codec, void* cuda_stream) {
  if (!codec) {
    set_error("null codec");
    return SX_E_INVALID;
  }
  codec->stream = static_cast<cudaStream_t>(cuda_stream);
  return SX_OK;
}

int sx_codec_decode(sx_codec* codec, const uint32_t* codes, int32_t n_codebooks, int32_t n_frames,
                    float* wav_out, size_t wav_capacity) {
  SX_GUARD({
    if (!codec || !codes || !wav_out) {
      set_error("null argument");
      return SX_E_INVALID;
    }
    int rc = codec_check_shape(codec, n_codebooks, n_frames);
    if (rc) return rc;
    const size_t n_wav = (size_t)n_frames * (size_t)codec->hop;
    if (wav_capacity < n_wav) {
      set_error("codec decode: wav_out holds " + std::to_string(wav_capacity) + " samples, " +
                std::to_string(n_wav) + " needed");
      return SX_E_RANGE;
    }
    if (n_frames == 0) return SX_OK;
    rc = codec_device(codec);
    if (rc) return rc;
    if ((size_t)n_frames > codec->io_frames) {
      cudaFree(codec->codes_dev);
      cudaFree(codec->wav_dev);
      codec->codes_dev = nullptr, codec->wav_dev = nullptr, codec->io_frames = 0;
      const size_t ncb_max = (size_t)(1 + codec->n_res);
      if (cudaMalloc((void**)&codec->codes_dev, ncb_max * n_frames * sizeof(uint32_t)) != cudaSuccess ||
          cudaMalloc((void**)&codec->wav_dev, n_wav * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        set_error("codec decode: device allocation failed");
        return SX_E_OOM;
      }
      codec->io_frames = (size_t)n_frames;
    }
    cudaStream_t st = codec->stream;
    if (cudaMemcpyAsync(codec->codes_dev, codes, (size_t)n_codebooks * n_frames * sizeof(uint32_t),
                        cudaMemcpyHostToDevice, st) != cudaSuccess) {
      set_error("codec decode: codes upload failed");
      return SX_E_CUDA;
    }
    std::string err;
    rc = codec->decode_device(codec->codes_dev, n_codebooks, n_frames, codec->wav_dev, &err);
    if (rc) {
      set_error(err);
      return rc;
    }
    int flag = 0;
    if (cudaMemcpyAsync(wav_out, codec->wav_dev, n_wav * sizeof(float), cudaMemcpyDeviceToHost, st) !=
            cudaSuccess ||
        cudaMemcpyAsync(&flag, codec->err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess) {
      set_error(std::string("codec decode: ") + cudaGetErrorString(cudaGetLastError()));
      return SX_E_CUDA;
    }
    if (flag != 0) {
      cudaMemset(codec->err, 0, sizeof(int));
      set_error("codec decode: a tensor-core pipeline wait timed out");
      return SX_E_DEVICE;
    }
    return SX_OK;
  })
}

int sx_codec_decode_device(sx_codec* codec, const uint32_t* codes_dev, int32_t n_codebooks,
                           int32_t n_frames, float* wav_dev) {
  SX_GUARD({
    if (!codec || !codes_dev || !wav_dev) {
      set_error("null argument");
      return SX_E_INVALID;
    }
    int rc = codec_check_shape(codec, n_codebooks, n_frames);
    if (rc) return rc;
    rc = codec_device(codec);
    if (rc) return rc;
    std::string err;
    rc = codec->decode_device(codes_dev, n_codebooks, n_frames, wav_dev, &err);
    if (rc) set_error(err);
    return rc;
  })
}

}  // extern "C"
