// model.cu — model upload/repack, sessions, and the decode orchestration on one GPU.
//
// The per-layer kernel sequence (5 launches, all programmatic-dependent):
//   1 gemv  wqkv   prologue RMSNorm(attention_norm), + qkv bias        (s2/nn.rs:309-313)
//   2 attn  QK-norm, RoPE, KV append, split-K GQA softmax(QK^T)V       (s2/nn.rs:315-352)
//   3 gemv  wo     epilogue + bias, residual add                        (s2/slow_ar.rs:195)
//   4 gemv  w1|w3  prologue RMSNorm(ffn_norm), epilogue SiLU(g)*u      (s2/nn.rs:452-456)
//   5 gemv  w2     epilogue residual add                                (s2/slow_ar.rs:198)
// A greedy frame (head -> semantic -> fast AR x C -> MCF embed -> slow stack -> advance)
// is captured once into a CUDA graph and replayed per frame with no host round trip
// (the driver loop of crates/syrinx-fish/src/common/dualar.rs:188-219 with top_k = 1).
#include "model.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <cstdlib>

#include "sx_internal.hpp"

namespace sx {

size_t DevMat::bytes() const {
  switch (dtype) {
    case SX_DTYPE_Q8_0: return (size_t)q8_tiles(rows) * (cols / 32) * kQ8Rec;
    case SX_DTYPE_Q4_K: return (size_t)rows * cols / 2 + (size_t)rows * (cols / 256) * 16;
    case kDtypeQ4KT: return (size_t)q8_tiles(rows) * (cols / 256) * kQ4Rec;
    case SX_DTYPE_F32: return (size_t)rows * cols * 4;
  }
  return 0;
}

namespace {

#define SX_CU(expr)                                                                   \
  do {                                                                                \
    cudaError_t e_ = (expr);                                                          \
    if (e_ != cudaSuccess) {                                                          \
      set_error(std::string(#expr) + ": " + cudaGetErrorString(e_));                  \
      return SX_E_CUDA;                                                               \
    }                                                                                 \
  } while (0)

#define SX_RC(expr)        \
  do {                     \
    int rc_ = (expr);      \
    if (rc_) return rc_;   \
  } while (0)

template <class T>
int dalloc(std::vector<void*>& allocs, T** p, size_t count) {
  *p = nullptr;
  if (count == 0) count = 1;
  cudaError_t e = cudaMalloc((void**)p, count * sizeof(T));
  if (e != cudaSuccess) {
    set_error(std::string("cudaMalloc(") + std::to_string(count * sizeof(T)) + "): " + cudaGetErrorString(e));
    return SX_E_OOM;
  }
  allocs.push_back(*p);
  return SX_OK;
}

int check_tdesc(const sx_transformer_desc& t, const char* what) {
  if (t.dim <= 0 || t.n_layer < 0 || t.n_head <= 0 || t.n_local_heads <= 0 || t.intermediate_size <= 0) {
    set_error(std::string(what) + ": non-positive dimension");
    return SX_E_INVALID;
  }
  if (t.head_dim != 32 && t.head_dim != 64 && t.head_dim != 128) {
    set_error(std::string(what) + ": head_dim must be 32, 64 or 128");
    return SX_E_UNSUPPORTED;
  }
  if (t.n_head % t.n_local_heads || t.n_head / t.n_local_heads > kMaxGroup) {
    set_error(std::string(what) + ": n_head must be a multiple (<= 8x) of n_local_heads");
    return SX_E_UNSUPPORTED;
  }
  if (t.dim % 32 || t.intermediate_size % 32 || (t.n_head * t.head_dim) % 32) {
    set_error(std::string(what) + ": dims must be multiples of 32");
    return SX_E_UNSUPPORTED;
  }
  return SX_OK;
}

struct Loader {
  sx_model* m;
  BlobIndex idx;
  uint8_t* staging = nullptr;
  size_t staging_cap = 0;
  ~Loader() {
    if (staging) cudaFree(staging);
  }

  const BlobTensor* get(const std::string& name, int64_t rows, int64_t cols) {
    auto it = idx.t.find(name);
    if (it == idx.t.end()) {
      set_error("weight blob: missing tensor " + name);
      return nullptr;
    }
    if (it->second.rows != rows || it->second.cols != cols) {
      set_error("weight blob: shape mismatch for " + name + " (expected " + std::to_string(rows) + "x" +
                std::to_string(cols) + ")");
      return nullptr;
    }
    return &it->second;
  }

  int vec(const std::string& name, int64_t n, float** out) {
    const BlobTensor* t = get(name, 1, n);
    if (!t) return SX_E_BLOB;
    if (t->dtype != SX_DTYPE_F32) {
      set_error("weight blob: " + name + " must be f32");
      return SX_E_BLOB;
    }
    SX_RC(dalloc(m->allocs, out, (size_t)n));
    SX_CU(cudaMemcpy(*out, t->data, (size_t)n * 4, cudaMemcpyHostToDevice));
    m->weight_bytes += (size_t)n * 4;
    return SX_OK;
  }

  // A tensor-parallel shard of a blob tensor: the listed row ranges, concatenated, and the
  // element columns [c0, c0 + cols) (cols < 0: all), block-aligned for quantized types.
  struct Slice {
    std::vector<std::pair<int64_t, int64_t>> rows;  // (first row, count)
    int64_t c0 = 0, cols = -1;
  };

  int slice(const BlobTensor& t, const Slice& sl, std::vector<uint8_t>* host, BlobTensor* v) {
    const int64_t per = t.dtype == SX_DTYPE_Q8_0 ? 32 : t.dtype == SX_DTYPE_Q4_K ? 256 : 1;
    const size_t bb = t.dtype == SX_DTYPE_Q8_0 ? 34 : t.dtype == SX_DTYPE_Q4_K ? 144 : 4;
    const int64_t cols = sl.cols < 0 ? t.cols : sl.cols;
    if (sl.c0 % per || cols % per || sl.c0 < 0 || sl.c0 + cols > t.cols) {
      set_error("tensor-parallel shard of " + t.name + " is not aligned to its quantization blocks");
      return SX_E_UNSUPPORTED;
    }
    int64_t nrows = 0;
    for (const auto& r : sl.rows) {
      if (r.first < 0 || r.first + r.second > t.rows) {
        set_error("tensor-parallel shard of " + t.name + " is out of range");
        return SX_E_INVALID;
      }
      nrows += r.second;
    }
    const size_t src_row = row_bytes(t.dtype, t.cols), dst_row = (size_t)(cols / per) * bb;
    const size_t off = (size_t)(sl.c0 / per) * bb;
    host->resize((size_t)nrows * dst_row);
    uint8_t* dst = host->data();
    for (const auto& r : sl.rows)
      for (int64_t i = r.first; i < r.first + r.second; i++, dst += dst_row)
        std::memcpy(dst, t.data + (size_t)i * src_row + off, dst_row);
    *v = t;
    v->rows = nrows;
    v->cols = cols;
    v->data = host->data();
    v->nbytes = host->size();
    return SX_OK;
  }

  int vec_slice(const std::string& name, int64_t n, const Slice& sl, float** out) {
    const BlobTensor* t = get(name, 1, n);
    if (!t) return SX_E_BLOB;
    if (t->dtype != SX_DTYPE_F32) {
      set_error("weight blob: " + name + " must be f32");
      return SX_E_BLOB;
    }
    std::vector<float> v;
    for (const auto& r : sl.rows)
      v.insert(v.end(), (const float*)t->data + r.first, (const float*)t->data + r.first + r.second);
    SX_RC(dalloc(m->allocs, out, v.size()));
    SX_CU(cudaMemcpy(*out, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
    m->weight_bytes += v.size() * 4;
    return SX_OK;
  }

  // Upload `name` [rows x cols] (or its shard `sl`) into dst at destination rows
  // r*row_mul + row_add; dst spans total_rows rows and is allocated on first use.
  // A layer matrix (`tiled`) in Q4_K becomes tile records for the integer tensor-core GEMV.
  int mat(const std::string& name, int64_t rows, int64_t cols, DevMat* dst, int64_t total_rows,
          int row_mul = 1, int row_add = 0, const Slice* sl = nullptr, bool tiled = false) {
    const BlobTensor* full = get(name, rows, cols);
    if (!full) return SX_E_BLOB;
    BlobTensor view = *full;
    std::vector<uint8_t> host;
    if (sl) SX_RC(slice(*full, *sl, &host, &view));
    const BlobTensor* t = &view;
    rows = t->rows;
    cols = t->cols;
    if (t->dtype != SX_DTYPE_Q8_0 && t->dtype != SX_DTYPE_Q4_K && t->dtype != SX_DTYPE_F32) {
      set_error("weight blob: " + name + " has an unsupported dtype (Q8_0, Q4_K or F32)");
      return SX_E_UNSUPPORTED;
    }
    const int dtype = (tiled && t->dtype == SX_DTYPE_Q4_K) ? kDtypeQ4KT : t->dtype;
    if (dst->dtype < 0) {
      dst->dtype = dtype;
      dst->rows = total_rows;
      dst->cols = cols;
      if (dtype == SX_DTYPE_Q8_0 || dtype == kDtypeQ4KT) {
        uint8_t* q;
        SX_RC(dalloc(m->allocs, &q, dst->bytes()));
        SX_CU(cudaMemset(q, 0, dst->bytes()));  // rows past N of the last tile stay zero
        dst->q = q;
      } else if (t->dtype == SX_DTYPE_Q4_K) {
        uint8_t* q;
        SX_RC(dalloc(m->allocs, &q, (size_t)total_rows * cols / 2));
        SX_RC(dalloc(m->allocs, &dst->meta, (size_t)total_rows * (cols / 256) * 16));
        dst->q = q;
      } else {
        float* q;
        SX_RC(dalloc(m->allocs, &q, (size_t)total_rows * cols));
        dst->q = q;
      }
      m->weight_bytes += dst->bytes();
    } else if (dst->dtype != dtype) {
      set_error("weight blob: " + name + " dtype differs from its fused partner");
      return SX_E_BLOB;
    }
    if (t->dtype == SX_DTYPE_F32) {
      SX_CU(cudaMemcpy2D((float*)dst->q + (size_t)row_add * cols, (size_t)row_mul * cols * 4, t->data,
                         (size_t)cols * 4, (size_t)cols * 4, (size_t)rows, cudaMemcpyHostToDevice));
      return SX_OK;
    }
    if (t->nbytes > staging_cap) {
      if (staging) cudaFree(staging);
      staging = nullptr;
      SX_CU(cudaMalloc((void**)&staging, t->nbytes));
      staging_cap = t->nbytes;
    }
    SX_CU(cudaMemcpy(staging, t->data, t->nbytes, cudaMemcpyHostToDevice));
    // Q8_0 interleaves w1/w3 per 16-row tile (8 gate rows, then their 8 up rows)
    if (t->dtype == SX_DTYPE_Q8_0)
      SX_CU(repack_q8_0(staging, rows, cols, (uint8_t*)dst->q, row_mul, row_add, row_mul == 2 ? 8 : 1, 0));
    else if (dtype == kDtypeQ4KT)
      SX_CU(repack_q4k_tiles(staging, rows, cols, (uint8_t*)dst->q, row_mul, row_add, row_mul == 2 ? 8 : 1, 0));
    else
      SX_CU(repack_q4_k(staging, rows, cols, (uint8_t*)dst->q, dst->meta, row_mul, row_add, 0));
    SX_CU(cudaStreamSynchronize(0));
    return SX_OK;
  }

  // One transformer stack in the blob's (global) geometry `td`. Under tensor parallelism
  // rank r keeps query heads [r*H/tp, (r+1)*H/tp) and kv heads [r*Hkv/tp, ...) of wqkv (its
  // q, k and v rows), FFN rows [r*F/tp, (r+1)*F/tp) of w1 and w3, and the matching input
  // columns of wo and w2, whose outputs the residual merge adds up across ranks.
  int layers(const sx_transformer_desc& td, const char* prefix, std::vector<DevLayer>* out) {
    const int tp = m->tp_size, r = m->tp_rank;
    const int64_t hd = td.head_dim, H = td.n_head, Hkv = td.n_local_heads, F = td.intermediate_size;
    const int64_t Hl = H / tp, Hkvl = Hkv / tp, Fl = F / tp;
    const int64_t qkv = (H + 2 * Hkv) * hd, qkv_l = (Hl + 2 * Hkvl) * hd;
    Slice s_qkv, s_wo, s_f, s_w2;
    s_qkv.rows = {{r * Hl * hd, Hl * hd}, {H * hd + r * Hkvl * hd, Hkvl * hd},
                  {(H + Hkv) * hd + r * Hkvl * hd, Hkvl * hd}};
    s_wo.rows = {{0, td.dim}};
    s_wo.c0 = r * Hl * hd;
    s_wo.cols = Hl * hd;
    s_f.rows = {{r * Fl, Fl}};
    s_w2.rows = {{0, td.dim}};
    s_w2.c0 = r * Fl;
    s_w2.cols = Fl;
    const bool sh = tp > 1;
    for (int l = 0; l < td.n_layer; l++) {
      const std::string p = std::string(prefix) + "." + std::to_string(l) + ".";
      DevLayer L;
      SX_RC(vec(p + "attention_norm.weight", td.dim, &L.attn_norm));
      SX_RC(mat(p + "attention.wqkv.weight", qkv, td.dim, &L.wqkv, qkv_l, 1, 0, sh ? &s_qkv : nullptr, true));
      if (td.qkv_bias) {
        if (sh)
          SX_RC(vec_slice(p + "attention.wqkv.bias", qkv, s_qkv, &L.bqkv));
        else
          SX_RC(vec(p + "attention.wqkv.bias", qkv, &L.bqkv));
      }
      if (td.qk_norm) {
        SX_RC(vec(p + "attention.q_norm.weight", td.head_dim, &L.qn));
        SX_RC(vec(p + "attention.k_norm.weight", td.head_dim, &L.kn));
      }
      SX_RC(mat(p + "attention.wo.weight", td.dim, H * hd, &L.wo, td.dim, 1, 0, sh ? &s_wo : nullptr, true));
      if (td.o_bias) SX_RC(vec(p + "attention.wo.bias", td.dim, &L.bo));
      SX_RC(vec(p + "ffn_norm.weight", td.dim, &L.ffn_norm));
      SX_RC(mat(p + "feed_forward.w1.weight", F, td.dim, &L.w13, 2 * Fl, 2, 0, sh ? &s_f : nullptr, true));
      SX_RC(mat(p + "feed_forward.w3.weight", F, td.dim, &L.w13, 2 * Fl, 2, 1, sh ? &s_f : nullptr, true));
      SX_RC(mat(p + "feed_forward.w2.weight", td.dim, F, &L.w2, td.dim, 1, 0, sh ? &s_w2 : nullptr, true));
      out->push_back(L);
    }
    return SX_OK;
  }
};

// RoPE inverse frequencies 1 / base^(2i/hd) evaluated in f32 on the host, as the
// reference tables are (s2/nn.rs:125-127, cv2/attention.rs:110-112).
int upload_inv_freq(sx_model* m, const sx_transformer_desc& td, float** out) {
  std::vector<float> f(td.head_dim / 2);
  for (int i = 0; i < td.head_dim / 2; i++)
    f[i] = 1.0f / std::pow(td.rope_base, (2.0f * (float)i) / (float)td.head_dim);
  SX_RC(dalloc(m->allocs, out, f.size()));
  SX_CU(cudaMemcpy(*out, f.data(), f.size() * 4, cudaMemcpyHostToDevice));
  return SX_OK;
}

// The persistent decode kernel's per-layer records: only for stacks whose four matrices are
// all Q8_0 tile records.
int upload_stack(sx_model* m, const std::vector<DevLayer>& layers, StackLayer** out) {
  *out = nullptr;
  if (layers.empty()) return SX_OK;
  std::vector<StackLayer> h;
  for (const DevLayer& L : layers) {
    for (const DevMat* w : {&L.wqkv, &L.wo, &L.w13, &L.w2})
      if (w->dtype != SX_DTYPE_Q8_0) return SX_OK;
    StackLayer s;
    s.wqkv = (const uint8_t*)L.wqkv.q;
    s.wo = (const uint8_t*)L.wo.q;
    s.w13 = (const uint8_t*)L.w13.q;
    s.w2 = (const uint8_t*)L.w2.q;
    s.attn_norm = L.attn_norm;
    s.bqkv = L.bqkv;
    s.qn = L.qn;
    s.kn = L.kn;
    s.bo = L.bo;
    s.ffn_norm = L.ffn_norm;
    h.push_back(s);
  }
  SX_RC(dalloc(m->allocs, out, h.size()));
  SX_CU(cudaMemcpy(*out, h.data(), h.size() * sizeof(StackLayer), cudaMemcpyHostToDevice));
  return SX_OK;
}

}  // namespace

// A transformer stack divides over tp ranks when its heads, kv heads and FFN rows do, and
// the wo / w2 input-column shards stay whole Q8_0 blocks (Q4_K super-blocks).
int check_tp(const sx_transformer_desc& t, int tp, const char* what) {
  if (t.n_layer <= 0 || tp == 1) return SX_OK;
  if (t.n_head % tp || t.n_local_heads % tp || t.intermediate_size % tp ||
      ((int64_t)t.n_head / tp * t.head_dim) % 32 || (t.intermediate_size / tp) % 32) {
    set_error(std::string(what) + ": heads, kv heads and FFN rows must split evenly over the " +
              "tensor-parallel ranks into shards of whole 32-column blocks");
    return SX_E_UNSUPPORTED;
  }
  return SX_OK;
}

int model_create(const sx_model_desc* desc, const void* blob, size_t size, int device, sx_model** out,
                 int tp_rank, int tp_size) {
  if (!desc || !blob || !out) {
    set_error("sx_model_create: null argument");
    return SX_E_INVALID;
  }
  if (tp_size < 1 || tp_size > kMaxTp || tp_rank < 0 || tp_rank >= tp_size) {
    set_error("sx_model_create_tp: need 1 <= tp_size <= 8 and 0 <= tp_rank < tp_size");
    return SX_E_INVALID;
  }
  const sx_model_desc& d = *desc;
  SX_RC(check_tdesc(d.slow, "slow"));
  if (d.fast.n_layer > 0) {
    SX_RC(check_tdesc(d.fast, "fast"));
    if (d.fast.dim != d.slow.dim) {
      set_error("fast.dim != slow.dim needs fast_project_in, which this build does not load");
      return SX_E_UNSUPPORTED;
    }
    if (d.num_codebooks < 2 || d.codebook_size <= 0) {
      set_error("a fast AR needs num_codebooks >= 2 and codebook_size > 0");
      return SX_E_INVALID;
    }
  }
  if (d.num_codebooks < 0 || d.num_codebooks > 64 || d.vocab_size <= 0 || d.num_stop_tokens < 0 ||
      d.num_stop_tokens > kMaxStops || d.semantic_end_id < d.semantic_begin_id ||
      (int64_t)d.stop_token_id + d.num_stop_tokens > d.vocab_size) {
    set_error("sx_model_desc: bad vocab / codebook / stop configuration");
    return SX_E_INVALID;
  }
  if (d.num_stop_tokens > 4 && !stops_adjacent(d)) {
    // a wide stop set (CosyVoice3: 200 control ids) must continue the semantic range, so the
    // head reads it as one widened row range
    set_error("sx_model_desc: more than 4 stop ids must sit right after (or before) the semantic range");
    return SX_E_UNSUPPORTED;
  }
  SX_RC(check_tp(d.slow, tp_size, "slow"));
  SX_RC(check_tp(d.fast, tp_size, "fast"));
  int ndev = 0;
  SX_CU(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) {
    set_error("sx_model_create: no such CUDA device");
    return SX_E_INVALID;
  }
  SX_CU(cudaSetDevice(device));
  auto m = new sx_model();
  m->d = d;
  m->device = device;
  m->tp_rank = tp_rank;
  m->tp_size = tp_size;
  Loader L{m};
  std::string err;
  int rc = parse_blob(blob, size, &L.idx, &err);
  if (rc) {
    set_error(err);
    delete m;
    return rc;
  }
  auto fail = [&](int r) {
    model_destroy(m);
    return r;
  };
  if ((rc = L.layers(d.slow, "layers", &m->slow))) return fail(rc);
  if ((rc = L.mat("embeddings.weight", d.vocab_size, d.slow.dim, &m->emb, d.vocab_size))) return fail(rc);
  if ((rc = L.vec("norm.weight", d.slow.dim, &m->norm))) return fail(rc);
  if (d.tie_word_embeddings) {
    m->out_w = m->emb;
  } else if ((rc = L.mat("output.weight", d.vocab_size, d.slow.dim, &m->out_w, d.vocab_size))) {
    return fail(rc);
  }
  if (d.head_bias && (rc = L.vec("output.bias", d.vocab_size, &m->out_b))) return fail(rc);
  if (d.num_codebooks > 0) {
    const int64_t n = (int64_t)d.num_codebooks * d.codebook_size;
    if ((rc = L.mat("codebook_embeddings.weight", n, d.slow.dim, &m->cb_emb, n))) return fail(rc);
  }
  if (d.fast.n_layer > 0) {
    if ((rc = L.layers(d.fast, "fast_layers", &m->fast))) return fail(rc);
    if ((rc = L.vec("fast_norm.weight", d.fast.dim, &m->fast_norm))) return fail(rc);
    if ((rc = L.mat("fast_output.weight", d.codebook_size, d.fast.dim, &m->fast_out, d.codebook_size)))
      return fail(rc);
    if ((rc = L.mat("fast_embeddings.weight", d.codebook_size, d.fast.dim, &m->fast_emb, d.codebook_size)))
      return fail(rc);
  }
  if ((rc = upload_inv_freq(m, d.slow, &m->inv_slow))) return fail(rc);
  if (d.fast.n_layer > 0 && (rc = upload_inv_freq(m, d.fast, &m->inv_fast))) return fail(rc);
  if (tp_size == 1) {
    if ((rc = upload_stack(m, m->slow, &m->slow_stack))) return fail(rc);
    if ((rc = upload_stack(m, m->fast, &m->fast_stack))) return fail(rc);
  }
  // every later use sees this rank's geometry
  for (sx_transformer_desc* t : {&m->d.slow, &m->d.fast}) {
    t->n_head /= tp_size;
    t->n_local_heads /= tp_size;
    t->intermediate_size /= tp_size;
  }
  *out = m;
  return SX_OK;
}

void model_destroy(sx_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  for (void* p : m->allocs) cudaFree(p);
  delete m;
}

// ---------------------------------------------------------------------------------------
// sessions
// ---------------------------------------------------------------------------------------
int session_create(sx_model* m, int max_batch, int max_ctx, int kv_dtype, sx_session** out) {
  if (!m || !out || max_batch < 1 || max_batch > kMaxTok || max_ctx < 1) {
    set_error("sx_session_create: max_batch must be 1..8 and max_ctx >= 1");
    return SX_E_INVALID;
  }
  if (kv_dtype != SX_DTYPE_F32 && kv_dtype != SX_DTYPE_BF16) {
    set_error("sx_session_create: kv_dtype must be SX_DTYPE_F32 or SX_DTYPE_BF16");
    return SX_E_UNSUPPORTED;
  }
  SX_CU(cudaSetDevice(m->device));
  const sx_model_desc& d = m->d;
  auto s = new sx_session();
  s->m = m;
  s->max_batch = max_batch;
  s->max_ctx = max_ctx;
  s->kv_f32 = kv_dtype == SX_DTYPE_F32;
  s->kv_elem = s->kv_f32 ? 4 : 2;
  s->len.assign(max_batch, 0);
  s->synthetic_len.assign(max_batch, 0);
  auto fail = [&](int r) {
    session_destroy(s);
    return r;
  };
  if (cudaStreamCreateWithFlags(&s->own_st, cudaStreamNonBlocking) != cudaSuccess) {
    set_error("cudaStreamCreate failed");
    return fail(SX_E_CUDA);
  }
  s->st = s->own_st;
  const auto& sl = d.slow;
  s->pages_per_seq = (max_ctx + kPage - 1) / kPage;
  s->n_pages = max_batch * s->pages_per_seq;
  s->kv_layer_elems = (size_t)2 * s->n_pages * sl.n_local_heads * kPage * sl.head_dim;
  int rc;
  if ((rc = dalloc(s->allocs, &s->kv, s->kv_layer_elems * sl.n_layer * s->kv_elem))) return fail(rc);
  if ((rc = dalloc(s->allocs, &s->page_table, (size_t)s->n_pages))) return fail(rc);
  {
    std::vector<int> pt(s->n_pages);
    for (int i = 0; i < s->n_pages; i++) pt[i] = i;  // sequence b owns pages [b*pps, (b+1)*pps)
    if (cudaMemcpy(s->page_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      return fail(SX_E_CUDA);
  }
  const int C = d.num_codebooks;
  const bool has_fast = d.fast.n_layer > 0;
  if (has_fast) {
    const auto& f = d.fast;
    s->fkv_layer_elems = (size_t)2 * max_batch * f.n_local_heads * kPage * f.head_dim;
    if ((rc = dalloc(s->allocs, &s->fkv, s->fkv_layer_elems * f.n_layer * s->kv_elem))) return fail(rc);
    if ((rc = dalloc(s->allocs, &s->fpage_table, (size_t)max_batch))) return fail(rc);
    std::vector<int> pt(max_batch);
    for (int i = 0; i < max_batch; i++) pt[i] = i;
    if (cudaMemcpy(s->fpage_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      return fail(SX_E_CUDA);
  }
  const int width = 1 + C;
  auto qkv_w = [](const sx_transformer_desc& t) { return (t.n_head + 2 * t.n_local_heads) * t.head_dim; };
  const int max_qkv = std::max(qkv_w(sl), has_fast ? qkv_w(d.fast) : 0);
  const int max_att = std::max(sl.n_head * sl.head_dim, has_fast ? d.fast.n_head * d.fast.head_dim : 0);
  const int max_F = std::max(sl.intermediate_size, has_fast ? d.fast.intermediate_size : 0);
  const int dim = sl.dim;
  s->ring_frames = max_ctx;
  if ((rc = dalloc(s->allocs, &s->tok_seq, kMaxTok)) || (rc = dalloc(s->allocs, &s->tok_pos, kMaxTok)) ||
      (rc = dalloc(s->allocs, &s->ptok_seq, kMaxPrefillTok)) || (rc = dalloc(s->allocs, &s->ptok_pos, kMaxPrefillTok)) ||
      (rc = dalloc(s->allocs, &s->seq_len, max_batch)) || (rc = dalloc(s->allocs, &s->done, max_batch)) ||
      (rc = dalloc(s->allocs, &s->frame_count, max_batch)) || (rc = dalloc(s->allocs, &s->err, 1)) ||
      (rc = dalloc(s->allocs, &s->frames, (size_t)max_batch * width)) ||
      (rc = dalloc(s->allocs, &s->ring, (size_t)s->ring_frames * max_batch * width)) ||
      (rc = dalloc(s->allocs, &s->prompt, (size_t)width * max_ctx)) ||
      (rc = dalloc(s->allocs, &s->h, (size_t)max_batch * dim)) ||
      (rc = dalloc(s->allocs, &s->hp, (size_t)kMaxPrefillTok * dim)) ||
      (rc = dalloc(s->allocs, &s->fx, (size_t)max_batch * dim)) ||
      (rc = dalloc(s->allocs, &s->xqkv, (size_t)kMaxPrefillTok * max_qkv)) ||
      (rc = dalloc(s->allocs, &s->attn, (size_t)kMaxPrefillTok * max_att)) ||
      (rc = dalloc(s->allocs, &s->act, (size_t)kMaxPrefillTok * max_F)) ||
      (rc = dalloc(s->allocs, &s->logits, (size_t)max_batch * d.vocab_size)) ||
      (rc = dalloc(s->allocs, &s->fast_logits, (size_t)max_batch * std::max(1, d.codebook_size))) ||
      (rc = dalloc(s->allocs, &s->hidden, (size_t)max_batch * dim)) ||
      (rc = dalloc(s->allocs, &s->amax, (size_t)max_batch)) || (rc = dalloc(s->allocs, &s->sstate, 1)) ||
      (rc = dalloc(s->allocs, &s->dparams, 1)))
    return fail(rc);
  {
    // partial sums of the largest Q8_0 GEMV at the most tokens one launch takes: a prefill
    // chunk for the layer matrices, a decode batch for the heads
    size_t cap = 0;
    auto need = [&](const DevMat& w, int M) {
      if (w.dtype == SX_DTYPE_Q8_0 || w.dtype == kDtypeQ4KT) cap = std::max(cap, q8_part_floats(w, w.rows, M));
    };
    for (const auto* ls : {&m->slow, &m->fast})
      for (const DevLayer& L : *ls) {
        need(L.wqkv, kMaxPrefillTok);
        need(L.wo, kMaxPrefillTok);
        need(L.w13, kMaxPrefillTok);
        need(L.w2, kMaxPrefillTok);
      }
    for (const DevMat* w : {&m->emb, &m->cb_emb, &m->out_w, &m->fast_out, &m->fast_emb}) need(*w, kMaxTok);
    s->q8_part_cap = cap;
    // the tensor-core prefill GEMM's B operands at the widest K of any layer matrix
    size_t kmax = 0;
    for (const auto* ls : {&m->slow, &m->fast})
      for (const DevLayer& L : *ls)
        for (const DevMat* w : {&L.wqkv, &L.wo, &L.w13, &L.w2}) kmax = std::max(kmax, (size_t)w->cols);
    s->tc_scratch_bytes = gemm_tc_scratch_bytes((int)kmax, kMaxPrefillTok);
    if ((rc = dalloc(s->allocs, &s->tc_scratch, std::max<size_t>(s->tc_scratch_bytes, 16)))) return fail(rc);
    if ((rc = dalloc(s->allocs, &s->q8_part, std::max<size_t>(cap, 1)))) return fail(rc);
    // one-token w1|w3 partials, kept apart from q8_part because the w2 GEMV that reads them
    // writes its own partials there
    size_t cap2 = 0;
    for (const auto* ls : {&m->slow, &m->fast})
      for (const DevLayer& L : *ls)
        if (L.w13.dtype == SX_DTYPE_Q8_0) cap2 = std::max(cap2, q8_part_floats(L.w13, L.w13.rows, 1));
    s->q8_part2_cap = cap2;
    if (cap2 && (rc = dalloc(s->allocs, &s->q8_part2, cap2))) return fail(rc);
  }
  {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, m->device);
    (void)sms;
    size_t attn_floats = stack_attn_part_floats(kMaxTok, sl.n_head, sl.head_dim);
    if (has_fast) attn_floats = std::max(attn_floats, stack_attn_part_floats(kMaxTok, d.fast.n_head, d.fast.head_dim));
    if ((rc = dalloc(s->allocs, &s->stack_xb, (size_t)max_batch * dim)) ||
        (rc = dalloc(s->allocs, &s->stack_attn, attn_floats)) ||
        (rc = dalloc(s->allocs, &s->stack_ss, (size_t)2 * kMaxTok * 64)) || (rc = dalloc(s->allocs, &s->stack_bar, 1)))
      return fail(rc);
    if (cudaMemset(s->stack_bar, 0, 8) != cudaSuccess) return fail(SX_E_CUDA);
    const char* env = getenv("SYRINX_STACK");
    s->stack_enabled = env && env[0] == '1';
  }
  if (m->tp_size > 1) {
    // receive region rx [2][kMaxTp][xb_cap] 8-byte words; peers map it by IPC
    const int xb_cap = kMaxPrefillTok * dim;
    s->tp_region_bytes = (size_t)2 * kMaxTp * xb_cap * 8;
    uint8_t* region = nullptr;
    uint32_t* epochs = nullptr;
    if ((rc = dalloc(s->allocs, &region, s->tp_region_bytes)) || (rc = dalloc(s->allocs, &epochs, (size_t)xb_cap)))
      return fail(rc);
    if (cudaMemset(region, 0, s->tp_region_bytes) != cudaSuccess ||
        cudaMemset(epochs, 0, (size_t)xb_cap * 4) != cudaSuccess)
      return fail(SX_E_CUDA);
    s->tp_region = region;
    s->tp.rank = m->tp_rank;
    s->tp.size = m->tp_size;
    s->tp.xb_cap = xb_cap;
    s->tp.rx[m->tp_rank] = reinterpret_cast<uint64_t*>(region);
    s->tp.slot_epochs = epochs;
    s->tp.err = s->err;
  }
  if (cudaMemset(s->amax, 0, (size_t)max_batch * 8) != cudaSuccess ||
      cudaMemset(s->err, 0, 4) != cudaSuccess || cudaMemset(s->frames, 0, (size_t)max_batch * width * 4) != cudaSuccess)
    return fail(SX_E_CUDA);
  *out = s;
  return SX_OK;
}

void session_destroy(sx_session* s) {
  if (!s) return;
  cudaSetDevice(s->m->device);
  if (s->st) cudaStreamSynchronize(s->st);
  if (s->own_st) cudaStreamSynchronize(s->own_st);
  for (void* p : s->tp_opened) cudaIpcCloseMemHandle(p);
  for (auto& g : s->graphs)
    if (g.exec) cudaGraphExecDestroy(g.exec);
  for (void* p : s->allocs) cudaFree(p);
  if (s->own_st) cudaStreamDestroy(s->own_st);
  delete s;
}

// Handle record: cudaIpcMemHandle_t (64 B) | device UUID (16 B) | rank | size (int32 each).
int session_tp_handle(sx_session* s, void* out) {
  if (!s || !out) {
    set_error("sx_session_tp_handle: null argument");
    return SX_E_INVALID;
  }
  if (s->m->tp_size < 2) {
    set_error("sx_session_tp_handle: the model is not tensor-parallel");
    return SX_E_INVALID;
  }
  if (s->tp_connected) {
    set_error("sx_session_tp_handle: disconnect first (the handle starts a fresh exchange state)");
    return SX_E_STATE;
  }
  SX_CU(cudaSetDevice(s->m->device));
  // A fresh exchange state: receive region, slot epochs and the error flag at zero. Every rank
  // does this before the handle exchange, which no rank passes before all have, so no peer
  // pushes into a region that is still being cleared.
  SX_CU(cudaStreamSynchronize(s->st));
  SX_CU(cudaMemset(s->tp_region, 0, s->tp_region_bytes));
  SX_CU(cudaMemset(s->tp.slot_epochs, 0, (size_t)s->tp.xb_cap * 4));
  SX_CU(cudaMemset(s->err, 0, 4));
  SX_CU(cudaDeviceSynchronize());
  s->tp_failed = false;
  cudaIpcMemHandle_t h;
  SX_CU(cudaIpcGetMemHandle(&h, s->tp_region));
  cudaDeviceProp prop;
  SX_CU(cudaGetDeviceProperties(&prop, s->m->device));
  uint8_t* o = static_cast<uint8_t*>(out);
  std::memset(o, 0, SX_TP_HANDLE_BYTES);
  std::memcpy(o, &h, sizeof(h));
  std::memcpy(o + 64, &prop.uuid, 16);
  const int32_t rs[2] = {s->m->tp_rank, s->m->tp_size};
  std::memcpy(o + 80, rs, 8);
  return SX_OK;
}

int session_tp_connect(sx_session* s, const void* handles) {
  if (!s || !handles) {
    set_error("sx_session_tp_connect: null argument");
    return SX_E_INVALID;
  }
  const int tp = s->m->tp_size, me = s->m->tp_rank;
  if (tp < 2 || s->tp_connected) {
    set_error("sx_session_tp_connect: not a tensor-parallel session, or already connected");
    return SX_E_INVALID;
  }
  const uint8_t* h = static_cast<const uint8_t*>(handles);
  for (int q = 0; q < tp; q++) {
    int32_t rs[2];
    std::memcpy(rs, h + (size_t)q * SX_TP_HANDLE_BYTES + 80, 8);
    if (rs[0] != q || rs[1] != tp) {
      set_error("sx_session_tp_connect: handle " + std::to_string(q) + " is not rank " + std::to_string(q) +
                " of " + std::to_string(tp));
      return SX_E_INVALID;
    }
    for (int p = 0; p < q; p++)
      if (!std::memcmp(h + (size_t)q * SX_TP_HANDLE_BYTES + 64, h + (size_t)p * SX_TP_HANDLE_BYTES + 64, 16)) {
        // ranks that wait on one another must never share a GPU
        set_error("sx_session_tp_connect: ranks " + std::to_string(p) + " and " + std::to_string(q) +
                  " are on the same GPU");
        return SX_E_INVALID;
      }
  }
  SX_CU(cudaSetDevice(s->m->device));
  for (int q = 0; q < tp; q++) {
    if (q == me) continue;
    cudaIpcMemHandle_t ih;
    std::memcpy(&ih, h + (size_t)q * SX_TP_HANDLE_BYTES, sizeof(ih));
    void* p = nullptr;
    SX_CU(cudaIpcOpenMemHandle(&p, ih, cudaIpcMemLazyEnablePeerAccess));
    s->tp_opened.push_back(p);
    s->tp.rx[q] = static_cast<uint64_t*>(p);
  }
  s->tp_connected = true;
  return SX_OK;
}

int session_tp_disconnect(sx_session* s) {
  if (!s) {
    set_error("sx_session_tp_disconnect: null argument");
    return SX_E_INVALID;
  }
  SX_CU(cudaSetDevice(s->m->device));
  SX_CU(cudaStreamSynchronize(s->st));
  for (void* p : s->tp_opened) SX_CU(cudaIpcCloseMemHandle(p));
  s->tp_opened.clear();
  for (int q = 0; q < kMaxTp; q++)
    if (q != s->tp.rank) s->tp.rx[q] = nullptr;
  s->tp_connected = false;
  return SX_OK;
}

int session_tp_set_timeout(sx_session* s, int64_t timeout_ns) {
  if (!s || timeout_ns <= 0) {
    set_error("sx_session_tp_set_timeout: null session or non-positive limit");
    return SX_E_INVALID;
  }
  if (s->m->tp_size < 2) {
    set_error("sx_session_tp_set_timeout: the model is not tensor-parallel");
    return SX_E_INVALID;
  }
  if (!s->graphs.empty()) {
    set_error("sx_session_tp_set_timeout: set the limit before the first decode loop (its graphs hold the limit)");
    return SX_E_STATE;
  }
  s->tp.wait_ns = (uint64_t)timeout_ns;
  return SX_OK;
}

int session_reset(sx_session* s) {
  std::fill(s->len.begin(), s->len.end(), 0);
  std::fill(s->synthetic_len.begin(), s->synthetic_len.end(), 0);
  return SX_OK;
}

namespace {

// Splits of the key axis (a cluster per token and kv head): about 64 keys per CTA of 8
// warps at the session's longest context, i.e. one 8-key chunk per warp whose loads go out
// before the query work; long contexts get up to kMaxCluster CTAs per (token, kv head).
int n_split_for(const sx_session* s, int /*M*/, int /*Hkv*/) {
  return std::max(1, std::min(kMaxCluster, (s->max_ctx + 63) / 64));
}

// Every GEMV gets the session's Q8_0 partial-sum buffer; residual adds of a tensor-parallel
// model (wo, w2: input columns split over the ranks) also get the exchange communicator.
int gemv(GemvArgs a, Epi epi, sx_session* s) {
  if (!a.part) {  // the session's partial buffer unless the caller chose another
    a.part = s->q8_part;
    a.part_cap = s->q8_part_cap;
  }
  a.err = s->err;
  a.tc_scratch = s->tc_scratch;
  a.tc_scratch_bytes = s->tc_scratch_bytes;
  if (epi == EPI_ADD && s->m->tp_size > 1) {
    if (!s->tp_connected) {
      set_error("tensor-parallel session: call sx_session_tp_connect before decoding");
      return SX_E_INVALID;
    }
    if (s->tp_failed) {
      set_error("tensor-parallel session: an earlier residual exchange failed; reconnect the group "
                "(sx_session_tp_disconnect, then handle / connect on every rank) and reset");
      return SX_E_STATE;
    }
    if (a.w.dtype != SX_DTYPE_Q8_0) {
      set_error("tensor parallelism needs Q8_0 weights");
      return SX_E_UNSUPPORTED;
    }
    a.tp = s->tp;
  }
  SX_CU(launch_gemv(a, epi, s->st));
  return SX_OK;
}

int num_sms_of(int device) {
  static int cached[64] = {0};
  if (device >= 0 && device < 64 && cached[device]) return cached[device];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  if (device >= 0 && device < 64) cached[device] = n;
  return n;
}

// The persistent decode kernel for a whole stack (stack.cu), when the stack and the launch
// qualify: Q8_0 matrices, decode (each token appends its own K/V), M <= 8, one GPU.
// Returns 1 when it launched, 0 when the caller should run the per-kernel chain.
bool stack_args(sx_session* s, bool fast, int M, float* resid, const int* tok_seq, const int* tok_pos,
                int const_pos, StackArgs* out) {
  sx_model* m = s->m;
  const StackLayer* layers = fast ? m->fast_stack : m->slow_stack;
  if (!layers || M > kMaxTok || m->tp_size > 1) return false;
  const sx_transformer_desc& td = fast ? m->d.fast : m->d.slow;
  const int sms = num_sms_of(m->device);
  StackArgs a;
  a.layers = layers;
  a.n_layer = td.n_layer;
  a.dim = td.dim;
  a.H = td.n_head;
  a.Hkv = td.n_local_heads;
  a.hd = td.head_dim;
  a.F = td.intermediate_size;
  a.eps = td.norm_eps;
  a.inv_freq = fast ? m->inv_fast : m->inv_slow;
  a.interleaved = td.rope_interleaved;
  a.scale = (float)(1.0 / std::sqrt((double)td.head_dim));
  a.kv = fast ? s->fkv : s->kv;
  a.kv_layer_elems = fast ? s->fkv_layer_elems : s->kv_layer_elems;
  a.kv_f32 = s->kv_f32;
  a.page_table = fast ? s->fpage_table : s->page_table;
  a.pt_stride = fast ? 1 : s->pages_per_seq;
  a.tok_seq = tok_seq;
  a.tok_pos = tok_pos;
  a.const_pos = const_pos;
  a.M = M;
  const int ctx = fast ? std::max(1, m->d.num_codebooks) : s->max_ctx;
  a.n_split = std::max(1, std::min(stack_max_splits(sms, M, a.Hkv), (ctx + 31) / 32));
  a.x = resid;
  a.xb = s->stack_xb;
  auto geo = [](int64_t rows, int64_t cols) {
    StackGeo g;
    g.K = (int)cols;
    g.nb = (int)(cols / 32);
    g.nc = (g.nb + kStackChunkBlocks - 1) / kStackChunkBlocks;
    g.n_vt = (int)q8_tiles(rows);
    return g;
  };
  a.geo[0] = geo((int64_t)(a.H + 2 * a.Hkv) * a.hd, a.dim);
  a.geo[1] = geo(a.dim, (int64_t)a.H * a.hd);
  a.geo[2] = geo((int64_t)2 * a.F, a.dim);
  a.geo[3] = geo(a.dim, a.F);
  a.nc_dim = a.geo[0].nc;
  int mt = 1;
  while (mt < M) mt <<= 1;
  size_t need = 0;
  for (int i = 0; i < 4; i++) need = std::max(need, stack_part_floats(a.geo[i], mt));
  need = (need + 3) & ~(size_t)3;  // keep the second buffer 16-byte aligned
  if (2 * need > s->q8_part_cap || !stack_supported(a, sms)) return false;
  a.part0 = s->q8_part;
  a.part1 = s->q8_part + need;
  a.attn_part = s->stack_attn;
  a.ss = s->stack_ss;
  a.bar = s->stack_bar;
  a.err = s->err;
  if (const char* v = getenv("SYRINX_STACK_INFLIGHT")) a.inflight = atoi(v);  // profiling knob
  if (const char* v = getenv("SYRINX_STACK_L2")) a.l2_ahead = atoi(v);        // profiling knob
  *out = a;
  return true;
}

int try_stack(sx_session* s, bool fast, int M, float* resid, const int* tok_seq, const int* tok_pos, int const_pos,
              bool append) {
  if (!s->stack_enabled || !append) return 0;
  StackArgs a;
  if (!stack_args(s, fast, M, resid, tok_seq, tok_pos, const_pos, &a)) return 0;
  cudaError_t e = launch_stack(a, num_sms_of(s->m->device), s->st);
  if (e != cudaSuccess) {
    set_error(std::string("persistent decode stack: ") + cudaGetErrorString(e));
    return -1;
  }
  return 1;
}

// Decode steps leave the wqkv GEMV's k-chunk partials to the attention kernel, which adds
// them in the merge kernel's order (bit-identical), so the merge launch drops out of every
// layer. SYRINX_QKV_MERGE=1 keeps the separate merge (for measurement).
bool qkv_fold_enabled() {
  static const bool on = [] {
    const char* v = getenv("SYRINX_QKV_MERGE");
    return !(v && v[0] == '1');
  }();
  return on;
}

// k-chunks of the wqkv GEMV when the decode attention can add its partials (0: it cannot)
int qkv_fold_chunks(const DevMat& w, int M, bool append) {
  if (!append || M > kMaxTok || !qkv_fold_enabled()) return 0;
  if (w.dtype != SX_DTYPE_Q8_0 && w.dtype != kDtypeQ4KT) return 0;
  const int nc = (int)((w.cols / 32 + 7) / 8);  // 8 blocks of 32 per k-chunk (gemv_q8.cu)
  return nc <= kQkvChunks ? nc : 0;
}

// One-token steps leave the w1|w3 GEMV's k-chunk partials (in q8_part2) to the w2 GEMV, which
// forms silu(gate) * up from them in the merge kernel's order (bit-identical), so the SwiGLU
// merge launch drops out of every layer. SYRINX_GLU_MERGE=1 keeps the separate merge.
bool glu_fold_enabled() {
  static const bool on = [] {
    const char* v = getenv("SYRINX_GLU_MERGE");
    return !(v && v[0] == '1');
  }();
  return on;
}

// k-chunks of the w1|w3 GEMV when the w2 GEMV can form its input from their partials (0: no)
int glu_fold_chunks(const sx_session* s, const DevLayer& L, int M) {
  if (M != 1 || !glu_fold_enabled() || !s->q8_part2) return 0;
  if (L.w13.dtype != SX_DTYPE_Q8_0 || L.w2.dtype != SX_DTYPE_Q8_0) return 0;
  if (L.w13.rows != 2 * L.w2.cols || L.w2.cols % 32) return 0;
  if (q8_part_floats(L.w13, L.w13.rows, 1) > s->q8_part2_cap) return 0;
  const int nc = (int)((L.w13.cols / 32 + 7) / 8);
  return nc <= kQkvChunks ? nc : 0;
}

// One transformer stack over M tokens. resid [M][dim] is updated in place.
int run_stack(sx_session* s, bool fast, int M, float* resid, const int* tok_seq, const int* tok_pos,
              int const_pos, bool append) {
  const int ts = try_stack(s, fast, M, resid, tok_seq, tok_pos, const_pos, append);
  if (ts < 0) return SX_E_CUDA;
  if (ts > 0) return SX_OK;
  sx_model* m = s->m;
  const sx_transformer_desc& td = fast ? m->d.fast : m->d.slow;
  const std::vector<DevLayer>& layers = fast ? m->fast : m->slow;
  const int qkv_w = (td.n_head + 2 * td.n_local_heads) * td.head_dim;
  const size_t layer_elems = fast ? s->fkv_layer_elems : s->kv_layer_elems;
  const size_t half = layer_elems / 2;
  for (size_t l = 0; l < layers.size(); l++) {
    const DevLayer& L = layers[l];
    GemvArgs g;
    g.w = L.wqkv;
    g.x = resid;
    g.norm_w = L.attn_norm;
    g.eps = td.norm_eps;
    g.bias = L.bqkv;
    g.y = s->xqkv;
    g.ldy = qkv_w;
    g.M = M;
    g.n_range = qkv_w;
    const int fold_nc = qkv_fold_chunks(L.wqkv, M, append);
    SX_RC(gemv(g, fold_nc ? EPI_NONE : EPI_STORE, s));

    AttnArgs a;
    a.qkv = s->xqkv;
    if (fold_nc) {
      a.qkv_part = s->q8_part;
      a.qkv_nc = fold_nc;
      int mt = 1;
      while (mt < M) mt <<= 1;
      a.qkv_mt = mt;
      a.qkv_bias = L.bqkv;
    }
    a.out = s->attn;
    uint8_t* base = (fast ? s->fkv : s->kv) + l * layer_elems * s->kv_elem;
    a.kbase = base;
    a.vbase = base + half * s->kv_elem;
    a.kv_f32 = s->kv_f32;
    a.page_table = fast ? s->fpage_table : s->page_table;
    a.pt_stride = fast ? 1 : s->pages_per_seq;
    a.tok_seq = tok_seq;
    a.tok_pos = tok_pos;
    a.const_pos = const_pos;
    a.qn = L.qn;
    a.kn = L.kn;
    a.eps = td.norm_eps;
    a.inv_freq = fast ? m->inv_fast : m->inv_slow;
    a.interleaved = td.rope_interleaved;
    a.scale = (float)(1.0 / std::sqrt((double)td.head_dim));
    a.H = td.n_head;
    a.Hkv = td.n_local_heads;
    a.hd = td.head_dim;
    a.n_split = fast ? 1 : n_split_for(s, M, td.n_local_heads);
    a.append = append ? 1 : 0;
    a.M = M;
    if (append) {
      SX_CU(launch_attention(a, s->st));
    } else {  // a prompt chunk of one sequence: its K/V first, then the tiled prefill kernel
      SX_CU(launch_kv_append(a, s->st));
      SX_CU(launch_attention_prefill(a, s->st));
    }

    GemvArgs o;
    o.w = L.wo;
    o.x = s->attn;
    o.bias = L.bo;
    o.y = resid;
    o.ldy = td.dim;
    o.M = M;
    o.n_range = td.dim;
    SX_RC(gemv(o, EPI_ADD, s));

    GemvArgs f;
    f.w = L.w13;
    f.x = resid;
    f.norm_w = L.ffn_norm;
    f.eps = td.norm_eps;
    f.y = s->act;
    f.ldy = td.intermediate_size;
    f.M = M;
    f.n_range = 2 * td.intermediate_size;
    const int glu_nc = glu_fold_chunks(s, L, M);
    if (glu_nc) {
      f.part = s->q8_part2;
      f.part_cap = s->q8_part2_cap;
    }
    SX_RC(gemv(f, glu_nc ? EPI_NONE : EPI_SWIGLU, s));

    GemvArgs w2;
    w2.w = L.w2;
    w2.x = s->act;
    w2.y = resid;
    w2.ldy = td.dim;
    w2.M = M;
    w2.n_range = td.dim;
    if (glu_nc) {
      w2.glu_part = s->q8_part2;
      w2.glu_nc = glu_nc;
    }
    SX_RC(gemv(w2, EPI_ADD, s));
  }
  return SX_OK;
}

int upload_tokens(sx_session* s, int* dseq, int* dpos, const std::vector<int>& seq, const std::vector<int>& pos) {
  SX_CU(cudaMemcpyAsync(dseq, seq.data(), seq.size() * 4, cudaMemcpyHostToDevice, s->st));
  SX_CU(cudaMemcpyAsync(dpos, pos.data(), pos.size() * 4, cudaMemcpyHostToDevice, s->st));
  return SX_OK;
}

int check_err(sx_session* s) {
  int e = 0;
  SX_CU(cudaMemcpyAsync(&e, s->err, 4, cudaMemcpyDeviceToHost, s->st));
  SX_CU(cudaStreamSynchronize(s->st));
  if (!e) return SX_OK;
  if (e == 3) {
    // The flag stays raised on the device (later exchanges push poison words instead of
    // values) and the session refuses to decode until the group reconnects.
    s->tp_failed = true;
    set_error("a tensor-parallel peer did not complete a residual exchange in time (or reported a failure)");
    return SX_E_DEVICE;
  }
  SX_CU(cudaMemsetAsync(s->err, 0, 4, s->st));
  SX_CU(cudaStreamSynchronize(s->st));
  if (e == 2) {
    set_error("a kernel's bounded pipeline wait timed out (device error flag)");
    return SX_E_DEVICE;
  }
  set_error("token id or codebook code out of range");
  return SX_E_INVALID;
}

EmbedArgs embed_args(sx_session* s) {
  const sx_model_desc& d = s->m->d;
  EmbedArgs e;
  e.emb = s->m->emb;
  e.cb_emb = s->m->cb_emb;
  e.dim = d.slow.dim;
  e.C = d.num_codebooks;
  e.R = d.codebook_size;
  e.vocab = d.vocab_size;
  e.sem_lo = d.semantic_begin_id;
  e.sem_hi = d.semantic_end_id;
  e.scale_cb = d.scale_codebook_embeddings;
  e.err = s->err;
  return e;
}

}  // namespace

namespace {
// Seeded pseudo-random K/V values in [-1, 1) for positions [0, len) of one sequence, every
// slow layer (SplitMix64 of seed and the element's coordinates).
__global__ void k_fill_kv(uint8_t* kv, size_t layer_elems, int n_layer, int first_page, int Hkv, int hd, int len,
                          int kv_f32, uint64_t seed) {
  const size_t half = layer_elems / 2;
  const size_t per_layer = (size_t)2 * len * Hkv * hd;
  const size_t total = per_layer * n_layer;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    size_t r = i;
    const int d = (int)(r % hd);
    r /= hd;
    const int h = (int)(r % Hkv);
    r /= Hkv;
    const int pos = (int)(r % len);
    r /= len;
    const int which = (int)(r % 2);
    const int l = (int)(r / 2);
    uint64_t z = seed + 0x9E3779B97F4A7C15ull * (i + 1);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    const float v = (float)(z >> 40) * (1.0f / 8388608.0f) - 1.0f;
    const size_t page = (size_t)first_page + pos / kPage;
    const size_t e = (size_t)l * layer_elems + which * half + ((page * Hkv + h) * kPage + pos % kPage) * hd + d;
    if (kv_f32)
      reinterpret_cast<float*>(kv)[e] = v;
    else
      reinterpret_cast<__nv_bfloat16*>(kv)[e] = __float2bfloat16(v);
  }
}
}  // namespace

// Benchmark surface: sequence `seq` (empty) gets a slow-AR KV cache of `len` positions of
// seeded values, as if that many tokens had been prefilled; a following prefill appends to
// it and decoding attends over all of it.
int fill_kv_synthetic(sx_session* s, int seq, int len, uint64_t seed) {
  if (!s || seq < 0 || seq >= s->max_batch || len < 1 || len > s->max_ctx) {
    set_error("sx_session_fill_kv_synthetic: bad sequence or length");
    return SX_E_INVALID;
  }
  if (s->len[seq] != 0) {
    set_error("sx_session_fill_kv_synthetic: the sequence is not empty");
    return SX_E_STATE;
  }
  const auto& sl = s->m->d.slow;
  (void)cudaGetLastError();
  k_fill_kv<<<1184, 256, 0, s->st>>>(s->kv, s->kv_layer_elems, sl.n_layer, seq * s->pages_per_seq, sl.n_local_heads,
                                     sl.head_dim, len, s->kv_f32, seed);
  SX_CU(cudaGetLastError());
  SX_CU(cudaStreamSynchronize(s->st));
  s->len[seq] = len;
  s->synthetic_len[seq] = len;
  return SX_OK;
}

int prefill_seq(sx_session* s, int seq, const uint32_t* prompt, int T) {
  const sx_model_desc& d = s->m->d;
  const int rows = 1 + d.num_codebooks;
  if (T <= 0) {
    set_error("prefill: empty prompt");
    return SX_E_INVALID;
  }
  if (s->len[seq] + T > s->max_ctx) {
    set_error("prefill: prompt exceeds the session's max_ctx");
    return SX_E_RANGE;
  }
  SX_CU(cudaMemcpyAsync(s->prompt, prompt, (size_t)rows * T * 4, cudaMemcpyHostToDevice, s->st));
  const int base = s->len[seq];
  int last_M = 0;
  for (int c0 = 0; c0 < T; c0 += kMaxPrefillTok) {
    const int M = std::min(kMaxPrefillTok, T - c0);
    std::vector<int> ts(M, seq), tp(M);
    for (int i = 0; i < M; i++) tp[i] = base + c0 + i;
    SX_RC(upload_tokens(s, s->ptok_seq, s->ptok_pos, ts, tp));
    EmbedArgs e = embed_args(s);
    e.ids = s->prompt;
    e.T = T;
    e.t0 = c0;
    e.h = s->hp;
    e.M = M;
    SX_CU(launch_embed(e, s->st));
    SX_RC(run_stack(s, false, M, s->hp, s->ptok_seq, s->ptok_pos, 0, false));
    last_M = M;
  }
  SX_CU(cudaMemcpyAsync(s->h + (size_t)seq * d.slow.dim, s->hp + (size_t)(last_M - 1) * d.slow.dim,
                        (size_t)d.slow.dim * 4, cudaMemcpyDeviceToDevice, s->st));
  SX_RC(check_err(s));
  s->len[seq] = base + T;
  return SX_OK;
}

// Prefill from caller-assembled input embeddings [T][dim] (host f32) instead of ids: the
// cached forward of `Qwen2Lm::step_logits_cached(embeds)` (cv2/generate.rs:119-123), whose
// inputs `build_lm_input` (cv2/generate.rs:92) assembles from several tables.
int prefill_seq_embeds(sx_session* s, int seq, const float* embeds, int T) {
  const sx_model_desc& d = s->m->d;
  const int dim = d.slow.dim;
  if (T <= 0) {
    set_error("lm_step_embeds: empty input");
    return SX_E_INVALID;
  }
  if (s->len[seq] + T > s->max_ctx) {
    set_error("lm_step_embeds: input exceeds the session's max_ctx");
    return SX_E_RANGE;
  }
  const int base = s->len[seq];
  int last_M = 0;
  for (int c0 = 0; c0 < T; c0 += kMaxPrefillTok) {
    const int M = std::min(kMaxPrefillTok, T - c0);
    std::vector<int> ts(M, seq), tp(M);
    for (int i = 0; i < M; i++) tp[i] = base + c0 + i;
    SX_RC(upload_tokens(s, s->ptok_seq, s->ptok_pos, ts, tp));
    SX_CU(cudaMemcpyAsync(s->hp, embeds + (size_t)c0 * dim, (size_t)M * dim * 4, cudaMemcpyHostToDevice, s->st));
    SX_RC(run_stack(s, false, M, s->hp, s->ptok_seq, s->ptok_pos, 0, false));
    last_M = M;
  }
  SX_CU(cudaMemcpyAsync(s->h + (size_t)seq * dim, s->hp + (size_t)(last_M - 1) * dim, (size_t)dim * 4,
                        cudaMemcpyDeviceToDevice, s->st));
  SX_RC(check_err(s));
  s->len[seq] = base + T;
  return SX_OK;
}

// The slow step of n tokens (token i = sequence i), enqueued on the session stream: argument
// checks, frame and position upload, MCF embed, the slow stack. Nothing waits for the device
// and the cached lengths do not advance; the caller checks the error flag, then advances them.
int slow_step_enqueue(sx_session* s, const int* seqs, const uint32_t* frames, int n) {
  const sx_model_desc& d = s->m->d;
  const int width = 1 + d.num_codebooks;
  std::vector<int> ts(n), tp(n);
  for (int i = 0; i < n; i++) {
    if (seqs[i] != i) {
      set_error("slow_step: token i must be sequence i");
      return SX_E_INVALID;
    }
    if (s->len[i] <= 0) {
      set_error("slow_step before prefill");
      return SX_E_STATE;
    }
    if (s->len[i] + 1 > s->max_ctx) {
      set_error("slow_step: context exceeds the session's max_ctx");
      return SX_E_RANGE;
    }
    ts[i] = i;
    tp[i] = s->len[i];
  }
  SX_CU(cudaMemcpyAsync(s->frames, frames, (size_t)n * width * 4, cudaMemcpyHostToDevice, s->st));
  SX_RC(upload_tokens(s, s->tok_seq, s->tok_pos, ts, tp));
  EmbedArgs e = embed_args(s);
  e.tok_seq = s->tok_seq;
  e.frames = s->frames;
  e.frame_stride = width;
  e.h = s->h;
  e.M = n;
  SX_CU(launch_embed(e, s->st));
  return run_stack(s, false, n, s->h, s->tok_seq, s->tok_pos, 0, true);
}

int slow_step_seqs(sx_session* s, const int* seqs, const uint32_t* frames, int n) {
  SX_RC(slow_step_enqueue(s, seqs, frames, n));
  SX_RC(check_err(s));
  for (int i = 0; i < n; i++) s->len[i] += 1;
  return SX_OK;
}

// Rows the greedy / sampled head reads: the semantic range, plus the stop ids unless masked.
// Stop ids adjacent to the range widen it; others (at most 4) are extra rows.
void head_rows(const sx_model_desc& d, bool mask_stop, GemvArgs* g) {
  const uint32_t sem_hi = std::min<uint32_t>(d.semantic_end_id, (uint32_t)d.vocab_size - 1);
  uint32_t lo = d.semantic_begin_id, hi = sem_hi + 1;
  g->n_extra = 0;
  if (!mask_stop && d.num_stop_tokens > 0) {
    const uint32_t t0 = d.stop_token_id, t1 = d.stop_token_id + (uint32_t)d.num_stop_tokens;
    if (stops_adjacent(d)) {
      lo = std::min(lo, t0);
      hi = std::max(hi, t1);
    } else {
      for (uint32_t id = t0; id < t1; id++)
        if ((id < lo || id >= hi) && id < (uint32_t)d.vocab_size) g->extra[g->n_extra++] = (int)id;
    }
  }
  g->row_base = (int)lo;
  g->n_range = (int)(hi - lo);
}

int run_head(sx_session* s, int n, bool want_logits, bool want_argmax, bool mask_stop) {
  sx_model* m = s->m;
  const sx_model_desc& d = m->d;
  GemvArgs g;
  g.w = m->out_w;
  g.x = s->h;
  g.norm_w = m->norm;
  g.eps = d.slow.norm_eps;
  g.bias = m->out_b;
  g.M = n;
  const uint32_t sem_hi = std::min<uint32_t>(d.semantic_end_id, (uint32_t)d.vocab_size - 1);
  if (want_logits) {
    g.y = s->logits;
    g.ldy = d.vocab_size;
    g.n_range = d.vocab_size;
  } else {
    head_rows(d, mask_stop, &g);
  }
  if (want_argmax) {
    g.amax = s->amax;
    g.allow_lo = d.semantic_begin_id;
    g.allow_hi = sem_hi;
    if (!mask_stop) {
      g.stop_lo = d.stop_token_id;
      g.stop_hi = d.stop_token_id + d.num_stop_tokens;
    }
    return gemv(g, EPI_ARGMAX, s);
  }
  return gemv(g, EPI_STORE, s);
}

int make_hidden(sx_session* s, int n) {
  const sx_model_desc& d = s->m->d;
  if (d.norm_fastlayer_input)
    SX_CU(launch_final_norm(s->h, s->m->norm, d.slow.norm_eps, d.slow.dim, n, s->hidden, s->st));
  else
    SX_CU(cudaMemcpyAsync(s->hidden, s->h, (size_t)n * d.slow.dim * 4, cudaMemcpyDeviceToDevice, s->st));
  return SX_OK;
}

namespace {

FrameArgs frame_args(sx_session* s, int n) {
  const sx_model_desc& d = s->m->d;
  FrameArgs f;
  f.M = n;
  f.tok_seq = s->tok_seq;
  f.frames = s->frames;
  f.frame_stride = 1 + d.num_codebooks;
  f.sem_begin = d.semantic_begin_id;
  f.R = std::max(1, d.codebook_size);
  f.dim = d.slow.dim;
  return f;
}

int fast_head(sx_session* s, int n, Epi epi) {
  sx_model* m = s->m;
  GemvArgs g;
  g.w = m->fast_out;
  g.x = s->fx;
  g.norm_w = m->fast_norm;
  g.eps = m->d.fast.norm_eps;
  g.M = n;
  g.n_range = m->d.codebook_size;
  if (epi == EPI_ARGMAX) {
    g.amax = s->amax;
    g.allow_lo = 0;
    g.allow_hi = (uint32_t)m->d.codebook_size - 1;
  } else {
    g.y = s->fast_logits;
    g.ldy = m->d.codebook_size;
  }
  return gemv(g, epi, s);
}

}  // namespace

namespace {
// Draw arguments of the device sampler over rows [0, R) of the fast head's logits.
SampleArgs codebook_sample_args(sx_session* s) {
  const sx_model_desc& d = s->m->d;
  SampleArgs a;
  a.logits = s->fast_logits;
  a.ranges = 1;
  a.lo[0] = 0;
  a.hi[0] = (uint32_t)d.codebook_size;
  a.params = s->dparams;
  a.full_last = (uint32_t)d.codebook_size - 1;
  a.st = s->sstate;
  a.amax = s->amax;
  return a;
}
}  // namespace

int fast_expand_rows(sx_session* s, int n, const int* /*seqs*/, bool sampled) {
  sx_model* m = s->m;
  const int C = m->d.num_codebooks;
  SX_RC(run_stack(s, true, n, s->fx, s->tok_seq, nullptr, 0, true));
  FrameArgs f = frame_args(s, n);
  f.slot = 1;
  f.emb = m->fast_emb;
  f.x = s->fx;
  SX_CU(launch_take_code(f, s->st));
  for (int cb = 1; cb < C; cb++) {
    SX_RC(run_stack(s, true, n, s->fx, s->tok_seq, nullptr, cb, true));
    if (sampled) {
      SX_RC(fast_head(s, n, EPI_STORE));
      SX_CU(launch_sample(codebook_sample_args(s), s->st));
    } else {
      SX_RC(fast_head(s, n, EPI_ARGMAX));
    }
    FrameArgs t = frame_args(s, n);
    t.amax = s->amax;
    t.slot = 1 + cb;
    if (cb < C - 1) {
      t.emb = m->fast_emb;
      t.x = s->fx;
    }
    SX_CU(launch_take_code(t, s->st));
  }
  return SX_OK;
}

int fast_expand_sampled(sx_session* s, uint32_t first_code, sx_sample_fn fn, void* user, uint32_t* codes_out) {
  sx_model* m = s->m;
  const sx_model_desc& d = m->d;
  const int C = d.num_codebooks, R = d.codebook_size;
  if (first_code >= (uint32_t)R) {
    set_error("fast_expand: first_code out of range");
    return SX_E_INVALID;
  }
  const std::vector<int> ts{0}, tp{s->len[0]};
  SX_RC(upload_tokens(s, s->tok_seq, s->tok_pos, ts, tp));
  SX_RC(make_hidden(s, 1));
  SX_CU(cudaMemcpyAsync(s->fx, s->hidden, (size_t)d.slow.dim * 4, cudaMemcpyDeviceToDevice, s->st));
  SX_CU(cudaMemcpyAsync(s->frames + 1, &first_code, 4, cudaMemcpyHostToDevice, s->st));
  SX_RC(run_stack(s, true, 1, s->fx, s->tok_seq, nullptr, 0, true));
  FrameArgs f = frame_args(s, 1);
  f.slot = 1;
  f.emb = m->fast_emb;
  f.x = s->fx;
  SX_CU(launch_take_code(f, s->st));
  codes_out[0] = first_code;
  std::vector<float> logits(R);
  for (int cb = 1; cb < C; cb++) {
    SX_RC(run_stack(s, true, 1, s->fx, s->tok_seq, nullptr, cb, true));
    SX_RC(fast_head(s, 1, EPI_STORE));
    SX_CU(cudaMemcpyAsync(logits.data(), s->fast_logits, (size_t)R * 4, cudaMemcpyDeviceToHost, s->st));
    SX_CU(cudaStreamSynchronize(s->st));
    const uint32_t code = fn(user, logits.data(), R);
    if (code >= (uint32_t)R) {
      set_error("fast_expand: sampler returned an out-of-range code");
      return SX_E_INVALID;
    }
    codes_out[cb] = code;
    if (cb < C - 1) {
      SX_CU(cudaMemcpyAsync(s->frames + 1 + cb, &codes_out[cb], 4, cudaMemcpyHostToDevice, s->st));
      FrameArgs t = frame_args(s, 1);
      t.slot = 1 + cb;
      t.emb = m->fast_emb;
      t.x = s->fx;
      SX_CU(launch_take_code(t, s->st));
    }
  }
  SX_CU(cudaStreamSynchronize(s->st));
  return SX_OK;
}

namespace {

// The semantic constraint's allowed ids (sampling.rs:84-106) as ascending disjoint ranges:
// the semantic range [begin, end] and the stop ids.
bool semantic_sample_args(sx_session* s, SampleArgs* a) {
  const sx_model_desc& d = s->m->d;
  const uint32_t sem_hi = std::min<uint32_t>(d.semantic_end_id, (uint32_t)d.vocab_size - 1);
  const uint32_t s0 = d.semantic_begin_id, s1 = sem_hi + 1;
  const uint32_t t0 = d.stop_token_id, t1 = d.stop_token_id + (uint32_t)d.num_stop_tokens;
  a->logits = s->logits;
  a->ranges = 1;
  a->lo[0] = s0;
  a->hi[0] = s1;
  if (t1 > t0 && !(t0 >= s0 && t1 <= s1)) {
    if (t1 <= s0) {
      a->ranges = 2, a->lo[0] = t0, a->hi[0] = t1, a->lo[1] = s0, a->hi[1] = s1;
    } else if (t0 >= s1 && t1 <= (uint32_t)d.vocab_size) {
      a->ranges = 2, a->lo[1] = t0, a->hi[1] = t1;
    } else {
      return false;  // stop ids straddle the semantic range
    }
  }
  a->params = s->dparams;
  a->semantic = 1;
  a->sem_lo = s0;
  a->sem_hi = sem_hi;
  a->stop_lo = t0;
  a->stop_hi = t1;
  a->full_last = (uint32_t)d.vocab_size - 1;
  a->st = s->sstate;
  a->amax = s->amax;
  return true;
}

// head -> semantic -> (fast AR) for rows [0, n): leaves the frame in s->frames. Sampled
// (one sequence): the head stores the allowed rows' logits and the device sampler draws.
int greedy_frame_front(sx_session* s, int n, int mask_stop, bool sampled) {
  sx_model* m = s->m;
  const sx_model_desc& d = m->d;
  if (sampled) {
    SampleArgs sa;
    if (!semantic_sample_args(s, &sa)) {
      set_error("decode_sample: stop ids straddle the semantic range");
      return SX_E_UNSUPPORTED;
    }
    GemvArgs g;
    g.w = m->out_w;
    g.x = s->h;
    g.norm_w = m->norm;
    g.eps = d.slow.norm_eps;
    g.bias = m->out_b;
    g.M = 1;
    g.y = s->logits;
    g.ldy = d.vocab_size;
    head_rows(d, false, &g);
    SX_RC(gemv(g, EPI_STORE, s));
    SX_CU(launch_sample(sa, s->st));
  } else {
    SX_RC(run_head(s, n, false, true, mask_stop != 0));
  }
  FrameArgs f = frame_args(s, n);
  f.amax = s->amax;
  f.slot = 0;
  f.write_first_code = d.num_codebooks > 0;
  f.done = s->done;
  f.stop_lo = d.stop_token_id;
  f.stop_hi = d.stop_token_id + d.num_stop_tokens;
  if (d.fast.n_layer > 0) {
    f.x = s->fx;
    f.h_last = s->h;
    f.norm_w = d.norm_fastlayer_input ? m->norm : nullptr;
    f.eps = d.slow.norm_eps;
  }
  SX_CU(launch_take_semantic(f, s->st));
  if (d.fast.n_layer > 0) SX_RC(fast_expand_rows(s, n, nullptr, sampled));
  return SX_OK;
}

// Captures what body() enqueues on the session stream into an executable graph.
template <class F>
int capture_graph(sx_session* s, F&& body, cudaGraphExec_t* exec) {
  SX_CU(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
  int rc = body();
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(s->st, &graph);
  if (rc) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) {
    set_error(std::string("graph capture: ") + cudaGetErrorString(e));
    return SX_E_CUDA;
  }
  e = cudaGraphInstantiateWithFlags(exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    set_error(std::string("graph instantiate: ") + cudaGetErrorString(e));
    return SX_E_CUDA;
  }
  return SX_OK;
}

// sx_frame_step_greedy's frame: the slow step of the frame in s->frames at the position in
// s->tok_pos (MCF embed, slow stack), then the greedy front (head, first code, fast AR).
int build_frame_step_graph(sx_session* s, int mask_stop, cudaGraphExec_t* exec) {
  const int width = 1 + s->m->d.num_codebooks;
  return capture_graph(
      s,
      [&]() -> int {
        EmbedArgs e = embed_args(s);
        e.tok_seq = s->tok_seq;
        e.frames = s->frames;
        e.frame_stride = width;
        e.h = s->h;
        e.M = 1;
        SX_CU(launch_embed(e, s->st));
        SX_RC(run_stack(s, false, 1, s->h, s->tok_seq, s->tok_pos, 0, true));
        return greedy_frame_front(s, 1, mask_stop, false);
      },
      exec);
}

int build_graph(sx_session* s, int n, int mask_stop, bool sampled, cudaGraphExec_t* exec) {
  const sx_model_desc& d = s->m->d;
  const int width = 1 + d.num_codebooks;
  SX_CU(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
  auto body = [&]() -> int {
    SX_RC(greedy_frame_front(s, n, mask_stop, sampled));
    EmbedArgs e = embed_args(s);
    e.tok_seq = s->tok_seq;
    e.frames = s->frames;
    e.frame_stride = width;
    e.h = s->h;
    e.M = n;
    SX_CU(launch_embed(e, s->st));
    SX_RC(run_stack(s, false, n, s->h, s->tok_seq, s->tok_pos, 0, true));
    AdvanceArgs a;
    a.M = n;
    a.tok_seq = s->tok_seq;
    a.tok_pos = s->tok_pos;
    a.seq_len = s->seq_len;
    a.done = s->done;
    a.frames = s->frames;
    a.frame_stride = width;
    a.ring = s->ring;
    a.ring_frames = s->ring_frames;
    a.frame_count = s->frame_count;
    a.batch = s->max_batch;
    SX_CU(launch_advance(a, s->st));
    return SX_OK;
  };
  int rc = body();
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(s->st, &graph);
  if (rc) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) {
    set_error(std::string("graph capture: ") + cudaGetErrorString(e));
    return SX_E_CUDA;
  }
  e = cudaGraphInstantiateWithFlags(exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    set_error(std::string("graph instantiate: ") + cudaGetErrorString(e));
    return SX_E_CUDA;
  }
  return SX_OK;
}

}  // namespace

namespace {
int run_frames(sx_session* s, int n, int n_frames, int mask_stop, bool sampled, uint32_t* frames_out,
               int* n_frames_out);
}  // namespace

int decode_greedy(sx_session* s, int n, int n_frames, int mask_stop, uint32_t* frames_out, int* n_frames_out) {
  return run_frames(s, n, n_frames, mask_stop, false, frames_out, n_frames_out);
}

int decode_sample(sx_session* s, int n_frames, uint64_t seed, const sx_sampling_params* p, uint32_t* frames_out,
                  int* n_frames_out) {
  if (!p || p->ras_win_size > kMaxRasWin) {
    set_error("decode_sample: null parameters or ras_win_size above 64");
    return SX_E_INVALID;
  }
  SampleState st{};
  st.rng = seed;
  SX_CU(cudaMemcpyAsync(s->sstate, &st, sizeof(st), cudaMemcpyHostToDevice, s->st));
  SX_CU(cudaMemcpyAsync(s->dparams, p, sizeof(*p), cudaMemcpyHostToDevice, s->st));
  return run_frames(s, 1, n_frames, 0, true, frames_out, n_frames_out);
}

namespace {
int run_frames(sx_session* s, int n, int n_frames, int mask_stop, bool sampled, uint32_t* frames_out,
               int* n_frames_out) {
  const sx_model_desc& d = s->m->d;
  const int width = 1 + d.num_codebooks;
  if (n < 1 || n > s->max_batch || n_frames < 0) {
    set_error("decode_greedy: bad batch or frame count");
    return SX_E_INVALID;
  }
  if (s->tp_failed) {
    set_error("tensor-parallel session: an earlier residual exchange failed; reconnect the group and reset");
    return SX_E_STATE;
  }
  int max_len = 0;
  for (int i = 0; i < n; i++) {
    if (s->len[i] <= 0) {
      set_error("decode_greedy before prefill");
      return SX_E_STATE;
    }
    max_len = std::max(max_len, s->len[i]);
  }
  // each frame's trailing slow step writes position len + f
  n_frames = std::min(n_frames, s->max_ctx - max_len);
  n_frames = std::min(n_frames, s->ring_frames);
  std::vector<int> ts(n), tp(n), zeros(n, 0);
  for (int i = 0; i < n; i++) {
    ts[i] = i;
    tp[i] = s->len[i];
  }
  SX_RC(upload_tokens(s, s->tok_seq, s->tok_pos, ts, tp));
  SX_CU(cudaMemcpyAsync(s->seq_len, tp.data(), n * 4, cudaMemcpyHostToDevice, s->st));
  SX_CU(cudaMemcpyAsync(s->done, zeros.data(), n * 4, cudaMemcpyHostToDevice, s->st));
  SX_CU(cudaMemcpyAsync(s->frame_count, zeros.data(), n * 4, cudaMemcpyHostToDevice, s->st));
  GreedyGraph* gg = nullptr;
  for (auto& g : s->graphs)
    if (!g.frame_step && g.M == n && g.mask_stop == mask_stop && g.sampled == (int)sampled) gg = &g;
  if (!gg) {
    GreedyGraph g;
    g.M = n;
    g.mask_stop = mask_stop;
    g.sampled = sampled;
    SX_RC(build_graph(s, n, mask_stop, sampled, &g.exec));
    s->graphs.push_back(g);
    gg = &s->graphs.back();
  }
  for (int f = 0; f < n_frames; f++) SX_CU(cudaGraphLaunch(gg->exec, s->st));
  std::vector<int> counts(n), lens(n);
  SX_CU(cudaMemcpyAsync(counts.data(), s->frame_count, n * 4, cudaMemcpyDeviceToHost, s->st));
  SX_CU(cudaMemcpyAsync(lens.data(), s->seq_len, n * 4, cudaMemcpyDeviceToHost, s->st));
  std::vector<uint32_t> ring((size_t)std::max(1, n_frames) * s->max_batch * width);
  if (n_frames > 0)
    SX_CU(cudaMemcpyAsync(ring.data(), s->ring, (size_t)n_frames * s->max_batch * width * 4,
                          cudaMemcpyDeviceToHost, s->st));
  SX_CU(cudaStreamSynchronize(s->st));
  for (int i = 0; i < n; i++) {
    const int c = std::min(counts[i], n_frames);
    if (n_frames_out) n_frames_out[i] = c;
    s->len[i] = lens[i];
    if (frames_out)
      for (int f = 0; f < c; f++)
        std::memcpy(frames_out + ((size_t)i * n_frames + f) * width, ring.data() + ((size_t)f * s->max_batch + i) * width,
                    width * 4);
  }
  return check_err(s);
}
}  // namespace

int profile_gemv(sx_session* s, int kind, int n_launches) {
  sx_model* m = s->m;
  const sx_transformer_desc& td = m->d.slow;
  if (kind < 0 || kind > 4 || n_launches < 0 || m->slow.empty()) {
    set_error("profile_gemv: kind must be 0..4");
    return SX_E_INVALID;
  }
  for (int i = 0; i < n_launches; i++) {
    const DevLayer& L = m->slow[i % m->slow.size()];
    GemvArgs g;
    g.M = 1;
    Epi epi = EPI_STORE;
    if (kind == 0) {
      g.w = L.wqkv;
      g.x = s->h;
      g.norm_w = L.attn_norm;
      g.eps = td.norm_eps;
      g.bias = L.bqkv;
      g.y = s->xqkv;
      g.ldy = (int)L.wqkv.rows;
      g.n_range = (int)L.wqkv.rows;
    } else if (kind == 1) {
      g.w = L.wo;
      g.x = s->attn;
      g.y = s->hp;
      g.ldy = td.dim;
      g.n_range = td.dim;
    } else if (kind == 2 || kind == 4) {
      g.w = L.w13;
      g.x = s->h;
      g.norm_w = L.ffn_norm;
      g.eps = td.norm_eps;
      g.y = s->act;
      g.ldy = td.intermediate_size;
      g.n_range = 2 * td.intermediate_size;
      epi = EPI_SWIGLU;
      if (kind == 4) {  // as a one-token step runs it: partials only, the merge left to w2
        if (!glu_fold_chunks(s, L, 1)) {
          set_error("profile_gemv: kind 4 needs Q8_0 w1|w3 and w2 with the SwiGLU fold enabled");
          return SX_E_UNSUPPORTED;
        }
        g.part = s->q8_part2;
        g.part_cap = s->q8_part2_cap;
        epi = EPI_NONE;
      }
    } else {
      g.w = L.w2;
      g.x = s->act;
      g.y = s->hp;
      g.ldy = td.dim;
      g.n_range = td.dim;
    }
    SX_RC(gemv(g, epi, s));
  }
  return SX_OK;
}

// One launch of the persistent stack for sequence 0 at its current position with the phase
// trace on. out[0] total us, out[1] setup before the first phase, out[2] the final phase; then
// per phase p (wqkv, attention, wo, w1|w3, w2), averaged over the layers, out[3 + 4p + i]:
// i = 0 the phase (its start to the next phase's start, CTA 0), 1 the slowest CTA's prologue,
// 2 the slowest CTA's arrival after the phase start, 3 the barrier (the last arrival to the
// next phase's start on CTA 0).
int profile_stack(sx_session* s, int fast, float* out) {
  if (s->len[0] <= 0) {
    set_error("profile_stack: prefill first");
    return SX_E_STATE;
  }
  const std::vector<int> ts{0}, tp{s->len[0]};
  SX_RC(upload_tokens(s, s->tok_seq, s->tok_pos, ts, tp));
  StackArgs a;
  float* resid = fast ? s->fx : s->h;
  if (!stack_args(s, fast != 0, 1, resid, s->tok_seq, fast ? nullptr : s->tok_pos, 0, &a)) {
    set_error("profile_stack: this stack does not run on the persistent kernel");
    return SX_E_UNSUPPORTED;
  }
  const int sms = num_sms_of(s->m->device);
  const int L = a.n_layer;
  const size_t per = (size_t)L * 15 + 3;
  unsigned long long* tr = nullptr;
  SX_CU(cudaMalloc((void**)&tr, (per + (size_t)L * 4) * sms * 8));
  a.trace = tr;
  cudaError_t e = launch_stack(a, sms, s->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->st);
  std::vector<unsigned long long> h((per + (size_t)L * 4) * sms);
  if (e == cudaSuccess) e = cudaMemcpy(h.data(), tr, h.size() * 8, cudaMemcpyDeviceToHost);
  cudaFree(tr);
  if (e != cudaSuccess) {
    set_error(std::string("profile_stack: ") + cudaGetErrorString(e));
    return SX_E_CUDA;
  }
  auto T = [&](int cta, size_t i) { return (double)h[(size_t)cta * per + i]; };
  auto at = [&](int l, int p, int k) { return (size_t)1 + ((size_t)l * 5 + p) * 3 + k; };
  const size_t fin = 1 + (size_t)L * 15, end = 2 + (size_t)L * 15;
  for (int i = 0; i < 28; i++) out[i] = 0.f;
  out[0] = (float)((T(0, end) - T(0, 0)) * 1e-3);
  out[1] = (float)((T(0, at(0, 0, 0)) - T(0, 0)) * 1e-3);
  out[2] = (float)((T(0, end) - T(0, fin)) * 1e-3);
  for (int l = 0; l < L; l++)
    for (int p = 0; p < 5; p++) {
      const double start = T(0, at(l, p, 0));
      const double next = (l == L - 1 && p == 4) ? T(0, fin) : T(0, p == 4 ? at(l + 1, 0, 0) : at(l, p + 1, 0));
      double pro = 0, arr = 0;
      for (int c = 0; c < sms; c++) {
        pro = std::max(pro, T(c, at(l, p, 1)) - T(c, at(l, p, 0)));
        arr = std::max(arr, T(c, at(l, p, 2)));
      }
      out[3 + 4 * p + 0] += (float)((next - start) * 1e-3 / L);
      out[3 + 4 * p + 1] += (float)(pro * 1e-3 / L);
      out[3 + 4 * p + 2] += (float)((arr - start) * 1e-3 / L);
      out[3 + 4 * p + 3] += (float)((next - arr) * 1e-3 / L);
    }
  // attention on CTA 0: merge loads + denominators, scale, norm/rope/append, key loop, write-out
  const unsigned long long* sub = h.data() + per * sms;
  for (int l = 0; l < L; l++) {
    const double st = T(0, at(l, 1, 0)), en = T(0, at(l, 1, 1));
    const double p0 = (double)sub[l * 4 + 0], p1 = (double)sub[l * 4 + 1], p2 = (double)sub[l * 4 + 2],
                 p3 = (double)sub[l * 4 + 3];
    out[23] += (float)((p0 - st) * 1e-3 / L);
    out[24] += (float)((p1 - p0) * 1e-3 / L);
    out[25] += (float)((p2 - p1) * 1e-3 / L);
    out[26] += (float)((p3 - p2) * 1e-3 / L);
    out[27] += (float)((en - p3) * 1e-3 / L);
  }
  return check_err(s);
}

int frame_step_greedy(sx_session* s, const uint32_t* frame_in, int mask_stop, uint32_t* frame_out, int* stopped) {
  const sx_model_desc& d = s->m->d;
  const int width = 1 + d.num_codebooks;
  if (s->len[0] <= 0) {
    set_error("frame_step before prefill");
    return SX_E_STATE;
  }
  // One synchronisation per frame: the slow step and the front run as one captured graph and
  // the error flag is read after the frame (a bad frame still runs the front, whose results
  // are discarded; the cached length advances only when the step succeeded).
  if (frame_in) {
    if (s->len[0] + 1 > s->max_ctx) {
      set_error("frame_step: context exceeds the session's max_ctx");
      return SX_E_RANGE;
    }
    // the frame and its position go to device memory; the captured frame graph reads them
    const std::vector<int> ts{0}, tp{s->len[0]};
    SX_CU(cudaMemcpyAsync(s->frames, frame_in, (size_t)width * 4, cudaMemcpyHostToDevice, s->st));
    SX_RC(upload_tokens(s, s->tok_seq, s->tok_pos, ts, tp));
    GreedyGraph* gg = nullptr;
    for (auto& g : s->graphs)
      if (g.frame_step && g.mask_stop == (mask_stop != 0)) gg = &g;
    if (!gg) {
      GreedyGraph g;
      g.M = 1;
      g.mask_stop = mask_stop != 0;
      g.frame_step = 1;
      SX_RC(build_frame_step_graph(s, g.mask_stop, &g.exec));
      s->graphs.push_back(g);
      gg = &s->graphs.back();
    }
    SX_CU(cudaGraphLaunch(gg->exec, s->st));
  } else {
    const std::vector<int> ts{0}, tp{s->len[0]};
    SX_RC(upload_tokens(s, s->tok_seq, s->tok_pos, ts, tp));
    SX_RC(greedy_frame_front(s, 1, mask_stop, false));
  }
  SX_CU(cudaMemcpyAsync(frame_out, s->frames, (size_t)width * 4, cudaMemcpyDeviceToHost, s->st));
  SX_RC(check_err(s));
  if (frame_in) s->len[0] += 1;
  if (stopped)
    *stopped = frame_out[0] >= d.stop_token_id && frame_out[0] < d.stop_token_id + (uint32_t)d.num_stop_tokens;
  return SX_OK;
}

}  // namespace sx
