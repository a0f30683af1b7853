// blob.cpp — the SXW1 weight container: parser and the seeded synthetic-weight writer.
//
// Tensor names follow the reference's weight naming after its load-time remap
// (crates/syrinx-fish/src/s2/load.rs:150-310): `layers.{l}.attention.wqkv.weight` holds the
// fused q|k|v rows in that order (fuse_qkv, s2/load.rs:271-310), the head is tied to
// `embeddings.weight` unless `output.weight` is present (s2/slow_ar.rs:216-221), and the
// fast AR uses `fast_layers.*`, `fast_norm`, `fast_output`, `fast_embeddings`
// (s2/fast_ar.rs). Quantized tensors hold GGML blocks along the input dimension, as the
// reference's `QTensor::quantize` produces them (crates/syrinx-lm/src/cv2/load.rs:99-105).
#include "blob.hpp"

#include <omp.h>

#include <cmath>
#include <cstring>

namespace sx {

namespace {

uint16_t f32_to_f16_rne(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000;
  const uint32_t ax = x & 0x7fffffff;
  if (ax >= 0x7f800000) return (uint16_t)(sign | 0x7c00 | (ax > 0x7f800000 ? 0x200 : 0));
  if (ax >= 0x477ff000) return (uint16_t)(sign | 0x7c00);
  if (ax < 0x38800000) {
    float v;
    std::memcpy(&v, &ax, 4);
    return (uint16_t)(sign | (uint16_t)std::nearbyint(v * 16777216.0f));
  }
  const uint32_t e = (ax >> 23) - 127 + 15;
  const uint32_t m = ax & 0x7fffff;
  uint32_t h = (e << 10) | (m >> 13);
  const uint32_t rem = m & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
  return (uint16_t)(sign | h);
}

float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      int e = -1;
      do {
        e++;
        man <<= 1;
      } while ((man & 0x400) == 0);
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ff) << 13);
    }
  } else if (exp == 0x1f) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Counter-based approximately-normal value: the sum of four 16-bit uniforms of one
// SplitMix64 output (Irwin-Hall, n = 4), centred and scaled to unit variance.
inline float synth_normal(uint64_t key, uint64_t i, float std) {
  const uint64_t z = mix64(key + (i + 1) * 0x9E3779B97F4A7C15ull);
  const double s = (double)(z & 0xffff) + (double)((z >> 16) & 0xffff) + (double)((z >> 32) & 0xffff) +
                   (double)(z >> 48);
  const double u = (s + 2.0) / 65536.0 - 2.0;  // sum of 4 U(0,1) centred: var 1/3
  return (float)(u * 1.7320508075688772 * (double)std);
}

// ggml quantize_row_q8_0_ref: d = amax/127, q = round(x / d) half away from zero.
void quant_q8_0_row(const float* x, int64_t n, uint8_t* out) {
  for (int64_t b = 0; b < n / 32; b++) {
    const float* xb = x + b * 32;
    float amax = 0.f;
    for (int j = 0; j < 32; j++) amax = std::fmax(amax, std::fabs(xb[j]));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint8_t* o = out + b * 34;
    const uint16_t dh = f32_to_f16_rne(d);
    std::memcpy(o, &dh, 2);
    for (int j = 0; j < 32; j++) ((int8_t*)(o + 2))[j] = (int8_t)std::round(xb[j] * id);
  }
}

// Q4_K min/max quantizer: per 32-element sub-block scale = (max - min)/15 and min = -min
// (clamped so the minimum is <= 0), 6-bit sub-block scales/mins relative to the f16
// super-block d / dmin, then the nibbles re-quantized against the stored scales. It is a
// plain min/max fit, not ggml's iterative make_qkx2_quants search; the produced blocks are
// valid Q4_K and dequantize exactly like ggml's.
void quant_q4_k_row(const float* x, int64_t n, uint8_t* out) {
  for (int64_t b = 0; b < n / 256; b++) {
    const float* xb = x + b * 256;
    float scale[8], mins[8];
    float max_scale = 0.f, max_min = 0.f;
    for (int j = 0; j < 8; j++) {
      float mn = xb[32 * j], mx = xb[32 * j];
      for (int l = 1; l < 32; l++) {
        mn = std::fmin(mn, xb[32 * j + l]);
        mx = std::fmax(mx, xb[32 * j + l]);
      }
      if (mn > 0.f) mn = 0.f;
      scale[j] = (mx - mn) / 15.0f;
      mins[j] = -mn;
      max_scale = std::fmax(max_scale, scale[j]);
      max_min = std::fmax(max_min, mins[j]);
    }
    const float d = max_scale / 63.0f, dmin = max_min / 63.0f;
    const uint16_t dh = f32_to_f16_rne(d), mh = f32_to_f16_rne(dmin);
    const float dq = f16_to_f32(dh), mq = f16_to_f32(mh);
    uint8_t sc[8], mm[8];
    for (int j = 0; j < 8; j++) {
      int s = dq > 0.f ? (int)std::lround(scale[j] / dq) : 0;
      int m = mq > 0.f ? (int)std::lround(mins[j] / mq) : 0;
      sc[j] = (uint8_t)std::min(63, std::max(0, s));
      mm[j] = (uint8_t)std::min(63, std::max(0, m));
    }
    uint8_t* o = out + b * 144;
    std::memcpy(o, &dh, 2);
    std::memcpy(o + 2, &mh, 2);
    uint8_t* s12 = o + 4;
    for (int j = 0; j < 4; j++) {
      s12[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
      s12[j + 4] = (uint8_t)((mm[j] & 63) | ((mm[j + 4] >> 4) << 6));
      s12[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mm[j + 4] & 0xF) << 4));
    }
    uint8_t q[256];
    for (int j = 0; j < 8; j++) {
      const float D = dq * (float)sc[j], Mn = mq * (float)mm[j];
      for (int l = 0; l < 32; l++) {
        int v = D > 0.f ? (int)std::lround((xb[32 * j + l] + Mn) / D) : 0;
        q[32 * j + l] = (uint8_t)std::min(15, std::max(0, v));
      }
    }
    uint8_t* qs = o + 16;
    for (int j = 0; j < 4; j++)
      for (int l = 0; l < 32; l++) qs[32 * j + l] = (uint8_t)(q[64 * j + l] | (q[64 * j + 32 + l] << 4));
  }
}

}  // namespace

size_t row_bytes(int dtype, int64_t cols) {
  switch (dtype) {
    case SX_DTYPE_F32: return (size_t)cols * 4;
    case SX_DTYPE_F16:
    case SX_DTYPE_BF16: return (size_t)cols * 2;
    case SX_DTYPE_Q8_0: return cols % 32 ? 0 : (size_t)(cols / 32) * 34;
    case SX_DTYPE_Q4_K: return cols % 256 ? 0 : (size_t)(cols / 256) * 144;
  }
  return 0;
}

int parse_blob(const void* blob, size_t size, BlobIndex* out, std::string* err) {
  const uint8_t* b = (const uint8_t*)blob;
  if (!b || size < 24 || std::memcmp(b, "SXW1", 4) != 0) {
    *err = "weight blob: bad magic";
    return SX_E_BLOB;
  }
  uint32_t version, n;
  uint64_t data_off;
  std::memcpy(&version, b + 4, 4);
  std::memcpy(&n, b + 8, 4);
  std::memcpy(&data_off, b + 16, 8);
  if (version != 1) {
    *err = "weight blob: unsupported version";
    return SX_E_BLOB;
  }
  size_t off = 24;
  for (uint32_t i = 0; i < n; i++) {
    uint32_t nl, dtype, ndim;
    if (off + 4 > size) goto trunc;
    std::memcpy(&nl, b + off, 4);
    off += 4;
    if (nl > 4096 || off + nl + 8 > size) goto trunc;
    {
      BlobTensor t;
      t.name.assign((const char*)b + off, nl);
      off += nl;
      std::memcpy(&dtype, b + off, 4);
      std::memcpy(&ndim, b + off + 4, 4);
      off += 8;
      if (ndim < 1 || ndim > 3 || off + 8 * ndim + 16 > size) {
        *err = "weight blob: bad rank for " + t.name;
        return SX_E_BLOB;
      }
      uint64_t shape[3] = {1, 1, 1};
      for (uint32_t d = 0; d < ndim; d++) std::memcpy(&shape[d], b + off + 8 * d, 8);
      off += 8 * ndim;
      if (ndim == 3 && (dtype != SX_DTYPE_F32 || shape[1] > (1ull << 31) || shape[2] > (1ull << 31))) {
        *err = "weight blob: rank-3 tensors must be f32: " + t.name;
        return SX_E_BLOB;
      }
      uint64_t toff, nbytes;
      std::memcpy(&toff, b + off, 8);
      std::memcpy(&nbytes, b + off + 8, 8);
      off += 16;
      t.dtype = (int)dtype;
      t.ndim = (int)ndim;
      for (uint32_t d = 0; d < ndim; d++) t.shape[d] = (int64_t)shape[d];
      t.rows = ndim == 1 ? 1 : (int64_t)shape[0];
      t.cols = ndim == 1 ? (int64_t)shape[0] : (int64_t)(shape[1] * shape[2]);
      const size_t rb = row_bytes(t.dtype, t.cols);
      if (rb == 0) {
        *err = "weight blob: unsupported dtype / block alignment for " + t.name;
        return SX_E_BLOB;
      }
      if (rb * (size_t)t.rows != nbytes || data_off + toff + nbytes > size) {
        *err = "weight blob: size mismatch for " + t.name;
        return SX_E_BLOB;
      }
      t.data = b + data_off + toff;
      t.nbytes = nbytes;
      out->t[t.name] = t;
    }
  }
  return SX_OK;
trunc:
  *err = "weight blob: truncated header";
  return SX_E_BLOB;
}

std::vector<SynthTensor> synth_tensors(const sx_model_desc& d, int wtype) {
  std::vector<SynthTensor> v;
  auto mat = [&](const std::string& name, int64_t r, int64_t c) { v.push_back({name, wtype, r, c, 0}); };
  auto gain = [&](const std::string& name, int64_t n) { v.push_back({name, SX_DTYPE_F32, 1, n, 1}); };
  auto bias = [&](const std::string& name, int64_t n) { v.push_back({name, SX_DTYPE_F32, 1, n, 2}); };
  auto stack = [&](const sx_transformer_desc& t, const char* prefix) {
    const int64_t qkv = (int64_t)(t.n_head + 2 * t.n_local_heads) * t.head_dim;
    for (int l = 0; l < t.n_layer; l++) {
      const std::string p = std::string(prefix) + "." + std::to_string(l) + ".";
      gain(p + "attention_norm.weight", t.dim);
      mat(p + "attention.wqkv.weight", qkv, t.dim);
      if (t.qkv_bias) bias(p + "attention.wqkv.bias", qkv);
      if (t.qk_norm) {
        gain(p + "attention.q_norm.weight", t.head_dim);
        gain(p + "attention.k_norm.weight", t.head_dim);
      }
      mat(p + "attention.wo.weight", t.dim, (int64_t)t.n_head * t.head_dim);
      if (t.o_bias) bias(p + "attention.wo.bias", t.dim);
      gain(p + "ffn_norm.weight", t.dim);
      mat(p + "feed_forward.w1.weight", t.intermediate_size, t.dim);
      mat(p + "feed_forward.w3.weight", t.intermediate_size, t.dim);
      mat(p + "feed_forward.w2.weight", t.dim, t.intermediate_size);
    }
  };
  mat("embeddings.weight", d.vocab_size, d.slow.dim);
  if (d.num_codebooks > 0) mat("codebook_embeddings.weight", (int64_t)d.num_codebooks * d.codebook_size, d.slow.dim);
  stack(d.slow, "layers");
  gain("norm.weight", d.slow.dim);
  if (!d.tie_word_embeddings) mat("output.weight", d.vocab_size, d.slow.dim);
  if (d.head_bias) bias("output.bias", d.vocab_size);
  if (d.fast.n_layer > 0) {
    stack(d.fast, "fast_layers");
    gain("fast_norm.weight", d.fast.dim);
    mat("fast_output.weight", d.codebook_size, d.fast.dim);
    mat("fast_embeddings.weight", d.codebook_size, d.fast.dim);
  }
  return v;
}

int synth_layout(const sx_model_desc& d, int wtype, std::vector<SynthTensor>* ts, size_t* header,
                 size_t* total) {
  if (wtype != SX_DTYPE_Q8_0 && wtype != SX_DTYPE_Q4_K && wtype != SX_DTYPE_F32) return SX_E_UNSUPPORTED;
  *ts = synth_tensors(d, wtype);
  size_t h = 24;
  for (auto& t : *ts) h += 4 + t.name.size() + 8 + 8 * (t.rows == 1 && t.kind ? 1 : 2) + 16;
  h = (h + 63) & ~(size_t)63;
  size_t off = 0;
  for (auto& t : *ts) {
    const size_t rb = row_bytes(t.dtype, t.cols);
    if (rb == 0) return SX_E_UNSUPPORTED;
    t.offset = off;
    t.nbytes = rb * (size_t)t.rows;
    off = (off + t.nbytes + 63) & ~(size_t)63;
  }
  *header = h;
  *total = h + off;
  return SX_OK;
}

int synth_write(const sx_model_desc& d, int wtype, uint64_t seed, void* out, size_t size) {
  std::vector<SynthTensor> ts;
  size_t header, total;
  int rc = synth_layout(d, wtype, &ts, &header, &total);
  if (rc) return rc;
  if (size < total) return SX_E_INVALID;
  uint8_t* b = (uint8_t*)out;
  std::memset(b, 0, header);
  std::memcpy(b, "SXW1", 4);
  const uint32_t version = 1, n = (uint32_t)ts.size(), reserved = 0;
  const uint64_t data_off = header;
  std::memcpy(b + 4, &version, 4);
  std::memcpy(b + 8, &n, 4);
  std::memcpy(b + 12, &reserved, 4);
  std::memcpy(b + 16, &data_off, 8);
  size_t off = 24;
  for (auto& t : ts) {
    const uint32_t nl = (uint32_t)t.name.size();
    std::memcpy(b + off, &nl, 4);
    std::memcpy(b + off + 4, t.name.data(), nl);
    off += 4 + nl;
    const uint32_t dt = (uint32_t)t.dtype, ndim = (t.rows == 1 && t.kind) ? 1 : 2;
    std::memcpy(b + off, &dt, 4);
    std::memcpy(b + off + 4, &ndim, 4);
    off += 8;
    const uint64_t shape[2] = {(uint64_t)t.rows, (uint64_t)t.cols};
    if (ndim == 1) {
      std::memcpy(b + off, &shape[1], 8);
      off += 8;
    } else {
      std::memcpy(b + off, shape, 16);
      off += 16;
    }
    const uint64_t toff = t.offset, nb = t.nbytes;
    std::memcpy(b + off, &toff, 8);
    std::memcpy(b + off + 8, &nb, 8);
    off += 16;
  }
  const float std = 0.02f;
  for (size_t ti = 0; ti < ts.size(); ti++) {
    const SynthTensor& t = ts[ti];
    uint8_t* dst = b + header + t.offset;
    const uint64_t key = mix64(seed * 0x9E3779B97F4A7C15ull + (uint64_t)(ti + 1) * 0xD1B54A32D192ED03ull);
    const size_t rb = row_bytes(t.dtype, t.cols);
    if (t.kind == 1) {  // RMSNorm gains: 1.0
      float* f = (float*)dst;
      for (int64_t i = 0; i < t.cols; i++) f[i] = 1.0f;
      continue;
    }
#pragma omp parallel
    {
      std::vector<float> row((size_t)t.cols);
#pragma omp for schedule(static)
      for (int64_t r = 0; r < t.rows; r++) {
        for (int64_t c = 0; c < t.cols; c++) row[c] = synth_normal(key, (uint64_t)r * t.cols + c, std);
        uint8_t* o = dst + rb * (size_t)r;
        if (t.dtype == SX_DTYPE_F32)
          std::memcpy(o, row.data(), rb);
        else if (t.dtype == SX_DTYPE_Q8_0)
          quant_q8_0_row(row.data(), t.cols, o);
        else
          quant_q4_k_row(row.data(), t.cols, o);
      }
    }
  }
  return SX_OK;
}

}  // namespace sx
