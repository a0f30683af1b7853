// oracle.cpp — CPU restatement of the reference's quantized dual-AR decode path.
//
// TEST INFRASTRUCTURE ONLY (see oracle.h): the checker the B200 kernels are compared
// against, and the CPU baseline timed beside them. Never part of the product path.
//
// Reference behaviour restated here, by file (paths inside voldiguarddevelopment/syrinx):
//   block formats ........ GGML Q8_0 quantize_row_q8_0_ref / dequantize_row_q8_0 and Q4_K
//                          dequantize_row_q4_K, as implemented bit-exactly by gguf-py
//                          (gguf/quants.py Q8_0, Q4_K); called by candle QMatMul
//                          (crates/syrinx-lm/src/cv2/load.rs:99-105)
//   rms_norm_w ........... crates/syrinx-fish/src/s2/nn.rs:100-106 (x / sqrt(mean(x^2)+eps) * w)
//   precompute_rope ...... s2/nn.rs:117-141 ; apply_rotary_emb (interleaved) s2/nn.rs:154-166
//   rotate-half rope ..... crates/syrinx-lm/src/cv2/attention.rs:82-88, 108-119
//   attention ............ s2/nn.rs:284-360 (wqkv split q|k|v, QK-norm, RoPE, cache append,
//                          repeat_kv GQA, scale 1/sqrt(hd), softmax, wo)
//   swiglu ............... s2/nn.rs:452-457
//   MCF embed ............ s2/slow_ar.rs:101-161 (s1: s1/slow_ar.rs:85-127, no scale)
//   run_layers / head .... s2/slow_ar.rs:166-246 (s1 head: s1/slow_ar.rs:171-195)
//   fast AR .............. s2/fast_ar.rs:67-154
//   drive ................ crates/syrinx-fish/src/common/dualar.rs:161-230
//   Sampler .............. crates/syrinx-fish/src/common/sampling.rs:19-268
#include "oracle.h"
#include "../syrinx_b200/csrc/blob.hpp"

#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

thread_local std::string g_err;
int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

// ---------------------------------------------------------------------------------------
// half / bfloat16 conversions
// ---------------------------------------------------------------------------------------
float h2f(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: renormalise
      int e = -1;
      do {
        e++;
        man <<= 1;
      } while ((man & 0x400) == 0);
      man &= 0x3ff;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 0x1f) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// round-to-nearest-even f32 -> f16
uint16_t f2h(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000;
  uint32_t ax = x & 0x7fffffff;
  if (ax >= 0x7f800000) return (uint16_t)(sign | 0x7c00 | (ax > 0x7f800000 ? 0x200 : 0));
  if (ax >= 0x477ff000) return (uint16_t)(sign | 0x7c00);  // rounds to >= 65520 -> inf
  if (ax < 0x38800000) {                                  // result is subnormal or zero
    // value = ax as float; subnormal f16 unit = 2^-24
    float v;
    std::memcpy(&v, &ax, 4);
    float scaled = v * 16777216.0f;  // exact (power of two)
    // round half to even
    float r = std::nearbyint(scaled);
    return (uint16_t)(sign | (uint16_t)r);
  }
  uint32_t e = (ax >> 23) - 127 + 15;
  uint32_t m = ax & 0x7fffff;
  uint32_t h = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
  return (uint16_t)(sign | h);
}

uint16_t f2bf(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  if ((x & 0x7fffffff) > 0x7f800000) return (uint16_t)((x >> 16) | 0x40);
  uint32_t r = x + 0x7fff + ((x >> 16) & 1);
  return (uint16_t)(r >> 16);
}
float bf2f(uint16_t b) {
  uint32_t x = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}
float round_bf16(float f) { return bf2f(f2bf(f)); }

// ---------------------------------------------------------------------------------------
// GGML blocks
// ---------------------------------------------------------------------------------------
constexpr int QK8_0 = 32;
constexpr int Q8_0_BYTES = 34;
constexpr int QK_K = 256;
constexpr int Q4_K_BYTES = 144;

void q8_0_dequant_block(const uint8_t* b, float* y) {
  uint16_t dh;
  std::memcpy(&dh, b, 2);
  const float d = h2f(dh);
  const int8_t* q = (const int8_t*)(b + 2);
  for (int j = 0; j < QK8_0; j++) y[j] = (float)q[j] * d;
}

// get_scale_min_k4: the 6-bit sub-block scale / min packing of Q4_K.
inline void q4k_scale_min(int j, const uint8_t* q, uint8_t* sc, uint8_t* m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

void q4_k_dequant_block(const uint8_t* b, float* y) {
  uint16_t dh, mh;
  std::memcpy(&dh, b, 2);
  std::memcpy(&mh, b + 2, 2);
  const float d = h2f(dh);
  const float dmin = h2f(mh);
  const uint8_t* scales = b + 4;
  const uint8_t* qs = b + 16;
  for (int j = 0; j < 4; j++) {
    uint8_t sc, m;
    q4k_scale_min(2 * j, scales, &sc, &m);
    const float d1 = d * (float)sc;
    const float m1 = dmin * (float)m;
    q4k_scale_min(2 * j + 1, scales, &sc, &m);
    const float d2 = d * (float)sc;
    const float m2 = dmin * (float)m;
    for (int l = 0; l < 32; l++) y[64 * j + l] = d1 * (float)(qs[32 * j + l] & 0xF) - m1;
    for (int l = 0; l < 32; l++) y[64 * j + 32 + l] = d2 * (float)(qs[32 * j + l] >> 4) - m2;
  }
}

// ---------------------------------------------------------------------------------------
// tensors and the blob container
// ---------------------------------------------------------------------------------------
struct OT {
  int dtype = -1;
  int64_t rows = 0, cols = 0;
  const uint8_t* p = nullptr;
  size_t nbytes = 0;
};

size_t row_bytes(int dtype, int64_t cols) {
  switch (dtype) {
    case SX_DTYPE_F32: return (size_t)cols * 4;
    case SX_DTYPE_F16:
    case SX_DTYPE_BF16: return (size_t)cols * 2;
    case SX_DTYPE_Q8_0: return (size_t)(cols / QK8_0) * Q8_0_BYTES;
    case SX_DTYPE_Q4_K: return (size_t)(cols / QK_K) * Q4_K_BYTES;
  }
  return 0;
}

void deq_row(const OT& t, int64_t r, float* out) {
  const uint8_t* p = t.p + row_bytes(t.dtype, t.cols) * (size_t)r;
  switch (t.dtype) {
    case SX_DTYPE_F32: std::memcpy(out, p, t.cols * 4); break;
    case SX_DTYPE_F16:
      for (int64_t c = 0; c < t.cols; c++) {
        uint16_t h;
        std::memcpy(&h, p + 2 * c, 2);
        out[c] = h2f(h);
      }
      break;
    case SX_DTYPE_BF16:
      for (int64_t c = 0; c < t.cols; c++) {
        uint16_t h;
        std::memcpy(&h, p + 2 * c, 2);
        out[c] = bf2f(h);
      }
      break;
    case SX_DTYPE_Q8_0:
      for (int64_t b = 0; b < t.cols / QK8_0; b++)
        q8_0_dequant_block(p + b * Q8_0_BYTES, out + b * QK8_0);
      break;
    case SX_DTYPE_Q4_K:
      for (int64_t b = 0; b < t.cols / QK_K; b++)
        q4_k_dequant_block(p + b * Q4_K_BYTES, out + b * QK_K);
      break;
  }
}

float dot(const float* a, const float* b, int64_t n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int64_t i = 0;
  for (; i + 8 <= n; i += 8)
    for (int j = 0; j < 8; j++) acc[j] += a[i + j] * b[i + j];
  for (; i < n; i++) acc[i & 7] += a[i] * b[i];
  return ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
}

// Matmul numerics for quantized weights. Mode A (the default, what the B200 kernels
// compute) multiplies the exactly dequantized weights by the f32 activations with f32 sums.
// Mode B (oc_set_qmode(1), for analysis) restates Candle's CPU QMatMul for Q8_0 weights,
// which follows ggml: every activation row is quantized to Q8_0 blocks (quantize_row_q8_0:
// d = amax/127, q = round(x/d), d stored as f16) and each block contributes
// (float)sumi * (d_w * d_x), sumi the exact int32 dot, in block order (vec_dot_q8_0_q8_0;
// candle-core 0.8.x is not vendored here, so the published ggml form stands in). Mode B is
// chaotic in its inputs: a 1-ulp change of the normed activations moves config-1 logits by
// ~5e-2 (mode A: ~3e-6), so it cannot serve as a parity target for any implementation with
// another reduction order. Mode B for Q4_K weights: linear_q4_k_b below.
int g_qmode = 0;

void q8_0_quantize_act(const float* x, int64_t K, int8_t* q, float* d) {
  for (int64_t b = 0; b < K / QK8_0; b++) {
    const float* xb = x + b * QK8_0;
    float amax = 0.0f;
    for (int j = 0; j < QK8_0; j++) amax = std::max(amax, std::fabs(xb[j]));
    const float dd = amax / 127.0f;
    const float id = dd != 0.0f ? 1.0f / dd : 0.0f;
    d[b] = h2f(f2h(dd));
    for (int j = 0; j < QK8_0; j++) q[b * QK8_0 + j] = (int8_t)std::round(xb[j] * id);
  }
}

void linear_q8_0_b(const OT& W, const float* b, const float* x, int M, float* y) {
  const int64_t N = W.rows, K = W.cols, nb = K / QK8_0;
  std::vector<int8_t> xq((size_t)M * K);
  std::vector<float> xd((size_t)M * nb);
  for (int m = 0; m < M; m++) q8_0_quantize_act(x + (size_t)m * K, K, xq.data() + (size_t)m * K, xd.data() + (size_t)m * nb);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < N; r++) {
    const uint8_t* row = W.p + (size_t)r * nb * Q8_0_BYTES;
    for (int m = 0; m < M; m++) {
      const int8_t* qx = xq.data() + (size_t)m * K;
      float sumf = 0.0f;
      for (int64_t bk = 0; bk < nb; bk++) {
        const uint8_t* blk = row + bk * Q8_0_BYTES;
        uint16_t dh;
        std::memcpy(&dh, blk, 2);
        const int8_t* qw = (const int8_t*)(blk + 2);
        int32_t sumi = 0;
        for (int j = 0; j < QK8_0; j++) sumi += (int32_t)qw[j] * (int32_t)qx[bk * QK8_0 + j];
        sumf += (float)sumi * (h2f(dh) * xd[(size_t)m * nb + bk]);
      }
      y[(size_t)m * N + r] = b ? sumf + b[r] : sumf;
    }
  }
}

// Mode B for Q4_K weights, as candle-core's k-quants restate ggml for the CPU QMatMul (the
// portable form; candle-core 0.8.x is not vendored, so its published k_quants source stands in).
// Each activation row is quantized to Q8_K super-blocks of 256 (BlockQ8K::from_float: the
// element of largest magnitude, with its sign, sets iscale = -128 / max; q = min(127,
// round(iscale * x)) rounding halves away from zero; d = 1 / iscale kept in f32; bsums = the
// sums of each 16 consecutive q). Per super-block (BlockQ4K vec_dot): the nibbles widened to
// int8, int32 lane sums aux[l] += sc_j * (q8 * q4) over the eight lanes of every 8-element
// group, sumi = sum_j bsums[j] * m_{j/2}; then sums[l] += (d_w * d_x) * aux[l] for each lane
// and sumf -= (dmin_w * d_x) * sumi, in f32; the row is sumf + (sums[0] + ... + sums[7]).
struct Q8K {
  float d = 0.0f;
  int8_t qs[QK_K];
  int16_t bsums[QK_K / 16];
};

void q8_k_quantize_act(const float* x, int64_t K, Q8K* out) {
  for (int64_t b = 0; b < K / QK_K; b++) {
    const float* xb = x + b * QK_K;
    Q8K& y = out[b];
    float mx = 0.0f, amax = 0.0f;
    for (int j = 0; j < QK_K; j++)
      if (amax < std::fabs(xb[j])) {
        amax = std::fabs(xb[j]);
        mx = xb[j];
      }
    if (amax == 0.0f) {
      y.d = 0.0f;
      std::memset(y.qs, 0, sizeof(y.qs));
      std::memset(y.bsums, 0, sizeof(y.bsums));
      continue;
    }
    const float iscale = -128.0f / mx;
    for (int j = 0; j < QK_K; j++) y.qs[j] = (int8_t)std::min(127.0f, std::round(iscale * xb[j]));
    for (int j = 0; j < QK_K / 16; j++) {
      int32_t sum = 0;
      for (int i = 0; i < 16; i++) sum += y.qs[16 * j + i];
      y.bsums[j] = (int16_t)sum;
    }
    y.d = 1.0f / iscale;
  }
}

void linear_q4_k_b(const OT& W, const float* b, const float* x, int M, float* y) {
  const int64_t N = W.rows, K = W.cols, nb = K / QK_K;
  std::vector<Q8K> xq((size_t)M * nb);
  for (int m = 0; m < M; m++) q8_k_quantize_act(x + (size_t)m * K, K, xq.data() + (size_t)m * nb);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < N; r++) {
    const uint8_t* row = W.p + (size_t)r * nb * Q4_K_BYTES;
    for (int m = 0; m < M; m++) {
      float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      float sumf = 0.0f;
      for (int64_t bk = 0; bk < nb; bk++) {
        const uint8_t* blk = row + bk * Q4_K_BYTES;
        const Q8K& q8 = xq[(size_t)m * nb + bk];
        uint16_t dh, mh;
        std::memcpy(&dh, blk, 2);
        std::memcpy(&mh, blk + 2, 2);
        const uint8_t* qs = blk + 16;
        int8_t a[QK_K];
        for (int j = 0; j < 4; j++)
          for (int l = 0; l < 32; l++) {
            a[64 * j + l] = (int8_t)(qs[32 * j + l] & 0xF);
            a[64 * j + 32 + l] = (int8_t)(qs[32 * j + l] >> 4);
          }
        uint8_t sc[8], mn[8];
        for (int j = 0; j < 8; j++) q4k_scale_min(j, blk + 4, &sc[j], &mn[j]);
        int32_t sumi = 0;
        for (int j = 0; j < QK_K / 16; j++) sumi += (int32_t)q8.bsums[j] * (int32_t)mn[j / 2];
        int32_t aux[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < 8; j++)
          for (int g = 0; g < 4; g++)
            for (int l = 0; l < 8; l++) {
              const int k = 32 * j + 8 * g + l;
              aux[l] += (int32_t)sc[j] * (int32_t)(int16_t)(q8.qs[k] * a[k]);
            }
        const float d = h2f(dh) * q8.d;
        for (int l = 0; l < 8; l++) sums[l] += d * (float)aux[l];
        const float dmin = h2f(mh) * q8.d;
        sumf -= dmin * (float)sumi;
      }
      float tot = 0.0f;
      for (int l = 0; l < 8; l++) tot += sums[l];
      const float v = sumf + tot;
      y[(size_t)m * N + r] = b ? v + b[r] : v;
    }
  }
}

// y[M][N] = x[M][K] . W^T (+ b).
void linear(const OT& W, const OT* bias, const float* x, int M, float* y) {
  const int64_t N = W.rows, K = W.cols;
  const float* b = bias ? (const float*)bias->p : nullptr;
  if (W.dtype == SX_DTYPE_Q8_0 && g_qmode == 1) {
    linear_q8_0_b(W, b, x, M, y);
    return;
  }
  if (W.dtype == SX_DTYPE_Q4_K && g_qmode == 1) {
    linear_q4_k_b(W, b, x, M, y);
    return;
  }
#pragma omp parallel
  {
    std::vector<float> row(K);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < N; r++) {
      deq_row(W, r, row.data());
      for (int m = 0; m < M; m++) {
        float v = dot(row.data(), x + (size_t)m * K, K);
        if (b) v = v + b[r];
        y[(size_t)m * N + r] = v;
      }
    }
  }
}

void rmsnorm_rows(const float* x, const float* w, int rows, int n, float eps, float* y) {
  for (int r = 0; r < rows; r++) {
    const float* xr = x + (size_t)r * n;
    float* yr = y + (size_t)r * n;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i < n; i++) acc[i & 7] += xr[i] * xr[i];
    float ss = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    const float var = ss / (float)n;
    const float den = std::sqrt(var + eps);
    for (int i = 0; i < n; i++) yr[i] = (xr[i] / den) * w[i];
  }
}

// RoPE inverse frequencies exactly as precompute_rope (s2/nn.rs:125-127) and
// rope_cos_sin_at (cv2/attention.rs:110-112): 1 / base^(2i/hd) in f32.
std::vector<float> rope_inv_freq(int hd, float base) {
  std::vector<float> f(hd / 2);
  for (int i = 0; i < hd / 2; i++) f[i] = 1.0f / std::pow(base, (2.0f * (float)i) / (float)hd);
  return f;
}

// Rotate one head vector x[hd] at absolute position pos, in place.
void rope_head(float* x, int hd, int pos, const float* inv_freq, bool interleaved) {
  const int half = hd / 2;
  if (interleaved) {
    for (int i = 0; i < half; i++) {
      const float a = (float)pos * inv_freq[i];
      const float c = std::cos(a), s = std::sin(a);
      const float x0 = x[2 * i], x1 = x[2 * i + 1];
      x[2 * i] = x0 * c - x1 * s;
      x[2 * i + 1] = x1 * c + x0 * s;
    }
  } else {
    for (int i = 0; i < half; i++) {
      const float a = (float)pos * inv_freq[i];
      const float c = std::cos(a), s = std::sin(a);
      const float x1 = x[i], x2 = x[i + half];
      x[i] = x1 * c + (-x2) * s;
      x[i + half] = x2 * c + x1 * s;
    }
  }
}

float silu(float v) { return v / (1.0f + std::exp(-v)); }

// ---------------------------------------------------------------------------------------
// Blob parse (SXW1)
// ---------------------------------------------------------------------------------------
struct Blob {
  std::unordered_map<std::string, OT> t;
};

int parse_blob(const void* blob, size_t size, Blob* out) {
  const uint8_t* b = (const uint8_t*)blob;
  if (size < 24 || std::memcmp(b, "SXW1", 4) != 0) return fail(SX_E_BLOB, "bad blob magic");
  uint32_t version, n;
  uint64_t data_off;
  std::memcpy(&version, b + 4, 4);
  std::memcpy(&n, b + 8, 4);
  std::memcpy(&data_off, b + 16, 8);
  if (version != 1) return fail(SX_E_BLOB, "unsupported blob version");
  size_t off = 24;
  for (uint32_t i = 0; i < n; i++) {
    uint32_t nl, dtype, ndim;
    if (off + 4 > size) return fail(SX_E_BLOB, "truncated blob header");
    std::memcpy(&nl, b + off, 4);
    off += 4;
    if (off + nl + 8 > size) return fail(SX_E_BLOB, "truncated blob header");
    std::string name((const char*)b + off, nl);
    off += nl;
    std::memcpy(&dtype, b + off, 4);
    std::memcpy(&ndim, b + off + 4, 4);
    off += 8;
    if (ndim < 1 || ndim > 2 || off + 8 * ndim + 16 > size)
      return fail(SX_E_BLOB, "bad tensor rank for " + name);
    uint64_t shape[2] = {1, 1};
    for (uint32_t d = 0; d < ndim; d++) std::memcpy(&shape[d], b + off + 8 * d, 8);
    off += 8 * ndim;
    uint64_t toff, nbytes;
    std::memcpy(&toff, b + off, 8);
    std::memcpy(&nbytes, b + off + 8, 8);
    off += 16;
    OT t;
    t.dtype = (int)dtype;
    if (ndim == 1) {
      t.rows = 1;
      t.cols = (int64_t)shape[0];
    } else {
      t.rows = (int64_t)shape[0];
      t.cols = (int64_t)shape[1];
    }
    size_t rb = row_bytes(t.dtype, t.cols);
    if (rb == 0) return fail(SX_E_BLOB, "unsupported dtype for " + name);
    if (t.dtype == SX_DTYPE_Q8_0 && t.cols % QK8_0) return fail(SX_E_BLOB, "Q8_0 cols % 32 " + name);
    if (t.dtype == SX_DTYPE_Q4_K && t.cols % QK_K) return fail(SX_E_BLOB, "Q4_K cols % 256 " + name);
    if (rb * (size_t)t.rows != nbytes) return fail(SX_E_BLOB, "size mismatch for " + name);
    if (data_off + toff + nbytes > size) return fail(SX_E_BLOB, "tensor out of blob: " + name);
    t.p = b + data_off + toff;
    t.nbytes = nbytes;
    out->t[name] = t;
  }
  return SX_OK;
}

struct Layer {
  const OT *attn_norm = nullptr, *wqkv = nullptr, *bqkv = nullptr, *qn = nullptr, *kn = nullptr,
           *wo = nullptr, *bo = nullptr, *ffn_norm = nullptr, *w1 = nullptr, *w2 = nullptr,
           *w3 = nullptr;
};

}  // namespace

struct oc_model {
  sx_model_desc d;
  Blob blob;
  std::vector<Layer> slow, fast;
  const OT *emb = nullptr, *cb_emb = nullptr, *norm = nullptr, *out_w = nullptr, *out_b = nullptr;
  const OT *fast_norm = nullptr, *fast_out = nullptr, *fast_emb = nullptr;
  std::vector<float> inv_slow, inv_fast;
};

struct oc_session {
  oc_model* m;
  int max_ctx;
  bool kv_bf16;
  int len = 0;
  // slow cache: [L][Hkv][max_ctx][hd] for K and V
  std::vector<float> k, v;
  // fast cache: [Lf][Hkv][C][hd]
  std::vector<float> fk, fv;
  int fast_len = 0;
  // last prefill/step outputs
  std::vector<float> last_h;  // pre-norm residual of the last position [slow.dim]
};

namespace {

const OT* need(oc_model* m, const std::string& name, int* rc, int64_t rows, int64_t cols) {
  auto it = m->blob.t.find(name);
  if (it == m->blob.t.end()) {
    *rc = fail(SX_E_BLOB, "missing tensor " + name);
    return nullptr;
  }
  const OT& t = it->second;
  if ((rows >= 0 && t.rows != rows) || (cols >= 0 && t.cols != cols)) {
    *rc = fail(SX_E_BLOB, "shape mismatch for " + name);
    return nullptr;
  }
  return &t;
}

int bind_layers(oc_model* m, const sx_transformer_desc& td, const char* prefix, std::vector<Layer>* out) {
  int rc = SX_OK;
  const int qkv_rows = (td.n_head + 2 * td.n_local_heads) * td.head_dim;
  const int attn_w = td.n_head * td.head_dim;
  for (int l = 0; l < td.n_layer; l++) {
    std::string p = std::string(prefix) + "." + std::to_string(l) + ".";
    Layer L;
    L.attn_norm = need(m, p + "attention_norm.weight", &rc, 1, td.dim);
    L.wqkv = need(m, p + "attention.wqkv.weight", &rc, qkv_rows, td.dim);
    if (td.qkv_bias) L.bqkv = need(m, p + "attention.wqkv.bias", &rc, 1, qkv_rows);
    if (td.qk_norm) {
      L.qn = need(m, p + "attention.q_norm.weight", &rc, 1, td.head_dim);
      L.kn = need(m, p + "attention.k_norm.weight", &rc, 1, td.head_dim);
    }
    L.wo = need(m, p + "attention.wo.weight", &rc, td.dim, attn_w);
    if (td.o_bias) L.bo = need(m, p + "attention.wo.bias", &rc, 1, td.dim);
    L.ffn_norm = need(m, p + "ffn_norm.weight", &rc, 1, td.dim);
    L.w1 = need(m, p + "feed_forward.w1.weight", &rc, td.intermediate_size, td.dim);
    L.w3 = need(m, p + "feed_forward.w3.weight", &rc, td.intermediate_size, td.dim);
    L.w2 = need(m, p + "feed_forward.w2.weight", &rc, td.dim, td.intermediate_size);
    if (rc) return rc;
    out->push_back(L);
  }
  return rc;
}

bool is_allowed(const sx_model_desc& d, uint32_t id, bool mask_stop) {
  if (id >= d.semantic_begin_id && id <= d.semantic_end_id) return true;
  if (!mask_stop && id >= d.stop_token_id && id < d.stop_token_id + (uint32_t)d.num_stop_tokens)
    return true;
  return false;
}

// One transformer stack over M new tokens at absolute positions pos0..pos0+M-1 of one
// sequence, causally. `x` [M][dim] is updated in place (the residual stream).
void run_layers(oc_session* s, bool fast, float* x, int M, int pos0) {
  oc_model* m = s->m;
  const sx_transformer_desc& td = fast ? m->d.fast : m->d.slow;
  const std::vector<Layer>& layers = fast ? m->fast : m->slow;
  const int d = td.dim, H = td.n_head, Hkv = td.n_local_heads, hd = td.head_dim;
  const int F = td.intermediate_size, G = H / Hkv;
  const int qkv_w = (H + 2 * Hkv) * hd;
  const int cap = fast ? m->d.num_codebooks : s->max_ctx;
  const std::vector<float>& inv = fast ? m->inv_fast : m->inv_slow;
  std::vector<float>& kc = fast ? s->fk : s->k;
  std::vector<float>& vc = fast ? s->fv : s->v;
  const bool round_kv = s->kv_bf16;  // mirrors the device cache element type (slow and fast)
  const float scale = (float)(1.0 / std::sqrt((double)hd));

  std::vector<float> hn((size_t)M * d), qkv((size_t)M * qkv_w), ctx((size_t)M * H * hd);
  std::vector<float> o((size_t)M * d), g((size_t)M * F), u((size_t)M * F);
  for (size_t l = 0; l < layers.size(); l++) {
    const Layer& L = layers[l];
    rmsnorm_rows(x, (const float*)L.attn_norm->p, M, d, td.norm_eps, hn.data());
    linear(*L.wqkv, L.bqkv, hn.data(), M, qkv.data());
    for (int t = 0; t < M; t++) {
      float* q = qkv.data() + (size_t)t * qkv_w;
      float* k = q + H * hd;
      float* v = k + Hkv * hd;
      if (td.qk_norm) {
        rmsnorm_rows(q, (const float*)L.qn->p, H, hd, td.norm_eps, q);
        rmsnorm_rows(k, (const float*)L.kn->p, Hkv, hd, td.norm_eps, k);
      }
      for (int h = 0; h < H; h++) rope_head(q + h * hd, hd, pos0 + t, inv.data(), td.rope_interleaved);
      for (int h = 0; h < Hkv; h++) rope_head(k + h * hd, hd, pos0 + t, inv.data(), td.rope_interleaved);
      // KvCache::append: K post-RoPE and raw V at the token's absolute position.
      for (int h = 0; h < Hkv; h++) {
        float* kd = kc.data() + (((size_t)l * Hkv + h) * cap + (pos0 + t)) * hd;
        float* vd = vc.data() + (((size_t)l * Hkv + h) * cap + (pos0 + t)) * hd;
        for (int e = 0; e < hd; e++) {
          kd[e] = round_kv ? round_bf16(k[h * hd + e]) : k[h * hd + e];
          vd[e] = round_kv ? round_bf16(v[h * hd + e]) : v[h * hd + e];
        }
      }
    }
    // GQA scaled-dot-product attention with the causal mask.
#pragma omp parallel for collapse(2) schedule(static)
    for (int t = 0; t < M; t++) {
      for (int h = 0; h < H; h++) {
        const int kvh = h / G;
        const int n_keys = pos0 + t + 1;
        const float* q = qkv.data() + (size_t)t * qkv_w + h * hd;
        std::vector<float> sc(n_keys);
        float mx = -INFINITY;
        for (int j = 0; j < n_keys; j++) {
          const float* kr = kc.data() + (((size_t)l * Hkv + kvh) * cap + j) * hd;
          sc[j] = dot(q, kr, hd) * scale;
          mx = std::max(mx, sc[j]);
        }
        float sum = 0.f;
        for (int j = 0; j < n_keys; j++) {
          sc[j] = std::exp(sc[j] - mx);
          sum += sc[j];
        }
        for (int j = 0; j < n_keys; j++) sc[j] = sc[j] / sum;
        float* c = ctx.data() + (size_t)t * H * hd + h * hd;
        for (int e = 0; e < hd; e++) c[e] = 0.f;
        for (int j = 0; j < n_keys; j++) {
          const float* vr = vc.data() + (((size_t)l * Hkv + kvh) * cap + j) * hd;
          for (int e = 0; e < hd; e++) c[e] += sc[j] * vr[e];
        }
      }
    }
    linear(*L.wo, L.bo, ctx.data(), M, o.data());
    for (size_t i = 0; i < (size_t)M * d; i++) x[i] = x[i] + o[i];
    rmsnorm_rows(x, (const float*)L.ffn_norm->p, M, d, td.norm_eps, hn.data());
    linear(*L.w1, nullptr, hn.data(), M, g.data());
    linear(*L.w3, nullptr, hn.data(), M, u.data());
    for (size_t i = 0; i < (size_t)M * F; i++) g[i] = silu(g[i]) * u[i];
    linear(*L.w2, nullptr, g.data(), M, o.data());
    for (size_t i = 0; i < (size_t)M * d; i++) x[i] = x[i] + o[i];
  }
}

// MCF embedding of a [(1+C) x T] id matrix into x [T][dim].
int embed(oc_session* s, const uint32_t* ids, int T, float* x) {
  oc_model* m = s->m;
  const sx_model_desc& d = m->d;
  const int dim = d.slow.dim, C = d.num_codebooks, R = d.codebook_size;
  std::vector<float> row(dim), acc(dim);
  const float inv_scale = 1.0f / std::sqrt((float)C + 1.0f);
  for (int t = 0; t < T; t++) {
    const uint32_t tok = ids[t];
    if (tok >= (uint32_t)d.vocab_size) return fail(SX_E_INVALID, "token id out of range");
    float* xt = x + (size_t)t * dim;
    deq_row(*m->emb, tok, xt);
    if (C == 0) continue;
    for (int i = 0; i < C; i++) {
      const uint32_t code = ids[(size_t)(i + 1) * T + t];
      if (code >= (uint32_t)R) return fail(SX_E_INVALID, "codebook code out of range");
      deq_row(*m->cb_emb, (int64_t)code + (int64_t)i * R, row.data());
      if (i == 0)
        std::memcpy(acc.data(), row.data(), dim * 4);
      else
        for (int e = 0; e < dim; e++) acc[e] = acc[e] + row[e];
    }
    const bool sem = tok >= d.semantic_begin_id && tok <= d.semantic_end_id;
    const float mask = sem ? 1.0f : 0.0f;
    for (int e = 0; e < dim; e++) xt[e] = xt[e] + acc[e] * mask;
    if (d.scale_codebook_embeddings) {
      const float sc = sem ? inv_scale : 1.0f;
      for (int e = 0; e < dim; e++) xt[e] = xt[e] * sc;
    }
  }
  return SX_OK;
}

// Final RMSNorm -> head logits; hidden = post-norm (s2) or pre-norm (s1) last position.
void head(oc_session* s, const float* last, float* logits, float* hidden) {
  oc_model* m = s->m;
  const int dim = m->d.slow.dim;
  std::vector<float> normed(dim);
  rmsnorm_rows(last, (const float*)m->norm->p, 1, dim, m->d.slow.norm_eps, normed.data());
  if (logits) linear(*m->out_w, m->out_b, normed.data(), 1, logits);
  if (hidden) std::memcpy(hidden, m->d.norm_fastlayer_input ? normed.data() : last, dim * 4);
}

int forward_ids(oc_session* s, const uint32_t* ids, int T, float* logits, float* hidden) {
  oc_model* m = s->m;
  if (T <= 0) return fail(SX_E_INVALID, "empty input");
  if (s->len + T > s->max_ctx) return fail(SX_E_RANGE, "context exceeds session capacity");
  const int dim = m->d.slow.dim;
  std::vector<float> x((size_t)T * dim);
  int rc = embed(s, ids, T, x.data());
  if (rc) return rc;
  run_layers(s, false, x.data(), T, s->len);
  s->len += T;
  s->last_h.assign(x.end() - dim, x.end());
  head(s, s->last_h.data(), logits, hidden);
  return SX_OK;
}

// Qwen2Lm::step_logits_cached(embeds) (crates/syrinx-lm/src/cv2/generate.rs:119-123):
// caller-assembled input embeddings through the cached layers, last-position head.
int forward_embeds(oc_session* s, const float* embeds, int T, float* logits) {
  oc_model* m = s->m;
  if (T <= 0) return fail(SX_E_INVALID, "empty input");
  if (s->len + T > s->max_ctx) return fail(SX_E_RANGE, "context exceeds session capacity");
  const int dim = m->d.slow.dim;
  std::vector<float> x(embeds, embeds + (size_t)T * dim);
  run_layers(s, false, x.data(), T, s->len);
  s->len += T;
  s->last_h.assign(x.end() - dim, x.end());
  head(s, s->last_h.data(), logits, nullptr);
  return SX_OK;
}

uint32_t argmax_allowed(const sx_model_desc& d, const float* logits, bool mask_stop, float* margin) {
  float best = -INFINITY, second = -INFINITY;
  int64_t bi = -1;
  auto visit = [&](uint32_t id) {
    const float v = logits[id];
    if (bi < 0 || v > best) {
      second = best;
      best = v;
      bi = id;
    } else if (v > second) {
      second = v;
    }
  };
  for (uint32_t id = d.semantic_begin_id; id <= d.semantic_end_id && id < (uint32_t)d.vocab_size; id++)
    visit(id);
  if (!mask_stop)
    for (int i = 0; i < d.num_stop_tokens; i++) {
      const uint32_t id = d.stop_token_id + i;
      if (id < d.semantic_begin_id || id > d.semantic_end_id) {
        // keep ascending id order for ties: a stop id below the range wins ties
        const float v = logits[id];
        if (v > best || (v == best && (int64_t)id < bi)) {
          second = best;
          best = v;
          bi = id;
        } else if (v > second) {
          second = v;
        }
      }
    }
  if (margin) *margin = best - second;
  return (uint32_t)bi;
}

uint32_t argmax_all(const float* v, int n) {
  int bi = 0;
  for (int i = 1; i < n; i++)
    if (v[i] > v[bi]) bi = i;
  return (uint32_t)bi;
}

// ---------------------------------------------------------------------------------------
// Sampler (common/sampling.rs)
// ---------------------------------------------------------------------------------------
struct SplitMix64 {
  uint64_t state;
  uint64_t next_u64() {
    state += 0x9E3779B97F4A7C15ull;
    uint64_t z = state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  double next_f64() { return (double)(next_u64() >> 11) * (1.0 / (double)(1ull << 53)); }
};

std::vector<float> logits_to_probs(const float* logits, int n, float temperature, float top_p,
                                   int top_k) {
  std::vector<int> order(n);
  for (int i = 0; i < n; i++) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
    if (logits[b] < logits[a]) return true;
    if (logits[a] < logits[b]) return false;
    return a < b;
  });
  const float mx = n ? logits[order[0]] : 0.0f;
  std::vector<double> exps(n);
  double sum = 0.0;
  for (int r = 0; r < n; r++) {
    exps[r] = std::exp((double)(logits[order[r]] - mx));
  }
  for (int r = 0; r < n; r++) sum += exps[r];
  const int k_cap = top_k == 0 ? n : top_k;
  std::vector<char> keep(n, 0);
  double cum = 0.0;
  for (int r = 0; r < n; r++) {
    const int i = order[r];
    if (r == 0) {
      keep[i] = 1;
    } else if (cum <= (double)top_p && r < k_cap) {
      keep[i] = 1;
    } else {
      break;
    }
    cum += exps[r] / sum;
  }
  const float t = std::max(temperature, 1e-5f);
  float kept_max = -INFINITY;
  for (int i = 0; i < n; i++)
    if (keep[i]) kept_max = std::max(kept_max, logits[i] / t);
  std::vector<float> probs(n, 0.0f);
  double psum = 0.0;
  for (int i = 0; i < n; i++)
    if (keep[i]) {
      const double e = std::exp((double)(logits[i] / t - kept_max));
      probs[i] = (float)e;
      psum += e;
    }
  if (psum > 0.0)
    for (int i = 0; i < n; i++) probs[i] = (float)((double)probs[i] / psum);
  return probs;
}

int multinomial1(const std::vector<float>& probs, SplitMix64* rng) {
  double total = 0.0;
  for (float p : probs) total += (double)p;
  if (total <= 0.0) return 0;
  const double u = rng->next_f64() * total;
  double acc = 0.0;
  for (size_t i = 0; i < probs.size(); i++) {
    acc += (double)probs[i];
    if (u < acc) return (int)i;
  }
  return probs.empty() ? 0 : (int)probs.size() - 1;
}

struct Sampler {
  SplitMix64 rng;
  sx_sampling_params p;
  uint32_t sample_codebook(const float* logits, int n) {
    // repetition penalty over an empty `recent` list is a no-op (s2/fast_ar.rs:147)
    auto probs = logits_to_probs(logits, n, p.temperature, p.top_p, p.top_k);
    return (uint32_t)multinomial1(probs, &rng);
  }
  uint32_t sample_semantic(const sx_model_desc& d, const float* logits, int n,
                           const std::vector<uint32_t>& window) {
    std::vector<float> c(logits, logits + n);
    for (int i = 0; i < n; i++)
      if (!is_allowed(d, (uint32_t)i, false)) c[i] = -INFINITY;
    auto pn = logits_to_probs(c.data(), n, p.temperature, p.top_p, p.top_k);
    const uint32_t normal = (uint32_t)multinomial1(pn, &rng);
    auto ph = logits_to_probs(c.data(), n, p.ras_high_temp, p.ras_high_top_p, p.top_k);
    const uint32_t high = (uint32_t)multinomial1(ph, &rng);
    const bool in_window = std::find(window.begin(), window.end(), normal) != window.end();
    const bool sem = normal >= d.semantic_begin_id && normal <= d.semantic_end_id;
    return (in_window && sem) ? high : normal;
  }
};

int fast_step(oc_session* s, const float* xin, int pos, float* logits) {
  oc_model* m = s->m;
  const int fd = m->d.fast.dim;
  std::vector<float> x(xin, xin + fd);
  run_layers(s, true, x.data(), 1, pos);
  s->fast_len = pos + 1;
  if (logits) {
    std::vector<float> normed(fd);
    rmsnorm_rows(x.data(), (const float*)m->fast_norm->p, 1, fd, m->d.fast.norm_eps, normed.data());
    linear(*m->fast_out, nullptr, normed.data(), 1, logits);
  }
  return SX_OK;
}

template <class Pick>
int fast_expand(oc_session* s, const float* hidden, uint32_t first_code, uint32_t* codes,
                float* fast_logits, Pick pick) {
  oc_model* m = s->m;
  const int C = m->d.num_codebooks, R = m->d.codebook_size, fd = m->d.fast.dim;
  if (C == 0 || m->fast.empty()) return fail(SX_E_STATE, "model has no fast AR");
  if (first_code >= (uint32_t)R) return fail(SX_E_INVALID, "first_code out of range");
  std::fill(s->fk.begin(), s->fk.end(), 0.0f);
  std::fill(s->fv.begin(), s->fv.end(), 0.0f);
  fast_step(s, hidden, 0, nullptr);  // conditioning prefix; its logits are discarded
  codes[0] = first_code;
  std::vector<float> x(fd), logits(R);
  deq_row(*m->fast_emb, first_code, x.data());
  for (int cb = 1; cb < C; cb++) {
    fast_step(s, x.data(), cb, logits.data());
    if (fast_logits) std::memcpy(fast_logits + (size_t)(cb - 1) * R, logits.data(), R * 4);
    const uint32_t code = pick(logits.data(), R);
    codes[cb] = code;
    deq_row(*m->fast_emb, code, x.data());
  }
  return SX_OK;
}

}  // namespace

// =======================================================================================
// C ABI
// =======================================================================================
extern "C" {

const char* oc_last_error(void) { return g_err.c_str(); }
int oc_num_threads(void) { return omp_get_max_threads(); }
void oc_set_num_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}

void oc_set_qmode(int32_t mode) { g_qmode = mode ? 1 : 0; }
int32_t oc_get_qmode(void) { return g_qmode; }

void oc_linear_q8_0(const float* x, const uint8_t* blocks, int32_t M, int32_t N, int32_t K, float* y) {
  OT w;
  w.dtype = SX_DTYPE_Q8_0;
  w.rows = N;
  w.cols = K;
  w.p = blocks;
  w.nbytes = (size_t)N * (K / QK8_0) * Q8_0_BYTES;
  linear(w, nullptr, x, M, y);
}

void oc_linear_q4_k(const float* x, const uint8_t* blocks, int32_t M, int32_t N, int32_t K, float* y) {
  OT w;
  w.dtype = SX_DTYPE_Q4_K;
  w.rows = N;
  w.cols = K;
  w.p = blocks;
  w.nbytes = (size_t)N * (K / QK_K) * Q4_K_BYTES;
  linear(w, nullptr, x, M, y);
}

void oc_q8_0_quantize(const float* x, int64_t n, uint8_t* blocks) {
  for (int64_t b = 0; b < n / QK8_0; b++) {
    const float* xb = x + b * QK8_0;
    float amax = 0.0f;
    for (int j = 0; j < QK8_0; j++) amax = std::max(amax, std::fabs(xb[j]));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint8_t* o = blocks + b * Q8_0_BYTES;
    const uint16_t dh = f2h(d);
    std::memcpy(o, &dh, 2);
    for (int j = 0; j < QK8_0; j++) ((int8_t*)(o + 2))[j] = (int8_t)std::round(xb[j] * id);
  }
}
void oc_q8_0_dequantize(const uint8_t* blocks, int64_t n_blocks, float* out) {
  for (int64_t b = 0; b < n_blocks; b++) q8_0_dequant_block(blocks + b * Q8_0_BYTES, out + b * QK8_0);
}
void oc_q4_k_dequantize(const uint8_t* blocks, int64_t n_blocks, float* out) {
  for (int64_t b = 0; b < n_blocks; b++) q4_k_dequant_block(blocks + b * Q4_K_BYTES, out + b * QK_K);
}
float oc_f16_to_f32(uint16_t h) { return h2f(h); }
uint16_t oc_f32_to_f16(float f) { return f2h(f); }
uint16_t oc_f32_to_bf16(float f) { return f2bf(f); }

void oc_rmsnorm(const float* x, const float* w, int32_t rows, int32_t n, float eps, float* y) {
  rmsnorm_rows(x, w, rows, n, eps, y);
}
void oc_softmax(const float* x, int32_t rows, int32_t n, float* y) {
  for (int r = 0; r < rows; r++) {
    const float* xr = x + (size_t)r * n;
    float* yr = y + (size_t)r * n;
    float mx = -INFINITY;
    for (int i = 0; i < n; i++) mx = std::max(mx, xr[i]);
    float sum = 0.f;
    for (int i = 0; i < n; i++) {
      yr[i] = std::exp(xr[i] - mx);
      sum += yr[i];
    }
    for (int i = 0; i < n; i++) yr[i] = yr[i] / sum;
  }
}
void oc_silu(const float* x, int64_t n, float* y) {
  for (int64_t i = 0; i < n; i++) y[i] = silu(x[i]);
}
void oc_rope(float* x, int32_t T, int32_t n_heads, int32_t hd, const int32_t* positions, float theta,
             int32_t interleaved) {
  auto inv = rope_inv_freq(hd, theta);
  for (int t = 0; t < T; t++)
    for (int h = 0; h < n_heads; h++)
      rope_head(x + ((size_t)t * n_heads + h) * hd, hd, positions[t], inv.data(), interleaved != 0);
}
void oc_linear_f32(const float* x, const float* w, const float* b, int32_t M, int32_t N, int32_t K,
                   float* y) {
  for (int m = 0; m < M; m++)
    for (int n = 0; n < N; n++) {
      float v = dot(x + (size_t)m * K, w + (size_t)n * K, K);
      if (b) v = v + b[n];
      y[(size_t)m * N + n] = v;
    }
}

int oc_model_create(const sx_model_desc* desc, const void* blob, size_t blob_size, oc_model** out) {
  if (!desc || !blob || !out) return fail(SX_E_INVALID, "null argument");
  auto m = new oc_model();
  m->d = *desc;
  int rc = parse_blob(blob, blob_size, &m->blob);
  const sx_model_desc& d = m->d;
  const int dim = d.slow.dim;
  if (!rc) rc = bind_layers(m, d.slow, "layers", &m->slow);
  if (!rc) {
    m->emb = need(m, "embeddings.weight", &rc, d.vocab_size, dim);
    m->norm = need(m, "norm.weight", &rc, 1, dim);
    if (d.tie_word_embeddings)
      m->out_w = m->emb;
    else
      m->out_w = need(m, "output.weight", &rc, d.vocab_size, dim);
    if (d.head_bias) m->out_b = need(m, "output.bias", &rc, 1, d.vocab_size);
    if (d.num_codebooks > 0)
      m->cb_emb = need(m, "codebook_embeddings.weight", &rc,
                       (int64_t)d.num_codebooks * d.codebook_size, dim);
  }
  if (!rc && d.fast.n_layer > 0) {
    if (d.fast.dim != dim) rc = fail(SX_E_UNSUPPORTED, "fast_project_in (fast.dim != slow.dim)");
    if (!rc) rc = bind_layers(m, d.fast, "fast_layers", &m->fast);
    if (!rc) {
      m->fast_norm = need(m, "fast_norm.weight", &rc, 1, d.fast.dim);
      m->fast_out = need(m, "fast_output.weight", &rc, d.codebook_size, d.fast.dim);
      m->fast_emb = need(m, "fast_embeddings.weight", &rc, d.codebook_size, d.fast.dim);
    }
  }
  if (rc) {
    delete m;
    return rc;
  }
  m->inv_slow = rope_inv_freq(d.slow.head_dim, d.slow.rope_base);
  if (d.fast.n_layer > 0) m->inv_fast = rope_inv_freq(d.fast.head_dim, d.fast.rope_base);
  *out = m;
  return SX_OK;
}
void oc_model_destroy(oc_model* m) { delete m; }

int oc_tensor_rows(const oc_model* m, const char* name, int64_t r0, int64_t n, float* out) {
  auto it = m->blob.t.find(name);
  if (it == m->blob.t.end()) return fail(SX_E_INVALID, std::string("no tensor ") + name);
  const OT& t = it->second;
  if (r0 < 0 || r0 + n > t.rows) return fail(SX_E_RANGE, "row range");
  for (int64_t r = 0; r < n; r++) deq_row(t, r0 + r, out + r * t.cols);
  return SX_OK;
}
int oc_tensor_shape(const oc_model* m, const char* name, int64_t* rows, int64_t* cols, int32_t* dtype) {
  auto it = m->blob.t.find(name);
  if (it == m->blob.t.end()) return fail(SX_E_INVALID, std::string("no tensor ") + name);
  *rows = it->second.rows;
  *cols = it->second.cols;
  *dtype = it->second.dtype;
  return SX_OK;
}

int oc_session_create(oc_model* m, int32_t max_ctx, int32_t kv_bf16, oc_session** out) {
  if (!m || !out || max_ctx <= 0) return fail(SX_E_INVALID, "bad session args");
  auto s = new oc_session();
  s->m = m;
  s->max_ctx = max_ctx;
  s->kv_bf16 = kv_bf16 != 0;
  const auto& d = m->d;
  size_t n = (size_t)d.slow.n_layer * d.slow.n_local_heads * max_ctx * d.slow.head_dim;
  s->k.assign(n, 0.0f);
  s->v.assign(n, 0.0f);
  if (d.fast.n_layer > 0) {
    size_t nf = (size_t)d.fast.n_layer * d.fast.n_local_heads * d.num_codebooks * d.fast.head_dim;
    s->fk.assign(nf, 0.0f);
    s->fv.assign(nf, 0.0f);
  }
  *out = s;
  return SX_OK;
}
void oc_session_destroy(oc_session* s) { delete s; }
void oc_session_reset(oc_session* s) {
  s->len = 0;
  s->fast_len = 0;
}
int32_t oc_session_len(const oc_session* s) { return s->len; }

int oc_prefill(oc_session* s, const uint32_t* prompt, int32_t T, float* logits, float* hidden) {
  if (!s || !prompt) return fail(SX_E_INVALID, "null argument");
  if (s->len != 0) return fail(SX_E_STATE, "prefill on a non-empty session");
  return forward_ids(s, prompt, T, logits, hidden);
}
int oc_slow_step(oc_session* s, const uint32_t* frame, float* logits, float* hidden) {
  if (!s || !frame) return fail(SX_E_INVALID, "null argument");
  if (s->len == 0) return fail(SX_E_STATE, "slow_step before prefill");
  return forward_ids(s, frame, 1, logits, hidden);
}
int oc_lm_step_tokens(oc_session* s, const uint32_t* tokens, int32_t t_new, float* logits) {
  if (!s || !tokens) return fail(SX_E_INVALID, "null argument");
  if (s->m->d.num_codebooks != 0) return fail(SX_E_UNSUPPORTED, "not a plain LM");
  return forward_ids(s, tokens, t_new, logits, nullptr);
}
int oc_lm_step_embeds(oc_session* s, const float* embeds, int32_t t_new, float* logits) {
  if (!s || !embeds) return fail(SX_E_INVALID, "null argument");
  return forward_embeds(s, embeds, t_new, logits);
}
int oc_fast_expand_greedy(oc_session* s, const float* hidden, uint32_t first_code, uint32_t* codes,
                          float* fast_logits) {
  return fast_expand(s, hidden, first_code, codes, fast_logits,
                     [](const float* l, int n) { return argmax_all(l, n); });
}
uint32_t oc_first_code(const oc_model* m, uint32_t tok) {
  const int64_t raw = tok >= m->d.semantic_begin_id ? (int64_t)(tok - m->d.semantic_begin_id) : 0;
  const int64_t mx = (int64_t)m->d.codebook_size - 1;
  return (uint32_t)std::min<int64_t>(std::max<int64_t>(raw, 0), std::max<int64_t>(mx, 0));
}
uint32_t oc_greedy_semantic(const oc_model* m, const float* logits, int32_t mask_stop, float* margin) {
  return argmax_allowed(m->d, logits, mask_stop != 0, margin);
}

int oc_drive_greedy(oc_session* s, const uint32_t* prompt, int32_t T, int32_t n_frames,
                    int32_t mask_stop, uint32_t* frames_out, int32_t* n_out, float* margins_out) {
  oc_model* m = s->m;
  const auto& d = m->d;
  const int C = d.num_codebooks;
  oc_session_reset(s);
  std::vector<float> logits(d.vocab_size), hidden(d.slow.dim);
  int rc = oc_prefill(s, prompt, T, logits.data(), hidden.data());
  if (rc) return rc;
  int produced = 0;
  std::vector<uint32_t> frame(1 + C);
  for (int f = 0; f < n_frames; f++) {
    float margin = 0.f;
    const uint32_t sem = argmax_allowed(d, logits.data(), mask_stop != 0, &margin);
    if (margins_out) margins_out[f] = margin;
    if (sem >= d.stop_token_id && sem < d.stop_token_id + (uint32_t)d.num_stop_tokens) break;
    frame[0] = sem;
    if (C > 0) {
      rc = oc_fast_expand_greedy(s, hidden.data(), oc_first_code(m, sem), frame.data() + 1, nullptr);
      if (rc) return rc;
    }
    std::memcpy(frames_out + (size_t)f * (1 + C), frame.data(), (1 + C) * 4);
    produced++;
    if (f + 1 == n_frames) break;
    if (s->len + 1 > s->max_ctx) break;
    // the frame as a [(1+C) x 1] column: row r = frame[r]
    rc = forward_ids(s, frame.data(), 1, logits.data(), hidden.data());
    if (rc) return rc;
  }
  *n_out = produced;
  return SX_OK;
}

int oc_drive(oc_session* s, const uint32_t* prompt, int32_t T, int32_t max_frames, uint64_t seed,
             const sx_sampling_params* p, uint32_t* codes_out, int32_t* n_out) {
  oc_model* m = s->m;
  const auto& d = m->d;
  const int C = d.num_codebooks, R = d.codebook_size, V = d.vocab_size;
  oc_session_reset(s);
  Sampler smp{SplitMix64{seed}, *p};
  std::vector<float> logits(V), hidden(d.slow.dim);
  int rc = oc_prefill(s, prompt, T, logits.data(), hidden.data());
  if (rc) return rc;
  std::vector<uint32_t> window;
  const int ras_win = std::max(p->ras_win_size, 1);
  int pos = T, nf = 0;
  std::vector<uint32_t> frame(C > 0 ? C : 1), full(1 + C);
  for (;;) {
    const uint32_t sem = smp.sample_semantic(d, logits.data(), V, window);
    if (sem >= d.stop_token_id && sem < d.stop_token_id + (uint32_t)d.num_stop_tokens) break;
    const uint32_t first = oc_first_code(m, sem);
    if (C > 0) {
      rc = fast_expand(s, hidden.data(), first, frame.data(), nullptr,
                       [&](const float* l, int n) { return smp.sample_codebook(l, n); });
      if (rc) return rc;
      (void)R;
      for (int c = 0; c < C; c++) codes_out[(size_t)c * max_frames + nf] = frame[c];
    }
    nf++;
    window.push_back(sem);
    if ((int)window.size() > ras_win) window.erase(window.begin());
    if (nf >= max_frames) break;
    if (pos + 1 >= s->max_ctx) break;
    full[0] = sem;
    for (int c = 0; c < C; c++) full[1 + c] = frame[c];
    rc = forward_ids(s, full.data(), 1, logits.data(), hidden.data());
    if (rc) return rc;
    pos++;
  }
  *n_out = nf;
  return SX_OK;
}

int oc_synth_blob_size(const sx_model_desc* desc, int32_t wtype, size_t* size_out) {
  if (!desc || !size_out) return fail(SX_E_INVALID, "null argument");
  std::vector<sx::SynthTensor> ts;
  size_t header = 0;
  if (sx::synth_layout(*desc, wtype, &ts, &header, size_out)) return fail(SX_E_UNSUPPORTED, "synthetic blob layout");
  return SX_OK;
}
int oc_synth_blob_write(const sx_model_desc* desc, int32_t wtype, uint64_t seed, void* out, size_t size) {
  if (!desc || !out) return fail(SX_E_INVALID, "null argument");
  if (sx::synth_write(*desc, wtype, seed, out, size)) return fail(SX_E_INVALID, "synthetic blob write");
  return SX_OK;
}

uint64_t oc_splitmix64_next(uint64_t* state) {
  SplitMix64 r{*state};
  uint64_t v = r.next_u64();
  *state = r.state;
  return v;
}
void oc_logits_to_probs(const float* logits, int32_t n, float temperature, float top_p, int32_t top_k,
                        float* probs) {
  auto p = logits_to_probs(logits, n, temperature, top_p, top_k);
  std::memcpy(probs, p.data(), (size_t)n * 4);
}

}  // extern "C"
