// misc.cu — embedding gather, greedy frame bookkeeping, weight repack, exact dequant.
//
//   k_embed        MCF input embedding (crates/syrinx-fish/src/s2/slow_ar.rs:101-161; s1
//                  variant s1/slow_ar.rs:85-127; plain LM rows cv2/generate.rs:22-69):
//                  emb[tok] + sum_i cb_emb[code_i + i*R], codebook sum zeroed off the semantic
//                  range, x 1/sqrt(C+1) on semantic positions when the model scales it.
//   k_take_semantic greedy semantic id from the packed argmax (top_k = 1 draw of
//                  sample_semantic, common/sampling.rs:143-167), first_code
//                  (s2/fast_ar.rs:105-110), the fast-AR prefix hidden (post- or pre-norm,
//                  s2/slow_ar.rs:228-244 / s1/slow_ar.rs:186-193) and the stop check.
//   k_take_code    greedy residual code (sample_codebook, sampling.rs:132-137) and the next
//                  fast input fast_embeddings[code] (s2/fast_ar.rs:149-151).
//   k_advance      frame emission + cache length bookkeeping of the driver loop
//                  (common/dualar.rs:198-218).
#include <cuda_runtime.h>

#include <cstdlib>

#include "sx_device.cuh"
#include "sx_internal.hpp"

namespace sx {
namespace {

cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, cudaStream_t st, cudaLaunchAttribute* attr) {
  return launch_cfg(grid, block, 0, st, attr);
}

// Exact dequantized element (r, e) of a device matrix: the value ggml's dequantize_row_*
// produces (single f32 products, no fused multiply-add).
__device__ __forceinline__ float deq_elem(const DevMat& w, int64_t r, int64_t e) {
  const int64_t K = w.cols;
  if (w.dtype == SX_DTYPE_Q8_0) {
    const uint8_t* rec = (const uint8_t*)w.q + ((r / kQ8Tile) * (K / 32) + e / 32) * kQ8Rec;
    const int rr = (int)(r % kQ8Tile), kk = (int)(e % 32);
    const float d = __half2float(*reinterpret_cast<const __half*>(rec + q8_scale_off(rr)));
    return __fmul_rn((float)(int8_t)rec[q8_quant_off(rr, kk)], d);
  } else if (w.dtype == SX_DTYPE_Q4_K) {
    const uint8_t* meta = w.meta + (r * (K / 256) + e / 256) * 16;
    const float d = __half2float(*reinterpret_cast<const __half*>(meta));
    const float dmin = __half2float(*reinterpret_cast<const __half*>(meta + 2));
    const uint8_t* sc12 = meta + 4;
    const int in_sb = (int)(e % 256);
    const int jj = in_sb / 64, l = in_sb % 64;
    const int sub = 2 * jj + (l >= 32 ? 1 : 0);
    uint32_t sc, mn;
    if (sub < 4) {
      sc = sc12[sub] & 63;
      mn = sc12[sub + 4] & 63;
    } else {
      sc = (sc12[sub + 4] & 0xF) | ((sc12[sub - 4] >> 6) << 4);
      mn = (sc12[sub + 4] >> 4) | ((sc12[sub] >> 6) << 4);
    }
    const uint8_t byte = ((const uint8_t*)w.q)[r * (K / 2) + (e / 256) * 128 + jj * 32 + (l & 31)];
    const uint32_t q = l >= 32 ? (byte >> 4) : (byte & 0xF);
    const float d1 = __fmul_rn(d, (float)sc);
    const float m1 = __fmul_rn(dmin, (float)mn);
    return __fsub_rn(__fmul_rn(d1, (float)q), m1);
  }
  return ((const float*)w.q)[r * K + e];
}

__global__ void __launch_bounds__(256) k_embed(const EmbedArgs a, float inv_scale) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  __shared__ uint32_t ids[1 + 64];
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  __syncthreads();
  const int rows = 1 + a.C;
  if (threadIdx.x < rows) {
    uint32_t v;
    if (a.frames) {
      const int seq = a.tok_seq ? ld_cg(a.tok_seq + m) : 0;
      v = ld_cg(a.frames + (size_t)seq * a.frame_stride + threadIdx.x);
    } else {
      v = ld_cg(a.ids + (size_t)threadIdx.x * a.T + a.t0 + m);
    }
    ids[threadIdx.x] = v;
    const bool ok = threadIdx.x == 0 ? v < (uint32_t)a.vocab : v < (uint32_t)a.R;
    if (!ok) bad = 1;
  }
  __syncthreads();
  float* h = a.h + (size_t)m * a.dim;
  if (bad) {
    if (threadIdx.x == 0 && a.err) atomicExch(a.err, 1);
    for (int e = threadIdx.x; e < a.dim; e += blockDim.x) h[e] = 0.f;
    return;
  }
  const uint32_t tok = ids[0];
  const bool sem = tok >= a.sem_lo && tok <= a.sem_hi;
  const float mask = sem ? 1.0f : 0.0f;
  const float sc = sem ? inv_scale : 1.0f;
  for (int e = threadIdx.x; e < a.dim; e += blockDim.x) {
    float x = deq_elem(a.emb, tok, e);
    if (a.C > 0) {
      float acc = deq_elem(a.cb_emb, ids[1], e);
      for (int i = 1; i < a.C; i++)
        acc = __fadd_rn(acc, deq_elem(a.cb_emb, (int64_t)ids[1 + i] + (int64_t)i * a.R, e));
      x = __fadd_rn(x, __fmul_rn(acc, mask));
      if (a.scale_cb) x = __fmul_rn(x, sc);
    }
    h[e] = x;
  }
}

// One CTA per token. Consumes the packed argmax of the slow head.
__global__ void __launch_bounds__(256) k_take_semantic(const FrameArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  const int seq = a.tok_seq ? ld_cg(a.tok_seq + m) : 0;
  __shared__ float red[8];
  if (threadIdx.x == 0) {
    const unsigned long long key = atomicExch(a.amax + m, 0ull);  // read and re-arm
    const uint32_t tok = argmax_row(key);
    uint32_t* fr = a.frames + (size_t)seq * a.frame_stride;
    fr[0] = tok;
    if (a.write_first_code) {
      const uint32_t raw = tok >= a.sem_begin ? tok - a.sem_begin : 0u;
      fr[1] = min(raw, (uint32_t)(a.R - 1));
    }
    if (a.done && tok >= a.stop_lo && tok < a.stop_hi) a.done[seq] = 1;
  }
  if (!a.x) return;
  // fast-AR prefix: the (post-norm) slow hidden of this token
  const float* h = a.h_last + (size_t)m * a.dim;
  float* x = a.x + (size_t)m * a.dim;
  if (a.norm_w) {
    float ss = 0.f;
    for (int e = threadIdx.x; e < a.dim; e += blockDim.x) {
      const float v = ld_cg(h + e);
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += red[w];
    const float den = sqrtf(__fadd_rn(__fdiv_rn(t, (float)a.dim), a.eps));
    for (int e = threadIdx.x; e < a.dim; e += blockDim.x)
      x[e] = __fmul_rn(__fdiv_rn(ld_cg(h + e), den), a.norm_w[e]);
  } else {
    for (int e = threadIdx.x; e < a.dim; e += blockDim.x) x[e] = ld_cg(h + e);
  }
}

// One CTA per token: code for frame slot `slot` (from the argmax, or already in the frame
// when amax is null) and the next fast input fast_embeddings[code] (when emb is set).
__global__ void __launch_bounds__(256) k_take_code(const FrameArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  const int seq = a.tok_seq ? ld_cg(a.tok_seq + m) : 0;
  __shared__ uint32_t code_s;
  uint32_t* fr = a.frames + (size_t)seq * a.frame_stride;
  if (threadIdx.x == 0) {
    uint32_t code;
    if (a.amax) {
      code = argmax_row(atomicExch(a.amax + m, 0ull));  // read and re-arm
      fr[a.slot] = code;
    } else {
      code = ld_cg(fr + a.slot);
    }
    code_s = min(code, (uint32_t)(a.R - 1));
  }
  __syncthreads();
  if (!a.x) return;
  float* x = a.x + (size_t)m * a.dim;
  for (int e = threadIdx.x; e < a.dim; e += blockDim.x) x[e] = deq_elem(a.emb, code_s, e);
}

__global__ void __launch_bounds__(256) k_final_norm(const float* h, const float* w, float eps, int dim,
                                                    float* out) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[8];
  const int m = blockIdx.x;
  const float* hr = h + (size_t)m * dim;
  float ss = 0.f;
  for (int e = threadIdx.x; e < dim; e += blockDim.x) {
    const float v = ld_cg(hr + e);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.f;
  for (int k = 0; k < (int)(blockDim.x >> 5); k++) t += red[k];
  const float den = sqrtf(__fadd_rn(__fdiv_rn(t, (float)dim), eps));
  for (int e = threadIdx.x; e < dim; e += blockDim.x)
    out[(size_t)m * dim + e] = __fmul_rn(__fdiv_rn(ld_cg(hr + e), den), w[e]);
}

__global__ void k_advance(const AdvanceArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = threadIdx.x;
  if (m >= a.M) return;
  const int seq = a.tok_seq ? ld_cg(a.tok_seq + m) : m;
  if (a.done && ld_cg(a.done + seq)) return;
  const int f = ld_cg(a.frame_count + seq);
  const int width = a.frame_stride;
  if (f < a.ring_frames) {
    uint32_t* dst = a.ring + ((size_t)f * a.batch + seq) * width;
    for (int i = 0; i < width; i++) dst[i] = ld_cg(a.frames + (size_t)seq * width + i);
  }
  a.frame_count[seq] = f + 1;
  const int len = ld_cg(a.seq_len + seq) + 1;
  a.seq_len[seq] = len;
  a.tok_pos[m] = len;
}

// GGML Q8_0 blocks {f16 d; i8 q[32]} of source row r -> the tile records of destination row
// (r / grp) * grp * row_mul + row_add * grp + r % grp.
__global__ void k_repack_q8_0(const uint8_t* blocks, int64_t rows, int64_t cols, uint8_t* rec, int row_mul,
                              int row_add, int grp) {
  const int64_t nb = cols / 32;
  const int64_t total = rows * nb;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nb, b = i % nb;
    const uint8_t* src = blocks + i * 34;
    const int64_t dr = (r / grp) * grp * row_mul + (int64_t)row_add * grp + r % grp;
    const int rr = (int)(dr % kQ8Tile);
    uint8_t* dst = rec + ((dr / kQ8Tile) * nb + b) * kQ8Rec;
    dst[q8_scale_off(rr)] = src[0];
    dst[q8_scale_off(rr) + 1] = src[1];
    for (int kk = 0; kk < 32; kk++) dst[q8_quant_off(rr, kk)] = src[2 + kk];
  }
}

__global__ void k_repack_q4_k(const uint8_t* blocks, int64_t rows, int64_t cols, uint8_t* q, uint8_t* meta,
                              int row_mul, int row_add) {
  const int64_t nb = cols / 256;
  const int64_t total = rows * nb;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nb, b = i % nb;
    const uint4* src = reinterpret_cast<const uint4*>(blocks + i * 144);
    const int64_t dr = r * row_mul + row_add;
    reinterpret_cast<uint4*>(meta)[dr * nb + b] = src[0];
    uint4* dq = reinterpret_cast<uint4*>(q + dr * (cols / 2) + b * 128);
    for (int j = 0; j < 8; j++) dq[j] = src[1 + j];
  }
}

// GGML Q4_K super-blocks -> tile records (sx_internal.hpp, kQ4Rec): one thread per (row,
// super-block). The 6-bit scale / min of sub-block j unpacked as ggml's get_scale_min_k4 does;
// sub-block j's 32 nibbles are the low (even j) or high (odd j) halves of qs[32 (j / 2) ..].
// Rows land at dr = (r / grp) * grp * row_mul + row_add * grp + r % grp (w1 / w3 interleave per
// 16-row tile, as the Q8_0 records).
__global__ void k_repack_q4k_tiles(const uint8_t* blocks, int64_t rows, int64_t cols, uint8_t* rec, int row_mul,
                                   int row_add, int grp) {
  const int64_t nsb = cols / 256;
  const int64_t total = rows * nsb;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nsb, sb = i % nsb;
    const uint8_t* src = blocks + i * 144;
    const int64_t dr = (r / grp) * grp * row_mul + (int64_t)row_add * grp + r % grp;
    const int rr = (int)(dr % kQ8Tile);
    uint8_t* dst = rec + ((dr / kQ8Tile) * nsb + sb) * kQ4Rec;
    const uint8_t* sc12 = src + 4;
    const uint8_t* qs = src + 16;
    for (int j = 0; j < 8; j++) {
      uint32_t sc, mn;
      if (j < 4) {
        sc = sc12[j] & 63;
        mn = sc12[j + 4] & 63;
      } else {
        sc = (sc12[j + 4] & 0xF) | ((sc12[j - 4] >> 6) << 4);
        mn = (sc12[j + 4] >> 4) | ((sc12[j] >> 6) << 4);
      }
      dst[q4_sc_off(rr, j)] = (uint8_t)sc;
      dst[q4_sc_off(rr, j) + 128] = (uint8_t)mn;
      for (int k = 0; k < 16; k++) {
        const uint8_t b0 = qs[(j >> 1) * 32 + k], b1 = qs[(j >> 1) * 32 + k + 16];
        const uint8_t q0 = (j & 1) ? (b0 >> 4) : (b0 & 0xF), q1 = (j & 1) ? (b1 >> 4) : (b1 & 0xF);
        dst[q4_quant_off(rr, j, k)] = (uint8_t)(q0 | (q1 << 4));
      }
    }
    for (int b = 0; b < 4; b++) dst[q4_dd_off(rr) + b] = src[b];  // d, dmin (f16)
  }
}

__global__ void k_dequant(int dtype, const uint8_t* blocks, int64_t n_blocks, float* out) {
  const int64_t per = dtype == SX_DTYPE_Q8_0 ? 32 : 256;
  const int64_t total = n_blocks * per;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / per, e = i % per;
    if (dtype == SX_DTYPE_Q8_0) {
      const uint8_t* src = blocks + b * 34;
      const float d = __half2float(__ushort_as_half((unsigned short)(src[0] | (src[1] << 8))));
      out[i] = __fmul_rn((float)(int8_t)src[2 + e], d);
    } else {
      const uint8_t* src = blocks + b * 144;
      const float d = __half2float(__ushort_as_half((unsigned short)(src[0] | (src[1] << 8))));
      const float dmin = __half2float(__ushort_as_half((unsigned short)(src[2] | (src[3] << 8))));
      const uint8_t* sc12 = src + 4;
      const int jj = (int)(e / 64), l = (int)(e % 64);
      const int sub = 2 * jj + (l >= 32 ? 1 : 0);
      uint32_t sc, mn;
      if (sub < 4) {
        sc = sc12[sub] & 63;
        mn = sc12[sub + 4] & 63;
      } else {
        sc = (sc12[sub + 4] & 0xF) | ((sc12[sub - 4] >> 6) << 4);
        mn = (sc12[sub + 4] >> 4) | ((sc12[sub] >> 6) << 4);
      }
      const uint8_t byte = src[16 + jj * 32 + (l & 31)];
      const uint32_t qv = l >= 32 ? (byte >> 4) : (byte & 0xF);
      const float d1 = __fmul_rn(d, (float)sc);
      const float m1 = __fmul_rn(dmin, (float)mn);
      out[i] = __fsub_rn(__fmul_rn(d1, (float)qv), m1);
    }
  }
}

}  // namespace

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("SYRINX_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

cudaLaunchConfig_t launch_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t st, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cfg;
}

cudaError_t launch_embed(const EmbedArgs& a, cudaStream_t st) {
  if (a.C > 64) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(a.M), dim3(256), st, attr);
  const float inv_scale = 1.0f / sqrtf((float)a.C + 1.0f);
  return cudaLaunchKernelEx(&cfg, k_embed, a, inv_scale);
}

cudaError_t launch_take_semantic(const FrameArgs& a, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(a.M), dim3(256), st, attr);
  return cudaLaunchKernelEx(&cfg, k_take_semantic, a);
}

cudaError_t launch_take_code(const FrameArgs& a, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(a.M), dim3(256), st, attr);
  return cudaLaunchKernelEx(&cfg, k_take_code, a);
}

cudaError_t launch_final_norm(const float* h, const float* w, float eps, int dim, int M, float* out,
                              cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(M), dim3(256), st, attr);
  return cudaLaunchKernelEx(&cfg, k_final_norm, h, w, eps, dim, out);
}

cudaError_t launch_advance(const AdvanceArgs& a, cudaStream_t st) {
  if (a.M > 1024) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(1), dim3(((a.M + 31) / 32) * 32), st, attr);
  return cudaLaunchKernelEx(&cfg, k_advance, a);
}

cudaError_t repack_q8_0(const uint8_t* blocks, int64_t rows, int64_t cols, uint8_t* rec, int row_mul, int row_add,
                        int grp, cudaStream_t st) {
  if (grp < 1 || cols % 32) return cudaErrorInvalidValue;
  (void)cudaGetLastError();  // report this launch's status, not an earlier one
  k_repack_q8_0<<<1184, 256, 0, st>>>(blocks, rows, cols, rec, row_mul, row_add, grp);
  return cudaGetLastError();
}

cudaError_t repack_q4_k(const uint8_t* blocks, int64_t rows, int64_t cols, uint8_t* q, uint8_t* meta,
                        int row_mul, int row_add, cudaStream_t st) {
  (void)cudaGetLastError();  // report this launch's status, not an earlier one
  k_repack_q4_k<<<1184, 256, 0, st>>>(blocks, rows, cols, q, meta, row_mul, row_add);
  return cudaGetLastError();
}

cudaError_t repack_q4k_tiles(const uint8_t* blocks, int64_t rows, int64_t cols, uint8_t* rec, int row_mul,
                             int row_add, int grp, cudaStream_t st) {
  if (grp < 1 || cols % 256) return cudaErrorInvalidValue;
  (void)cudaGetLastError();  // report this launch's status, not an earlier one
  k_repack_q4k_tiles<<<1184, 256, 0, st>>>(blocks, rows, cols, rec, row_mul, row_add, grp);
  return cudaGetLastError();
}

cudaError_t dequant_blocks(int dtype, const uint8_t* blocks, int64_t n_blocks, float* out,
                           cudaStream_t st) {
  if (dtype != SX_DTYPE_Q8_0 && dtype != SX_DTYPE_Q4_K) return cudaErrorInvalidValue;
  (void)cudaGetLastError();  // report this launch's status, not an earlier one
  k_dequant<<<1184, 256, 0, st>>>(dtype, blocks, n_blocks, out);
  return cudaGetLastError();
}

}  // namespace sx
