// attention.cu — GQA decode attention over the paged KV cache (f32 or bf16 elements).
//
// Replaces the reference attention block after the wqkv projection
// (`attention`, crates/syrinx-fish/src/s2/nn.rs:315-352; `attn_cached`,
// crates/syrinx-lm/src/cv2/attention.rs:60-76):
//   split q|k|v -> per-head QK-RMSNorm (nn.rs:325-331) -> RoPE, interleaved (nn.rs:154-166)
//   or rotate-half (cv2/attention.rs:82-88) -> KV append (KvCache::append, nn.rs:244-254)
//   -> scores * 1/sqrt(hd) -> softmax -> P.V, per kv head for its whole query group, so
//   the repeat_kv copy (nn.rs:194-202) never exists.
//
// One CTA per (token, kv head, split of the key axis): the CTA streams its slice of the
// bf16 K/V pages once for all G query heads of the group, keeps an online softmax in f32,
// and the last CTA of a (token, kv head) to finish merges the split partials (flash-decoding).
// In decode (append = 1) the CTA whose slice contains the new position computes that
// token's normed, rotated K and V, writes them into the cache and uses them directly, so
// no other CTA reads a slot written in the same launch.
#include <cuda_runtime.h>

#include "sx_device.cuh"
#include "sx_internal.hpp"

namespace sx {
namespace {

constexpr int kWarpsA = kAttnThreads / 32;
constexpr int kSub = 128;  // keys per shared-memory score tile

// RMSNorm (optional) + RoPE of one head held in shared memory by one warp, in place.
template <int HD>
__device__ void norm_rope_head(float* buf, const float* nw, float eps, const float* inv_freq,
                               int interleaved, int pos, int lane) {
  if (nw) {
    float ss = 0.f;
    for (int e = lane; e < HD; e += 32) ss = fmaf(buf[e], buf[e], ss);
    ss = warp_sum(ss);
    const float den = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)HD), eps));
    __syncwarp();
    for (int e = lane; e < HD; e += 32) buf[e] = __fmul_rn(__fdiv_rn(buf[e], den), nw[e]);
    __syncwarp();
  }
  for (int i = lane; i < HD / 2; i += 32) {
    const float ang = __fmul_rn((float)pos, inv_freq[i]);
    float s, c;
    sincosf(ang, &s, &c);
    const int i0 = interleaved ? 2 * i : i;
    const int i1 = interleaved ? 2 * i + 1 : i + HD / 2;
    const float x0 = buf[i0], x1 = buf[i1];
    if (interleaved) {
      buf[i0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
      buf[i1] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
    } else {
      buf[i0] = __fadd_rn(__fmul_rn(x0, c), __fmul_rn(-x1, s));
      buf[i1] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
    }
  }
  __syncwarp();
}

__device__ __forceinline__ size_t kv_off(const AttnArgs& a, int seq, int t, int g, int HD) {
  const int page = a.page_table[(size_t)seq * a.pt_stride + t / kPage];
  return ((size_t)(page * a.Hkv + g) * kPage + (t % kPage)) * HD;
}

// KV element type: f32 (exact, the reference CPU path's cache) or bf16 (half the bytes).
__device__ __forceinline__ void kv_store(float* p, float v) { *p = v; }
__device__ __forceinline__ void kv_store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ float kv_load(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float kv_load(const __nv_bfloat16* p) { return __bfloat162float(__ldcg(p)); }

// EPL consecutive elements of a K row starting at p, as f32 (one vector load).
template <int EPL>
__device__ __forceinline__ void kv_load_row(const float* p, float (&v)[EPL]) {
  if constexpr (EPL == 4) {
    const float4 r = __ldcg(reinterpret_cast<const float4*>(p));
    v[0] = r.x; v[1] = r.y; v[2] = r.z; v[3] = r.w;
  } else if constexpr (EPL == 2) {
    const float2 r = __ldcg(reinterpret_cast<const float2*>(p));
    v[0] = r.x; v[1] = r.y;
  } else {
#pragma unroll
    for (int e = 0; e < EPL; e++) v[e] = __ldcg(p + e);
  }
}
template <int EPL>
__device__ __forceinline__ void kv_load_row(const __nv_bfloat16* p, float (&v)[EPL]) {
  if constexpr (EPL == 4) {
    const uint2 raw = __ldcg(reinterpret_cast<const uint2*>(p));
    const __nv_bfloat162 p0 = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 p1 = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    v[0] = __low2float(p0); v[1] = __high2float(p0); v[2] = __low2float(p1); v[3] = __high2float(p1);
  } else if constexpr (EPL == 2) {
    const unsigned int raw = __ldcg(reinterpret_cast<const unsigned int*>(p));
    const __nv_bfloat162 p0 = *reinterpret_cast<const __nv_bfloat162*>(&raw);
    v[0] = __low2float(p0); v[1] = __high2float(p0);
  } else {
#pragma unroll
    for (int e = 0; e < EPL; e++) v[e] = __bfloat162float(__ldcg(p + e));
  }
}

// Compute token m's K (normed, rotated) and V for kv head g and store them at position
// pos of its sequence. One warp; buf is HD floats of shared memory.
template <int HD, typename KT>
__device__ void append_kv(const AttnArgs& a, int m, int seq, int pos, int g, float* buf, int lane) {
  const float* kr = a.qkv + (size_t)m * (a.H + 2 * a.Hkv) * HD + (size_t)(a.H + g) * HD;
  const float* vr = kr + (size_t)a.Hkv * HD;
  for (int e = lane; e < HD; e += 32) buf[e] = ld_cg(kr + e);
  __syncwarp();
  norm_rope_head<HD>(buf, a.kn, a.eps, a.inv_freq, a.interleaved, pos, lane);
  const size_t off = kv_off(a, seq, pos, g, HD);
  for (int e = lane; e < HD; e += 32) {
    kv_store(static_cast<KT*>(a.kbase) + off + e, buf[e]);
    kv_store(static_cast<KT*>(a.vbase) + off + e, ld_cg(vr + e));
  }
}

template <int HD, typename KT>
__global__ void __launch_bounds__(kAttnThreads) k_attention(const AttnArgs a) {
  constexpr int EPL = HD / 32;           // key elements per lane in the score phase
  constexpr int NG = kAttnThreads / HD;  // token groups in the P.V phase
  __shared__ __align__(16) float qs[kMaxGroup][HD];
  __shared__ float sc[kMaxGroup][kSub];
  __shared__ float m_s[kMaxGroup], l_s[kMaxGroup], alpha_s[kMaxGroup];
  __shared__ float accx[NG][kMaxGroup][HD];
  __shared__ float kbuf[HD];
  __shared__ int is_last;

  pdl_launch_dependents();
  pdl_wait();

  const int m = blockIdx.x, g = blockIdx.y, s = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.H / a.Hkv;
  const int seq = a.tok_seq ? ld_cg(a.tok_seq + m) : 0;
  const int pos = a.tok_pos ? ld_cg(a.tok_pos + m) : a.const_pos;
  const int n_keys = pos + 1;
  const int chunk = (n_keys + a.n_split - 1) / a.n_split;
  const int t0 = min(n_keys, s * chunk);
  const int t1 = min(n_keys, t0 + chunk);
  const float scale = a.scale;

  // q heads of this group: norm + rope into shared memory
  const float* qrow = a.qkv + (size_t)m * (a.H + 2 * a.Hkv) * HD;
  for (int i = warp; i < G; i += kWarpsA) {
    const float* src = qrow + (size_t)(g * G + i) * HD;
    for (int e = lane; e < HD; e += 32) qs[i][e] = ld_cg(src + e);
    __syncwarp();
    norm_rope_head<HD>(qs[i], a.qn, a.eps, a.inv_freq, a.interleaved, pos, lane);
  }
  if (a.append && pos >= t0 && pos < t1 && warp == kWarpsA - 1)
    append_kv<HD, KT>(a, m, seq, pos, g, kbuf, lane);
  if (threadIdx.x < kMaxGroup) {
    m_s[threadIdx.x] = -INFINITY;
    l_s[threadIdx.x] = 0.f;
  }
  __syncthreads();

  float acc[kMaxGroup];
#pragma unroll
  for (int i = 0; i < kMaxGroup; i++) acc[i] = 0.f;
  const int e_pv = threadIdx.x % HD, grp = threadIdx.x / HD;

  for (int tb = t0; tb < t1; tb += kSub) {
    const int n = min(kSub, t1 - tb);
    // scores: one key row per warp iteration, lanes split the head dimension
    for (int t = warp; t < n; t += kWarpsA) {
      const KT* kr = static_cast<const KT*>(a.kbase) + kv_off(a, seq, tb + t, g, HD) + lane * EPL;
      float kv[EPL];
      kv_load_row<EPL>(kr, kv);
      for (int i = 0; i < G; i++) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; e++) d = fmaf(qs[i][lane * EPL + e], kv[e], d);
        d = warp_sum(d);
        if (lane == 0) sc[i][t] = __fmul_rn(d, scale);
      }
    }
    __syncthreads();
    // online softmax statistics: one warp per head
    for (int i = warp; i < G; i += kWarpsA) {
      float mx = -INFINITY;
      for (int t = lane; t < n; t += 32) mx = fmaxf(mx, sc[i][t]);
      mx = warp_max(mx);
      const float m_old = m_s[i];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.f;
      for (int t = lane; t < n; t += 32) {
        const float p = expf(sc[i][t] - m_new);
        sc[i][t] = p;
        sum += p;
      }
      sum = warp_sum(sum);
      __syncwarp();
      if (lane == 0) {
        const float al = expf(m_old - m_new);
        alpha_s[i] = al;
        l_s[i] = l_s[i] * al + sum;
        m_s[i] = m_new;
      }
    }
    __syncthreads();
    for (int i = 0; i < G; i++) acc[i] *= alpha_s[i];
    // P.V: thread (e, grp) accumulates keys t == grp (mod NG)
    for (int t = grp; t < n; t += NG) {
      const float v = kv_load(static_cast<const KT*>(a.vbase) + kv_off(a, seq, tb + t, g, HD) + e_pv);
      for (int i = 0; i < G; i++) acc[i] = fmaf(sc[i][t], v, acc[i]);
    }
    __syncthreads();
  }

  if constexpr (NG > 1) {
    for (int i = 0; i < G; i++) accx[grp][i][e_pv] = acc[i];
    __syncthreads();
    if (grp == 0)
      for (int i = 0; i < G; i++) {
        float t = 0.f;
        for (int q = 0; q < NG; q++) t += accx[q][i][e_pv];
        acc[i] = t;
      }
  }

  float* out = a.out + (size_t)m * a.H * HD + (size_t)g * G * HD;
  if (a.n_split == 1) {
    if (grp == 0)
      for (int i = 0; i < G; i++) out[(size_t)i * HD + e_pv] = __fdiv_rn(acc[i], l_s[i]);
    return;
  }

  // split partial: per head [m, l, acc[HD]]
  const size_t stride_h = HD + 2;
  float* part = a.part + (((size_t)m * a.Hkv + g) * a.n_split + s) * G * stride_h;
  if (threadIdx.x < G) {
    part[threadIdx.x * stride_h + 0] = m_s[threadIdx.x];
    part[threadIdx.x * stride_h + 1] = l_s[threadIdx.x];
  }
  if (grp == 0)
    for (int i = 0; i < G; i++) part[i * stride_h + 2 + e_pv] = acc[i];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(&a.counters[(size_t)m * a.Hkv + g], 1);
    is_last = (old == a.n_split - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const float* base = a.part + ((size_t)m * a.Hkv + g) * a.n_split * G * stride_h;
  if (grp == 0) {
    for (int i = 0; i < G; i++) {
      float M = -INFINITY;
      for (int q = 0; q < a.n_split; q++) M = fmaxf(M, __ldcg(base + ((size_t)q * G + i) * stride_h));
      float L = 0.f, O = 0.f;
      for (int q = 0; q < a.n_split; q++) {
        const float* p = base + ((size_t)q * G + i) * stride_h;
        const float w = expf(__ldcg(p) - M);
        L = fmaf(__ldcg(p + 1), w, L);
        O = fmaf(__ldcg(p + 2 + e_pv), w, O);
      }
      out[(size_t)i * HD + e_pv] = __fdiv_rn(O, L);
    }
  }
  if (threadIdx.x == 0) a.counters[(size_t)m * a.Hkv + g] = 0;
}

// Prefill: append the K/V of all M tokens first (tokens of one sequence attend to each
// other, so appends and reads cannot share a launch).
template <int HD, typename KT>
__global__ void __launch_bounds__(32) k_kv_append(const AttnArgs a) {
  __shared__ float buf[HD];
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x, g = blockIdx.y;
  const int seq = a.tok_seq ? ld_cg(a.tok_seq + m) : 0;
  const int pos = a.tok_pos ? ld_cg(a.tok_pos + m) : a.const_pos;
  append_kv<HD, KT>(a, m, seq, pos, g, buf, threadIdx.x);
}

cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, cudaStream_t st, cudaLaunchAttribute* attr) {
  return launch_cfg(grid, block, 0, st, attr);
}

}  // namespace

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st) {
  if (a.H % a.Hkv || a.H / a.Hkv > kMaxGroup || a.n_split < 1 || a.n_split > kMaxSplit)
    return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(a.M, a.Hkv, a.n_split), dim3(kAttnThreads), st, attr);
  switch (a.hd) {
    case 32: return a.kv_f32 ? cudaLaunchKernelEx(&cfg, k_attention<32, float>, a)
                             : cudaLaunchKernelEx(&cfg, k_attention<32, __nv_bfloat16>, a);
    case 64: return a.kv_f32 ? cudaLaunchKernelEx(&cfg, k_attention<64, float>, a)
                             : cudaLaunchKernelEx(&cfg, k_attention<64, __nv_bfloat16>, a);
    case 128: return a.kv_f32 ? cudaLaunchKernelEx(&cfg, k_attention<128, float>, a)
                              : cudaLaunchKernelEx(&cfg, k_attention<128, __nv_bfloat16>, a);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_kv_append(const AttnArgs& a, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(a.M, a.Hkv), dim3(32), st, attr);
  switch (a.hd) {
    case 32: return a.kv_f32 ? cudaLaunchKernelEx(&cfg, k_kv_append<32, float>, a)
                             : cudaLaunchKernelEx(&cfg, k_kv_append<32, __nv_bfloat16>, a);
    case 64: return a.kv_f32 ? cudaLaunchKernelEx(&cfg, k_kv_append<64, float>, a)
                             : cudaLaunchKernelEx(&cfg, k_kv_append<64, __nv_bfloat16>, a);
    case 128: return a.kv_f32 ? cudaLaunchKernelEx(&cfg, k_kv_append<128, float>, a)
                              : cudaLaunchKernelEx(&cfg, k_kv_append<128, __nv_bfloat16>, a);
  }
  return cudaErrorInvalidValue;
}

}  // namespace sx
