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
// One CTA of 8 warps per (token, kv head, split of the key axis); the splits of one
// (token, kv head) form a thread-block cluster. Each warp walks chunks of KC keys inside one
// KV page: one page-table lookup, then the K and V row loads of the whole chunk at once
// (lanes split the head dimension, so every row load is coalesced); the first chunk's loads
// go out before the query work. The KC x G dot products are reduced across lanes in
// independent shuffle chains and folded into an online softmax held in registers. The warps
// are merged through shared memory; the splits are merged by cluster rank 0 reading the
// other CTAs' partials through distributed shared memory after a cluster barrier
// (flash-decoding without a global round trip, atomics or a second pass).
// In decode (append = 1) the CTA whose slice contains the new position computes that
// token's normed, rotated K and V, writes them into the cache for later steps and keeps
// them in shared memory for its own warps, so no CTA reads a slot written in this launch.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "sx_device.cuh"
#include "sx_internal.hpp"

namespace cg = cooperative_groups;

namespace sx {
namespace {

constexpr int kWarpsA = kAttnThreads / 32;

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
// The value a read of the cache element returns after kv_store(p, v).
__device__ __forceinline__ float kv_round(float v, const float*) { return v; }
__device__ __forceinline__ float kv_round(float v, const __nv_bfloat16*) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// EPL consecutive elements of a K/V row starting at p, as f32 (one vector load, L2 only).
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
// pos of its sequence. One warp; buf is HD floats of shared memory. When vbuf is non-null
// the stored values (rounded to KT, as a later read of the cache returns them) are also
// left in buf / vbuf for the CTA's own readers.
template <int HD, typename KT>
__device__ void append_kv(const AttnArgs& a, int m, int seq, int pos, int g, float* buf, int lane,
                          float* vbuf = nullptr) {
  const float* kr = a.qkv + (size_t)m * (a.H + 2 * a.Hkv) * HD + (size_t)(a.H + g) * HD;
  const float* vr = kr + (size_t)a.Hkv * HD;
  for (int e = lane; e < HD; e += 32) buf[e] = ld_cg(kr + e);
  __syncwarp();
  norm_rope_head<HD>(buf, a.kn, a.eps, a.inv_freq, a.interleaved, pos, lane);
  const size_t off = kv_off(a, seq, pos, g, HD);
  for (int e = lane; e < HD; e += 32) {
    KT* kd = static_cast<KT*>(a.kbase) + off + e;
    KT* vd = static_cast<KT*>(a.vbase) + off + e;
    const float v = ld_cg(vr + e);
    kv_store(kd, buf[e]);
    kv_store(vd, v);
    if (vbuf) {
      buf[e] = kv_round(buf[e], kd);
      vbuf[e] = kv_round(v, vd);
    }
  }
}

// One q|k|v row of token m for the decode kernel. With the wqkv GEMV's partials (EPI_NONE) the
// row's k-chunk partials are loaded (all at once, zeros past qkv_nc); otherwise the merged row
// value goes to pv[0]. row < 0: nothing to load.
template <int NC>
__device__ __forceinline__ void qkv_fetch(const AttnArgs& a, int m, int row, float (&pv)[NC]) {
#pragma unroll
  for (int kc = 0; kc < NC; kc++) pv[kc] = 0.f;
  if (row < 0) return;
  if (a.qkv_part) {
    const float* p = a.qkv_part + ((size_t)(row >> 4) * a.qkv_nc * a.qkv_mt + m) * 16 + (row & 15);
#pragma unroll
    for (int kc = 0; kc < NC; kc++)
      if (kc < a.qkv_nc) pv[kc] = __ldcg(p + (size_t)kc * a.qkv_mt * 16);
  } else {
    pv[0] = ld_cg(a.qkv + (size_t)m * (a.H + 2 * a.Hkv) * a.hd + row);
  }
}

// The value k_merge_q8's store epilogue writes for the row (gemv_q8.cu), bit for bit: the
// k-chunks in four contiguous quarters, each added in chunk order starting from zero, the
// quarters added in order, then the bias.
template <int NC>
__device__ __forceinline__ float qkv_value(const AttnArgs& a, int row, const float (&pv)[NC]) {
  if (!a.qkv_part) return pv[0];
  float q[4];
#pragma unroll
  for (int qi = 0; qi < 4; qi++) {
    const int k0 = qi * a.qkv_nc / 4, k1 = (qi + 1) * a.qkv_nc / 4;
    float s = 0.f;
#pragma unroll
    for (int kc = 0; kc < NC; kc++)
      if (kc >= k0 && kc < k1) s += pv[kc];
    q[qi] = s;
  }
  float v = ((q[0] + q[1]) + q[2]) + q[3];
  if (a.qkv_bias) v = __fadd_rn(v, a.qkv_bias[row]);
  return v;
}

// Decode append: the token's raw K (kbuf) is normed and rotated, K and V are stored at
// position pos of its sequence, and kbuf / vbuf are left holding what a later read of the
// cache returns (rounded to KT). One warp.
template <int HD, typename KT>
__device__ void store_new_kv(const AttnArgs& a, int seq, int pos, int g, float* kbuf, float* vbuf, int lane) {
  norm_rope_head<HD>(kbuf, a.kn, a.eps, a.inv_freq, a.interleaved, pos, lane);
  const size_t off = kv_off(a, seq, pos, g, HD);
  for (int e = lane; e < HD; e += 32) {
    KT* kd = static_cast<KT*>(a.kbase) + off + e;
    KT* vd = static_cast<KT*>(a.vbase) + off + e;
    const float v = vbuf[e];
    kv_store(kd, kbuf[e]);
    kv_store(vd, v);
    kbuf[e] = kv_round(kbuf[e], kd);
    vbuf[e] = kv_round(v, vd);
  }
}

// GM: compile-time bound on the query heads per kv head (the loops over heads unroll and
// predicate on the runtime G <= GM).
template <int HD, typename KT, int GM>
__global__ void __launch_bounds__(kAttnThreads) k_attention(const AttnArgs a) {
  constexpr int EPL = HD / 32;          // head elements per lane
  constexpr int KC = GM <= 4 ? 8 : 4;   // keys per warp chunk
  __shared__ __align__(16) float qs[GM][HD];
  __shared__ __align__(16) float wacc[kWarpsA][GM][HD];
  __shared__ float wm[kWarpsA][GM], wl[kWarpsA][GM];
  __shared__ float kbuf[HD], vbuf[HD];
  __shared__ __align__(16) float co[GM][HD];  // this split's partial, read by cluster rank 0
  __shared__ float cm[GM], cl[GM];

  pdl_launch_dependents();
  pdl_wait();

  const int m = blockIdx.x, g = blockIdx.y, s = blockIdx.z;
  const int n_split = gridDim.z;  // the splits of (m, g) are one cluster along z
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.H / a.Hkv;
  // q of the group's heads, one element per thread and step: these loads do not depend on
  // the position, so they go out first
  constexpr int NQJ = (GM * HD + kAttnThreads - 1) / kAttnThreads;
  constexpr int NKJ = (2 * HD + kAttnThreads - 1) / kAttnThreads;
  const int nq = G * HD;
  float qp[NQJ][kQkvChunks];
#pragma unroll
  for (int j = 0; j < NQJ; j++) {
    const int idx = threadIdx.x + j * kAttnThreads;
    qkv_fetch<kQkvChunks>(a, m, idx < nq ? g * G * HD + idx : -1, qp[j]);
  }
  const int seq = a.tok_seq ? ld_cg(a.tok_seq + m) : 0;
  const int pos = a.tok_pos ? ld_cg(a.tok_pos + m) : a.const_pos;
  const int n_keys = pos + 1;
  // split lengths are whole chunks, so a chunk never straddles a KV page (kPage % KC == 0)
  const int chunk = ((n_keys + n_split - 1) / n_split + KC - 1) / KC * KC;
  const int t0 = min(n_keys, s * chunk);
  const int t1 = min(n_keys, t0 + chunk);
  const int n_chunks = (t1 - t0 + KC - 1) / KC;
  // in decode the new key is read back from shared memory (the append below), not the cache
  const bool own_new = a.append && pos >= t0 && pos < t1;

  const KT* kb = static_cast<const KT*>(a.kbase);
  const KT* vb = static_cast<const KT*>(a.vbase);
  float kv[KC][EPL], vv[KC][EPL];
  // K/V rows of chunk c: one page-table lookup, KC coalesced row loads each for K and V
  auto load_chunk = [&](int c) {
    const int base = t0 + c * KC;
    const int page = ld_cg(a.page_table + (size_t)seq * a.pt_stride + base / kPage);
    const size_t row0 = ((size_t)(page * a.Hkv + g) * kPage + (base % kPage)) * HD + lane * EPL;
#pragma unroll
    for (int j = 0; j < KC; j++) {
      if (base + j < t1 && !(own_new && base + j == pos)) {
        kv_load_row<EPL>(kb + row0 + (size_t)j * HD, kv[j]);
        kv_load_row<EPL>(vb + row0 + (size_t)j * HD, vv[j]);
      } else {
#pragma unroll
        for (int e = 0; e < EPL; e++) kv[j][e] = vv[j][e] = 0.f;
      }
    }
  };
  // the first chunk's loads go out before the query work, so their latency overlaps it
  if (warp < n_chunks) load_chunk(warp);

  // the new token's raw K and V, for the CTA that appends them
  float kp[NKJ][kQkvChunks];
#pragma unroll
  for (int j = 0; j < NKJ; j++) {
    const int idx = threadIdx.x + j * kAttnThreads;
    const int row = !own_new || idx >= 2 * HD ? -1
                    : idx < HD               ? (a.H + g) * HD + idx
                                             : (a.H + a.Hkv + g) * HD + (idx - HD);
    qkv_fetch<kQkvChunks>(a, m, row, kp[j]);
  }
  float* qflat = &qs[0][0];  // head i, element e at i * HD + e
#pragma unroll
  for (int j = 0; j < NQJ; j++) {
    const int idx = threadIdx.x + j * kAttnThreads;
    if (idx < nq) qflat[idx] = qkv_value<kQkvChunks>(a, g * G * HD + idx, qp[j]);
  }
#pragma unroll
  for (int j = 0; j < NKJ; j++) {
    const int idx = threadIdx.x + j * kAttnThreads;
    if (own_new && idx < 2 * HD) {
      if (idx < HD)
        kbuf[idx] = qkv_value<kQkvChunks>(a, (a.H + g) * HD + idx, kp[j]);
      else
        vbuf[idx - HD] = qkv_value<kQkvChunks>(a, (a.H + a.Hkv + g) * HD + (idx - HD), kp[j]);
    }
  }
  __syncthreads();

  // q heads of this group: norm + rope in shared memory; the appending CTA's last warp
  // stores the new K / V
  for (int i = warp; i < G; i += kWarpsA)
    norm_rope_head<HD>(qs[i], a.qn, a.eps, a.inv_freq, a.interleaved, pos, lane);
  if (own_new && warp == kWarpsA - 1) store_new_kv<HD, KT>(a, seq, pos, g, kbuf, vbuf, lane);
  __syncthreads();

  float qv[GM][EPL];
#pragma unroll
  for (int i = 0; i < GM; i++)
#pragma unroll
    for (int e = 0; e < EPL; e++) qv[i][e] = i < G ? qs[i][lane * EPL + e] : 0.f;
  float m_w[GM], l_w[GM], acc[GM][EPL];
#pragma unroll
  for (int i = 0; i < GM; i++) {
    m_w[i] = -INFINITY;
    l_w[i] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; e++) acc[i][e] = 0.f;
  }

  for (int c = warp; c < n_chunks; c += kWarpsA) {
    const int base = t0 + c * KC;
    if (c != warp) load_chunk(c);
    if (own_new) {
#pragma unroll
      for (int j = 0; j < KC; j++)
        if (base + j == pos)
#pragma unroll
          for (int e = 0; e < EPL; e++) {
            kv[j][e] = kbuf[lane * EPL + e];
            vv[j][e] = vbuf[lane * EPL + e];
          }
    }
    float sc[KC][GM];
#pragma unroll
    for (int j = 0; j < KC; j++)
#pragma unroll
      for (int i = 0; i < GM; i++) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; e++) d = fmaf(qv[i][e], kv[j][e], d);
        sc[j][i] = d;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int j = 0; j < KC; j++)
#pragma unroll
        for (int i = 0; i < GM; i++) sc[j][i] += __shfl_xor_sync(0xffffffffu, sc[j][i], o);
#pragma unroll
    for (int i = 0; i < GM; i++) {
      float cmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < KC; j++) {
        sc[j][i] = base + j < t1 ? __fmul_rn(sc[j][i], a.scale) : -INFINITY;
        cmax = fmaxf(cmax, sc[j][i]);
      }
      const float m_new = fmaxf(m_w[i], cmax);
      const float alpha = expf(m_w[i] - m_new);
      float lsum = l_w[i] * alpha;
#pragma unroll
      for (int e = 0; e < EPL; e++) acc[i][e] *= alpha;
#pragma unroll
      for (int j = 0; j < KC; j++) {
        const float p = base + j < t1 ? expf(sc[j][i] - m_new) : 0.f;
        lsum += p;
#pragma unroll
        for (int e = 0; e < EPL; e++) acc[i][e] = fmaf(p, vv[j][e], acc[i][e]);
      }
      l_w[i] = lsum;
      m_w[i] = m_new;
    }
  }

  // merge the warps of this CTA
#pragma unroll
  for (int i = 0; i < GM; i++) {
    if (lane == 0) {
      wm[warp][i] = m_w[i];
      wl[warp][i] = l_w[i];
    }
#pragma unroll
    for (int e = 0; e < EPL; e++) wacc[warp][i][lane * EPL + e] = acc[i][e];
  }
  __syncthreads();
  const int e_t = threadIdx.x % HD;   // element handled by this thread in the merges
  const int i_t0 = threadIdx.x / HD;  // first head handled by this thread
  constexpr int HSTEP = kAttnThreads / HD;
  float cta_m[GM], cta_l[GM], cta_o[GM];
#pragma unroll
  for (int i = 0; i < GM; i++) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarpsA; w++) M = fmaxf(M, wm[w][i]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarpsA; w++) {
        const float f = expf(wm[w][i] - M);
        L = fmaf(wl[w][i], f, L);
        O = fmaf(wacc[w][i][e_t], f, O);
      }
    }
    cta_m[i] = M;
    cta_l[i] = L;
    cta_o[i] = O;
  }

  float* out = a.out + (size_t)m * a.H * HD + (size_t)g * G * HD;
  if (n_split == 1) {
#pragma unroll
    for (int i = 0; i < GM; i++)
      if (i < G && (i % HSTEP) == i_t0) out[(size_t)i * HD + e_t] = __fdiv_rn(cta_o[i], cta_l[i]);
    return;
  }

  // this split's partial per head (m, l, acc[HD]) stays in shared memory; cluster rank 0
  // merges the splits in rank order through distributed shared memory
#pragma unroll
  for (int i = 0; i < GM; i++)
    if (i < G && (i % HSTEP) == i_t0) {
      if (e_t == 0) {
        cm[i] = cta_m[i];
        cl[i] = cta_l[i];
      }
      co[i][e_t] = cta_o[i];
    }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();  // every split's partial is visible to the cluster
  if (cluster.block_rank() == 0) {
#pragma unroll
    for (int i = 0; i < GM; i++)
      if (i < G && (i % HSTEP) == i_t0) {
        float M = -INFINITY;
        for (int r = 0; r < n_split; r++) M = fmaxf(M, *cluster.map_shared_rank(&cm[i], r));
        float L = 0.f, O = 0.f;
        for (int r = 0; r < n_split; r++) {
          const float w = expf(*cluster.map_shared_rank(&cm[i], r) - M);
          L = fmaf(*cluster.map_shared_rank(&cl[i], r), w, L);
          O = fmaf(*cluster.map_shared_rank(&co[i][e_t], r), w, O);
        }
        out[(size_t)i * HD + e_t] = __fdiv_rn(O, L);
      }
  }
  cluster.sync();  // no CTA leaves while rank 0 still reads its shared memory
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


// ---- prefill attention ------------------------------------------------------------------
// Causal attention of a prompt chunk (M tokens of ONE sequence, consecutive positions) whose
// K/V k_kv_append has already written. One CTA per (query tile of kPfTq tokens, kv head): its
// GM x kPfTq query rows (QK-normed and rotated once, in shared memory) share every tile of
// kPfKeys keys and values staged in shared memory, where the decode kernel re-reads the keys
// once per token. Per key tile: scores R x kPfKeys (each thread one key for R/4 rows, f32
// FMAs over the head dimension), an online softmax per row (one warp per row), then
// O += P.V (each thread R/8 rows x 4 elements). f32 throughout, as the decode path.
constexpr int kPfTq = 4;     // query tokens per CTA
constexpr int kPfKeys = 64;  // keys per shared-memory tile (one KV page)

template <int HD, int R>
struct PfSmem {
  float q[R][HD];
  float k[kPfKeys][HD + 4];  // padded rows: a quarter-warp's 16-byte loads hit distinct banks
  float v[kPfKeys][HD];
  float p[R][kPfKeys];
  float m[R], l[R], alpha[R];
};

template <int HD, typename KT, int GM>
__global__ void __launch_bounds__(256) k_attn_prefill(const AttnArgs a) {
  constexpr int R = GM * kPfTq;   // query rows: row = token * GM + head
  constexpr int RQ = R / 4;       // rows per thread in the scores (4 row groups of 64 threads)
  constexpr int RO = R / 8;       // rows per thread in P.V (8 warps)
  constexpr int EPL = HD / 32;
  extern __shared__ __align__(16) unsigned char pf_raw[];
  PfSmem<HD, R>& sm = *reinterpret_cast<PfSmem<HD, R>*>(pf_raw);
  pdl_launch_dependents();
  pdl_wait();
  const int tile = blockIdx.x, g = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.H / a.Hkv;
  const int m0 = tile * kPfTq;
  const int n_tok = min(kPfTq, a.M - m0);
  const int seq = ld_cg(a.tok_seq + m0);
  int qpos[kPfTq];
  int last = 0;  // the tile's last query position: keys beyond it are never read
#pragma unroll
  for (int j = 0; j < kPfTq; j++) {
    qpos[j] = j < n_tok ? ld_cg(a.tok_pos + m0 + j) : -1;
    last = max(last, qpos[j]);
  }

  // query rows: load, QK-norm, RoPE (one warp per row)
  for (int r = warp; r < R; r += 8) {
    const int j = r / GM, i = r % GM;
    if (j < n_tok && i < G) {
      const float* src = a.qkv + (size_t)(m0 + j) * (a.H + 2 * a.Hkv) * HD + (size_t)(g * G + i) * HD;
      for (int e = lane; e < HD; e += 32) sm.q[r][e] = ld_cg(src + e);
      __syncwarp();
      norm_rope_head<HD>(sm.q[r], a.qn, a.eps, a.inv_freq, a.interleaved, qpos[j], lane);
    } else {
      for (int e = lane; e < HD; e += 32) sm.q[r][e] = 0.f;
    }
    if (lane == 0) {
      sm.m[r] = -INFINITY;
      sm.l[r] = 0.f;
    }
  }
  float acc[RO][4];
#pragma unroll
  for (int i = 0; i < RO; i++)
#pragma unroll
    for (int e = 0; e < 4; e++) acc[i][e] = 0.f;
  const KT* kb = static_cast<const KT*>(a.kbase);
  const KT* vb = static_cast<const KT*>(a.vbase);
  const int key = threadIdx.x & (kPfKeys - 1), rg = threadIdx.x / kPfKeys;  // scores: key, row group
  const int d0 = (threadIdx.x & 31) * 4;  // P.V: 4 elements (HD = 128; at HD = 64 / 32 lanes past HD idle)

  for (int k0 = 0; k0 <= last; k0 += kPfKeys) {
    __syncthreads();  // the previous tile's readers are done
    {  // stage the tile's keys and values (one page) as f32
      const int page = ld_cg(a.page_table + (size_t)seq * a.pt_stride + k0 / kPage);
      const size_t base = ((size_t)(page * a.Hkv + g) * kPage) * HD;
      for (int kk = warp; kk < kPfKeys; kk += 8) {
        float kv[EPL], vv[EPL];
        if (k0 + kk <= last) {
          kv_load_row<EPL>(kb + base + (size_t)kk * HD + lane * EPL, kv);
          kv_load_row<EPL>(vb + base + (size_t)kk * HD + lane * EPL, vv);
        } else {
#pragma unroll
          for (int e = 0; e < EPL; e++) kv[e] = vv[e] = 0.f;
        }
#pragma unroll
        for (int e = 0; e < EPL; e++) {
          sm.k[kk][lane * EPL + e] = kv[e];
          sm.v[kk][lane * EPL + e] = vv[e];
        }
      }
    }
    __syncthreads();
    {  // scores of this thread's key for rows rg * RQ .. + RQ
      float sc[RQ];
#pragma unroll
      for (int i = 0; i < RQ; i++) sc[i] = 0.f;
#pragma unroll 4
      for (int d = 0; d < HD; d += 4) {
        const float4 kq = *reinterpret_cast<const float4*>(&sm.k[key][d]);
#pragma unroll
        for (int i = 0; i < RQ; i++) {
          const float4 qq = *reinterpret_cast<const float4*>(&sm.q[rg * RQ + i][d]);
          sc[i] = fmaf(qq.x, kq.x, sc[i]);
          sc[i] = fmaf(qq.y, kq.y, sc[i]);
          sc[i] = fmaf(qq.z, kq.z, sc[i]);
          sc[i] = fmaf(qq.w, kq.w, sc[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < RQ; i++) {
        const int r = rg * RQ + i, j = r / GM;
        const bool ok = j < n_tok && k0 + key <= qpos[j];
        sm.p[r][key] = ok ? __fmul_rn(sc[i], a.scale) : -INFINITY;
      }
    }
    __syncthreads();
    // online softmax per row: one warp per row, two keys per lane
    for (int r = warp; r < R; r += 8) {
      const float s0 = sm.p[r][lane], s1 = sm.p[r][lane + 32];
      const float mx = warp_max(fmaxf(s0, s1));
      const float m_old = sm.m[r];
      const float m_new = fmaxf(m_old, mx);
      const float e0 = m_new == -INFINITY ? 0.f : expf(s0 - m_new);
      const float e1 = m_new == -INFINITY ? 0.f : expf(s1 - m_new);
      sm.p[r][lane] = e0;
      sm.p[r][lane + 32] = e1;
      const float sum = warp_sum(e0 + e1);
      if (lane == 0) {
        const float al = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
        sm.alpha[r] = al;
        sm.l[r] = __fadd_rn(__fmul_rn(sm.l[r], al), sum);
        sm.m[r] = m_new;
      }
    }
    __syncthreads();
    if (d0 < HD) {  // O = O * alpha + P.V for rows warp * RO .. + RO, elements d0 .. d0 + 3
#pragma unroll
      for (int i = 0; i < RO; i++) {
        const float al = sm.alpha[warp * RO + i];
#pragma unroll
        for (int e = 0; e < 4; e++) acc[i][e] *= al;
      }
#pragma unroll 4
      for (int kk = 0; kk < kPfKeys; kk++) {
        const float4 vq = *reinterpret_cast<const float4*>(&sm.v[kk][d0]);
#pragma unroll
        for (int i = 0; i < RO; i++) {
          const float pr = sm.p[warp * RO + i][kk];
          acc[i][0] = fmaf(pr, vq.x, acc[i][0]);
          acc[i][1] = fmaf(pr, vq.y, acc[i][1]);
          acc[i][2] = fmaf(pr, vq.z, acc[i][2]);
          acc[i][3] = fmaf(pr, vq.w, acc[i][3]);
        }
      }
    }
  }
  __syncthreads();
  if (d0 < HD) {
#pragma unroll
    for (int i = 0; i < RO; i++) {
      const int r = warp * RO + i, j = r / GM, h = r % GM;
      if (j < n_tok && h < G) {
        float* out = a.out + (size_t)(m0 + j) * a.H * HD + (size_t)(g * G + h) * HD + d0;
        const float L = sm.l[r];
#pragma unroll
        for (int e = 0; e < 4; e++) out[e] = __fdiv_rn(acc[i][e], L);
      }
    }
  }
}

template <int HD, typename KT, int GM>
cudaError_t launch_pf_t(const AttnArgs& a, cudaStream_t st) {
  auto kern = k_attn_prefill<HD, KT, GM>;
  const size_t smem = sizeof(PfSmem<HD, GM * kPfTq>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = launch_cfg(dim3((a.M + kPfTq - 1) / kPfTq, a.Hkv), dim3(256), smem, st, attr);
  return cudaLaunchKernelEx(&cfg, kern, a);
}
template <int HD, typename KT>
cudaError_t launch_pf_hd(const AttnArgs& a, cudaStream_t st) {
  const int G = a.H / a.Hkv;
  if (G <= 2) return launch_pf_t<HD, KT, 2>(a, st);
  if (G <= 4) return launch_pf_t<HD, KT, 4>(a, st);
  return launch_pf_t<HD, KT, 8>(a, st);
}

template <int HD, typename KT>
cudaError_t launch_attention_hd(const AttnArgs& a, cudaLaunchConfig_t& cfg) {
  const int G = a.H / a.Hkv;
  if (G <= 1) return cudaLaunchKernelEx(&cfg, k_attention<HD, KT, 1>, a);
  if (G <= 2) return cudaLaunchKernelEx(&cfg, k_attention<HD, KT, 2>, a);
  if (G <= 4) return cudaLaunchKernelEx(&cfg, k_attention<HD, KT, 4>, a);
  return cudaLaunchKernelEx(&cfg, k_attention<HD, KT, 8>, a);
}

}  // namespace

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st) {
  if (a.H % a.Hkv || a.H / a.Hkv > kMaxGroup || a.n_split < 1 || a.n_split > kMaxCluster)
    return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = launch_cfg(dim3(a.M, a.Hkv, a.n_split), dim3(kAttnThreads), 0, st, attr);
  if (a.n_split > 1) {  // the splits of one (token, kv head) form a cluster
    cudaLaunchAttribute& c = attr[cfg.numAttrs++];
    c.id = cudaLaunchAttributeClusterDimension;
    c.val.clusterDim.x = 1;
    c.val.clusterDim.y = 1;
    c.val.clusterDim.z = (unsigned)a.n_split;
  }
  switch (a.hd) {
    case 32: return a.kv_f32 ? launch_attention_hd<32, float>(a, cfg) : launch_attention_hd<32, __nv_bfloat16>(a, cfg);
    case 64: return a.kv_f32 ? launch_attention_hd<64, float>(a, cfg) : launch_attention_hd<64, __nv_bfloat16>(a, cfg);
    case 128:
      return a.kv_f32 ? launch_attention_hd<128, float>(a, cfg) : launch_attention_hd<128, __nv_bfloat16>(a, cfg);
  }
  return cudaErrorInvalidValue;
}

// Prefill chunks (append = 0) of one sequence: the tiled kernel above. Its K/V must already be
// in the cache (launch_kv_append).
cudaError_t launch_attention_prefill(const AttnArgs& a, cudaStream_t st) {
  if (a.H % a.Hkv || a.H / a.Hkv > kMaxGroup || a.append || !a.tok_seq || !a.tok_pos || a.M < 1)
    return cudaErrorInvalidValue;
  switch (a.hd) {
    case 32: return a.kv_f32 ? launch_pf_hd<32, float>(a, st) : launch_pf_hd<32, __nv_bfloat16>(a, st);
    case 64: return a.kv_f32 ? launch_pf_hd<64, float>(a, st) : launch_pf_hd<64, __nv_bfloat16>(a, st);
    case 128: return a.kv_f32 ? launch_pf_hd<128, float>(a, st) : launch_pf_hd<128, __nv_bfloat16>(a, st);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_kv_append(const AttnArgs& a, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = launch_cfg(dim3(a.M, a.Hkv), dim3(32), 0, st, attr);
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
