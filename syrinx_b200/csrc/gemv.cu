// gemv.cu — fused dequant-GEMV for decode: y = x . W^T over Q4_K / F32 weights (Q8_0
// weights take the tensor-core kernel of gemv_q8.cu).
//
// Replaces the quantized linear of the reference hot path (`Weights::linear`,
// crates/syrinx-fish/src/s2/nn.rs:61-68; `Qwen2Lm::linear` over candle QMatMul,
// crates/syrinx-lm/src/cv2/mod.rs:195-211) at M = 1..8 tokens per launch (longer prefill
// chunks are split into launches of up to 8), with the neighbouring
// element-wise ops fused in:
//   prologue  RMSNorm of x with a gain vector (rms_norm_w, s2/nn.rs:100-106)
//   epilogue  + bias, residual add (s2/slow_ar.rs:195,198), SiLU(g)*u (s2/nn.rs:452-457),
//             or the greedy argmax of the head (sampling.rs:189-245 with top_k = 1).
//
// Memory-bound design (one pass over the weights at the HBM roofline):
//   * persistent grid: 1-2 CTAs of 8 warps per SM, each CTA owning a contiguous,
//     balanced range of row groups (RPW rows), so x is staged (and RMS-normalised) once per
//     CTA and every SM streams the same number of bytes;
//   * the CTA's work is split into items (row group, 512-element k-chunk); each warp takes a
//     contiguous run of items and streams them with 128-bit ld.global.nc.L1::no_allocate
//     loads, ping-ponging two register buffers so the next item's weights are in flight
//     while the current one is multiplied;
//   * Q4_K values are unpacked in registers (byte-permute into the 2^23 mantissa,
//     exact) and multiplied on the packed f32x2 FMA pipe against x in shared memory;
//   * a warp-shuffle reduction per run of items, partial sums per (row, k-chunk) in shared
//     memory, then a fixed-order sum in the epilogue (deterministic for a given grid);
//   * the first weight items are requested before griddepcontrol.wait, so under
//     programmatic dependent launch they stream while the producer of x drains.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>

#include "sx_device.cuh"
#include "sx_internal.hpp"

namespace sx {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

// Elements covered by one lane-chunk (16 bytes of packed weights).
template <int WT> struct Unit;
template <> struct Unit<SX_DTYPE_Q4_K> { static constexpr int elems = 32; };
template <> struct Unit<SX_DTYPE_F32> { static constexpr int elems = 4; };

template <int WT> struct Frag;
template <> struct Frag<SX_DTYPE_Q4_K> {
  uint4 q;
  uint4 meta;
};
template <> struct Frag<SX_DTYPE_F32> {
  uint4 q;
};

__device__ __forceinline__ int phys_row(const GemvArgs& a, int i) {
  return i < a.n_range ? a.row_base + i : a.extra[i - a.n_range];
}

template <int WT>
__device__ __forceinline__ void load_frag(const GemvArgs& a, int prow, int unit, Frag<WT>& f) {
  const int64_t K = a.w.cols;
  if constexpr (WT == SX_DTYPE_Q4_K) {
    const uint8_t* q = (const uint8_t*)a.w.q + (size_t)prow * (K / 2) + (size_t)unit * 16;
    f.q = ldg_stream(q);
    f.meta = __ldg((const uint4*)(a.w.meta + ((size_t)prow * (K / 256) + (unit >> 3)) * 16));
  } else {
    const float* q = (const float*)a.w.q + (size_t)prow * K + (size_t)unit * 4;
    f.q = ldg_stream(q);
  }
}

// Q4_K 6-bit sub-block scale / min of sub-block j from the 12 packed bytes.
__device__ __forceinline__ void q4k_sm(const uint8_t* sc12, int j, float& sc, float& m) {
  uint32_t s, mm;
  if (j < 4) {
    s = sc12[j] & 63;
    mm = sc12[j + 4] & 63;
  } else {
    s = (sc12[j + 4] & 0xF) | ((sc12[j - 4] >> 6) << 4);
    mm = (sc12[j + 4] >> 4) | ((sc12[j] >> 6) << 4);
  }
  sc = (float)s;
  m = (float)mm;
}

// x fragment of one lane-unit for M tokens (read from shared memory once, shared by the
// RPW rows of a row group).
template <int WT, int M> struct XFrag;
template <int M> struct XFrag<SX_DTYPE_Q4_K, M> {
  ulonglong2 lo[M][4], hi[M][4];  // the low- and high-nibble runs of 16 elements
  float slo[M], shi[M];           // their sums (for the sub-block minimum term)
};
template <int M> struct XFrag<SX_DTYPE_F32, M> {
  ulonglong2 v[M];  // 4 f32 as 2 f32x2
};

// Q4_K unit u: super-block u/8, 16-byte chunk c = u%8 -> 64-group c/2, offset 16*(c%2)
__device__ __forceinline__ int q4k_elem_lo(int unit) {
  const int c = unit & 7;
  return (unit >> 3) * 256 + (c >> 1) * 64 + (c & 1) * 16;
}

template <int WT, int M>
__device__ __forceinline__ void load_x(const float* xs, int K, int unit, const float* xsum16, XFrag<WT, M>& x) {
#pragma unroll
  for (int m = 0; m < M; m++) {
    if constexpr (WT == SX_DTYPE_Q4_K) {
      const int e = q4k_elem_lo(unit);
      const ulonglong2* pl = (const ulonglong2*)(xs + (size_t)m * K + e);
      const ulonglong2* ph = (const ulonglong2*)(xs + (size_t)m * K + e + 32);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        x.lo[m][j] = pl[j];
        x.hi[m][j] = ph[j];
      }
      x.slo[m] = xsum16[(size_t)m * (K / 16) + (e >> 4)];
      x.shi[m] = xsum16[(size_t)m * (K / 16) + ((e + 32) >> 4)];
    } else {
      x.v[m] = *(const ulonglong2*)(xs + (size_t)m * K + unit * 4);
    }
  }
}

// Dot of one weight fragment with the x fragment of M tokens, accumulated into acc.
template <int WT, int M>
__device__ __forceinline__ void frag_dot(const Frag<WT>& f, const XFrag<WT, M>& x, int unit, float (&acc)[M]) {
  if constexpr (WT == SX_DTYPE_Q4_K) {
    const int jj = (unit & 7) >> 1;
    const __half2 dd = *reinterpret_cast<const __half2*>(&f.meta.x);
    const float d = __low2float(dd), dmin = __high2float(dd);
    const uint8_t* sc12 = reinterpret_cast<const uint8_t*>(&f.meta) + 4;
    float sc_lo, m_lo, sc_hi, m_hi;
    q4k_sm(sc12, 2 * jj, sc_lo, m_lo);
    q4k_sm(sc12, 2 * jj + 1, sc_hi, m_hi);
    const float dl = d * sc_lo, ml = dmin * m_lo, dh = d * sc_hi, mh = dmin * m_hi;
    unsigned long long wl[8], wh[8];
    const uint32_t words[4] = {f.q.x, f.q.y, f.q.z, f.q.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      u4x4_to_f32x2x2(words[j] & 0x0F0F0F0Fu, wl[2 * j], wl[2 * j + 1]);
      u4x4_to_f32x2x2((words[j] >> 4) & 0x0F0F0F0Fu, wh[2 * j], wh[2 * j + 1]);
    }
#pragma unroll
    for (int m = 0; m < M; m++) {
      unsigned long long sl = 0, sh = 0;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        sl = fma2(wl[2 * j], x.lo[m][j].x, sl);
        sl = fma2(wl[2 * j + 1], x.lo[m][j].y, sl);
        sh = fma2(wh[2 * j], x.hi[m][j].x, sh);
        sh = fma2(wh[2 * j + 1], x.hi[m][j].y, sh);
      }
      float a0, a1, b0, b1;
      unpack2(sl, a0, a1);
      unpack2(sh, b0, b1);
      float r = dl * (a0 + a1) - ml * x.slo[m];
      r += dh * (b0 + b1) - mh * x.shi[m];
      acc[m] += r;
    }
  } else {
    const unsigned long long w0 = pack2u(f.q.x, f.q.y), w1 = pack2u(f.q.z, f.q.w);
#pragma unroll
    for (int m = 0; m < M; m++) {
      unsigned long long s = fma2(w0, x.v[m].x, 0ull);
      s = fma2(w1, x.v[m].y, s);
      float a0, a1;
      unpack2(s, a0, a1);
      acc[m] += a0 + a1;
    }
  }
}

// Per-CTA work geometry shared by the loader, the compute loop and the epilogue.
struct Geo {
  int K, units, n_kc, n_logical, rg0, rg1, it0, it1;
};

// Walk of a warp's items: (row group, k-chunk) advanced without divisions.
struct Cursor {
  int rg, kc, left;
};

template <int WT, int RPW>
__device__ __forceinline__ void row_ptrs(const GemvArgs& a, const Geo& g, int rg, int (&prow)[RPW]) {
#pragma unroll
  for (int r = 0; r < RPW; r++) {
    const int i = rg * RPW + r;
    prow[r] = phys_row(a, i < g.n_logical ? i : g.n_logical - 1);
  }
}

// Issue the loads of the next B items of the warp (those still to load).
template <int WT, int RPW, int B>
__device__ __forceinline__ void load_group(const GemvArgs& a, const Geo& g, Cursor& c, int (&prow)[RPW], int& prow_rg,
                                           int lane, Frag<WT> (&f)[B][RPW]) {
#pragma unroll
  for (int b = 0; b < B; b++) {
    if (c.left > 0) {
      if (c.rg != prow_rg) {
        row_ptrs<WT, RPW>(a, g, c.rg, prow);
        prow_rg = c.rg;
      }
      const int unit = c.kc * 32 + lane;
      if (unit < g.units)
#pragma unroll
        for (int r = 0; r < RPW; r++) load_frag<WT>(a, prow[r], unit, f[b][r]);
      if (++c.kc == g.n_kc) {
        c.kc = 0;
        c.rg++;
      }
      c.left--;
    }
  }
}

// Flush a run of items of row group rg (started at k-chunk kc0) into the partial sums.
template <int RPW, int M>
__device__ __forceinline__ void flush(float (&acc)[RPW][M], float* part, const Geo& g, int rg, int kc0, int lane) {
#pragma unroll
  for (int r = 0; r < RPW; r++)
#pragma unroll
    for (int m = 0; m < M; m++) {
      const float v = warp_sum(acc[r][m]);
      if (lane == 0) part[(((rg - g.rg0) * RPW + r) * g.n_kc + kc0) * M + m] = v;
      acc[r][m] = 0.f;
    }
}

template <int WT, int M, int RPW, int B>
__device__ __forceinline__ void compute_group(const Geo& g, Cursor& c, int lane, const Frag<WT> (&f)[B][RPW],
                                              const float* xs, const float* xsum16, float* part,
                                              float (&acc)[RPW][M], int& cur_rg, int& run_kc0) {
#pragma unroll
  for (int b = 0; b < B; b++) {
    if (c.left > 0) {
      if (c.rg != cur_rg) {
        if (cur_rg >= 0) flush<RPW, M>(acc, part, g, cur_rg, run_kc0, lane);
        cur_rg = c.rg;
        run_kc0 = c.kc;
      }
      const int unit = c.kc * 32 + lane;
      if (unit < g.units) {
        XFrag<WT, M> x;
        load_x<WT, M>(xs, g.K, unit, xsum16, x);
#pragma unroll
        for (int r = 0; r < RPW; r++) frag_dot<WT, M>(f[b][r], x, unit, acc[r]);
      }
      if (++c.kc == g.n_kc) {
        c.kc = 0;
        c.rg++;
      }
      c.left--;
    }
  }
}
template <int WT, int M, int RPW, int B, int EPI>
__global__ void __launch_bounds__(kThreads, 1) k_gemv(const GemvArgs a) {
  extern __shared__ __align__(16) float smem[];
  constexpr int UE = Unit<WT>::elems;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  Geo g;
  g.K = (int)a.w.cols;
  g.units = g.K / UE;
  g.n_kc = (g.units + 31) / 32;
  g.n_logical = a.n_range + a.n_extra;
  const int n_rg = (g.n_logical + RPW - 1) / RPW;
  g.rg0 = (int)((long long)blockIdx.x * n_rg / gridDim.x);
  g.rg1 = (int)((long long)(blockIdx.x + 1) * n_rg / gridDim.x);
  const int n_items = (g.rg1 - g.rg0) * g.n_kc;
  g.it0 = (int)((long long)warp * n_items / kWarps);
  g.it1 = (int)((long long)(warp + 1) * n_items / kWarps);

  pdl_launch_dependents();

  // The first weight items do not depend on the previous kernel: request them now.
  Cursor lc{g.rg0 + g.it0 / g.n_kc, g.it0 % g.n_kc, g.it1 - g.it0};
  Cursor cc = lc;
  int prow[RPW], prow_rg = -1;
  Frag<WT> fa[B][RPW], fb[B][RPW];
  load_group<WT, RPW, B>(a, g, lc, prow, prow_rg, lane, fa);

  pdl_wait();

  // ---- shared memory: x [M][K] | xsum16 [M][K/16] (Q4_K) | partials [rows][n_kc][M] ----
  float* xs = smem;
  float* xsum16 = xs + (size_t)M * g.K;
  float* part = xsum16 + (WT == SX_DTYPE_Q4_K ? (size_t)M * (g.K / 16) : 0);
  const int rows_cta = (g.rg1 - g.rg0) * RPW;
  __shared__ float red[kWarps][kMaxTok];
  __shared__ float den[kMaxTok];
  for (int i = threadIdx.x; i < rows_cta * g.n_kc * M; i += kThreads) part[i] = 0.f;
  if (a.norm_w) {
    float ss[M];
#pragma unroll
    for (int m = 0; m < M; m++) ss[m] = 0.f;
    for (int k = threadIdx.x; k < g.K; k += kThreads)
#pragma unroll
      for (int m = 0; m < M; m++) {
        const float v = (m < a.M) ? ld_cg(a.x + (size_t)m * g.K + k) : 0.f;
        xs[(size_t)m * g.K + k] = v;
        ss[m] = fmaf(v, v, ss[m]);
      }
#pragma unroll
    for (int m = 0; m < M; m++) {
      const float t = warp_sum(ss[m]);
      if (lane == 0) red[warp][m] = t;
    }
    __syncthreads();
    if (threadIdx.x < M) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; w++) t += red[w][threadIdx.x];
      den[threadIdx.x] = sqrtf(__fadd_rn(__fdiv_rn(t, (float)g.K), a.eps));
    }
    __syncthreads();
    for (int k = threadIdx.x; k < g.K; k += kThreads) {
      const float gk = a.norm_w[k];
#pragma unroll
      for (int m = 0; m < M; m++) {
        float* p = xs + (size_t)m * g.K + k;
        *p = __fmul_rn(__fdiv_rn(*p, den[m]), gk);
      }
    }
  } else {
    const int nv = g.K / 4;
    for (int i = threadIdx.x; i < nv; i += kThreads)
#pragma unroll
      for (int m = 0; m < M; m++) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (m < a.M) v = ld_cg4(a.x + (size_t)m * g.K + 4 * i);
        reinterpret_cast<float4*>(xs + (size_t)m * g.K)[i] = v;
      }
  }
  __syncthreads();
  if constexpr (WT == SX_DTYPE_Q4_K) {
    for (int q = threadIdx.x; q < g.K / 16; q += kThreads)
#pragma unroll
      for (int m = 0; m < M; m++) {
        const float* p = xs + (size_t)m * g.K + q * 16;
        float t = 0.f;
#pragma unroll
        for (int e = 0; e < 16; e++) t += p[e];
        xsum16[(size_t)m * (g.K / 16) + q] = t;
      }
    __syncthreads();
  }

  // ---- stream this warp's items, two register buffers in ping-pong ----
  float acc[RPW][M];
#pragma unroll
  for (int r = 0; r < RPW; r++)
#pragma unroll
    for (int m = 0; m < M; m++) acc[r][m] = 0.f;
  int cur_rg = -1, run_kc0 = 0;
  while (cc.left > 0) {
    load_group<WT, RPW, B>(a, g, lc, prow, prow_rg, lane, fb);
    compute_group<WT, M, RPW, B>(g, cc, lane, fa, xs, xsum16, part, acc, cur_rg, run_kc0);
    if (cc.left > 0) {
      load_group<WT, RPW, B>(a, g, lc, prow, prow_rg, lane, fa);
      compute_group<WT, M, RPW, B>(g, cc, lane, fb, xs, xsum16, part, acc, cur_rg, run_kc0);
    }
  }
  if (cur_rg >= 0) flush<RPW, M>(acc, part, g, cur_rg, run_kc0, lane);
  __syncthreads();

  // ---- epilogue: fixed-order sum of the k-chunk partials of each row ----
  const int row_lo = g.rg0 * RPW;
  auto row_sum = [&](int rl, int m) {
    float v = 0.f;
    for (int kc = 0; kc < g.n_kc; kc++) v += part[(rl * g.n_kc + kc) * M + m];
    return v;
  };
  if constexpr (EPI == EPI_SWIGLU) {
    // logical rows (2j, 2j+1) = (gate_j, up_j)
    const int pairs = rows_cta / 2;
    for (int t = threadIdx.x; t < pairs * M; t += kThreads) {
      const int p = t / M, m = t % M;
      const int i = row_lo + 2 * p;
      if (m < a.M && i + 1 < g.n_logical) {
        const float gv = row_sum(2 * p, m), uv = row_sum(2 * p + 1, m);
        a.y[(size_t)m * a.ldy + (i >> 1)] = __fmul_rn(silu_f(gv), uv);
      }
    }
  } else if constexpr (EPI == EPI_ARGMAX) {
    __shared__ unsigned long long best[kWarps][kMaxTok];
    unsigned long long bk[M];
#pragma unroll
    for (int m = 0; m < M; m++) bk[m] = 0ull;
    for (int rl = threadIdx.x; rl < rows_cta; rl += kThreads) {
      const int i = row_lo + rl;
      if (i >= g.n_logical) continue;
      const uint32_t pr = (uint32_t)phys_row(a, i);
      const bool allowed = (pr >= a.allow_lo && pr <= a.allow_hi) || (pr >= a.stop_lo && pr < a.stop_hi);
#pragma unroll
      for (int m = 0; m < M; m++)
        if (m < a.M) {
          float v = row_sum(rl, m);
          if (a.bias) v = __fadd_rn(v, a.bias[pr]);
          if (a.y) a.y[(size_t)m * a.ldy + pr] = v;
          if (allowed) {
            const unsigned long long key = argmax_key(v, pr);
            bk[m] = key > bk[m] ? key : bk[m];
          }
        }
    }
#pragma unroll
    for (int m = 0; m < M; m++) {
      unsigned long long b = bk[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, b, o);
        b = other > b ? other : b;
      }
      if (lane == 0) best[warp][m] = b;
    }
    __syncthreads();
    if (threadIdx.x < a.M && threadIdx.x < M) {
      unsigned long long b = 0ull;
#pragma unroll
      for (int w = 0; w < kWarps; w++) b = best[w][threadIdx.x] > b ? best[w][threadIdx.x] : b;
      if (b != 0ull) atomicMax(a.amax + threadIdx.x, b);
    }
  } else {
    for (int t = threadIdx.x; t < rows_cta * M; t += kThreads) {
      const int rl = t / M, m = t % M;
      const int i = row_lo + rl;
      if (m < a.M && i < g.n_logical) {
        const int pr = phys_row(a, i);
        float v = row_sum(rl, m);
        if (a.bias) v = __fadd_rn(v, a.bias[pr]);
        float* dst = a.y + (size_t)m * a.ldy + pr;
        if constexpr (EPI == EPI_ADD)
          *dst = __fadd_rn(ld_cg(dst), v);
        else
          *dst = v;
      }
    }
  }
}

int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <int WT, int M, int RPW, int B, int EPI>
cudaError_t launch_t(const GemvArgs& a, cudaStream_t st) {
  constexpr int UE = Unit<WT>::elems;
  const int n_logical = a.n_range + a.n_extra;
  const int K = (int)a.w.cols;
  const int n_kc = (K / UE + 31) / 32;
  const int n_rg = (n_logical + RPW - 1) / RPW;
  const size_t x_bytes = (size_t)M * K * sizeof(float) + (WT == SX_DTYPE_Q4_K ? (size_t)M * (K / 16) * sizeof(float) : 0);
  // persistent grid: as many CTAs as are co-resident (registers and shared memory, at
  // most three per SM), so every CTA streams an equal share of the rows in a single wave
  static const int sms = num_sms();
  auto kern = k_gemv<WT, M, RPW, B, EPI>;
  int per_sm = 3, grid = 0;
  size_t smem = 0;
  for (;;) {
    grid = std::min(n_rg, per_sm * sms);
    smem = x_bytes + (size_t)((n_rg + grid - 1) / grid) * RPW * n_kc * M * sizeof(float);
    if (smem > 220 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    int occ = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (occ >= per_sm || per_sm == 1 || grid < n_rg) {
      if (occ >= per_sm || per_sm == 1) break;
    }
    per_sm = std::max(1, std::min(per_sm - 1, occ));
  }
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = launch_cfg(dim3(grid), dim3(kThreads), smem, st, attr);
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int WT, int M>
cudaError_t dispatch_epi(const GemvArgs& a, Epi epi, cudaStream_t st) {
  // RPW = 4 rows share each x fragment; one item per register buffer
  constexpr int RPW = 4;
  constexpr int B = 1;
  switch (epi) {
    case EPI_STORE: return launch_t<WT, M, RPW, B, EPI_STORE>(a, st);
    case EPI_ADD: return launch_t<WT, M, RPW, B, EPI_ADD>(a, st);
    case EPI_SWIGLU: return launch_t<WT, M, RPW, B, EPI_SWIGLU>(a, st);
    case EPI_ARGMAX: return launch_t<WT, M, RPW, B, EPI_ARGMAX>(a, st);
  }
  return cudaErrorInvalidValue;
}

template <int WT>
cudaError_t dispatch_m(const GemvArgs& a, Epi epi, cudaStream_t st) {
  if (a.M <= 1) return dispatch_epi<WT, 1>(a, epi, st);
  if (a.M <= 2) return dispatch_epi<WT, 2>(a, epi, st);
  if (a.M <= 4) return dispatch_epi<WT, 4>(a, epi, st);
  return dispatch_epi<WT, 8>(a, epi, st);
}

}  // namespace

cudaError_t launch_gemv(const GemvArgs& a, Epi epi, cudaStream_t st) {
  if (a.M < 1 || a.M > kMaxPrefillTok || a.n_range + a.n_extra < 1) return cudaErrorInvalidValue;
  if (a.w.dtype == SX_DTYPE_Q8_0 || a.w.dtype == kDtypeQ4KT) return launch_gemv_q8(a, epi, st);
  if (epi == EPI_NONE) return cudaErrorInvalidValue;  // the row-layout kernel has no partials to leave
  // x and the row partial sums of all M tokens live in shared memory, sized by the
  // kernel's template M (1, 2, 4 or 8): split the tokens into launches that fit
  const size_t K = (size_t)a.w.cols;
  const int ue = a.w.dtype == SX_DTYPE_Q4_K ? 32 : 4;
  const size_t n_kc = (K / ue + 31) / 32;
  const size_t n_rg = (size_t)(a.n_range + a.n_extra + 3) / 4;  // row groups of 4
  static const int sms = num_sms();
  const size_t per_tok = K * 4 + (a.w.dtype == SX_DTYPE_Q4_K ? (K / 16) * 4 : 0) +
                         ((n_rg + sms - 1) / sms) * 4 * n_kc * 4;
  int max_m = kMaxTok;
  while (max_m > 1 && (size_t)max_m * per_tok > 200 * 1024) max_m >>= 1;
  for (int m0 = 0; m0 < a.M; m0 += max_m) {
    GemvArgs b = a;
    b.M = std::min(max_m, a.M - m0);
    b.x = a.x + (size_t)m0 * K;
    if (a.y) b.y = a.y + (size_t)m0 * a.ldy;
    if (a.amax) b.amax = a.amax + m0;
    cudaError_t e = cudaErrorInvalidValue;
    switch (a.w.dtype) {
      case SX_DTYPE_Q4_K: e = dispatch_m<SX_DTYPE_Q4_K>(b, epi, st); break;
      case SX_DTYPE_F32: e = dispatch_m<SX_DTYPE_F32>(b, epi, st); break;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace sx
