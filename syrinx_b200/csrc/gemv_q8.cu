// gemv_q8.cu — Q8_0 GEMV on int8 tensor-core fragments: decode (M = 1..8 tokens) and
// prefill chunks (up to 64 tokens), plus the merge kernels, including the tensor-parallel
// residual exchange.
//
// Replaces the quantized linear of the reference hot path (`Weights::linear`,
// crates/syrinx-fish/src/s2/nn.rs:61-68; `Qwen2Lm::linear` over candle QMatMul,
// crates/syrinx-lm/src/cv2/mod.rs:195-211) for Q8_0 weights, with the neighbouring
// element-wise ops fused in:
//   prologue  RMSNorm of x with a gain vector (rms_norm_w, s2/nn.rs:100-106)
//   epilogue  + bias, residual add (s2/slow_ar.rs:195,198), SiLU(g)*u (s2/nn.rs:452-457),
//             or the greedy argmax of the head (common/sampling.rs:189-245 with top_k = 1).
//
// Arithmetic. The product is the exact dequantized weight times f32 x. Per 32-wide block b
// and token m, x is written as sx * (l0 + l1/128 + l2/128^2 + l3/128^3), sx a power of two
// that puts the block's max |x| in [32, 64) and every limb l_i an integer in [-64, 64] (the
// split is exact to 2^-27 of the block max; x itself carries 24 bits). One
// mma.m16n8k32.s8 then yields, for a 16-row weight tile, the exact int32 sums
// S_i = sum_k q_k l_i,k of all four limbs of two tokens at once (B columns 0-3 token 2p,
// 4-7 token 2p+1). Each lane folds its two limb sums as S_0*128 + S_1 (or S_2*128 + S_3),
// converts once and accumulates d_row * sx * S in f32; the two halves are combined with
// weights 2^-7 and 2^-21. That is about 15 instructions per 512 weight bytes, so the
// stream is bound by HBM, not by issue.
//
// Work split. Items are (virtual tile, k-chunk of 8 blocks), ordered k-chunk-major over the
// whole grid, contiguous per CTA and per warp: a CTA touches one or two k-chunks, so it
// splits x into limbs only for those 8-16 blocks. Every item writes its 16 row sums per
// token to a partial buffer [vt][k-chunk][m][16]; a second small kernel (k_merge_q8) adds
// the k-chunks of each row in a fixed order and applies the epilogue. The result does not
// depend on the grid, on M, or on which warp ran which item.
#include <cuda_runtime.h>

#include <algorithm>

#include "sx_device.cuh"
#include "sx_internal.hpp"

namespace sx {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kCB = 8;  // 32-wide k blocks per item
// (block, token) units per warp whose x loads go out together: a warp has at most 2M units
// (a CTA spans at most 16 blocks), so small batches cover all of them in one round trip
__host__ __device__ constexpr int limb_batch(int M) { return M == 1 ? 2 : M == 2 ? 4 : M <= 8 ? 8 : 4; }

struct Q8Geo {
  int K, nb, nc;      // columns, 32-wide blocks, k-chunks of kCB blocks
  int t_first, n_rt;  // first physical tile of the row range, tiles covering the range
  int n_vt;           // virtual tiles: the range tiles, then one per extra row
};

__device__ __forceinline__ int vt_tile(const GemvArgs& a, const Q8Geo& g, int vt) {
  return vt < g.n_rt ? g.t_first + vt : (a.extra[vt - g.n_rt] >> 4);
}

struct Item {
  uint4 q[kCB];
  uint32_t s[kCB];
};

__device__ __forceinline__ void load_item(const uint8_t* W, const Q8Geo& g, int tile, int kc, int lane, Item& it) {
#pragma unroll
  for (int j = 0; j < kCB; j++) {
    const int b = kc * kCB + j;
    if (b < g.nb) {
      const uint8_t* r = W + ((size_t)tile * g.nb + b) * kQ8Rec;
      it.q[j] = ldg_stream(r + lane * 16);
      it.s[j] = ldg_stream32(r + 512 + (lane >> 2) * 4);
    }
  }
}

// RMSNorm denominators of the M rows of x over K: each thread sums the squares of k = tid,
// tid + 256, ... in k order, then the warps are added in order (the register kernel's order).
// KT > 0 loads KT elements per token and thread before the first is used, so K <= KT * 256
// costs one round trip to L2 (the guarded loads past K add exact zeros); KT = 0 keeps a
// four-step unrolled loop, for kernels without the registers to hold more loads.
template <int M, int KT>
__device__ __forceinline__ void rms_dens(const GemvArgs& a, int K, float (&red)[kWarps][M], float (&den)[M], int warp,
                                         int lane) {
  float ss[M];
#pragma unroll
  for (int m = 0; m < M; m++) ss[m] = 0.f;
  if constexpr (KT > 0) {
    for (int k0 = threadIdx.x; k0 < K; k0 += KT * kThreads) {
      float v[KT][M];
#pragma unroll
      for (int j = 0; j < KT; j++) {
        const int k = k0 + j * kThreads;
#pragma unroll
        for (int m = 0; m < M; m++) v[j][m] = (k < K && m < a.M) ? ld_cg(a.x + (size_t)m * K + k) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < KT; j++)
#pragma unroll
        for (int m = 0; m < M; m++) ss[m] = fmaf(v[j][m], v[j][m], ss[m]);
    }
  } else {
#pragma unroll(M <= 8 ? 4 : 1)
    for (int k = threadIdx.x; k < K; k += kThreads)
#pragma unroll
      for (int m = 0; m < M; m++) {
        const float v = (m < a.M) ? ld_cg(a.x + (size_t)m * K + k) : 0.f;
        ss[m] = fmaf(v, v, ss[m]);
      }
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
    den[threadIdx.x] = sqrtf(__fadd_rn(__fdiv_rn(t, (float)K), a.eps));
  }
  __syncthreads();
}

// x (and gain) of one batch of (block, token) units of the limb split: unit u0 + j * kWarps
// is block b_lo + u / M, token u % M, lane = column within the block. The gains are weights,
// so their loads may go out before the grid dependency wait; x only after it.
template <int LB, int M>
__device__ __forceinline__ void limb_gains(const GemvArgs& a, int b_lo, int n_units, int u0, int lane,
                                           float (&gv)[LB]) {
#pragma unroll
  for (int j = 0; j < LB; j++) {
    const int u = u0 + j * kWarps, m = u % M, k = (b_lo + u / M) * 32 + lane;
    gv[j] = (u < n_units && m < a.M && a.norm_w) ? a.norm_w[k] : 0.f;
  }
}
template <int LB, int M>
__device__ __forceinline__ void limb_x(const GemvArgs& a, int K, int b_lo, int n_units, int u0, int lane,
                                       float (&xv)[LB]) {
#pragma unroll
  for (int j = 0; j < LB; j++) {
    const int u = u0 + j * kWarps, m = u % M, k = (b_lo + u / M) * 32 + lane;
    xv[j] = (u < n_units && m < a.M) ? ld_cg(a.x + (size_t)m * K + k) : 0.f;
  }
}

// The decode prologue's shape per kernel (registers allow it at 80 per thread for Q8_0 up to
// two tokens, at 128 for Q4_K up to eight): RMSNorm loads per token and thread in one pass
// (rms_dens; 0 = the unrolled loop) and whether the first limb batch's loads go out with them
__host__ __device__ constexpr int rms_kt_q8(int M) { return M == 1 ? 16 : M == 2 ? 4 : 0; }
__host__ __device__ constexpr int rms_kt_q4k(int M) { return M == 1 ? 16 : M <= 4 ? 8 : M <= 8 ? 4 : 0; }

// x[j] of a w2 GEMV fed by the w1|w3 partials (GemvArgs::glu_part), feature j = 32 (b_lo + bi)
// + lane: tile 4 (b_lo + bi) + lane / 8 holds its gate (row lane % 8) and up (row 8 + lane % 8)
// partials, staged in shared memory from tile 4 b_lo on. Added exactly as k_merge_q8's SwiGLU
// epilogue adds them: four contiguous quarters of the k-chunks, each in order from zero, the
// quarters in order, then silu(gate) * up.
__device__ __forceinline__ float glu_value(const float* stage, int bi, int lane, int nc) {
  const float* p = stage + (size_t)(bi * 4 + (lane >> 3)) * nc * 16 + (lane & 7);
  float tg[4], tu[4];
#pragma unroll
  for (int qi = 0; qi < 4; qi++) {
    const int k0 = qi * nc / 4, k1 = (qi + 1) * nc / 4;
    float s0 = 0.f, s1 = 0.f;
    for (int kc = k0; kc < k1; kc++) {
      s0 += p[kc * 16];
      s1 += p[kc * 16 + 8];
    }
    tg[qi] = s0;
    tu[qi] = s1;
  }
  const float t0 = ((tg[0] + tg[1]) + tg[2]) + tg[3];
  const float t1 = ((tu[0] + tu[1]) + tu[2]) + tu[3];
  return __fmul_rn(silu_f(t0), t1);
}

// Up to 8 tokens (decode) at three CTAs per SM; prefill chunks of 16..64 tokens hold one
// accumulator pair per token pair and run one CTA per SM.
template <int M>
__global__ void __launch_bounds__(kThreads, M <= 8 ? 3 : 1) k_gemv_q8(const GemvArgs a, const Q8Geo g) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int NP = (M + 1) / 2;  // token pairs = tensor-core instructions per record
  __shared__ __align__(16) int8_t scr[kWarps][4][32];
  __shared__ float red[kWarps][M];
  __shared__ float den[M];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const long long I = (long long)g.n_vt * g.nc;
  const long long c0 = (long long)blockIdx.x * I / gridDim.x;
  const long long c1 = (long long)(blockIdx.x + 1) * I / gridDim.x;
  const int kc_lo = (int)(c0 / g.n_vt), kc_hi = c1 > c0 ? (int)((c1 - 1) / g.n_vt) : kc_lo;
  const int b_lo = kc_lo * kCB, b_hi = min(g.nb, (kc_hi + 1) * kCB);
  // one token: a w2 GEMV may form its x from the w1|w3 partials (glu_value)
  const bool glu = M == 1 && a.glu_part != nullptr;
  const int stage_f = glu ? (b_hi - b_lo) * 4 * a.glu_nc * 16 : 0;  // floats
  // shared: staged w1|w3 partials [4 (block - b_lo)][glu_nc][16] (glu only) | B fragments
  // [block - b_lo][NP][32 lanes] | block scales of x [block - b_lo][M]
  float* stage = reinterpret_cast<float*>(smem);
  uint2* bfr = reinterpret_cast<uint2*>(smem + (size_t)stage_f * 4);
  float* sxs = reinterpret_cast<float*>(smem + (size_t)stage_f * 4 + (size_t)(b_hi - b_lo) * NP * 256);
  const long long w0 = c0 + (c1 - c0) * warp / kWarps, w1 = c0 + (c1 - c0) * (warp + 1) / kWarps;
  int kc = (int)(w0 / g.n_vt), vt = (int)(w0 % g.n_vt), left = (int)(w1 - w0);
  const uint8_t* W = static_cast<const uint8_t*>(a.w.q);

  // x limbs of this CTA's blocks, one warp per (block, token) unit, in batches of up to 8
  // units per warp whose loads all go out before the first is used
  constexpr int LB = limb_batch(M);
  const int n_units = (b_hi - b_lo) * M;
  float xv[LB], gv[LB];

  constexpr bool early = rms_kt_q8(M) > 0;

  pdl_launch_dependents();
  // The first item's weights and the first batch's gains do not depend on the previous
  // kernel: request them now.
  Item it;
  if (left > 0) load_item(W, g, vt_tile(a, g, vt), kc, lane, it);
  if (early) limb_gains<LB, M>(a, b_lo, n_units, warp, lane, gv);
  pdl_wait();
  if (glu) {  // the w1|w3 partials of this CTA's blocks: one contiguous run, straight to shared memory
    const float* src = a.glu_part + (size_t)b_lo * 4 * a.glu_nc * 16;
    for (int i = threadIdx.x; i < stage_f / 4; i += kThreads) cp_async16(stage + 4 * i, src + 4 * i);
    cp_async_wait_all();
    __syncthreads();
  } else if (early) {
    // the first batch's x goes out together with the RMSNorm loads: one round trip for both
    limb_x<LB, M>(a, g.K, b_lo, n_units, warp, lane, xv);
  }

  // ---- RMSNorm denominators over the full K (same order as the register kernel) ----
  if (a.norm_w) rms_dens<M, rms_kt_q8(M)>(a, g.K, red, den, warp, lane);

  // ---- x limbs ----
  for (int u0 = warp; u0 < n_units; u0 += LB * kWarps) {
    if (!early || u0 != warp) {
      limb_gains<LB, M>(a, b_lo, n_units, u0, lane, gv);
      if (!glu) limb_x<LB, M>(a, g.K, b_lo, n_units, u0, lane, xv);
    }
#pragma unroll
    for (int j = 0; j < LB; j++) {
    const int u = u0 + j * kWarps;
    if (u >= n_units) break;
    const int bi = u / M, m = u % M;
    float v = 0.f;
    if (m < a.M) {
      v = glu ? glu_value(stage, bi, lane, a.glu_nc) : xv[j];
      if (a.norm_w) v = __fmul_rn(__fdiv_rn(v, den[m]), gv[j]);
    }
    const float mx = warp_max(fabsf(v));
    const int e = (__float_as_int(mx) >> 23) & 0xff;
    float sc = 0.f, sx = 0.f;
    if (e == 255 || __any_sync(0xffffffffu, v != v)) {
      sx = __int_as_float(0x7fc00000);  // inf / nan in the block: the result is nan
    } else if (e >= 6) {               // below 2^-121 the block contributes nothing
      sc = __int_as_float((259 - e) << 23);  // 2^(132 - e): max |x| * sc in [32, 64)
      sx = __int_as_float((e - 5) << 23);    // 1 / sc
    }
    const float s = v * sc;
    const float l0 = rintf(s);
    float r = (s - l0) * 128.f;
    const float l1 = rintf(r);
    r = (r - l1) * 128.f;
    const float l2 = rintf(r);
    r = (r - l2) * 128.f;
    const float l3 = rintf(r);
    scr[warp][0][lane] = (int8_t)(int)l0;
    scr[warp][1][lane] = (int8_t)(int)l1;
    scr[warp][2][lane] = (int8_t)(int)l2;
    scr[warp][3][lane] = (int8_t)(int)l3;
    __syncwarp();
    if (lane < 16) {  // B fragment: lane 4n + c holds limb n of k 4c..4c+3 and 16+4c..16+4c+3
      const int n = lane >> 2, c = lane & 3;
      uint2 w;
      w.x = *reinterpret_cast<const uint32_t*>(&scr[warp][n][4 * c]);
      w.y = *reinterpret_cast<const uint32_t*>(&scr[warp][n][16 + 4 * c]);
      bfr[(bi * NP + (m >> 1)) * 32 + (m & 1) * 16 + lane] = w;
    }
    if (lane == 0) sxs[bi * M + m] = sx;
    __syncwarp();
    }
  }
  __syncthreads();

  // ---- stream this warp's items ----
  // lane roles in the accumulator: rows g = lane/4 and g+8; token 2p + ((lane >> 1) & 1);
  // limb pair (0,1) on even lanes, (2,3) on odd lanes
  const int bl = M == 1 ? (lane & 15) : lane;
  while (left > 0) {
    float acc[NP][2];
#pragma unroll
    for (int p = 0; p < NP; p++) acc[p][0] = acc[p][1] = 0.f;
#pragma unroll
    for (int j = 0; j < kCB; j++) {
      const int b = kc * kCB + j;
      if (b < g.nb) {
        const int bi = b - b_lo;
        const float2 ds = __half22float2(*reinterpret_cast<const __half2*>(&it.s[j]));
#pragma unroll
        for (int p = 0; p < NP; p++) {
          const uint2 bf = bfr[(bi * NP + p) * 32 + bl];
          const int tok = M == 1 ? 0 : 2 * p + ((lane >> 1) & 1);
          const float sx = sxs[bi * M + tok];
          int d[4];
          mma_s8_16832(it.q[j], bf, d);
          acc[p][0] = fmaf(__fmul_rn(ds.x, sx), (float)(d[0] * 128 + d[1]), acc[p][0]);
          acc[p][1] = fmaf(__fmul_rn(ds.y, sx), (float)(d[2] * 128 + d[3]), acc[p][1]);
        }
      }
    }
    const int done_vt = vt, done_kc = kc;
    if (++vt == g.n_vt) {
      vt = 0;
      kc++;
    }
    left--;
    if (left > 0) load_item(W, g, vt_tile(a, g, vt), kc, lane, it);
    const float wgt = (lane & 1) ? 0x1p-21f : 0x1p-7f;
    float* P = a.part + ((size_t)done_vt * g.nc + done_kc) * M * 16;
#pragma unroll
    for (int p = 0; p < NP; p++) {
      float v0 = acc[p][0] * wgt, v1 = acc[p][1] * wgt;
      v0 += __shfl_down_sync(0xffffffffu, v0, 1);
      v1 += __shfl_down_sync(0xffffffffu, v1, 1);
      const int tok = 2 * p + ((lane >> 1) & 1);
      if ((lane & 1) == 0 && tok < M) {
        __stcg(P + tok * 16 + (lane >> 2), v0);
        __stcg(P + tok * 16 + (lane >> 2) + 8, v1);
      }
    }
  }
}

// ---- Q4_K tile records (sx_internal.hpp, kQ4Rec): the same integer tensor-core scheme ----
// A Q4_K weight of sub-block j is d * sc_j * q - dmin * m_j (q a nibble 0..15, sc_j / m_j 6-bit),
// so per row and sub-block sum_k w_k x_k = d * sc_j * sum_k q_k x_k - dmin * m_j * sum_k x_k.
// The first sum is exact on the tensor cores exactly as for Q8_0 (nibbles widened in the A
// fragment registers with one mask and one shift per word; d * sc_j is an exact f32); the
// second uses the block sum of the normed x, one warp sum per (block, token) beside the limb
// split, added on the lanes that carry the limb pair (0, 1). A k chunk is one super-block.
struct ItemQ4 {
  uint4 q[4];     // the 4 sub-block pairs' quants of this lane
  uint4 sc, mn;   // 6-bit scales / mins of rows g (x, y) and g + 8 (z, w)
  uint2 dd;       // {d, dmin} of row g, then of row g + 8 (f16)
};

__device__ __forceinline__ void load_item_q4(const uint8_t* W, const Q8Geo& g, int tile, int kc, int lane, ItemQ4& it) {
  const uint8_t* r = W + ((size_t)tile * g.nc + kc) * kQ4Rec;
#pragma unroll
  for (int jp = 0; jp < 4; jp++) it.q[jp] = ldg_stream(r + jp * 512 + lane * 16);
  it.sc = ldg_stream(r + 2048 + (lane >> 2) * 16);
  it.mn = ldg_stream(r + 2176 + (lane >> 2) * 16);
  it.dd.x = ldg_stream32(r + 2304 + (lane >> 2) * 8);
  it.dd.y = ldg_stream32(r + 2304 + (lane >> 2) * 8 + 4);
}

template <int M>
__global__ void __launch_bounds__(kThreads, M <= 8 ? 2 : 1) k_gemv_q4k(const GemvArgs a, const Q8Geo g) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int NP = (M + 1) / 2;
  __shared__ __align__(16) int8_t scr[kWarps][4][32];
  __shared__ float red[kWarps][M];
  __shared__ float den[M];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const long long I = (long long)g.n_vt * g.nc;
  const long long c0 = (long long)blockIdx.x * I / gridDim.x;
  const long long c1 = (long long)(blockIdx.x + 1) * I / gridDim.x;
  const int kc_lo = (int)(c0 / g.n_vt), kc_hi = c1 > c0 ? (int)((c1 - 1) / g.n_vt) : kc_lo;
  const int b_lo = kc_lo * kCB, b_hi = min(g.nb, (kc_hi + 1) * kCB);
  // shared: B fragments [block - b_lo][NP][32 lanes] | x scales [block - b_lo][M] | x block sums
  uint2* bfr = reinterpret_cast<uint2*>(smem);
  float* sxs = reinterpret_cast<float*>(smem + (size_t)(b_hi - b_lo) * NP * 256);
  float* xsum = sxs + (size_t)(b_hi - b_lo) * M;
  const long long w0 = c0 + (c1 - c0) * warp / kWarps, w1 = c0 + (c1 - c0) * (warp + 1) / kWarps;
  int kc = (int)(w0 / g.n_vt), vt = (int)(w0 % g.n_vt), left = (int)(w1 - w0);
  const uint8_t* W = static_cast<const uint8_t*>(a.w.q);

  constexpr int LB = limb_batch(M);
  const int n_units = (b_hi - b_lo) * M;
  float xv[LB], gv[LB];

  pdl_launch_dependents();
  // two items in registers: the next one loads while this one is multiplied
  ItemQ4 it0, it1;
  if (left > 0) load_item_q4(W, g, g.t_first + vt, kc, lane, it0);
  if (left > 1) {
    const int vt1 = vt + 1 == g.n_vt ? 0 : vt + 1, kc1 = vt + 1 == g.n_vt ? kc + 1 : kc;
    load_item_q4(W, g, g.t_first + vt1, kc1, lane, it1);
  }
  constexpr bool early = rms_kt_q4k(M) > 0;
  if (early) limb_gains<LB, M>(a, b_lo, n_units, warp, lane, gv);
  pdl_wait();
  if (early) limb_x<LB, M>(a, g.K, b_lo, n_units, warp, lane, xv);  // with the RMSNorm loads, as k_gemv_q8

  if (a.norm_w) rms_dens<M, rms_kt_q4k(M)>(a, g.K, red, den, warp, lane);

  // x limbs (as k_gemv_q8) and the block sums of x, one warp per (block, token)
  for (int u0 = warp; u0 < n_units; u0 += LB * kWarps) {
    if (!early || u0 != warp) {
      limb_gains<LB, M>(a, b_lo, n_units, u0, lane, gv);
      limb_x<LB, M>(a, g.K, b_lo, n_units, u0, lane, xv);
    }
#pragma unroll
    for (int j = 0; j < LB; j++) {
    const int u = u0 + j * kWarps;
    if (u >= n_units) break;
    const int bi = u / M, m = u % M;
    float v = 0.f;
    if (m < a.M) {
      v = xv[j];
      if (a.norm_w) v = __fmul_rn(__fdiv_rn(v, den[m]), gv[j]);
    }
    const float bsum = warp_sum(v);
    const float mx = warp_max(fabsf(v));
    const int e = (__float_as_int(mx) >> 23) & 0xff;
    float sc = 0.f, sx = 0.f;
    if (e == 255 || __any_sync(0xffffffffu, v != v)) {
      sx = __int_as_float(0x7fc00000);
    } else if (e >= 6) {
      sc = __int_as_float((259 - e) << 23);
      sx = __int_as_float((e - 5) << 23);
    }
    const float s = v * sc;
    const float l0 = rintf(s);
    float r = (s - l0) * 128.f;
    const float l1 = rintf(r);
    r = (r - l1) * 128.f;
    const float l2 = rintf(r);
    r = (r - l2) * 128.f;
    const float l3 = rintf(r);
    scr[warp][0][lane] = (int8_t)(int)l0;
    scr[warp][1][lane] = (int8_t)(int)l1;
    scr[warp][2][lane] = (int8_t)(int)l2;
    scr[warp][3][lane] = (int8_t)(int)l3;
    __syncwarp();
    if (lane < 16) {
      const int n = lane >> 2, c = lane & 3;
      uint2 w;
      w.x = *reinterpret_cast<const uint32_t*>(&scr[warp][n][4 * c]);
      w.y = *reinterpret_cast<const uint32_t*>(&scr[warp][n][16 + 4 * c]);
      bfr[(bi * NP + (m >> 1)) * 32 + (m & 1) * 16 + lane] = w;
    }
    if (lane == 0) {
      sxs[bi * M + m] = sx;
      xsum[bi * M + m] = bsum;
    }
    __syncwarp();
    }
  }
  __syncthreads();

  const int bl = M == 1 ? (lane & 15) : lane;
  const float mmul = (lane & 1) ? 0.f : -128.f;  // the min term rides on the limb-(0, 1) lanes
  // one item: multiply, then load the item after the next one into its registers
  auto run = [&](ItemQ4& it) {
    float acc[NP][2];
#pragma unroll
    for (int p = 0; p < NP; p++) acc[p][0] = acc[p][1] = 0.f;
    const float2 dg = __half22float2(*reinterpret_cast<const __half2*>(&it.dd.x));   // d, dmin of row g
    const float2 dg8 = __half22float2(*reinterpret_cast<const __half2*>(&it.dd.y));  // of row g + 8
#pragma unroll
    for (int j = 0; j < kCB; j++) {
      const int bi = kc * kCB + j - b_lo;
      const uint32_t w0 = (j & 1) ? it.q[j >> 1].z : it.q[j >> 1].x;
      const uint32_t w1 = (j & 1) ? it.q[j >> 1].w : it.q[j >> 1].y;
      uint4 af;
      af.x = w0 & 0x0F0F0F0Fu;
      af.y = w1 & 0x0F0F0F0Fu;
      af.z = (w0 >> 4) & 0x0F0F0F0Fu;
      af.w = (w1 >> 4) & 0x0F0F0F0Fu;
      const int sh = 8 * (j & 3);
      const uint32_t scg = (((j < 4) ? it.sc.x : it.sc.y) >> sh) & 0xff, scg8 = (((j < 4) ? it.sc.z : it.sc.w) >> sh) & 0xff;
      const uint32_t mng = (((j < 4) ? it.mn.x : it.mn.y) >> sh) & 0xff, mng8 = (((j < 4) ? it.mn.z : it.mn.w) >> sh) & 0xff;
      const float d1g = __fmul_rn(dg.x, (float)scg), d1g8 = __fmul_rn(dg8.x, (float)scg8);
      const float m1g = __fmul_rn(__fmul_rn(dg.y, (float)mng), mmul);
      const float m1g8 = __fmul_rn(__fmul_rn(dg8.y, (float)mng8), mmul);
#pragma unroll
      for (int p = 0; p < NP; p++) {
        const uint2 bf = bfr[(bi * NP + p) * 32 + bl];
        const int tok = M == 1 ? 0 : 2 * p + ((lane >> 1) & 1);
        const float sx = sxs[bi * M + tok];
        const float xs = xsum[bi * M + tok];
        int d[4];
        mma_s8_16832(af, bf, d);
        acc[p][0] = fmaf(__fmul_rn(d1g, sx), (float)(d[0] * 128 + d[1]), acc[p][0]);
        acc[p][1] = fmaf(__fmul_rn(d1g8, sx), (float)(d[2] * 128 + d[3]), acc[p][1]);
        acc[p][0] = fmaf(m1g, xs, acc[p][0]);
        acc[p][1] = fmaf(m1g8, xs, acc[p][1]);
      }
    }
    const int done_vt = vt, done_kc = kc;
    if (++vt == g.n_vt) {
      vt = 0;
      kc++;
    }
    left--;
    if (left > 1) {  // the item after the next one, into this buffer
      const int vt2 = vt + 1 == g.n_vt ? 0 : vt + 1, kc2 = vt + 1 == g.n_vt ? kc + 1 : kc;
      load_item_q4(W, g, g.t_first + vt2, kc2, lane, it);
    }
    const float wgt = (lane & 1) ? 0x1p-21f : 0x1p-7f;
    float* P = a.part + ((size_t)done_vt * g.nc + done_kc) * M * 16;
#pragma unroll
    for (int p = 0; p < NP; p++) {
      float v0 = acc[p][0] * wgt, v1 = acc[p][1] * wgt;
      v0 += __shfl_down_sync(0xffffffffu, v0, 1);
      v1 += __shfl_down_sync(0xffffffffu, v1, 1);
      const int tok = 2 * p + ((lane >> 1) & 1);
      if ((lane & 1) == 0 && tok < M) {
        __stcg(P + tok * 16 + (lane >> 2), v0);
        __stcg(P + tok * 16 + (lane >> 2) + 8, v1);
      }
    }
  };
  while (left > 0) {
    run(it0);
    if (left > 0) run(it1);
  }
}

// Row sums over the k-chunks in a fixed order (four lanes per output unit each add a
// contiguous quarter of the chunks, then the quarters are added in order), then the
// epilogue. Units: rows (STORE / ADD / ARGMAX) or gate/up row pairs (SWIGLU) per token.
template <int M, int EPI>
__global__ void __launch_bounds__(256) k_merge_q8(const GemvArgs a, const Q8Geo g) {
  pdl_launch_dependents();
  constexpr int R = EPI == EPI_SWIGLU ? 8 : 16;  // units per tile and token
  const int lane = threadIdx.x & 31, q4 = lane & 3;
  const long long u = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 2;
  const bool live = u < (long long)g.n_vt * R * M;
  const int vt = live ? (int)(u / (R * M)) : 0;
  const int m = live ? (int)((u / R) % M) : 0;
  const int r = live ? (int)(u % R) : 0;
  const bool lead = live && q4 == 0 && m < a.M;
  // the output row of a non-SwiGLU unit; its bias (a weight) is requested before the wait,
  // and the residual of an add together with the partials, after it
  int pr = 0;
  bool valid = false;
  if constexpr (EPI != EPI_SWIGLU) {
    if (vt < g.n_rt) {
      pr = (g.t_first + vt) * 16 + r;
      valid = pr >= a.row_base && pr < a.row_base + a.n_range;
    } else {
      pr = a.extra[vt - g.n_rt];
      valid = (pr & 15) == r;
    }
    valid = valid && lead;
  }
  const float bv = (valid && a.bias) ? a.bias[pr] : 0.f;
  pdl_wait();
  float res = 0.f;
  if constexpr (EPI == EPI_ADD)
    if (valid) res = ld_cg(a.y + (size_t)m * a.ldy + pr);
  float s0 = 0.f, s1 = 0.f;
  if (live) {
    const float* p = a.part + ((size_t)vt * g.nc * M + m) * 16 + r;
    const int k0 = q4 * g.nc / 4, k1 = (q4 + 1) * g.nc / 4;
    constexpr int KQ = 12;  // a quarter of up to 48 k-chunks (K <= 12288): every load out at once
    if (k1 - k0 <= KQ) {
      float v0[KQ], v1[KQ];
#pragma unroll
      for (int i = 0; i < KQ; i++) {
        v0[i] = k0 + i < k1 ? __ldcg(p + (size_t)(k0 + i) * M * 16) : 0.f;
        v1[i] = EPI == EPI_SWIGLU && k0 + i < k1 ? __ldcg(p + (size_t)(k0 + i) * M * 16 + 8) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < KQ; i++)
        if (k0 + i < k1) {  // the same additions in the same order as the loop below
          s0 += v0[i];
          if (EPI == EPI_SWIGLU) s1 += v1[i];
        }
    } else {
#pragma unroll 4
      for (int kc = k0; kc < k1; kc++) {
        s0 += __ldcg(p + (size_t)kc * M * 16);
        if (EPI == EPI_SWIGLU) s1 += __ldcg(p + (size_t)kc * M * 16 + 8);
      }
    }
  }
  const int base = lane & ~3;
  const float t0 = ((__shfl_sync(0xffffffffu, s0, base) + __shfl_sync(0xffffffffu, s0, base + 1)) +
                    __shfl_sync(0xffffffffu, s0, base + 2)) +
                   __shfl_sync(0xffffffffu, s0, base + 3);
  const float t1 = ((__shfl_sync(0xffffffffu, s1, base) + __shfl_sync(0xffffffffu, s1, base + 1)) +
                    __shfl_sync(0xffffffffu, s1, base + 2)) +
                   __shfl_sync(0xffffffffu, s1, base + 3);
  if constexpr (EPI == EPI_SWIGLU) {
    // tile j holds gate rows 8j..8j+7 (tile rows 0-7) and up rows 8j..8j+7 (rows 8-15)
    const int j = (g.t_first + vt) * 8 + r;
    if (lead && j < a.n_range / 2) a.y[(size_t)m * a.ldy + j] = __fmul_rn(silu_f(t0), t1);
  } else {
    float v = t0;
    if (valid && a.bias) v = __fadd_rn(v, bv);
    if constexpr (EPI == EPI_ARGMAX) {
      unsigned long long key = 0ull;
      if (valid) {
        if (a.y) a.y[(size_t)m * a.ldy + pr] = v;
        const uint32_t ur = (uint32_t)pr;
        if ((ur >= a.allow_lo && ur <= a.allow_hi) || (ur >= a.stop_lo && ur < a.stop_hi)) key = argmax_key(v, ur);
      }
      // a warp covers 8 consecutive units of one (tile, token): one atomic per warp
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
      }
      if (lane == 0 && key != 0ull) atomicMax(a.amax + m, key);
    } else if (valid) {
      float* dst = a.y + (size_t)m * a.ldy + pr;
      if constexpr (EPI == EPI_ADD)
        *dst = __fadd_rn(res, v);
      else
        *dst = v;
    }
  }
}

// Residual add of a K-split (tensor-parallel) GEMV. Each rank adds up its own k-chunk
// partials per row exactly as k_merge_q8 does; the lane that owns a row then stores the
// 8-byte word {row sum, exchange epoch} into that row's slot of every peer's receive region
// (over NVLink), polls its own region until every peer's word for the row carries the same
// epoch (bounded by %globaltimer), and adds all ranks' values in rank order, so every rank
// computes bit-identical residuals. No fence, flag or barrier sits on the path: the value
// and its tag arrive in one single-copy-atomic store. The epoch belongs to the slot (token,
// row): only exchanges that carry the slot advance it, the same way on every rank, so an
// old word can never show the epoch a receiver waits for. Exchange e of a slot uses parity
// e % 2: a rank starts exchange e + 2 only after its exchange e + 1 kernel completed, which
// needed every peer's e + 1 word, which each peer stores only after its exchange e kernel
// (and with it every read of parity e % 2) completed.
// A rank whose wait runs out (the session's limit, TpComm::wait_ns) raises the session's
// error flag (3) and from then on pushes poison words (epoch kTpPoison) instead of row sums,
// in this exchange and in every later one while the flag stays raised; a receiver that reads
// a poison word raises its own flag and stops waiting. So a lost or late peer makes every
// rank fail within one bounded wait, and no rank accepts a value computed from residuals the
// sender could not update. The host keeps the flag raised (the session refuses to decode)
// until the group reconnects, which zeroes the receive regions and the slot epochs.
constexpr uint32_t kTpPoison = 0xffffffffu;

template <int M>
__global__ void __launch_bounds__(256, 4) k_merge_q8_tp(const GemvArgs a, const Q8Geo g) {
  pdl_launch_dependents();
  pdl_wait();
  const TpComm& tp = a.tp;
  const int lane = threadIdx.x & 31, q4 = lane & 3;
  const long long n_units = (long long)g.n_vt * 16 * M;
  // grid-stride over units (4 lanes each), warp-uniform trip count: the grid is capped so
  // that every CTA of the exchange is co-resident, and a CTA waiting for its counterpart on
  // a peer never waits for a CTA that cannot be scheduled
  const long long stride = (long long)gridDim.x * (blockDim.x >> 2);
  bool ok = ld_cg(tp.err) == 0;
  for (long long u0 = ((long long)blockIdx.x * blockDim.x + (threadIdx.x & ~31)) >> 2; u0 < n_units; u0 += stride) {
    const long long u = u0 + (lane >> 2);
    const bool live = u < n_units;
    const int vt = live ? (int)(u / (16 * M)) : 0;
    const int m = live ? (int)((u / 16) % M) : 0;
    const int r = live ? (int)(u % 16) : 0;
    float s0 = 0.f;
    if (live) {
      const float* p = a.part + ((size_t)vt * g.nc * M + m) * 16 + r;
      const int k0 = q4 * g.nc / 4, k1 = (q4 + 1) * g.nc / 4;
#pragma unroll 4
      for (int kc = k0; kc < k1; kc++) s0 += __ldcg(p + (size_t)kc * M * 16);
    }
    const int base = lane & ~3;
    const float t0 = ((__shfl_sync(0xffffffffu, s0, base) + __shfl_sync(0xffffffffu, s0, base + 1)) +
                      __shfl_sync(0xffffffffu, s0, base + 2)) +
                     __shfl_sync(0xffffffffu, s0, base + 3);
    const int pr = (g.t_first + vt) * 16 + r;
    const bool valid = live && q4 == 0 && m < a.M && pr >= a.row_base && pr < a.row_base + a.n_range;
    if (!valid) continue;
    const size_t idx = (size_t)m * a.ldy + pr;
    const uint32_t ep = ld_cg(tp.slot_epochs + idx) + 1;  // only this thread touches slot idx here
    tp.slot_epochs[idx] = ep;
    const size_t par = (size_t)(ep & 1) * kMaxTp;
    const uint64_t word = ok ? ((uint64_t)ep << 32) | __float_as_uint(t0) : ((uint64_t)kTpPoison << 32);
    for (int p = 0; p < tp.size; p++)
      if (p != tp.rank) st_relaxed_sys_u64(tp.rx[p] + (par + tp.rank) * tp.xb_cap + idx, word);
    float tot = 0.f;
    for (int q = 0; q < tp.size && ok; q++) {
      float v = t0;
      if (q != tp.rank) {
        const uint64_t* src = tp.rx[tp.rank] + (par + q) * tp.xb_cap + idx;
        uint64_t w = ld_relaxed_sys_u64(src);
        const uint64_t t_start = global_ns();
        while ((uint32_t)(w >> 32) != ep) {
          if ((uint32_t)(w >> 32) == kTpPoison || global_ns() - t_start > tp.wait_ns) {
            ok = false;
            atomicExch(tp.err, 3);
            break;
          }
          w = ld_relaxed_sys_u64(src);
        }
        v = __uint_as_float((uint32_t)w);
      }
      tot += v;
    }
    if (!ok) continue;
    float v = tot;
    if (a.bias) v = __fadd_rn(v, a.bias[pr]);
    float* dst = a.y + (size_t)m * a.ldy + pr;
    *dst = __fadd_rn(ld_cg(dst), v);
  }
}

int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <int M, int EPI>
cudaError_t launch_merge(const GemvArgs& a, const Q8Geo& g, cudaStream_t st) {
  constexpr int R = EPI == EPI_SWIGLU ? 8 : 16;
  const long long threads = (long long)g.n_vt * R * M * 4;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = launch_cfg(dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, st, attr);
  return cudaLaunchKernelEx(&cfg, k_merge_q8<M, EPI>, a, g);
}

template <int M>
cudaError_t launch_epilogue(const GemvArgs& a, Epi epi, const Q8Geo& g, cudaStream_t st);

template <int M>
cudaError_t launch_m(const GemvArgs& a, Epi epi, const Q8Geo& g, cudaStream_t st) {
  constexpr int NP = (M + 1) / 2;
  static const int sms = num_sms();
  const bool q4 = a.w.dtype == kDtypeQ4KT;
  if (!q4 && M >= 16 && tc_enabled() && a.n_extra == 0 && g.t_first == 0) {
    // prefill chunks: the same partials from the tensor-core GEMM
    cudaError_t e = launch_gemm_tc(a, M, g.K, g.nb, g.nc, g.t_first, g.n_vt, sms, st);
    if (e != cudaSuccess) return e;
    return launch_epilogue<M>(a, epi, g, st);
  }
  auto kern = q4 ? k_gemv_q4k<M> : k_gemv_q8<M>;
  const long long I = (long long)g.n_vt * g.nc;
  // persistent grid of up to three CTAs per SM; shared memory holds the limbs of the
  // k-chunks a CTA spans (at most ceil(items per CTA / n_vt) + 1 of them)
  int per_sm = 3, grid = 1;
  size_t smem = 0;
  for (;;) {
    grid = (int)std::max(1LL, std::min(I, (long long)per_sm * sms));
    const long long ipc = (I + grid - 1) / grid;
    const long long spans = std::min<long long>(g.nc, (ipc + g.n_vt - 1) / g.n_vt + 1);
    smem = (size_t)spans * kCB * (NP * 256 + M * (q4 ? 8 : 4));
    if (a.glu_part) smem += (size_t)spans * kCB * 4 * a.glu_nc * 64;  // staged w1|w3 partials
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    int occ = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (occ >= per_sm || per_sm == 1) break;
    per_sm = std::max(1, std::min(per_sm - 1, occ));
  }
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = launch_cfg(dim3(grid), dim3(kThreads), smem, st, attr);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, g);
  if (e != cudaSuccess) return e;
  return launch_epilogue<M>(a, epi, g, st);
}

// The merge of the partials with the epilogue (or the tensor-parallel exchange).
template <int M>
cudaError_t launch_epilogue(const GemvArgs& a, Epi epi, const Q8Geo& g, cudaStream_t st) {
  static const int sms = num_sms();
  if (epi == EPI_ADD && a.tp.size > 1) {
    // no more CTAs than can be resident at once (at most four per SM by the launch bounds),
    // so every CTA of the exchange is co-resident once the GEMV drains
    int occ = 0;
    cudaError_t eo = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_merge_q8_tp<M>, 256, 0);
    if (eo != cudaSuccess) return eo;
    if (occ < 1) return cudaErrorInvalidConfiguration;
    const long long blocks =
        std::min<long long>(((long long)g.n_vt * 16 * M * 4 + 255) / 256, (long long)std::min(occ, 4) * sms);
    if (a.n_extra != 0 || (long long)M * a.ldy > a.tp.xb_cap) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr2[1];
    cudaLaunchConfig_t cfg2 = launch_cfg(dim3((unsigned)blocks), dim3(256), 0, st, attr2);
    return cudaLaunchKernelEx(&cfg2, k_merge_q8_tp<M>, a, g);
  }
  switch (epi) {
    case EPI_NONE: return cudaSuccess;  // the consumer adds the partials itself
    case EPI_STORE: return launch_merge<M, EPI_STORE>(a, g, st);
    case EPI_ADD: return launch_merge<M, EPI_ADD>(a, g, st);
    case EPI_SWIGLU: return launch_merge<M, EPI_SWIGLU>(a, g, st);
    case EPI_ARGMAX: return launch_merge<M, EPI_ARGMAX>(a, g, st);
  }
  return cudaErrorInvalidValue;
}

bool make_geo(const GemvArgs& a, Q8Geo* g) {
  const int64_t K = a.w.cols;
  if (K <= 0 || K % 32 || a.n_range < 0 || a.n_extra < 0 || a.n_extra > 4 || a.n_range + a.n_extra < 1) return false;
  if (a.row_base < 0 || (int64_t)a.row_base + a.n_range > a.w.rows) return false;
  for (int i = 0; i < a.n_extra; i++)
    if (a.extra[i] < 0 || a.extra[i] >= a.w.rows) return false;
  g->K = (int)K;
  g->nb = (int)(K / 32);
  g->nc = (g->nb + kCB - 1) / kCB;
  g->t_first = a.row_base / kQ8Tile;
  g->n_rt = a.n_range > 0 ? (a.row_base + a.n_range + kQ8Tile - 1) / kQ8Tile - g->t_first : 0;
  g->n_vt = g->n_rt + a.n_extra;
  return true;
}

}  // namespace

size_t q8_part_floats(const DevMat& w, int64_t n_rows, int M) {
  const int64_t nc = (w.cols / 32 + kCB - 1) / kCB;
  return (size_t)(q8_tiles(n_rows) + 1 + 4) * nc * M * 16;
}

cudaError_t launch_gemv_q8(const GemvArgs& a, Epi epi, cudaStream_t st) {
  Q8Geo g;
  if ((a.w.dtype != SX_DTYPE_Q8_0 && a.w.dtype != kDtypeQ4KT) || !a.part || a.M < 1 || a.M > kMaxPrefillTok ||
      !make_geo(a, &g))
    return cudaErrorInvalidValue;
  // Q4_K records: whole super-blocks, no extra rows
  if (a.w.dtype == kDtypeQ4KT && (g.nb % kCB || a.n_extra != 0)) return cudaErrorInvalidValue;
  // the SwiGLU pairing is per tile of the whole interleaved matrix
  if (epi == EPI_SWIGLU && (a.row_base != 0 || a.n_extra != 0)) return cudaErrorInvalidValue;
  // x from the w1|w3 partials: one token, Q8_0, no RMSNorm, at most kQkvChunks k-chunks
  if (a.glu_part && (a.M != 1 || a.w.dtype != SX_DTYPE_Q8_0 || a.norm_w || a.glu_nc < 1 || a.glu_nc > kQkvChunks))
    return cudaErrorInvalidValue;
  int Mt = 1;
  while (Mt < a.M) Mt <<= 1;
  if ((size_t)g.n_vt * g.nc * Mt * 16 > a.part_cap) return cudaErrorInvalidValue;
  switch (Mt) {
    case 1: return launch_m<1>(a, epi, g, st);
    case 2: return launch_m<2>(a, epi, g, st);
    case 4: return launch_m<4>(a, epi, g, st);
    case 8: return launch_m<8>(a, epi, g, st);
    case 16: return launch_m<16>(a, epi, g, st);
    case 32: return launch_m<32>(a, epi, g, st);
    default: return launch_m<64>(a, epi, g, st);
  }
}

}  // namespace sx
