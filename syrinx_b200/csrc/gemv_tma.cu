// gemv_tma.cu — batch-1 Q8_0 decode GEMV fed by the TMA engine.
//
// Same contract as the register-streaming GEMV in gemv.cu (y = x . W^T with the RMSNorm
// prologue and the store / residual / SwiGLU / argmax epilogues; the reference linear is
// `Weights::linear`, crates/syrinx-fish/src/s2/nn.rs:61-68, an f32 matmul against the
// dequantised weight), built for the M = 1 decode step:
//
//   * one persistent CTA per SM owns a balanced, contiguous range of weight rows. Rows of
//     the SoA Q8_0 layout are contiguous in HBM, so a stage of R whole rows is ONE bulk copy
//     of R*K quant bytes plus one of R*s_stride scales (about 40 KB per stage). The TMA
//     engine's cost is per copy (on B200 a CTA streams ~3.7 TB/s device-wide with 2 KB
//     copies but ~7 TB/s with 20-32 KB copies), so stages are sized by bytes, not rows;
//   * a producer warp fills a ring of such stages (at most 108 KB of shared memory, so two
//     CTAs fit on an SM: under programmatic dependent launch the next GEMV's producer fills
//     its ring before griddepcontrol.wait, and HBM keeps streaming across the boundary);
//   * consumer warps form G row groups x C column warps. Lane l of column warp c owns the
//     16-column unit(s) c*32 + l (+ 32*C): its slice of x, RMS-normalised, lives in
//     registers for the whole kernel. In every stage the warp computes its rows
//     g, g+G, g+2G, ... for its units — the same unrolled work in every lane — with an exact
//     int8 -> f32 unpack (byte-permute into the 2^23 mantissa) and f32x2 FMAs, releases the
//     ring slot at once (nothing else sits between a slot's data landing and its refill
//     being issued), reduces its rows over the lanes with a reduce-scatter and writes one
//     partial per (row, column warp) into a partials ring of depth 2*ns;
//   * the last warp to finish a stage (a shared counter) sums each row's C partials in a
//     fixed order (deterministic) and applies the epilogue. No warp can run more than ns
//     stages ahead of the slowest one, so a partials buffer is never rewritten before it
//     was read. There is no CTA-wide barrier per stage;
//   * every consumer passes every stage in order, so no thread is ever more than one phase
//     ahead of any mbarrier and the parity waits are unambiguous;
//   * every mbarrier wait is bounded in wall time (globaltimer). A timeout sets the device
//     error flag to 2 and a CTA-wide abort flag: no thread waits again, nothing more is
//     consumed, and the producer waits (bounded) for its copies in flight before the CTA
//     exits. A launch that finds the error flag already raised does no work.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>

#include "sx_device.cuh"
#include "sx_internal.hpp"

namespace sx {
namespace {

constexpr int kMaxWarps = 16;                      // consumer warps (the plan never needs more)
constexpr int kRMax = 32;                          // max rows per stage
constexpr int kMaxSlots = 8;
constexpr int kStageTarget = 40 * 1024;  // quant bytes per stage (two slots fit the budget)
constexpr size_t kSmemBudget = 108 * 1024;  // two CTAs (+1 KB reserved each) fit in 228 KB
constexpr uint64_t kWaitNs = 1000000000ull;  // bound on any single mbarrier wait (1 s)

// Launch plan of one weight matrix (host side).
struct TmaPlan {
  int upt = 1;         // x units per lane (1 or 2)
  int C = 0;           // column warps per row group
  int G = 0;           // row groups
  int R = 0;           // rows per stage (multiple of G; even for gate/up pairs)
  int nr = 0;          // rows per group per stage = R / G (template bound 2, 4 or 8)
  int ns = 0;          // ring slots
  int slot_q = 0;      // byte offset of the scale block inside a slot
  int slot_bytes = 0;  // bytes per slot (multiple of 128)
  size_t smem = 0;
};

int round128(int v) { return (v + 127) & ~127; }

// Fills `p`; returns false when the shape does not fit the kernel.
bool make_plan(int64_t K64, int64_t s_stride, bool pairs, TmaPlan* p) {
  if (K64 <= 0 || K64 % 32 || K64 > 16384) return false;
  const int K = (int)K64, U = K / 16;
  const int upt = (U + 31) / 32 <= 16 ? 1 : 2;
  const int C = (U + 32 * upt - 1) / (32 * upt);
  if (C > 16) return false;
  int R = std::max(1, std::min(kRMax, kStageTarget / K));
  // row groups so that each warp computes about 8 rows per stage: the per-stage work
  // (wait, release, reduce-scatter, partials) is then spread over 8 rows
  const int G = std::max(1, std::min(kMaxWarps / C, R / 8));
  if (G * C > kMaxWarps) return false;
  const int step = (pairs && G % 2) ? 2 * G : G;
  R = std::min(R, 8 * G);
  R = std::max(step, R / step * step);
  if (R > kRMax || R / G > 8) return false;
  const int slot_q = round128(R * K);
  const int slot_bytes = slot_q + round128(R * (int)s_stride * 2);
  const size_t red = (size_t)2 * R * C * sizeof(float);  // partials: two per ring slot
  const size_t fixed = 3 * kMaxSlots * sizeof(uint64_t);  // full[8], empty[8], cnt[16]
  const int ns = (int)std::min<size_t>(kMaxSlots, (kSmemBudget - fixed) / (slot_bytes + red));
  if (ns < 2) return false;
  p->upt = upt;
  p->C = C;
  p->G = G;
  p->R = R;
  p->nr = R / G;
  p->ns = ns;
  p->slot_q = slot_q;
  p->slot_bytes = slot_bytes;
  p->smem = (size_t)ns * (slot_bytes + red) + fixed;
  return true;
}

struct KParams {
  int C, G, R, ns, slot_q, slot_bytes;
};

// 1: the phase completed; 0: another warp aborted the CTA; -1: timed out.
__device__ __forceinline__ int wait_phase(uint64_t* bar, uint32_t parity, const volatile int* abort_flag) {
  if (mbar_test_wait(bar, parity)) return 1;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait_hint(bar, parity, kTryWaitHintNs)) return 1;
    if (*abort_flag) return 0;
    if (global_ns() - t0 > kWaitNs) return -1;
  }
}

// A bounded wait gave up: raise the CTA-wide abort flag (first report prints where) and
// the device error flag.
__device__ void tma_timeout(int* err, int* abort_flag, const char* what, int s, int slot, int ns, int K) {
  if (atomicExch(abort_flag, 1) == 0)
    printf("syrinx gemv_tma: %s wait timed out (cta %d warp %d stage %d slot %d slots %d K %d)\n", what,
           (int)blockIdx.x, (int)(threadIdx.x >> 5), s, slot, ns, K);
  if (err) atomicExch(err, 2);
}

__device__ __forceinline__ int phys_row_t(const GemvArgs& a, int i) {
  return i < a.n_range ? a.row_base + i : a.extra[i - a.n_range];
}

// Logical rows of the stage starting at logical row `i` (CTA range end r1): up to R rows of
// the contiguous range part, or a single extra row.
__device__ __forceinline__ int stage_rows(const GemvArgs& a, int i, int r1, int R) {
  return i < a.n_range ? min(R, min(r1, a.n_range) - i) : 1;
}

// dot of one 16-column unit: exact int8 -> f32, two f32x2 chains
__device__ __forceinline__ float dot16(const uint4 wq, const ulonglong2 (&xv)[4]) {
  unsigned long long wv[8];
  u8b4_to_f32x2x2(wq.x, wv[0], wv[1]);
  u8b4_to_f32x2x2(wq.y, wv[2], wv[3]);
  u8b4_to_f32x2x2(wq.z, wv[4], wv[5]);
  u8b4_to_f32x2x2(wq.w, wv[6], wv[7]);
  unsigned long long s0 = 0ull, s1 = 0ull;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    s0 = fma2(wv[2 * i], xv[i].x, s0);
    s1 = fma2(wv[2 * i + 1], xv[i].y, s1);
  }
  float a0, a1;
  unpack2(add2(s0, s1), a0, a1);
  return a0 + a1;
}

// Recursive-halving reduce-scatter of NR per-lane values over a warp: afterwards v[0] of
// lane l holds the warp-wide sum of value l >> (5 - log2 NR). NR - 1 + 5 - log2 NR shuffles
// (6 for NR = 4) instead of 5 NR, in a fixed tree.
template <int NR>
__device__ __forceinline__ void reduce_scatter(float (&v)[NR], int lane) {
#pragma unroll
  for (int h = NR / 2, o = 16; h >= 1; h >>= 1, o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < h; i++) {
      const float send = upper ? v[i] : v[i + h];
      const float keep = upper ? v[i + h] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  constexpr int m = NR == 2 ? 1 : (NR == 4 ? 2 : 3);
#pragma unroll
  for (int o = 16 >> m; o > 0; o >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
}

template <int EPI, int UPT, int NR>
__global__ void __maxnreg__(UPT == 1 ? 80 : 96) k_gemv_q8_tma(const GemvArgs a, const KParams kp) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ float ssq[kMaxWarps];
  __shared__ unsigned long long cta_best;
  __shared__ int abort_flag;

  const int K = (int)a.w.cols;
  const int U = K / 16;
  const int C = kp.C, G = kp.G, R = kp.R, ns = kp.ns;
  const int W = C * G;  // consumer warps
  const int n_logical = a.n_range + a.n_extra;
  constexpr int g2 = (EPI == EPI_SWIGLU) ? 2 : 1;  // gate/up pairs never straddle CTAs or stages
  const int n_units = n_logical / g2;
  const int r0 = (int)((long long)blockIdx.x * n_units / gridDim.x) * g2;
  const int r1 = (int)((long long)(blockIdx.x + 1) * n_units / gridDim.x) * g2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  uint8_t* ring = sm;
  float* red = reinterpret_cast<float*>(sm + (size_t)ns * kp.slot_bytes);  // [2 ns][R][C]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + (size_t)2 * ns * R * C);
  uint64_t* empty = full + kMaxSlots;
  int* cnt = reinterpret_cast<int*>(empty + kMaxSlots);  // [2 ns]

  if (threadIdx.x == 0) {
    for (int i = 0; i < ns; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], W);
    }
    for (int i = 0; i < 2 * ns; i++) cnt[i] = 0;
    abort_flag = 0;
    cta_best = 0ull;
    mbar_fence_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == W) {
    // ------------- producer: weights do not depend on the previous kernel -------------
    if (lane == 0) {
      const int8_t* q = (const int8_t*)a.w.q;
      const __half* sc = a.w.s;
      const int64_t ss = a.w.s_stride;
      int issued = 0;
      for (int i = r0, s = 0; i < r1; s++) {
        const int rows = stage_rows(a, i, r1, R);
        const int slot = s % ns, round = s / ns;
        if (round > 0) {
          const int w = wait_phase(&empty[slot], (uint32_t)(round - 1) & 1, &abort_flag);
          if (w <= 0) {
            if (w < 0) tma_timeout(a.err, &abort_flag, "empty", s, slot, ns, K);
            break;
          }
        } else if (*(volatile int*)&abort_flag) {
          break;
        }
        const int pr = phys_row_t(a, i);
        const uint32_t qb = (uint32_t)rows * (uint32_t)K, sb = (uint32_t)rows * (uint32_t)ss * 2u;
        mbar_arrive_expect_tx(&full[slot], qb + sb);
        uint8_t* dst = ring + (size_t)slot * kp.slot_bytes;
        bulk_g2s(dst, q + (size_t)pr * K, qb, &full[slot]);
        bulk_g2s(dst + kp.slot_q, sc + (size_t)pr * ss, sb, &full[slot]);
        issued = s + 1;
        i += rows;
      }
      // Copies still in flight must land before this CTA's shared memory is released.
      for (int s = max(0, issued - ns); s < issued; s++)
        (void)mbar_wait_bounded(&full[s % ns], (uint32_t)(s / ns) & 1, kWaitNs);
    }
    pdl_wait();
    return;
  }

  // ------------------------------- consumers -------------------------------
  const int g = warp / C, c = warp % C;
  int uk[UPT];
  bool uv[UPT];
#pragma unroll
  for (int k = 0; k < UPT; k++) {
    uk[k] = c * 32 + lane + k * 32 * C;
    uv[k] = uk[k] < U;
  }
  // norm gains are weights: read before waiting on the previous kernel
  float4 nw[UPT][4];
#pragma unroll
  for (int k = 0; k < UPT; k++)
#pragma unroll
    for (int i = 0; i < 4; i++)
      nw[k][i] = (a.norm_w && uv[k]) ? *reinterpret_cast<const float4*>(a.norm_w + uk[k] * 16 + i * 4)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
  pdl_wait();
  if (threadIdx.x == 0 && a.err && ld_cg(a.err) != 0) atomicExch(&abort_flag, 1);  // an earlier kernel gave up
  float4 xf[UPT][4];
#pragma unroll
  for (int k = 0; k < UPT; k++)
#pragma unroll
    for (int i = 0; i < 4; i++) xf[k][i] = uv[k] ? ld_cg4(a.x + uk[k] * 16 + i * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
  if (a.norm_w) {
    // each unit is counted once, by row group 0
    float s2 = 0.f;
    if (g == 0) {
#pragma unroll
      for (int k = 0; k < UPT; k++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
          s2 = fmaf(xf[k][i].x, xf[k][i].x, s2);
          s2 = fmaf(xf[k][i].y, xf[k][i].y, s2);
          s2 = fmaf(xf[k][i].z, xf[k][i].z, s2);
          s2 = fmaf(xf[k][i].w, xf[k][i].w, s2);
        }
      s2 = warp_sum(s2);
      if (lane == 0) ssq[warp] = s2;
    }
    named_bar_sync(1, W * 32);
    float t = 0.f;
    for (int w = 0; w < C; w++) t += ssq[w];
    const float den = sqrtf(__fadd_rn(__fdiv_rn(t, (float)K), a.eps));
#pragma unroll
    for (int k = 0; k < UPT; k++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        xf[k][i].x = __fmul_rn(__fdiv_rn(xf[k][i].x, den), nw[k][i].x);
        xf[k][i].y = __fmul_rn(__fdiv_rn(xf[k][i].y, den), nw[k][i].y);
        xf[k][i].z = __fmul_rn(__fdiv_rn(xf[k][i].z, den), nw[k][i].z);
        xf[k][i].w = __fmul_rn(__fdiv_rn(xf[k][i].w, den), nw[k][i].w);
      }
  } else {
    named_bar_sync(1, W * 32);  // the abort flag from the error check is visible to all
  }
  ulonglong2 xr[UPT][4];
#pragma unroll
  for (int k = 0; k < UPT; k++)
#pragma unroll
    for (int i = 0; i < 4; i++) {
      xr[k][i].x = pack2(xf[k][i].x, xf[k][i].y);
      xr[k][i].y = pack2(xf[k][i].z, xf[k][i].w);
    }

  const int srow = (int)a.w.s_stride * 2;
  bool aborted = false;  // warp-uniform
  for (int i = r0, s = 0; i < r1; s++) {
    const int rows = stage_rows(a, i, r1, R);
    const int row0 = i;
    i += rows;
    if (aborted) continue;
    const int slot = s % ns;
    const int w = wait_phase(&full[slot], (uint32_t)(s / ns) & 1, &abort_flag);
    const bool all_ok = __all_sync(0xffffffffu, w == 1);
    if (!all_ok) {
      aborted = true;  // after an abort nothing is consumed or released
      if (__any_sync(0xffffffffu, w < 0) && lane == 0) tma_timeout(a.err, &abort_flag, "full", s, slot, ns, K);
      continue;
    }
    const uint8_t* base = ring + (size_t)slot * kp.slot_bytes;
    const uint8_t* sbase = base + kp.slot_q;
    const int ps = s % (2 * ns);  // partials slot
    float* rd = red + (size_t)ps * R * C;
    // this warp's rows g, g+G, ...: every lane does the same work
    float acc[NR];
#pragma unroll
    for (int j = 0; j < NR; j++) {
      acc[j] = 0.f;
      const int r = g + G * j;
      if (j * G < R && r < rows) {
#pragma unroll
        for (int k = 0; k < UPT; k++)
          if (uv[k]) {
            const uint4 wq = *reinterpret_cast<const uint4*>(base + (size_t)r * K + uk[k] * 16);
            const float d = __half2float(*reinterpret_cast<const __half*>(sbase + r * srow + (uk[k] >> 1) * 2));
            acc[j] = fmaf(d, dot16(wq, xr[k]), acc[j]);
          }
      }
    }
    // the ring slot is free as soon as this warp's reads of it are done
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    // row sums over the lanes: recursive-halving reduce-scatter; afterwards lane l holds
    // the full sum of value j = l >> (5 - log2 NR)
    reduce_scatter<NR>(acc, lane);
    constexpr int kShift = 5 - (NR == 2 ? 1 : (NR == 4 ? 2 : 3));
    {
      const int j = lane >> kShift, r = g + G * j;
      if ((lane & ((1 << kShift) - 1)) == 0 && j * G < R && r < rows) rd[r * C + c] = acc[0];
    }
    // the last warp to finish this stage sums its rows (partials ring of depth 2 ns: a warp
    // can be at most ns stages ahead of the slowest, so no partial is rewritten early)
    __syncwarp();
    int prev = 0;
    if (lane == 0) {
      __threadfence_block();
      prev = atomicAdd(&cnt[ps], 1);
    }
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev == W - 1) {
      __threadfence_block();
      if constexpr (EPI == EPI_SWIGLU) {
        for (int p = lane; 2 * p < rows; p += 32) {
          float gs = 0.f, us = 0.f;
          for (int q = 0; q < C; q++) {
            gs += rd[(2 * p) * C + q];
            us += rd[(2 * p + 1) * C + q];
          }
          a.y[(row0 + 2 * p) >> 1] = __fmul_rn(silu_f(gs), us);
        }
      } else {
        for (int r = lane; r < rows; r += 32) {
          float v = 0.f;
          for (int q = 0; q < C; q++) v += rd[r * C + q];
          const int pr = phys_row_t(a, row0 + r);
          if (a.bias) v = __fadd_rn(v, a.bias[pr]);
          if constexpr (EPI == EPI_ARGMAX) {
            if (a.y) a.y[pr] = v;
            const uint32_t upr = (uint32_t)pr;
            if ((upr >= a.allow_lo && upr <= a.allow_hi) || (upr >= a.stop_lo && upr < a.stop_hi))
              atomicMax(&cta_best, argmax_key(v, upr));
          } else if constexpr (EPI == EPI_ADD) {
            a.y[pr] = __fadd_rn(ld_cg(a.y + pr), v);
          } else {
            a.y[pr] = v;
          }
        }
      }
      if (lane == 0) cnt[ps] = 0;
      __syncwarp();
    }
  }
  if constexpr (EPI == EPI_ARGMAX) {
    named_bar_sync(1, W * 32);
    if (threadIdx.x == 0 && !*(volatile int*)&abort_flag && cta_best != 0ull) atomicMax(a.amax, cta_best);
  }
}

int sms_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <int EPI, int UPT, int NR>
cudaError_t launch_tma_x(const GemvArgs& a, const TmaPlan& p, int grid, cudaStream_t st) {
  auto kern = k_gemv_q8_tma<EPI, UPT, NR>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = launch_cfg(dim3(grid), dim3((p.C * p.G + 1) * 32), p.smem, st, attr);
  const KParams kp{p.C, p.G, p.R, p.ns, p.slot_q, p.slot_bytes};
  return cudaLaunchKernelEx(&cfg, kern, a, kp);
}

template <int EPI, int UPT>
cudaError_t launch_tma_u(const GemvArgs& a, const TmaPlan& p, int grid, cudaStream_t st) {
  if (p.nr <= 2) return launch_tma_x<EPI, UPT, 2>(a, p, grid, st);
  if (p.nr <= 4) return launch_tma_x<EPI, UPT, 4>(a, p, grid, st);
  return launch_tma_x<EPI, UPT, 8>(a, p, grid, st);
}

template <int EPI>
cudaError_t launch_tma_t(const GemvArgs& a, cudaStream_t st) {
  static const int sms = sms_count();
  TmaPlan p;
  if (!make_plan(a.w.cols, a.w.s_stride, EPI == EPI_SWIGLU, &p)) return cudaErrorInvalidValue;
  const int n_units = (a.n_range + a.n_extra) / (EPI == EPI_SWIGLU ? 2 : 1);
  if (n_units <= 0) return cudaErrorInvalidValue;
  const int grid = std::min(n_units, sms);
  return p.upt == 1 ? launch_tma_u<EPI, 1>(a, p, grid, st) : launch_tma_u<EPI, 2>(a, p, grid, st);
}

}  // namespace

bool gemv_tma_eligible(const GemvArgs& a) {
  // Q8_0, one token, K a multiple of 32 with the padded scale layout, a plan that fits
  TmaPlan p;
  const int n_logical = a.n_range + a.n_extra;
  return a.w.dtype == SX_DTYPE_Q8_0 && a.M == 1 && a.w.s_stride == q8_scale_stride(a.w.cols) && n_logical > 0 &&
         make_plan(a.w.cols, a.w.s_stride, false, &p) && make_plan(a.w.cols, a.w.s_stride, true, &p);
}

cudaError_t launch_gemv_tma(const GemvArgs& a, Epi epi, cudaStream_t st) {
  (void)cudaGetLastError();
  switch (epi) {
    case EPI_STORE: return launch_tma_t<EPI_STORE>(a, st);
    case EPI_ADD: return launch_tma_t<EPI_ADD>(a, st);
    case EPI_SWIGLU:
      if (a.n_extra != 0 || (a.n_range & 1)) return cudaErrorInvalidValue;
      return launch_tma_t<EPI_SWIGLU>(a, st);
    case EPI_ARGMAX: return launch_tma_t<EPI_ARGMAX>(a, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace sx
