// stack.cu — the persistent decode kernel: every layer of one transformer stack (the slow AR's
// 36 layers, or the fast AR's 4 for one codebook step) for a decode batch of 1..8 tokens in
// ONE cooperative launch of one CTA per SM.
//
// Replaces, for Q8_0 weights, the per-layer kernel chain of the decoder block
// (crates/syrinx-fish/src/s2/slow_ar.rs:166-202; attention s2/nn.rs:284-360, swiglu
// s2/nn.rs:452-457; the CosyVoice2 block cv2/mod.rs:261-279, cv2/attention.rs:46-78) — nine
// launches per layer, each paying its own ramp-up, drain and dependency wait — with one
// kernel whose HBM stream never stops between phases.
//
// Warp roles. Warps 0-7 compute; one lane of warp 8 is the producer. The producer walks every
// weight item this CTA will need in the order the consumers use them (per layer: wqkv, wo,
// w1|w3, w2) and copies each item (8 consecutive 544-byte tile records of one 16-row tile:
// 4352 contiguous bytes) into a ring of shared-memory slots with cp.async.bulk, completion
// counted on the slot's mbarrier. It depends on nothing but free slots, so while the
// consumers wait at a grid barrier or run attention, the next matrices are already streaming
// into shared memory. Plain bulk copies of this GPU's own memory: no tensor map, no multicast.
//
// Phases of a layer, separated by grid barriers (a monotonically increasing u64 counter; every
// wait is bounded by %globaltimer and raises the error flag instead of hanging):
//   P1 wqkv   prologue: x = x + (w2 partials of the previous layer) — the residual add of the
//             previous layer, folded in here — for this CTA's k range only; the CTA owning a
//             256-wide k chunk writes x back and that chunk's sum of squares. Limbs of x * g.
//   P2 attn   one CTA per (token, kv head, split of the key axis): merge the wqkv partials of
//             its heads, divide by the RMS denominator (from the chunk sums), + bias, QK-norm,
//             RoPE, KV append by the split that holds the new position, online softmax over
//             its key slice; writes (max, sum, acc) per head.
//   P3 wo     prologue: merge the attention splits for this CTA's k range.
//   P4 w1|w3  prologue: x = x + (wo partials) + bias, chunk owners write x and sums of squares.
//   P5 w2     prologue: act = silu(g / den) * (u / den) from the w1|w3 partials.
// and a final phase adds the last w2 partials into x.
//
// The RMSNorm is applied after the GEMV: rms_norm(x) . W^T = (x * g) . W^T / den, den a scalar
// per token (s2/nn.rs:100-106). The GEMV arithmetic is that of gemv_q8.cu: exact int32 block
// sums of the int8 quants against the four int8 limbs of (x * g), scaled per block in f32.
// Every partial is added in a fixed order, so the result does not depend on the schedule.
#include <cuda_runtime.h>

#include <algorithm>

#include "sx_device.cuh"
#include "sx_internal.hpp"

namespace sx {
namespace {

constexpr int kCW = 8;                 // consumer warps
constexpr int kCT = kCW * 32;          // consumer threads
constexpr int kThreadsStack = kCT + 32;  // + the producer warp
constexpr int kIB = kStackChunkBlocks;  // 32-wide k blocks per item (one k chunk of 512)
constexpr int kItemBytes = kIB * kQ8Rec;  // 8704
constexpr int kSpanBlocks = 32;        // k blocks a CTA's item range may span in one matrix
constexpr int kNCMax = 20;             // k chunks of any matrix (K <= 10240)
constexpr int kMaxSplit = 32;          // splits of the key axis (one per lane in the merge)
constexpr int kInflight = 10;          // weight items a CTA's producer keeps in flight (87 KB)
// prologue units (block, token) a warp gathers per batch (register budget: <= ~80 loads)
constexpr int kUBResid = 3, kUBAttn = 2, kUBSwiglu = 2;
constexpr uint64_t kBarWaitNs = 2000000000ull;  // grid / mbarrier wait limit

struct MatGeo {
  const uint8_t* w;  // unused on the host side of the geometry
  int K, nb, nc, n_vt;
};

__device__ __forceinline__ void cta_items(int n_vt, int nc, long long* c0, long long* c1) {
  const long long I = (long long)n_vt * nc;
  *c0 = (long long)blockIdx.x * I / gridDim.x;
  *c1 = (long long)(blockIdx.x + 1) * I / gridDim.x;
}

// ---- grid barrier ---------------------------------------------------------------------
// Arrive: every consumer thread's writes are ordered by the named barrier, thread 0 makes
// them visible at GPU scope and counts the CTA in. Returns the count that completes it.
__device__ __forceinline__ unsigned long long grid_arrive(const StackArgs& a) {
  bar_sync_n(1, kCT);
  unsigned long long target = 0;
  if (threadIdx.x == 0) {
    // a release at GPU scope after the CTA barrier: cumulative over the consumer threads'
    // writes that the named barrier ordered before it (no full fence needed)
    unsigned long long old;
    asm volatile("atom.add.release.gpu.global.u64 %0, [%1], 1;" : "=l"(old) : "l"(a.bar) : "memory");
    target = (old / gridDim.x + 1) * gridDim.x;
  }
  return target;
}
__device__ __forceinline__ void grid_wait(const StackArgs& a, unsigned long long target) {
  if (threadIdx.x == 0) {
    const uint64_t t0 = global_ns();
    while (ld_acquire_gpu(a.bar) < target) {
      if (ld_cg(a.err) != 0) break;  // another CTA gave up: do not wait out the limit again
      if (global_ns() - t0 > kBarWaitNs) {
        atomicExch(a.err, 2);
        break;
      }
    }
  }
  bar_sync_n(1, kCT);
}

// Bounded wait on a ring slot's mbarrier. Past 1 ms it also gives up when another wait of the
// launch has already failed, so a broken launch ends after one limit, not one per item.
__device__ __forceinline__ void mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    const uint64_t dt = global_ns() - t0;
    if (dt > 1000000ull && __ldcg(err) != 0) return;
    if (dt > kBarWaitNs) {
      atomicExch(err, 2);
      return;
    }
  }
}

// ---- shared memory ----------------------------------------------------------------------
constexpr int kSpanHeads = 16;  // attention heads a CTA's wo k range may touch (32 blocks / hd 64)
template <int MT>
struct Smem {
  static constexpr int NP = (MT + 1) / 2;  // token pairs (tensor-core B columns 0-3 / 4-7)
  // limb B fragments [block][NP][32 lanes] and per-(block, token) scales / sums of squares
  uint2 bfr[kSpanBlocks][NP][32];
  float sxs[kSpanBlocks][MT];
  float ssb[kSpanBlocks][MT];
  int8_t scr[kCW][4][32];
  float den[kMaxTok];
  // attention-split merge weights of the heads in the wo k range [head][token][split]
  float wts[kSpanHeads][MT][kMaxSplit];
  float lsum[kSpanHeads][MT];
};
template <int HD>
struct AttnSmem {
  float qs[kMaxGroup][HD];
  float wacc[kCW][kMaxGroup][HD];
  float wm[kCW][kMaxGroup], wl[kCW][kMaxGroup];
  float kbuf[HD], vbuf[HD];
  float den[kMaxTok];
};

template <int MT, int HD>
constexpr size_t scratch_bytes() {
  return sizeof(Smem<MT>) > sizeof(AttnSmem<HD>) ? sizeof(Smem<MT>) : sizeof(AttnSmem<HD>);
}

// ---- the limb split of one (block, token) of x (as gemv_q8.cu: exact to 2^-27 of the block max)
template <int MT>
__device__ __forceinline__ void split_limbs(Smem<MT>& sm, int warp, int lane, int bi, int m, float v) {
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
  sm.scr[warp][0][lane] = (int8_t)(int)l0;
  sm.scr[warp][1][lane] = (int8_t)(int)l1;
  sm.scr[warp][2][lane] = (int8_t)(int)l2;
  sm.scr[warp][3][lane] = (int8_t)(int)l3;
  __syncwarp();
  if (lane < 16) {
    const int n = lane >> 2, c = lane & 3;
    uint2 w;
    w.x = *reinterpret_cast<const uint32_t*>(&sm.scr[warp][n][4 * c]);
    w.y = *reinterpret_cast<const uint32_t*>(&sm.scr[warp][n][16 + 4 * c]);
    sm.bfr[bi][m >> 1][(m & 1) * 16 + lane] = w;
  }
  if (lane == 0) sm.sxs[bi][m] = sx;
  __syncwarp();
}

// Sum of partials of output row `row` (tile row r of virtual tile vt) over the k chunks: every
// load is issued before the first add (one L2 round trip), the adds run in chunk order.
template <int MT>
__device__ __forceinline__ float sum_part(const float* part, int nc, int row, int m) {
  const float* p = part + ((size_t)(row >> 4) * nc * MT + m) * 16 + (row & 15);
  float v[kNCMax];
#pragma unroll
  for (int kc = 0; kc < kNCMax; kc++) v[kc] = kc < nc ? __ldcg(p + (size_t)kc * MT * 16) : 0.f;
  float s = 0.f;
#pragma unroll
  for (int kc = 0; kc < kNCMax; kc++)
    if (kc < nc) s += v[kc];
  return s;
}

// RMS denominators of the tokens from the per-chunk sums of squares, by warp 0 (one chunk per
// lane, a butterfly sum that every lane and every CTA evaluates identically) into den[MT].
template <int MT>
__device__ __forceinline__ void rms_den_all(const StackArgs& a, const float* ss, float* den) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
#pragma unroll
    for (int m = 0; m < MT; m++) {
      const float v = (lane < a.nc_dim && m < a.M) ? __ldcg(ss + (size_t)m * 64 + lane) : 0.f;
      const float t = warp_sum(v);
      if (lane == 0) den[m] = sqrtf(__fadd_rn(__fdiv_rn(t, (float)a.dim), a.eps));
    }
  }
}

// ---- GEMV phase ------------------------------------------------------------------------
// Consumes this CTA's items [c0, c1) of one matrix from the ring (item j of the phase by warp
// j % 8) and writes each item's 16 row sums per token to `part` [vt][kc][MT][16].
template <int MT>
__device__ void gemv_consume(Smem<MT>& sm, uint8_t* ring, uint64_t* full, uint64_t* empty, int nslot,
                             long long& ctr, const MatGeo& g, long long c0, long long c1, int b_lo, int M,
                             float* part, int* err) {
  constexpr int NP = Smem<MT>::NP;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bl = MT == 1 ? (lane & 15) : lane;
  const int n = (int)(c1 - c0);
  // this warp's items j = warp, warp + 8, ...: (k chunk, tile) and (slot, round) advance
  // incrementally, no division per item
  int kc = (int)((c0 + warp) / g.n_vt), vt = (int)((c0 + warp) % g.n_vt);
  int slot = (int)((ctr + warp) % nslot), round = (int)((ctr + warp) / nslot);
  for (int j = warp; j < n; j += kCW) {
    const uint32_t par = (uint32_t)(round & 1);
    mbar_wait_bounded(&full[slot], par, err);
    const uint8_t* rec = ring + (size_t)slot * kItemBytes;
    float acc[NP][2];
#pragma unroll
    for (int p = 0; p < NP; p++) acc[p][0] = acc[p][1] = 0.f;
#pragma unroll
    for (int i = 0; i < kIB; i++) {
      const int b = kc * kIB + i;
      if (b < g.nb) {
        const uint4 q = lds128(rec + i * kQ8Rec + lane * 16);
        const uint32_t sw = lds32(rec + i * kQ8Rec + 512 + (lane >> 2) * 4);
        const float2 ds = __half22float2(*reinterpret_cast<const __half2*>(&sw));
        const int bi = b - b_lo;
#pragma unroll
        for (int p = 0; p < NP; p++) {
          const uint2 bf = sm.bfr[bi][p][bl];
          const int tok = MT == 1 ? 0 : 2 * p + ((lane >> 1) & 1);
          const float sx = sm.sxs[bi][tok < MT ? tok : 0];
          int d[4];
          mma_s8_16832(q, bf, d);
          acc[p][0] = fmaf(__fmul_rn(ds.x, sx), (float)(d[0] * 128 + d[1]), acc[p][0]);
          acc[p][1] = fmaf(__fmul_rn(ds.y, sx), (float)(d[2] * 128 + d[3]), acc[p][1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    const float wgt = (lane & 1) ? 0x1p-21f : 0x1p-7f;
    float* P = part + ((size_t)vt * g.nc + kc) * MT * 16;
#pragma unroll
    for (int p = 0; p < NP; p++) {
      float v0 = acc[p][0] * wgt, v1 = acc[p][1] * wgt;
      v0 += __shfl_down_sync(0xffffffffu, v0, 1);
      v1 += __shfl_down_sync(0xffffffffu, v1, 1);
      const int tok = 2 * p + ((lane >> 1) & 1);
      if ((lane & 1) == 0 && tok < MT) {
        __stcg(P + tok * 16 + (lane >> 2), v0);
        __stcg(P + tok * 16 + (lane >> 2) + 8, v1);
      }
    }
    slot += kCW;
    if (slot >= nslot) slot -= nslot, round++;
    vt += kCW;
    while (vt >= g.n_vt) vt -= g.n_vt, kc++;
  }
  (void)M;
  ctr += n;
}

// k range [b_lo, b_hi) of this CTA's items of a matrix (blocks of 32)
__device__ __forceinline__ void k_range(const MatGeo& g, long long c0, long long c1, int* b_lo, int* b_hi,
                                        int* kc_lo, int* kc_hi) {
  *kc_lo = (int)(c0 / g.n_vt);
  *kc_hi = c1 > c0 ? (int)((c1 - 1) / g.n_vt) : *kc_lo;
  *b_lo = *kc_lo * kIB;
  *b_hi = min(g.nb, (*kc_hi + 1) * kIB);
  if (c1 <= c0) *b_hi = *b_lo;
}

// ---- residual prologue (P1 and P4): x_new = x + partials (+ bias) for this CTA's k range;
// the owner of each k chunk writes x_new and the chunk's sum of squares; limbs of x_new * g.
// A warp's units (block, token) go in batches of kUBResid whose loads are all issued before any use.
template <int MT>
__device__ void resid_prologue(Smem<MT>& sm, const StackArgs& a, const MatGeo& g, long long c0, long long c1,
                               const float* x_in, float* x_out, const float* part, int nc_part,
                               const float* bias, const float* gain, float* ss_out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int b_lo, b_hi, kc_lo, kc_hi;
  k_range(g, c0, c1, &b_lo, &b_hi, &kc_lo, &kc_hi);
  const int dim = a.dim, n_units = (b_hi - b_lo) * MT;
  const int npart = part ? nc_part : 0;
  for (int u0 = warp; u0 < n_units; u0 += kUBResid * kCW) {
    float xv[kUBResid], pv[kUBResid][kNCMax];
#pragma unroll
    for (int j = 0; j < kUBResid; j++) {
      const int u = u0 + j * kCW, bi = u / MT, m = u % MT, k = (b_lo + bi) * 32 + lane;
      const bool ok = u < n_units && m < a.M;
      xv[j] = ok ? __ldcg(x_in + (size_t)m * dim + k) : 0.f;
      const float* p = part + ((size_t)(k >> 4) * nc_part * MT + m) * 16 + (k & 15);
#pragma unroll
      for (int kc = 0; kc < kNCMax; kc++) pv[j][kc] = (ok && kc < npart) ? __ldcg(p + (size_t)kc * MT * 16) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kUBResid; j++) {
      const int u = u0 + j * kCW;
      if (u >= n_units) break;
      const int bi = u / MT, m = u % MT, k = (b_lo + bi) * 32 + lane;
      float v = 0.f;
      if (m < a.M) {
        float x = xv[j];
        if (npart) {
          float t = 0.f;
#pragma unroll
          for (int kc = 0; kc < kNCMax; kc++)
            if (kc < npart) t += pv[j][kc];
          if (bias) t = __fadd_rn(t, bias[k]);
          x = __fadd_rn(x, t);
        }
        const int kc = (b_lo + bi) / kIB;
        const bool owner = (long long)kc * g.n_vt >= c0 && (long long)kc * g.n_vt < c1;
        if (owner) __stcg(x_out + (size_t)m * dim + k, x);
        const float sq = warp_sum(x * x);
        if (lane == 0) sm.ssb[bi][m] = sq;
        v = __fmul_rn(x, gain[k]);
      } else if (lane == 0) {
        sm.ssb[bi][m] = 0.f;
      }
      split_limbs<MT>(sm, warp, lane, bi, m, v);
    }
  }
  bar_sync_n(1, kCT);
  // owners: the sum of squares of each owned chunk, its blocks added in order
  if (threadIdx.x < MT * (kc_hi - kc_lo + 1)) {
    const int m = threadIdx.x % MT, kc = kc_lo + threadIdx.x / MT;
    if ((long long)kc * g.n_vt >= c0 && (long long)kc * g.n_vt < c1 && m < a.M) {
      float s = 0.f;
      for (int b = kc * kIB; b < min(g.nb, (kc + 1) * kIB); b++) s += sm.ssb[b - b_lo][m];
      __stcg(ss_out + (size_t)m * 64 + kc, s);
    }
  }
}

// ---- P3 prologue: attention output for this CTA's k range (merge of the key-axis splits).
// Each warp first issues the accumulator loads of its units (one split per register), then
// computes, one split per lane, the weights exp(m_s - max) and the denominator of the
// (head, token) pairs it owns; after a CTA barrier the units combine the two.
template <int MT>
__device__ void attn_out_prologue(Smem<MT>& sm, const StackArgs& a, const MatGeo& g, long long c0, long long c1) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int b_lo, b_hi, kc_lo, kc_hi;
  k_range(g, c0, c1, &b_lo, &b_hi, &kc_lo, &kc_hi);
  const int G = a.H / a.Hkv, hd = a.hd, ns = a.n_split;
  const size_t per = (size_t)kMaxGroup * (hd + 2);  // floats per split
  auto head_base = [&](int m, int h) {  // split 0 of (token m, head h)
    return a.attn_part + (size_t)((m * a.Hkv + h / G) * ns) * per + (size_t)(h % G) * (hd + 2);
  };
  const int h_lo = (b_lo * 32) / hd;
  const int nh = b_hi > b_lo ? ((b_hi * 32 - 1) / hd) - h_lo + 1 : 0;
  const int n_units = (b_hi - b_lo) * MT;
  for (int u0 = warp; u0 < n_units || u0 == warp; u0 += kUBAttn * kCW) {
    float o[kUBAttn][kMaxSplit];
#pragma unroll
    for (int j = 0; j < kUBAttn; j++) {
      const int u = u0 + j * kCW, bi = u / MT, m = u % MT, k = (b_lo + bi) * 32 + lane;
      const bool ok = u < n_units && m < a.M;
      const float* p = ok ? head_base(m, k / hd) + k % hd : a.attn_part;
#pragma unroll
      for (int sp = 0; sp < kMaxSplit; sp++) o[j][sp] = (ok && sp < ns) ? __ldcg(p + (size_t)sp * per) : 0.f;
    }
    if (u0 == warp) {  // the first batch: this warp's (head, token) weights, in the loads' shadow
      for (int v = warp; v < nh * MT; v += kCW) {
        const int hl = v / MT, m = v % MT;
        float ms = -INFINITY, ls = 0.f;
        if (m < a.M && lane < ns) {
          const float* p = head_base(m, h_lo + hl) + (size_t)lane * per;
          ms = __ldcg(p + hd);
          ls = __ldcg(p + hd + 1);
        }
        const float M_ = warp_max(ms);
        const float w = ms == -INFINITY ? 0.f : expf(ms - M_);
        const float L = warp_sum(ls * w);
        sm.wts[hl][m][lane] = w;
        if (lane == 0) sm.lsum[hl][m] = L;
      }
      bar_sync_n(1, kCT);
    }
#pragma unroll
    for (int j = 0; j < kUBAttn; j++) {
      const int u = u0 + j * kCW;
      if (u >= n_units) break;
      const int bi = u / MT, m = u % MT, k = (b_lo + bi) * 32 + lane;
      float v = 0.f;
      if (m < a.M) {
        const int hl = k / hd - h_lo;
        float O = 0.f;
#pragma unroll
        for (int sp = 0; sp < kMaxSplit; sp++)
          if (sp < ns) O = fmaf(o[j][sp], sm.wts[hl][m][sp], O);
        v = __fdiv_rn(O, sm.lsum[hl][m]);
      }
      split_limbs<MT>(sm, warp, lane, bi, m, v);
    }
  }
  bar_sync_n(1, kCT);
}

// ---- P5 prologue: act = silu(g / den) * (u / den) for this CTA's k range; the partial loads
// of a warp's units and warp 0's sum-of-squares loads go out together.
template <int MT>
__device__ void swiglu_prologue(Smem<MT>& sm, const StackArgs& a, const MatGeo& g, long long c0, long long c1,
                                const float* part13, int nc13) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int b_lo, b_hi, kc_lo, kc_hi;
  k_range(g, c0, c1, &b_lo, &b_hi, &kc_lo, &kc_hi);
  const int n_units = (b_hi - b_lo) * MT;
  bool first = true;
  for (int u0 = warp; u0 < n_units || first; u0 += kUBSwiglu * kCW) {
    float gv[kUBSwiglu][kNCMax], uv[kUBSwiglu][kNCMax];
#pragma unroll
    for (int j = 0; j < kUBSwiglu; j++) {
      const int u = u0 + j * kCW, bi = u / MT, m = u % MT, k = (b_lo + bi) * 32 + lane;
      const bool ok = u < n_units && m < a.M;
      // tile j holds gate rows 8j..8j+7 (tile rows 0-7) and up rows 8j..8j+7 (rows 8-15)
      const int row_g = (k >> 3) * 16 + (k & 7);
      const float* p = part13 + ((size_t)(row_g >> 4) * nc13 * MT + m) * 16 + (row_g & 15);
#pragma unroll
      for (int kc = 0; kc < kNCMax; kc++) {
        gv[j][kc] = (ok && kc < nc13) ? __ldcg(p + (size_t)kc * MT * 16) : 0.f;
        uv[j][kc] = (ok && kc < nc13) ? __ldcg(p + (size_t)kc * MT * 16 + 8) : 0.f;
      }
    }
    if (first) {
      rms_den_all<MT>(a, a.ss + (size_t)64 * MT, sm.den);
      bar_sync_n(1, kCT);
      first = false;
    }
#pragma unroll
    for (int j = 0; j < kUBSwiglu; j++) {
      const int u = u0 + j * kCW;
      if (u >= n_units) break;
      const int bi = u / MT, m = u % MT;
      float v = 0.f;
      if (m < a.M) {
        float gs = 0.f, us = 0.f;
#pragma unroll
        for (int kc = 0; kc < kNCMax; kc++)
          if (kc < nc13) {
            gs += gv[j][kc];
            us += uv[j][kc];
          }
        const float den = sm.den[m];
        v = __fmul_rn(silu_f(__fdiv_rn(gs, den)), __fdiv_rn(us, den));
      }
      split_limbs<MT>(sm, warp, lane, bi, m, v);
    }
  }
  bar_sync_n(1, kCT);
}

// ---- P2: attention of one (token, kv head, split) unit --------------------------------
template <int HD>
__device__ void norm_rope(float* buf, const float* nw, float eps, const float* inv_freq, int interleaved, int pos,
                          int lane) {
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

__device__ __forceinline__ void kv_put(float* p, float v) { *p = v; }
__device__ __forceinline__ void kv_put(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ float kv_back(float v, const float*) { return v; }
__device__ __forceinline__ float kv_back(float v, const __nv_bfloat16*) { return __bfloat162float(__float2bfloat16_rn(v)); }
template <int EPL>
__device__ __forceinline__ void kv_row(const float* p, float (&v)[EPL]) {
  if constexpr (EPL == 4) {
    const float4 r = __ldcg(reinterpret_cast<const float4*>(p));
    v[0] = r.x; v[1] = r.y; v[2] = r.z; v[3] = r.w;
  } else {
    const float2 r = __ldcg(reinterpret_cast<const float2*>(p));
    v[0] = r.x; v[1] = r.y;
  }
}
template <int EPL>
__device__ __forceinline__ void kv_row(const __nv_bfloat16* p, float (&v)[EPL]) {
  if constexpr (EPL == 4) {
    const uint2 raw = __ldcg(reinterpret_cast<const uint2*>(p));
    const __nv_bfloat162 p0 = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 p1 = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    v[0] = __low2float(p0); v[1] = __high2float(p0); v[2] = __low2float(p1); v[3] = __high2float(p1);
  } else {
    const unsigned int raw = __ldcg(reinterpret_cast<const unsigned int*>(p));
    const __nv_bfloat162 p0 = *reinterpret_cast<const __nv_bfloat162*>(&raw);
    v[0] = __low2float(p0); v[1] = __high2float(p0);
  }
}

template <int MT, int HD, typename KT>
__device__ void attention_unit(AttnSmem<HD>& sm, const StackArgs& a, const StackLayer& L, int layer,
                               const float* part_qkv, int nc_qkv, unsigned long long* sub) {
  auto substamp = [&](int i) {
    if (sub && threadIdx.x == 0) sub[i] = global_ns();
  };
  constexpr int EPL = HD / 32;
  constexpr int GM = kMaxGroup;
  constexpr int KC = 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ns = a.n_split;
  const int unit = blockIdx.x;
  if (unit >= a.M * a.Hkv * ns) return;
  const int m = unit / (a.Hkv * ns), g = (unit / ns) % a.Hkv, s = unit % ns;
  const int G = a.H / a.Hkv;
  const int seq = a.tok_seq ? __ldcg(a.tok_seq + m) : 0;
  const int pos = a.tok_pos ? __ldcg(a.tok_pos + m) : a.const_pos;
  const int n_keys = pos + 1;
  const int chunk = ((n_keys + ns - 1) / ns + KC - 1) / KC * KC;
  const int t0 = min(n_keys, s * chunk);
  const int t1 = min(n_keys, t0 + chunk);
  const int n_chunks = (t1 - t0 + KC - 1) / KC;
  const bool own_new = pos >= t0 && pos < t1;
  KT* kb = reinterpret_cast<KT*>(a.kv + (size_t)layer * a.kv_layer_elems * sizeof(KT));
  KT* vb = kb + a.kv_layer_elems / 2;

  // This warp's first key chunk: its page and K/V rows are requested first, so their latency
  // overlaps the partial merges below (the new position itself comes from shared memory).
  float kv0[KC][EPL], vv0[KC][EPL];
  if (warp < n_chunks) {
    const int base = t0 + warp * KC;
    const int page = __ldcg(a.page_table + (size_t)seq * a.pt_stride + base / kPage);
    const size_t row0 = ((size_t)(page * a.Hkv + g) * kPage + (base % kPage)) * HD + lane * EPL;
#pragma unroll
    for (int j = 0; j < KC; j++) {
      if (base + j < t1 && !(own_new && base + j == pos)) {
        kv_row<EPL>(kb + row0 + (size_t)j * HD, kv0[j]);
        kv_row<EPL>(vb + row0 + (size_t)j * HD, vv0[j]);
      } else {
#pragma unroll
        for (int e = 0; e < EPL; e++) kv0[j][e] = vv0[j][e] = 0.f;
      }
    }
  }
  // q rows of the group's heads (and, for the split that holds the new position, k and v):
  // the merged wqkv partials, then / den + bias once warp 0 has the denominators
  const int n_rows = G * HD + (own_new ? 2 * HD : 0);
  // up to (8 + 2) * 128 rows over 256 threads: every thread's rows' loads go out together
  constexpr int kRowsPT = ((kMaxGroup + 2) * HD + kCT - 1) / kCT;
  float raw[kRowsPT];
#pragma unroll
  for (int rr = 0; rr < kRowsPT; rr++) {
    const int t = threadIdx.x + rr * kCT;
    int row = 0;
    if (t < G * HD)
      row = (g * G + t / HD) * HD + t % HD;
    else if (t < G * HD + HD)
      row = (a.H + g) * HD + (t - G * HD);
    else
      row = (a.H + a.Hkv + g) * HD + (t - G * HD - HD);
    raw[rr] = t < n_rows ? sum_part<MT>(part_qkv, nc_qkv, row, m) : 0.f;
  }
  rms_den_all<MT>(a, a.ss, sm.den);
  bar_sync_n(1, kCT);
  substamp(0);
  const float den = sm.den[m];
#pragma unroll
  for (int rr = 0; rr < kRowsPT; rr++) {
    const int t = threadIdx.x + rr * kCT;
    if (t < n_rows) {
      int row;
      float* dst;
      if (t < G * HD) {
        row = (g * G + t / HD) * HD + t % HD;
        dst = &sm.qs[t / HD][t % HD];
      } else if (t < G * HD + HD) {
        row = (a.H + g) * HD + (t - G * HD);
        dst = &sm.kbuf[t - G * HD];
      } else {
        row = (a.H + a.Hkv + g) * HD + (t - G * HD - HD);
        dst = &sm.vbuf[t - G * HD - HD];
      }
      float v = __fdiv_rn(raw[rr], den);
      if (L.bqkv) v = __fadd_rn(v, L.bqkv[row]);
      *dst = v;
    }
  }
  bar_sync_n(1, kCT);
  substamp(1);
  for (int i = warp; i < G; i += kCW) norm_rope<HD>(sm.qs[i], L.qn, a.eps, a.inv_freq, a.interleaved, pos, lane);
  if (own_new && warp == kCW - 1) {
    norm_rope<HD>(sm.kbuf, L.kn, a.eps, a.inv_freq, a.interleaved, pos, lane);
    const int page = __ldcg(a.page_table + (size_t)seq * a.pt_stride + pos / kPage);
    const size_t off = ((size_t)(page * a.Hkv + g) * kPage + (pos % kPage)) * HD;
    for (int e = lane; e < HD; e += 32) {
      kv_put(kb + off + e, sm.kbuf[e]);
      kv_put(vb + off + e, sm.vbuf[e]);
      sm.kbuf[e] = kv_back(sm.kbuf[e], kb);
      sm.vbuf[e] = kv_back(sm.vbuf[e], vb);
    }
  }
  bar_sync_n(1, kCT);
  substamp(2);

  float qv[GM][EPL];
#pragma unroll
  for (int i = 0; i < GM; i++)
#pragma unroll
    for (int e = 0; e < EPL; e++) qv[i][e] = i < G ? sm.qs[i][lane * EPL + e] : 0.f;
  float m_w[GM], l_w[GM], acc[GM][EPL];
#pragma unroll
  for (int i = 0; i < GM; i++) {
    m_w[i] = -INFINITY;
    l_w[i] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; e++) acc[i][e] = 0.f;
  }
  for (int c = warp; c < n_chunks; c += kCW) {
    const int base = t0 + c * KC;
    float kv[KC][EPL], vv[KC][EPL];
    if (c == warp) {
#pragma unroll
      for (int j = 0; j < KC; j++)
#pragma unroll
        for (int e = 0; e < EPL; e++) kv[j][e] = kv0[j][e], vv[j][e] = vv0[j][e];
    } else {
      const int page = __ldcg(a.page_table + (size_t)seq * a.pt_stride + base / kPage);
      const size_t row0 = ((size_t)(page * a.Hkv + g) * kPage + (base % kPage)) * HD + lane * EPL;
#pragma unroll
      for (int j = 0; j < KC; j++) {
        if (base + j < t1 && !(own_new && base + j == pos)) {
          kv_row<EPL>(kb + row0 + (size_t)j * HD, kv[j]);
          kv_row<EPL>(vb + row0 + (size_t)j * HD, vv[j]);
        } else {
#pragma unroll
          for (int e = 0; e < EPL; e++) kv[j][e] = vv[j][e] = 0.f;
        }
      }
    }
    if (own_new) {
#pragma unroll
      for (int j = 0; j < KC; j++)
        if (base + j == pos)
#pragma unroll
          for (int e = 0; e < EPL; e++) {
            kv[j][e] = sm.kbuf[lane * EPL + e];
            vv[j][e] = sm.vbuf[lane * EPL + e];
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
      if (i >= G) continue;
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
  substamp(3);
#pragma unroll
  for (int i = 0; i < GM; i++) {
    if (i >= G) continue;
    if (lane == 0) {
      sm.wm[warp][i] = m_w[i];
      sm.wl[warp][i] = l_w[i];
    }
#pragma unroll
    for (int e = 0; e < EPL; e++) sm.wacc[warp][i][lane * EPL + e] = acc[i][e];
  }
  bar_sync_n(1, kCT);
  // this unit's partial per head: (acc[HD], max, sum) merged over the warps in order
  float* out = a.attn_part + (size_t)unit * kMaxGroup * (HD + 2);
  for (int t = threadIdx.x; t < G * HD; t += kCT) {
    const int i = t / HD, e = t % HD;
    float M_ = -INFINITY;
#pragma unroll
    for (int w = 0; w < kCW; w++) M_ = fmaxf(M_, sm.wm[w][i]);
    float Lsum = 0.f, O = 0.f;
    if (M_ != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kCW; w++) {
        const float f = expf(sm.wm[w][i] - M_);
        Lsum = fmaf(sm.wl[w][i], f, Lsum);
        O = fmaf(sm.wacc[w][i][e], f, O);
      }
    }
    __stcg(out + (size_t)i * (HD + 2) + e, O);
    if (e == 0) {
      __stcg(out + (size_t)i * (HD + 2) + HD, M_);
      __stcg(out + (size_t)i * (HD + 2) + HD + 1, Lsum);
    }
  }
}

// ---- the kernel ------------------------------------------------------------------------
template <int MT, int HD, typename KT>
__global__ void __launch_bounds__(kThreadsStack, 1) k_stack(const StackArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int nslot = a.nslot;
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)nslot * kItemBytes);
  uint64_t* empty = full + nslot;
  uint8_t* scratch = reinterpret_cast<uint8_t*>(empty + nslot);
  Smem<MT>& sm = *reinterpret_cast<Smem<MT>*>(scratch);
  AttnSmem<HD>& am = *reinterpret_cast<AttnSmem<HD>*>(scratch);

  if (threadIdx.x == 0) {
    for (int i = 0; i < nslot; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();

  const MatGeo G4[4] = {{nullptr, a.geo[0].K, a.geo[0].nb, a.geo[0].nc, a.geo[0].n_vt},
                        {nullptr, a.geo[1].K, a.geo[1].nb, a.geo[1].nc, a.geo[1].n_vt},
                        {nullptr, a.geo[2].K, a.geo[2].nb, a.geo[2].nc, a.geo[2].n_vt},
                        {nullptr, a.geo[3].K, a.geo[3].nb, a.geo[3].nc, a.geo[3].n_vt}};

  if (threadIdx.x >= kCT) {
    // ---- producer: one lane streams every item of every layer in consumption order ----
    if (threadIdx.x != kCT) return;
    // incremental slot / round / (k chunk, tile) counters: no division per item
    int slot = 0, round = 0, issued = 0;
    for (int l = 0; l < a.n_layer; l++) {
      const StackLayer& L = a.layers[l];
      const uint8_t* W[4] = {L.wqkv, L.wo, L.w13, L.w2};
      for (int mi = 0; mi < 4; mi++) {
        const MatGeo& g = G4[mi];
        long long c0, c1;
        cta_items(g.n_vt, g.nc, &c0, &c1);
        int kc = (int)(c0 / g.n_vt), vt = (int)(c0 % g.n_vt);
        for (int n = (int)(c1 - c0); n > 0; n--) {
          if (round > 0) mbar_wait_bounded(&empty[slot], (uint32_t)((round - 1) & 1), a.err);
          // at most kInflight items in flight: enough to keep HBM busy (Little's law), few
          // enough that the phases' small dependent loads do not queue behind the stream
          if (issued >= kInflight) {
            int ps = slot - kInflight, pr = round;
            if (ps < 0) ps += nslot, pr--;
            mbar_wait_bounded(&full[ps], (uint32_t)(pr & 1), a.err);
          }
          issued++;
          const int nrec = min(kIB, g.nb - kc * kIB);
          const uint32_t bytes = (uint32_t)nrec * kQ8Rec;
          mbar_arrive_expect_tx(&full[slot], bytes);
          bulk_g2s(ring + (size_t)slot * kItemBytes, W[mi] + ((size_t)vt * g.nb + (size_t)kc * kIB) * kQ8Rec, bytes,
                   &full[slot]);
          if (++slot == nslot) slot = 0, round++;
          if (++vt == g.n_vt) vt = 0, kc++;
        }
      }
    }
    return;
  }

  // ---- consumers ----
  // optional phase trace: thread 0 of each CTA stamps %globaltimer at every phase start
  // per CTA: [0] start, [1 + (l * 5 + p) * 3 + {0,1,2}] phase start / prologue end / arrival,
  // [1 + n_layer * 15] final phase start, [2 + n_layer * 15] end
  unsigned long long* tr = a.trace ? a.trace + (size_t)blockIdx.x * (a.n_layer * 15 + 3) : nullptr;
  auto stamp = [&](int l, int p, int k) {
    if (tr && threadIdx.x == 0) tr[1 + (l * 5 + p) * 3 + k] = global_ns();
  };
  if (tr && threadIdx.x == 0) tr[0] = global_ns();
  long long ctr = 0;
  float* xa = a.x;   // the residual stream (in / out)
  float* xb = a.xb;  // the other buffer of the two a residual update alternates between
  unsigned long long target = 0;
  for (int l = 0; l < a.n_layer; l++) {
    const StackLayer& L = a.layers[l];
    long long c0, c1;
    int b_lo, b_hi, kc_lo, kc_hi;
    // P1: wqkv (x += previous layer's w2 partials)
    if (l > 0) grid_wait(a, target);
    stamp(l, 0, 0);
    cta_items(G4[0].n_vt, G4[0].nc, &c0, &c1);
    resid_prologue<MT>(sm, a, G4[0], c0, c1, xa, xb, l > 0 ? a.part1 : nullptr, G4[3].nc, nullptr, L.attn_norm,
                       a.ss);
    k_range(G4[0], c0, c1, &b_lo, &b_hi, &kc_lo, &kc_hi);
    stamp(l, 0, 1);
    gemv_consume<MT>(sm, ring, full, empty, nslot, ctr, G4[0], c0, c1, b_lo, a.M, a.part0, a.err);
    stamp(l, 0, 2);
    target = grid_arrive(a);
    // P2: attention
    grid_wait(a, target);
    stamp(l, 1, 0);
    attention_unit<MT, HD, KT>(am, a, L, l, a.part0, G4[0].nc,
                               tr ? a.trace + (size_t)gridDim.x * (a.n_layer * 15 + 3) +
                                        ((size_t)blockIdx.x * a.n_layer + l) * 4
                                  : nullptr);
    stamp(l, 1, 1);
    stamp(l, 1, 2);
    target = grid_arrive(a);
    // P3: wo
    grid_wait(a, target);
    stamp(l, 2, 0);
    cta_items(G4[1].n_vt, G4[1].nc, &c0, &c1);
    attn_out_prologue<MT>(sm, a, G4[1], c0, c1);
    k_range(G4[1], c0, c1, &b_lo, &b_hi, &kc_lo, &kc_hi);
    stamp(l, 2, 1);
    gemv_consume<MT>(sm, ring, full, empty, nslot, ctr, G4[1], c0, c1, b_lo, a.M, a.part1, a.err);
    stamp(l, 2, 2);
    target = grid_arrive(a);
    // P4: w1|w3 (x += wo partials + bias)
    grid_wait(a, target);
    stamp(l, 3, 0);
    cta_items(G4[2].n_vt, G4[2].nc, &c0, &c1);
    resid_prologue<MT>(sm, a, G4[2], c0, c1, xb, xa, a.part1, G4[1].nc, L.bo, L.ffn_norm, a.ss + (size_t)64 * MT);
    k_range(G4[2], c0, c1, &b_lo, &b_hi, &kc_lo, &kc_hi);
    stamp(l, 3, 1);
    gemv_consume<MT>(sm, ring, full, empty, nslot, ctr, G4[2], c0, c1, b_lo, a.M, a.part0, a.err);
    stamp(l, 3, 2);
    target = grid_arrive(a);
    // P5: w2
    grid_wait(a, target);
    stamp(l, 4, 0);
    cta_items(G4[3].n_vt, G4[3].nc, &c0, &c1);
    swiglu_prologue<MT>(sm, a, G4[3], c0, c1, a.part0, G4[2].nc);
    k_range(G4[3], c0, c1, &b_lo, &b_hi, &kc_lo, &kc_hi);
    stamp(l, 4, 1);
    gemv_consume<MT>(sm, ring, full, empty, nslot, ctr, G4[3], c0, c1, b_lo, a.M, a.part1, a.err);
    stamp(l, 4, 2);
    target = grid_arrive(a);
  }
  // final: x += last w2 partials, rows spread over the CTAs
  grid_wait(a, target);
  if (tr && threadIdx.x == 0) tr[1 + a.n_layer * 15] = global_ns();
  const int rows = a.M * a.dim;
  for (int t = blockIdx.x * kCT + threadIdx.x; t < rows; t += gridDim.x * kCT) {
    const int m = t / a.dim, k = t % a.dim;
    xa[t] = __fadd_rn(__ldcg(xa + t), sum_part<MT>(a.part1, G4[3].nc, k, m));
  }
  if (tr) {
    bar_sync_n(1, kCT);
    if (threadIdx.x == 0) tr[2 + a.n_layer * 15] = global_ns();
  }
}

template <int MT, int HD, typename KT>
cudaError_t launch_t(StackArgs a, int sms, cudaStream_t st) {
  auto kern = k_stack<MT, HD, KT>;
  const size_t fixed = scratch_bytes<MT, HD>() + 128;
  int max_optin = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t avail = (size_t)max_optin - fixed;
  a.nslot = (int)std::min<size_t>(64, avail / (kItemBytes + 16));
  if (a.nslot < 8) return cudaErrorInvalidConfiguration;
  const size_t smem = (size_t)a.nslot * (kItemBytes + 16) + fixed;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int occ = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreadsStack, smem);
  if (e != cudaSuccess) return e;
  if (occ < 1) return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(kThreadsStack);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA co-resident: the grid barriers need it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int MT>
cudaError_t launch_m(const StackArgs& a, int sms, cudaStream_t st) {
  if (a.hd == 128) return a.kv_f32 ? launch_t<MT, 128, float>(a, sms, st) : launch_t<MT, 128, __nv_bfloat16>(a, sms, st);
  return a.kv_f32 ? launch_t<MT, 64, float>(a, sms, st) : launch_t<MT, 64, __nv_bfloat16>(a, sms, st);
}

}  // namespace

// Host-side checks: the persistent kernel takes Q8_0 stacks of head_dim 64 / 128 whose item
// ranges per CTA span at most kSpanBlocks k blocks in every matrix.
bool stack_supported(const StackArgs& a, int sms) {
  if (a.M < 1 || a.M > 8 || (a.hd != 64 && a.hd != 128) || a.H % a.Hkv || a.H / a.Hkv > kMaxGroup) return false;
  if (a.dim % 32 || a.nc_dim > 64 || a.M * a.Hkv > sms || a.n_split > kMaxSplit) return false;
  // a k range is whole 512-wide chunks, so it covers whole heads: at most 1024 / hd of them
  if (kSpanBlocks * 32 / a.hd > kSpanHeads) return false;
  for (int i = 0; i < 4; i++) {
    const StackGeo& g = a.geo[i];
    if (g.nc > kNCMax) return false;
    const long long I = (long long)g.n_vt * g.nc;
    const long long ipc = (I + sms - 1) / sms;
    const long long spans = std::min<long long>(g.nc, (ipc + g.n_vt - 1) / g.n_vt + 1);
    if (spans * kIB > kSpanBlocks) return false;
  }
  return true;
}

size_t stack_attn_part_floats(int sms, int hd) { return (size_t)sms * kMaxGroup * (hd + 2); }

int stack_max_splits(int sms, int M, int Hkv) { return std::max(1, std::min(kMaxSplit, sms / (M * Hkv))); }

cudaError_t launch_stack(const StackArgs& a, int sms, cudaStream_t st) {
  if (!stack_supported(a, sms) || a.n_split < 1 || a.M * a.Hkv * a.n_split > sms) return cudaErrorInvalidValue;
  if (a.M == 1) return launch_m<1>(a, sms, st);
  if (a.M == 2) return launch_m<2>(a, sms, st);
  if (a.M <= 4) return launch_m<4>(a, sms, st);
  return launch_m<8>(a, sms, st);
}

}  // namespace sx
