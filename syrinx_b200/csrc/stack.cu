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
// w1|w3, w2) and copies each item (16 consecutive 544-byte tile records of one 16-row tile:
// 8704 contiguous bytes) into a ring of shared-memory slots with cp.async.bulk, completion
// counted on the slot's mbarrier. It depends on nothing but free slots and keeps at most
// kInflight items in flight (enough for HBM's bandwidth-latency product, few enough that the
// phases' own small loads do not queue behind the stream). Plain bulk copies of this GPU's
// own memory: no tensor map, no multicast.
//
// Phases of a layer, separated by grid barriers (a monotonically increasing u64 counter; every
// wait is bounded by %globaltimer and raises the error flag instead of hanging):
//   P1 wqkv   prologue: x = x + (w2 partials of the previous layer) — the residual add of the
//             previous layer, folded in here — for this CTA's k range only; the CTA owning a
//             512-wide k chunk writes x back and that chunk's sum of squares. Limbs of x * g.
//   P2 attn   one CTA per (token, kv head, split of the key axis): merge the wqkv partials of
//             its heads, divide by the RMS denominator (from the chunk sums), + bias, QK-norm,
//             RoPE, KV append by the split that holds the new position, online softmax over
//             its key slice; writes (max, sum, acc) per head and split.
//   P3 wo     prologue: merge the attention splits for this CTA's k range.
//   P4 w1|w3  prologue: x = x + (wo partials) + bias, chunk owners write x and sums of squares.
//   P5 w2     prologue: act = silu(g / den) * (u / den) from the w1|w3 partials.
// and a final phase adds the last w2 partials into x.
//
// Two costs shape the code. (1) Every dependent global round trip is slow while HBM streams,
// so each prologue gathers what it needs in one batch: GEMV partials are stored row-major,
// [token][row][k chunk padded to 4], and attention partials [token][head][element][split
// padded to 4], so a row's (element's) partials arrive in a few 16-byte loads. (2) The kernel
// must fit the instruction cache: loops are kept compact and the per-CTA work ranges are
// computed once, not per item.
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

constexpr int kCW = 8;                   // consumer warps
constexpr int kCT = kCW * 32;            // consumer threads
constexpr int kThreadsStack = kCT + 32;  // + the producer warp
constexpr int kIB = kStackChunkBlocks;   // 32-wide k blocks per item (one 512-wide k chunk)
constexpr int kItemBytes = kIB * kQ8Rec;  // 8704
constexpr int kSpanBlocks = 32;          // k blocks a CTA's item range may span in one matrix
constexpr int kNCMax = 20;               // k chunks of any matrix (K <= 10240)
constexpr int kNQ = kNCMax / 4;          // their 16-byte groups
constexpr int kMaxSplit = 32;            // splits of the key axis (one per lane in the merge)
constexpr int kInflight = 10;            // weight items a CTA's producer keeps in flight (87 KB)
constexpr int kSpanHeads = 16;           // attention heads a CTA's wo k range may touch
constexpr int kUB = 2;                   // prologue units (block, token) gathered per batch
constexpr uint64_t kBarWaitNs = 2000000000ull;  // grid / mbarrier wait limit
constexpr int kStackMaxLayers = 64;
constexpr int kKvSeg = 4;  // key-range segments (pages) prefetched per layer              // layers whose weight pointers the producer keeps

__host__ __device__ constexpr int pad4(int n) { return (n + 3) & ~3; }

// matrix mi (0 wqkv, 1 wo, 2 w1|w3, 3 w2) of a layer
__device__ __forceinline__ const uint8_t* layer_w(const StackLayer& L, int mi) {
  return mi == 0 ? L.wqkv : mi == 1 ? L.wo : mi == 2 ? L.w13 : L.w2;
}

// This CTA's share of one matrix: items [c0, c0 + n) in k-chunk-major order
struct Plan {
  int c0, n;          // first item, item count
  int kc0, vt0;       // the first item's k chunk and tile
  int kc_lo, kc_hi;   // the k chunks the items touch
  int b_lo, b_hi;     // their 32-wide k blocks
};
__device__ Plan make_plan(const StackGeo& g) {
  Plan p;
  const long long I = (long long)g.n_vt * g.nc;
  const long long c0 = (long long)blockIdx.x * I / gridDim.x, c1 = (long long)(blockIdx.x + 1) * I / gridDim.x;
  p.c0 = (int)c0;
  p.n = (int)(c1 - c0);
  p.kc0 = (int)(c0 / g.n_vt);
  p.vt0 = (int)(c0 % g.n_vt);
  p.kc_lo = p.kc0;
  p.kc_hi = c1 > c0 ? (int)((c1 - 1) / g.n_vt) : p.kc0;
  p.b_lo = p.kc_lo * kIB;
  p.b_hi = c1 > c0 ? min(g.nb, (p.kc_hi + 1) * kIB) : p.b_lo;
  return p;
}
// does this CTA own k chunk kc (hold the chunk's first item)?
__device__ __forceinline__ bool owns_chunk(const Plan& p, const StackGeo& g, int kc) {
  const int first = kc * g.n_vt;
  return first >= p.c0 && first < p.c0 + p.n;
}

// ---- grid barrier ---------------------------------------------------------------------
// Arrive: every consumer thread's writes are ordered by the named barrier, thread 0 counts the
// CTA in with a release at GPU scope (cumulative over what the named barrier ordered before
// it). Returns, on thread 0 only, the count that completes the barrier (0 on every other thread).
__device__ __forceinline__ unsigned long long grid_arrive(const StackArgs& a) {
  bar_sync_n(1, kCT);
  unsigned long long target = 0;
  if (threadIdx.x == 0) {
    unsigned long long old;
    asm volatile("atom.add.release.gpu.global.u64 %0, [%1], 1;" : "=l"(old) : "l"(a.bar) : "memory");
    target = (old / gridDim.x + 1) * gridDim.x;
  }
  return target;
}
__device__ __noinline__ void grid_wait(const StackArgs& a, unsigned long long target) {
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
__device__ __noinline__ void mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = global_ns();
  while (!mbar_wait_sleep(bar, parity)) {
    const uint64_t dt = global_ns() - t0;
    if (dt > 1000000ull && __ldcg(err) != 0) return;
    if (dt > kBarWaitNs) {
      atomicExch(err, 2);
      return;
    }
  }
}

// ---- shared memory ----------------------------------------------------------------------
template <int MT>
struct Smem {
  static constexpr int NP = (MT + 1) / 2;  // token pairs (tensor-core B columns 0-3 / 4-7)
  // limb B fragments [block][NP][32 lanes] and per-(block, token) scales / sums of squares
  uint2 bfr[kSpanBlocks][NP][32];
  float sxs[kSpanBlocks][MT];
  float ssb[kSpanBlocks][MT];
  int8_t scr[kCW][4][32];
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
  float qn[HD], kn[HD];  // QK-norm weights of the layer
};
// Everything the kernel reads more than once that does not change during the launch lives in
// shared memory: with the ring taking most of the SM's 256 KB, L1 keeps almost nothing, and a
// miss costs a full L2 round trip.
struct Common {  // outside the union of the two
  StackArgs args;                     // the launch arguments
  StackLayer lay[kStackMaxLayers];    // every layer's weight and vector pointers
  float inv_freq[64];                 // RoPE inverse frequencies (head_dim / 2 <= 64)
  Plan plan[4];
  float den[kMaxTok];
  // this CTA's attention key range as contiguous segments of a layer's K (and V) region:
  // element offset and length per page, recorded by the first layer's attention unit so that
  // later layers prefetch their keys and values into L2 a phase ahead
  long long kvp_off[kKvSeg];
  int kvp_len[kKvSeg];
  int kvp_n;
};

template <int MT, int HD>
constexpr size_t scratch_bytes() {
  return sizeof(Smem<MT>) > sizeof(AttnSmem<HD>) ? sizeof(Smem<MT>) : sizeof(AttnSmem<HD>);
}

// ---- the limb split of one (block, token) of x (as gemv_q8.cu: exact to 2^-27 of the block max)
template <int MT>
__device__ __noinline__ void split_limbs(Smem<MT>& sm, int warp, int lane, int bi, int m, float v) {
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

// The GEMV partials of output row `row`, token m: a row of pad4(nc) floats, chunks in order.
__device__ __forceinline__ const float* part_row(const float* part, const StackGeo& g, int m, int row) {
  return part + ((size_t)m * g.n_vt * 16 + row) * pad4(g.nc);
}
// Load the first nq 16-byte groups of a partial row (the rest zero).
__device__ __forceinline__ void load_row(const float* p, bool ok, int nq, float4 (&v)[kNQ]) {
#pragma unroll
  for (int q = 0; q < kNQ; q++)
    v[q] = (ok && q < nq) ? __ldcg(reinterpret_cast<const float4*>(p) + q) : float4{0.f, 0.f, 0.f, 0.f};
}
// Their sum over the nc chunks, in chunk order.
__device__ __forceinline__ float sum_row(const float4 (&v)[kNQ], int nc) {
  float s = 0.f;
#pragma unroll
  for (int q = 0; q < kNQ; q++) {
    if (4 * q < nc) s += v[q].x;
    if (4 * q + 1 < nc) s += v[q].y;
    if (4 * q + 2 < nc) s += v[q].z;
    if (4 * q + 3 < nc) s += v[q].w;
  }
  return s;
}

// The same for rows of at most 8 chunks (the matrices whose K is the model width).
__device__ __forceinline__ void load_row2(const float* p, bool ok, int nq, float4 (&v)[2]) {
  v[0] = ok ? __ldcg(reinterpret_cast<const float4*>(p)) : float4{0.f, 0.f, 0.f, 0.f};
  v[1] = (ok && nq > 1) ? __ldcg(reinterpret_cast<const float4*>(p) + 1) : float4{0.f, 0.f, 0.f, 0.f};
}
__device__ __forceinline__ float sum_row2(const float4 (&v)[2], int nc) {
  float s = 0.f;
  if (nc > 0) s += v[0].x;
  if (nc > 1) s += v[0].y;
  if (nc > 2) s += v[0].z;
  if (nc > 3) s += v[0].w;
  if (nc > 4) s += v[1].x;
  if (nc > 5) s += v[1].y;
  if (nc > 6) s += v[1].z;
  if (nc > 7) s += v[1].w;
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
// Consumes this CTA's items of one matrix from the ring (item j of the phase by warp j % 8)
// and writes each item's 16 row sums per token into the row-major partials.
template <int MT>
__device__ __noinline__ void gemv_consume(Smem<MT>& sm, uint8_t* ring, uint64_t* full, uint64_t* empty, int nslot,
                                          int& ctr, const StackGeo& g, const Plan& p, float* part, int* err) {
  constexpr int NP = Smem<MT>::NP;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bl = MT == 1 ? (lane & 15) : lane;
  const int ncp = pad4(g.nc), NR = g.n_vt * 16;
  // this warp's items j = warp, warp + 8, ...: (k chunk, tile) and (slot, round) advance
  // incrementally
  int vt = p.vt0 + warp, kc = p.kc0;
  while (vt >= g.n_vt) vt -= g.n_vt, kc++;
  int slot = (ctr + warp) % nslot, round = (ctr + warp) / nslot;
  for (int j = warp; j < p.n; j += kCW) {
    mbar_wait_bounded(&full[slot], (uint32_t)(round & 1), err);
    const uint8_t* rec = ring + (size_t)slot * kItemBytes;
    float acc[NP][2];
#pragma unroll
    for (int q = 0; q < NP; q++) acc[q][0] = acc[q][1] = 0.f;
#pragma unroll
    for (int i = 0; i < kIB; i++) {
      const int b = kc * kIB + i;
      if (b < g.nb) {
        const uint4 qv = lds128(rec + i * kQ8Rec + lane * 16);
        const uint32_t sw = lds32(rec + i * kQ8Rec + 512 + (lane >> 2) * 4);
        const float2 ds = __half22float2(*reinterpret_cast<const __half2*>(&sw));
        const int bi = b - p.b_lo;
#pragma unroll
        for (int q = 0; q < NP; q++) {
          const uint2 bf = sm.bfr[bi][q][bl];
          const int tok = MT == 1 ? 0 : 2 * q + ((lane >> 1) & 1);
          const float sx = sm.sxs[bi][tok < MT ? tok : 0];
          int d[4];
          mma_s8_16832(qv, bf, d);
          acc[q][0] = fmaf(__fmul_rn(ds.x, sx), (float)(d[0] * 128 + d[1]), acc[q][0]);
          acc[q][1] = fmaf(__fmul_rn(ds.y, sx), (float)(d[2] * 128 + d[3]), acc[q][1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    const float wgt = (lane & 1) ? 0x1p-21f : 0x1p-7f;
#pragma unroll
    for (int q = 0; q < NP; q++) {
      float v0 = acc[q][0] * wgt, v1 = acc[q][1] * wgt;
      v0 += __shfl_down_sync(0xffffffffu, v0, 1);
      v1 += __shfl_down_sync(0xffffffffu, v1, 1);
      const int tok = 2 * q + ((lane >> 1) & 1);
      if ((lane & 1) == 0 && tok < MT) {
        float* P = part + ((size_t)tok * NR + vt * 16 + (lane >> 2)) * ncp + kc;
        __stcg(P, v0);
        __stcg(P + (size_t)8 * ncp, v1);
      }
    }
    slot += kCW;
    if (slot >= nslot) slot -= nslot, round++;
    vt += kCW;
    while (vt >= g.n_vt) vt -= g.n_vt, kc++;
  }
  ctr += p.n;
}

// ---- residual prologue (P1 and P4): x_new = x + partials (+ bias) for this CTA's k range;
// the owner of each k chunk writes x_new and the chunk's sum of squares; limbs of x_new * g.
// `pg` is the geometry of the matrix whose partials are added (null: none). x, the gains and
// the bias do not depend on the phase that just ended, so the first batch requests them before
// the grid barrier (when `wait`); the partials go out right after it, and at batch 1
// every unit of this CTA is in one batch, so the prologue costs one round trip to L2.
template <int MT>
__device__ __noinline__ void resid_prologue(Smem<MT>& sm, const StackArgs& a, const StackGeo& g, const Plan& p,
                                            const float* x_in, float* x_out, const float* part,
                                            const StackGeo* pg, const float* bias, const float* gain, float* ss_out,
                                            bool wait, unsigned long long target, unsigned long long* ts) {
  constexpr int UB = MT == 1 ? 3 : 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dim = a.dim, n_units = (p.b_hi - p.b_lo) * MT;
  const int nq = pg ? pad4(pg->nc) / 4 : 0, nc = pg ? pg->nc : 0;
  bool first = true;
#pragma unroll 1
  for (int u0 = warp; u0 < n_units || first; u0 += UB * kCW) {
    float xv[UB], gv[UB], bv[UB];
    float4 pv[UB][kNQ];
#pragma unroll
    for (int j = 0; j < UB; j++) {  // what the ended phase did not write
      const int u = u0 + j * kCW, m = u % MT, k = (p.b_lo + u / MT) * 32 + lane;
      const bool ok = u < n_units && m < a.M;
      xv[j] = ok ? __ldcg(x_in + (size_t)m * dim + k) : 0.f;
      gv[j] = ok ? gain[k] : 0.f;
      bv[j] = (ok && bias) ? bias[k] : 0.f;
    }
    if (first) {
      if (wait) grid_wait(a, target);  // `wait` is uniform; `target` is thread 0's alone
      if (ts && threadIdx.x == 0) *ts = global_ns();  // profiling: the phase starts here
      first = false;
    }
#pragma unroll
    for (int j = 0; j < UB; j++) {  // the partials of the ended phase
      const int u = u0 + j * kCW, m = u % MT, k = (p.b_lo + u / MT) * 32 + lane;
      const bool ok = u < n_units && m < a.M;
      load_row(pg ? part_row(part, *pg, m, k) : x_in, ok && pg, nq, pv[j]);
    }
#pragma unroll  // constant indices keep the batch in registers (not local memory)
    for (int j = 0; j < UB; j++) {
      const int u = u0 + j * kCW;
      if (u >= n_units) break;
      const int bi = u / MT, m = u % MT, k = (p.b_lo + bi) * 32 + lane;
      float v = 0.f;
      if (m < a.M) {
        float x = xv[j];
        if (pg) {
          float t = sum_row(pv[j], nc);
          if (bias) t = __fadd_rn(t, bv[j]);
          x = __fadd_rn(x, t);
        }
        if (owns_chunk(p, g, (p.b_lo + bi) / kIB)) __stcg(x_out + (size_t)m * dim + k, x);
        const float sq = warp_sum(x * x);
        if (lane == 0) sm.ssb[bi][m] = sq;
        v = __fmul_rn(x, gv[j]);
      } else if (lane == 0) {
        sm.ssb[bi][m] = 0.f;
      }
      split_limbs<MT>(sm, warp, lane, bi, m, v);
    }
  }
  bar_sync_n(1, kCT);
  // owners: the sum of squares of each owned chunk, its blocks added in order
  if (threadIdx.x < MT * (p.kc_hi - p.kc_lo + 1)) {
    const int m = threadIdx.x % MT, kc = p.kc_lo + threadIdx.x / MT;
    if (owns_chunk(p, g, kc) && m < a.M) {
      float s = 0.f;
      for (int b = kc * kIB; b < min(g.nb, (kc + 1) * kIB); b++) s += sm.ssb[b - p.b_lo][m];
      __stcg(ss_out + (size_t)m * 64 + kc, s);
    }
  }
}

// Attention partials: [token][head][element][split] and [token][head][2][split] (max, sum),
// splits padded to 4, so the merge reads a row of splits in 16-byte loads.
__device__ __forceinline__ size_t ao_off(const StackArgs& a, int m, int h, int e) {
  return (((size_t)m * a.H + h) * a.hd + e) * pad4(a.n_split);
}
__device__ __forceinline__ size_t aml_off(const StackArgs& a, int m, int h) {
  return (size_t)a.M * a.H * a.hd * pad4(a.n_split) + ((size_t)m * a.H + h) * 2 * pad4(a.n_split);
}

// ---- P3 prologue: attention output for this CTA's k range (merge of the key-axis splits).
// A batch's accumulator loads go out first; the first batch then computes, one split per
// lane, the weights exp(m_s - max) and the denominators of the (head, token) pairs it owns.
template <int MT>
__device__ __noinline__ void attn_out_prologue(Smem<MT>& sm, const StackArgs& a, const Plan& p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = a.hd, ns = a.n_split, nsq = pad4(ns) / 4;
  const int h_lo = (p.b_lo * 32) / hd;
  const int nh = p.b_hi > p.b_lo ? ((p.b_hi * 32 - 1) / hd) - h_lo + 1 : 0;
  const int n_units = (p.b_hi - p.b_lo) * MT;
  constexpr int SQ = kMaxSplit / 4;
  bool first = true;
#pragma unroll 1
  for (int u0 = warp; u0 < n_units || first; u0 += kUB * kCW) {
    float4 o[kUB][SQ];
#pragma unroll
    for (int j = 0; j < kUB; j++) {
      const int u = u0 + j * kCW, m = u % MT, k = (p.b_lo + u / MT) * 32 + lane;
      const bool ok = u < n_units && m < a.M;
      const float4* src = reinterpret_cast<const float4*>(a.attn_part + (ok ? ao_off(a, m, k / hd, k % hd) : 0));
#pragma unroll
      for (int q = 0; q < SQ; q++) o[j][q] = (ok && q < nsq) ? __ldcg(src + q) : float4{0.f, 0.f, 0.f, 0.f};
    }
    if (first) {
#pragma unroll 1
      for (int v = warp; v < nh * MT; v += kCW) {
        const int hl = v / MT, m = v % MT;
        float ms = -INFINITY, ls = 0.f;
        if (m < a.M && lane < ns) {
          const float* pm = a.attn_part + aml_off(a, m, h_lo + hl);
          ms = __ldcg(pm + lane);
          ls = __ldcg(pm + pad4(ns) + lane);
        }
        const float M_ = warp_max(ms);
        const float w = ms == -INFINITY ? 0.f : __expf(ms - M_);
        const float L = warp_sum(ls * w);
        sm.wts[hl][m][lane] = w;
        if (lane == 0) sm.lsum[hl][m] = L;
      }
      bar_sync_n(1, kCT);
      first = false;
    }
#pragma unroll  // constant indices keep the batch in registers (not local memory)
    for (int j = 0; j < kUB; j++) {
      const int u = u0 + j * kCW;
      if (u >= n_units) break;
      const int bi = u / MT, m = u % MT, k = (p.b_lo + bi) * 32 + lane;
      float v = 0.f;
      if (m < a.M) {
        const float* w = sm.wts[k / hd - h_lo][m];
        float O = 0.f;
#pragma unroll
        for (int q = 0; q < SQ; q++) {
          if (4 * q < ns) O = fmaf(o[j][q].x, w[4 * q], O);
          if (4 * q + 1 < ns) O = fmaf(o[j][q].y, w[4 * q + 1], O);
          if (4 * q + 2 < ns) O = fmaf(o[j][q].z, w[4 * q + 2], O);
          if (4 * q + 3 < ns) O = fmaf(o[j][q].w, w[4 * q + 3], O);
        }
        v = __fdiv_rn(O, sm.lsum[k / hd - h_lo][m]);
      }
      split_limbs<MT>(sm, warp, lane, bi, m, v);
    }
  }
  bar_sync_n(1, kCT);
}

// ---- P5 prologue: act = silu(g / den) * (u / den) for this CTA's k range; a batch's partial
// loads and (first batch) warp 0's sum-of-squares loads go out together.
template <int MT>
__device__ __noinline__ void swiglu_prologue(Smem<MT>& sm, Common& cm, const StackArgs& a, const Plan& p,
                                             const float* part13, const StackGeo& g13) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_units = (p.b_hi - p.b_lo) * MT, nq = pad4(g13.nc) / 4;
  constexpr int UB = MT == 1 ? 3 : 2;
  bool first = true;
#pragma unroll 1
  for (int u0 = warp; u0 < n_units || first; u0 += UB * kCW) {
    float4 gv[UB][2], uv[UB][2];
#pragma unroll
    for (int j = 0; j < UB; j++) {
      const int u = u0 + j * kCW, m = u % MT, k = (p.b_lo + u / MT) * 32 + lane;
      const bool ok = u < n_units && m < a.M;
      // tile j holds gate rows 8j..8j+7 (tile rows 0-7) and up rows 8j..8j+7 (rows 8-15)
      const int row_g = (k >> 3) * 16 + (k & 7);
      load_row2(part_row(part13, g13, m, row_g), ok, nq, gv[j]);
      load_row2(part_row(part13, g13, m, row_g + 8), ok, nq, uv[j]);
    }
    if (first) {
      rms_den_all<MT>(a, a.ss + (size_t)64 * MT, cm.den);
      bar_sync_n(1, kCT);
      first = false;
    }
#pragma unroll  // constant indices keep the batch in registers (not local memory)
    for (int j = 0; j < UB; j++) {
      const int u = u0 + j * kCW;
      if (u >= n_units) break;
      const int bi = u / MT, m = u % MT;
      float v = 0.f;
      if (m < a.M) {
        const float den = cm.den[m];
        v = __fmul_rn(silu_f(__fdiv_rn(sum_row2(gv[j], g13.nc), den)), __fdiv_rn(sum_row2(uv[j], g13.nc), den));
      }
      split_limbs<MT>(sm, warp, lane, bi, m, v);
    }
  }
  bar_sync_n(1, kCT);
}

// ---- P2: attention of one (token, kv head, split) unit --------------------------------
template <int HD>
__device__ __noinline__ void norm_rope(float* buf, const float* nw, float eps, const float* inv_freq, int interleaved,
                                       int pos, int lane) {
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
__device__ __noinline__ void attention_unit(AttnSmem<HD>& sm, Common& cm, const StackArgs& a, const StackLayer& L,
                                            int layer, const float* part_qkv, const StackGeo& gq,
                                            unsigned long long target, unsigned long long* ts,
                                            unsigned long long* sub) {
  constexpr int EPL = HD / 32;
  constexpr int GQ = 4;  // query heads per compute pass
  constexpr int KC = 4;  // keys per warp chunk
  auto substamp = [&](int i) {
    if (sub && threadIdx.x == 0) sub[i] = global_ns();
  };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ns = a.n_split;
  const int unit = blockIdx.x;
  // The grid barrier that ends the wqkv phase is taken inside (by every consumer thread of
  // every CTA): what does not depend on that phase (positions, pages, the first keys and values,
  // norm weights, biases) is requested before it.
  auto wait_phase = [&]() {
    grid_wait(a, target);
    if (ts && threadIdx.x == 0) *ts = global_ns();  // profiling: the phase starts here
  };
  if (unit >= a.M * a.Hkv * ns) {
    wait_phase();
    return;
  }
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
  if (layer == 0 && threadIdx.x == kCT - 1) {  // the keys [t0, t1) before the new position, per page
    int n = 0;
    for (int t = t0; t < min(t1, pos) && n < kKvSeg;) {
      const int pg = t / kPage, e = min(min(t1, pos), (pg + 1) * kPage);
      const int page = __ldcg(a.page_table + (size_t)seq * a.pt_stride + pg);
      cm.kvp_off[n] = ((long long)(page * a.Hkv + g) * kPage + (t % kPage)) * HD;
      cm.kvp_len[n] = (e - t) * HD;
      n++;
      t = e;
    }
    cm.kvp_n = n;
  }

  // K/V rows of chunk c (not the new position, which comes from shared memory)
  auto load_chunk = [&](int c, float (&kv)[KC][EPL], float (&vv)[KC][EPL]) {
    const int base = t0 + c * KC;
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
  };
  // this warp's first key chunk goes out before the partial merges, so its latency overlaps them
  float kv0[KC][EPL], vv0[KC][EPL];
  if (warp < n_chunks) load_chunk(warp, kv0, vv0);

  // q rows of the group's heads (and, for the split that holds the new position, k and v):
  // the merged wqkv partials, every row's loads out at once, then / den + bias
  const int n_rows = G * HD + (own_new ? 2 * HD : 0);
  constexpr int kRowsPT = ((kMaxGroup + 2) * HD + kCT - 1) / kCT;
  const int nq = pad4(gq.nc) / 4;
  auto row_of = [&](int t) {
    if (t < G * HD) return (g * G + t / HD) * HD + t % HD;
    if (t < G * HD + HD) return (a.H + g) * HD + (t - G * HD);
    return (a.H + a.Hkv + g) * HD + (t - G * HD - HD);
  };
  float bq[kRowsPT];
#pragma unroll
  for (int rr = 0; rr < kRowsPT; rr++) {
    const int t = threadIdx.x + rr * kCT;
    bq[rr] = (L.bqkv && t < n_rows) ? L.bqkv[row_of(t)] : 0.f;
  }
  for (int e = threadIdx.x; e < HD; e += kCT) {
    if (L.qn) sm.qn[e] = L.qn[e];
    if (L.kn) sm.kn[e] = L.kn[e];
  }
  const int new_page = own_new ? __ldcg(a.page_table + (size_t)seq * a.pt_stride + pos / kPage) : 0;
  wait_phase();
  float4 pv[kRowsPT][2];  // wqkv has at most 8 k chunks here (gq.nc <= 8, checked on the host)
#pragma unroll
  for (int rr = 0; rr < kRowsPT; rr++) {
    const int t = threadIdx.x + rr * kCT;
    const float4* src = reinterpret_cast<const float4*>(part_row(part_qkv, gq, m, t < n_rows ? row_of(t) : 0));
    pv[rr][0] = (t < n_rows) ? __ldcg(src) : float4{0.f, 0.f, 0.f, 0.f};
    pv[rr][1] = (t < n_rows && nq > 1) ? __ldcg(src + 1) : float4{0.f, 0.f, 0.f, 0.f};
  }
  rms_den_all<MT>(a, a.ss, cm.den);
  bar_sync_n(1, kCT);
  substamp(0);
  const float den = cm.den[m];
#pragma unroll
  for (int rr = 0; rr < kRowsPT; rr++) {
    const int t = threadIdx.x + rr * kCT;
    if (t < n_rows) {
      const float c[8] = {pv[rr][0].x, pv[rr][0].y, pv[rr][0].z, pv[rr][0].w,
                          pv[rr][1].x, pv[rr][1].y, pv[rr][1].z, pv[rr][1].w};
      float raw = 0.f;
#pragma unroll
      for (int i = 0; i < 8; i++)
        if (i < gq.nc) raw += c[i];
      const int row = row_of(t);
      float v = __fdiv_rn(raw, den);
      if (L.bqkv) v = __fadd_rn(v, bq[rr]);
      float* dst = t < G * HD        ? &sm.qs[t / HD][t % HD]
                   : t < G * HD + HD ? &sm.kbuf[t - G * HD]
                                     : &sm.vbuf[t - G * HD - HD];
      *dst = v;
    }
  }
  bar_sync_n(1, kCT);
  substamp(1);
  for (int i = warp; i < G; i += kCW)
    norm_rope<HD>(sm.qs[i], L.qn ? sm.qn : nullptr, a.eps, cm.inv_freq, a.interleaved, pos, lane);
  if (own_new && warp == kCW - 1) {
    norm_rope<HD>(sm.kbuf, L.kn ? sm.kn : nullptr, a.eps, cm.inv_freq, a.interleaved, pos, lane);
    const size_t off = ((size_t)(new_page * a.Hkv + g) * kPage + (pos % kPage)) * HD;
    for (int e = lane; e < HD; e += 32) {
      kv_put(kb + off + e, sm.kbuf[e]);
      kv_put(vb + off + e, sm.vbuf[e]);
      sm.kbuf[e] = kv_back(sm.kbuf[e], kb);
      sm.vbuf[e] = kv_back(sm.vbuf[e], vb);
    }
  }
  bar_sync_n(1, kCT);
  substamp(2);

  // the query heads in groups of GQ (the compute loop exists once, for GQ heads)
#pragma unroll 1
  for (int hg = 0; hg < G; hg += GQ) {
    float qv[GQ][EPL];
#pragma unroll
    for (int i = 0; i < GQ; i++)
#pragma unroll
      for (int e = 0; e < EPL; e++) qv[i][e] = hg + i < G ? sm.qs[hg + i][lane * EPL + e] : 0.f;
    float m_w[GQ], l_w[GQ], acc[GQ][EPL];
#pragma unroll
    for (int i = 0; i < GQ; i++) {
      m_w[i] = -INFINITY;
      l_w[i] = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; e++) acc[i][e] = 0.f;
    }
#pragma unroll 1
    for (int c = warp; c < n_chunks; c += kCW) {
      const int base = t0 + c * KC;
      float kv[KC][EPL], vv[KC][EPL];
      if (c == warp) {
#pragma unroll
        for (int j = 0; j < KC; j++)
#pragma unroll
          for (int e = 0; e < EPL; e++) kv[j][e] = kv0[j][e], vv[j][e] = vv0[j][e];
      } else {
        load_chunk(c, kv, vv);
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
      float sc[KC][GQ];
#pragma unroll
      for (int j = 0; j < KC; j++)
#pragma unroll
        for (int i = 0; i < GQ; i++) {
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
          for (int i = 0; i < GQ; i++) sc[j][i] += __shfl_xor_sync(0xffffffffu, sc[j][i], o);
#pragma unroll
      for (int i = 0; i < GQ; i++) {
        float cmax = -INFINITY;
#pragma unroll
        for (int j = 0; j < KC; j++) {
          sc[j][i] = base + j < t1 ? __fmul_rn(sc[j][i], a.scale) : -INFINITY;
          cmax = fmaxf(cmax, sc[j][i]);
        }
        const float m_new = fmaxf(m_w[i], cmax);
        const float alpha = __expf(m_w[i] - m_new);
        float lsum = l_w[i] * alpha;
#pragma unroll
        for (int e = 0; e < EPL; e++) acc[i][e] *= alpha;
#pragma unroll
        for (int j = 0; j < KC; j++) {
          const float pr = base + j < t1 ? __expf(sc[j][i] - m_new) : 0.f;
          lsum += pr;
#pragma unroll
          for (int e = 0; e < EPL; e++) acc[i][e] = fmaf(pr, vv[j][e], acc[i][e]);
        }
        l_w[i] = lsum;
        m_w[i] = m_new;
      }
    }
#pragma unroll
    for (int i = 0; i < GQ; i++) {
      if (hg + i >= G) continue;
      if (lane == 0) {
        sm.wm[warp][hg + i] = m_w[i];
        sm.wl[warp][hg + i] = l_w[i];
      }
#pragma unroll
      for (int e = 0; e < EPL; e++) sm.wacc[warp][hg + i][lane * EPL + e] = acc[i][e];
    }
  }
  substamp(3);
  bar_sync_n(1, kCT);
  // this split's partial per head: (acc[HD], max, sum) merged over the warps in order
  const int nsp = pad4(ns);
#pragma unroll 1
  for (int t = threadIdx.x; t < G * HD; t += kCT) {
    const int i = t / HD, e = t % HD;
    float M_ = -INFINITY;
#pragma unroll
    for (int w = 0; w < kCW; w++) M_ = fmaxf(M_, sm.wm[w][i]);
    float Lsum = 0.f, O = 0.f;
    if (M_ != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kCW; w++) {
        const float f = __expf(sm.wm[w][i] - M_);
        Lsum = fmaf(sm.wl[w][i], f, Lsum);
        O = fmaf(sm.wacc[w][i][e], f, O);
      }
    }
    const int h = g * G + i;
    __stcg(a.attn_part + ao_off(a, m, h, e) + s, O);
    if (e == 0) {
      float* pm = a.attn_part + aml_off(a, m, h);
      __stcg(pm + s, M_);
      __stcg(pm + nsp + s, Lsum);
    }
  }
}

// ---- the kernel ------------------------------------------------------------------------
template <int MT, int HD, typename KT>
__global__ void __launch_bounds__(kThreadsStack, 1) k_stack(const __grid_constant__ StackArgs a_in) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int nslot = a_in.nslot;
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)nslot * kItemBytes);
  uint64_t* empty = full + nslot;
  Common& cm = *reinterpret_cast<Common*>(empty + nslot);
  const StackArgs& a = cm.args;
  uint8_t* scratch = reinterpret_cast<uint8_t*>(&cm) + ((sizeof(Common) + 15) & ~(size_t)15);
  Smem<MT>& sm = *reinterpret_cast<Smem<MT>*>(scratch);
  AttnSmem<HD>& am = *reinterpret_cast<AttnSmem<HD>*>(scratch);

  if (threadIdx.x == 0) {
    for (int i = 0; i < nslot; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_fence_init();
    for (int i = 0; i < 4; i++) cm.plan[i] = make_plan(a_in.geo[i]);
    cm.args = a_in;
    cm.kvp_n = 0;
  }
  for (int l = threadIdx.x; l < a_in.n_layer; l += blockDim.x) cm.lay[l] = a_in.layers[l];
  for (int i = threadIdx.x; i < a_in.hd / 2; i += blockDim.x) cm.inv_freq[i] = a_in.inv_freq[i];
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();

  if (threadIdx.x >= kCT) {
    // ---- producer: one lane streams every item of every layer in consumption order ----
    // Besides the ring it runs an L2 prefetch cursor up to a.l2_ahead items ahead of the ring
    // (cp.async.bulk.prefetch.L2 of this GPU's own memory): while the consumers sit in a grid
    // barrier, a prologue or attention and the ring is full, HBM keeps streaming into L2, and
    // the ring refills from L2 when they resume.
    if (threadIdx.x != kCT) return;
    int slot = 0, round = 0, issued = 0;
    int pl = 0, pm = 0, pn = cm.plan[0].n, pkc = cm.plan[0].kc0, pvt = cm.plan[0].vt0, pf = 0;
    bool pf_done = a.l2_ahead <= 0;
    // advance the prefetch cursor by one item, prefetching it unless the ring has it already
    auto pf_one = [&]() {
      while (pn == 0) {
        if (++pm == 4) {
          pm = 0;
          if (++pl == a.n_layer) {
            pf_done = true;
            return;
          }
        }
        pn = cm.plan[pm].n;
        pkc = cm.plan[pm].kc0;
        pvt = cm.plan[pm].vt0;
      }
      const StackGeo& g = a.geo[pm];
      if (pf >= issued) {
        const int nrec = min(kIB, g.nb - pkc * kIB);
        bulk_prefetch_l2(layer_w(cm.lay[pl], pm) + ((size_t)pvt * g.nb + (size_t)pkc * kIB) * kQ8Rec,
                         (uint32_t)nrec * kQ8Rec);
      }
      pn--;
      pf++;
      if (++pvt == g.n_vt) pvt = 0, pkc++;
    };
    // bounded wait on a ring mbarrier that prefetches while it waits
    auto pwait = [&](uint64_t* bar, uint32_t parity) {
      if (mbar_try_wait(bar, parity)) return;
      const uint64_t t0 = global_ns();
      for (;;) {
        const bool more = !pf_done && pf < issued + a.l2_ahead;  // prefetch work while waiting
        if (more ? mbar_try_wait(bar, parity) : mbar_wait_sleep(bar, parity)) return;
        if (more) {
          pf_one();
          continue;
        }
        const uint64_t dt = global_ns() - t0;
        if (dt > 1000000ull && __ldcg(a.err) != 0) return;
        if (dt > kBarWaitNs) {
          atomicExch(a.err, 2);
          return;
        }
      }
    };
    for (int l = 0; l < a.n_layer; l++) {
      for (int mi = 0; mi < 4; mi++) {
        const StackGeo& g = a.geo[mi];
        const Plan& p = cm.plan[mi];
        const uint8_t* W = layer_w(cm.lay[l], mi);
        int kc = p.kc0, vt = p.vt0;
        for (int n = p.n; n > 0; n--) {
          if (round > 0) pwait(&empty[slot], (uint32_t)((round - 1) & 1));
          if (issued >= a.inflight) {  // keep at most `inflight` items in flight
            int ps = slot - a.inflight, pr = round;
            if (ps < 0) ps += nslot, pr--;
            pwait(&full[ps], (uint32_t)(pr & 1));
          }
          issued++;
          const int nrec = min(kIB, g.nb - kc * kIB);
          const uint32_t bytes = (uint32_t)nrec * kQ8Rec;
          mbar_arrive_expect_tx(&full[slot], bytes);
          bulk_g2s(ring + (size_t)slot * kItemBytes, W + ((size_t)vt * g.nb + (size_t)kc * kIB) * kQ8Rec, bytes,
                   &full[slot]);
          if (++slot == nslot) slot = 0, round++;
          if (++vt == g.n_vt) vt = 0, kc++;
        }
      }
    }
    return;
  }

  // ---- consumers ----
  // optional trace: per CTA [0] start, [1 + (l * 5 + p) * 3 + {0,1,2}] phase start / prologue
  // end / arrival, [1 + n_layer * 15] final phase start, [2 + n_layer * 15] end
  unsigned long long* tr = a.trace ? a.trace + (size_t)blockIdx.x * (a.n_layer * 15 + 3) : nullptr;
  auto stamp = [&](int l, int p, int k) {
    if (tr && threadIdx.x == 0) tr[1 + (l * 5 + p) * 3 + k] = global_ns();
  };
  if (tr && threadIdx.x == 0) tr[0] = global_ns();
  int ctr = 0;
  float* xa = a.x;   // the residual stream (in / out)
  float* xb = a.xb;  // the other buffer of the two a residual update alternates between
  unsigned long long target = 0;
  const Plan* P = cm.plan;
  for (int l = 0; l < a.n_layer; l++) {
    const StackLayer& L = cm.lay[l];
    // P1: wqkv (x += previous layer's w2 partials); the grid barrier is inside the prologue.
    // This layer's keys and values for the attention unit go to L2 first (HBM latency under the
    // weight stream is several microseconds; the attention phase starts one phase later).
    if (l > 0 && threadIdx.x == 32) {
      const size_t esz = a.kv_f32 ? 4 : 2;
      const uint8_t* kb = a.kv + (size_t)l * a.kv_layer_elems * esz;
      const uint8_t* vb = kb + a.kv_layer_elems / 2 * esz;
      for (int i = 0; i < cm.kvp_n; i++) {
        bulk_prefetch_l2(kb + cm.kvp_off[i] * esz, (uint32_t)(cm.kvp_len[i] * esz));
        bulk_prefetch_l2(vb + cm.kvp_off[i] * esz, (uint32_t)(cm.kvp_len[i] * esz));
      }
    }
    resid_prologue<MT>(sm, a, a.geo[0], P[0], xa, xb, a.part1, l > 0 ? &a.geo[3] : nullptr, nullptr, L.attn_norm,
                       a.ss, l > 0, target, tr ? tr + 1 + (l * 5 + 0) * 3 : nullptr);
    stamp(l, 0, 1);
    gemv_consume<MT>(sm, ring, full, empty, nslot, ctr, a.geo[0], P[0], a.part0, a.err);
    stamp(l, 0, 2);
    target = grid_arrive(a);
    // P2: attention (the grid barrier is inside)
    attention_unit<MT, HD, KT>(am, cm, a, L, l, a.part0, a.geo[0], target, tr ? tr + 1 + (l * 5 + 1) * 3 : nullptr,
                               tr ? a.trace + (size_t)gridDim.x * (a.n_layer * 15 + 3) +
                                        ((size_t)blockIdx.x * a.n_layer + l) * 4
                                  : nullptr);
    stamp(l, 1, 1);
    stamp(l, 1, 2);
    target = grid_arrive(a);
    // P3: wo
    grid_wait(a, target);
    stamp(l, 2, 0);
    attn_out_prologue<MT>(sm, a, P[1]);
    stamp(l, 2, 1);
    gemv_consume<MT>(sm, ring, full, empty, nslot, ctr, a.geo[1], P[1], a.part1, a.err);
    stamp(l, 2, 2);
    target = grid_arrive(a);
    // P4: w1|w3 (x += wo partials + bias); the grid barrier is inside the prologue
    resid_prologue<MT>(sm, a, a.geo[2], P[2], xb, xa, a.part1, &a.geo[1], L.bo, L.ffn_norm, a.ss + (size_t)64 * MT,
                       true, target, tr ? tr + 1 + (l * 5 + 3) * 3 : nullptr);
    stamp(l, 3, 1);
    gemv_consume<MT>(sm, ring, full, empty, nslot, ctr, a.geo[2], P[2], a.part0, a.err);
    stamp(l, 3, 2);
    target = grid_arrive(a);
    // P5: w2
    grid_wait(a, target);
    stamp(l, 4, 0);
    swiglu_prologue<MT>(sm, cm, a, P[3], a.part0, a.geo[2]);
    stamp(l, 4, 1);
    gemv_consume<MT>(sm, ring, full, empty, nslot, ctr, a.geo[3], P[3], a.part1, a.err);
    stamp(l, 4, 2);
    target = grid_arrive(a);
  }
  // final: x += last w2 partials, rows spread over the CTAs
  grid_wait(a, target);
  if (tr && threadIdx.x == 0) tr[1 + a.n_layer * 15] = global_ns();
  const int rows = a.M * a.dim, nq = pad4(a.geo[3].nc) / 4;
#pragma unroll 1
  for (int t = blockIdx.x * kCT + threadIdx.x; t < rows; t += gridDim.x * kCT) {
    const int m = t / a.dim, k = t % a.dim;
    float4 v[kNQ];
    load_row(part_row(a.part1, a.geo[3], m, k), true, nq, v);
    xa[t] = __fadd_rn(__ldcg(xa + t), sum_row(v, a.geo[3].nc));
  }
  if (tr) {
    bar_sync_n(1, kCT);
    if (threadIdx.x == 0) tr[2 + a.n_layer * 15] = global_ns();
  }
}

template <int MT, int HD, typename KT>
cudaError_t launch_t(StackArgs a, int sms, cudaStream_t st) {
  auto kern = k_stack<MT, HD, KT>;
  const size_t fixed = ((sizeof(Common) + 15) & ~(size_t)15) + scratch_bytes<MT, HD>() + 128;
  int max_optin = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t avail = (size_t)max_optin - fixed;
  a.nslot = (int)std::min<size_t>(64, avail / (kItemBytes + 16));
  if (a.nslot < kInflight + kCW) return cudaErrorInvalidConfiguration;
  if (a.inflight < 1 || a.inflight > a.nslot - kCW) a.inflight = kInflight;
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
  if (a.n_layer < 1 || a.n_layer > kStackMaxLayers) return false;
  if (a.dim % 32 || a.nc_dim > 64 || a.M * a.Hkv > sms || a.n_split > kMaxSplit) return false;
  // a k range is whole 512-wide chunks, so it covers whole heads: at most 1024 / hd of them
  if (kSpanBlocks * 32 / a.hd > kSpanHeads) return false;
  if (a.geo[0].nc > 8) return false;  // the attention unit merges at most 8 wqkv chunks
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

// floats of the attention partials: [M][H][hd][splits] + [M][H][2][splits], splits padded to 4
size_t stack_attn_part_floats(int max_tok, int H, int hd) { return (size_t)max_tok * H * (hd + 2) * kMaxSplit; }

// floats of one GEMV partial buffer: [M][rows][k chunks padded to 4]
size_t stack_part_floats(const StackGeo& g, int M) { return (size_t)M * g.n_vt * 16 * pad4(g.nc); }

int stack_max_splits(int sms, int M, int Hkv) { return std::max(1, std::min(kMaxSplit, sms / (M * Hkv))); }

cudaError_t launch_stack(const StackArgs& a, int sms, cudaStream_t st) {
  if (!stack_supported(a, sms) || a.n_split < 1 || a.M * a.Hkv * a.n_split > sms) return cudaErrorInvalidValue;
  if (a.M == 1) return launch_m<1>(a, sms, st);
  if (a.M == 2) return launch_m<2>(a, sms, st);
  if (a.M <= 4) return launch_m<4>(a, sms, st);
  return launch_m<8>(a, sms, st);
}

}  // namespace sx
