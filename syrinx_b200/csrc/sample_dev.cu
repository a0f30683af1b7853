// sample_dev.cu — the reference sampler on the device, one CTA per draw.
//
// Restates crates/syrinx-fish/src/common/sampling.rs for one sequence: the semantic
// constraint (84-106), logits_to_probs (189-245: stable sort descending with ties by lower
// index, rank-order softmax sum for the top-p / top-k cut that always keeps the top id, then
// a temperature softmax over the kept ids in index order), multinomial1 (254-268: inverse
// CDF in index order on a SplitMix64 draw) and the RAS rule of sample_semantic (143-167:
// a second draw at the high temperature / top-p replaces a semantic draw found in the
// window of recent semantic ids). Every floating-point step follows the host restatement
// (syrinx_b200/csrc/sampling.cpp) in the same order and precision, except the softmax
// normaliser of the top-p cut (a fixed-order tree sum instead of one thread's rank-order
// loop), so the device draws the same ids from the same logits and seed; that sum and the
// last bit of the f64 exp can only matter when a top-p or draw comparison lands within an
// ulp. The kept ids' sums (the probabilities and the draw) keep the reference's index order.
//
// Ids outside the constraint carry -inf logits in the reference: they sort last, add exact
// zeros to every sum and are never drawn, so the kernel works on the allowed ids only.
// The pick is written as a packed argmax key into the session's argmax slot, where the
// greedy loop's k_take_semantic / k_take_code read it.
#include <cuda_runtime.h>

#include "sx_device.cuh"
#include "sx_internal.hpp"

namespace sx {
namespace {

constexpr int kThreadsS = 1024;

__device__ __forceinline__ uint32_t id_of(const SampleArgs& a, int i) {
  const int n0 = (int)(a.hi[0] - a.lo[0]);
  return i < n0 ? a.lo[0] + (uint32_t)i : a.lo[1] + (uint32_t)(i - n0);
}

// SplitMix64 (sampling.rs:19-41): the next f64 in [0, 1) from the state in global memory.
__device__ double next_f64(SampleState* st) {
  uint64_t s = __ldcg(reinterpret_cast<const unsigned long long*>(&st->rng)) + 0x9E3779B97F4A7C15ull;
  st->rng = s;
  uint64_t z = s;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (double)(z >> 11) * (1.0 / 9007199254740992.0);
}

// Whether shared memory also holds the kept ids' f64 softmax terms (8 bytes per id), so that
// every thread makes them: up to 4096-odd ids (the Fish semantic and codebook draws); the
// CosyVoice heads (6564 / 6761 ids) make them on one thread.
__host__ __device__ __forceinline__ bool sample_smem_par(int n) {
  int np = 1;
  while (np < n) np <<= 1;
  return (size_t)np * 8 + (size_t)n * (8 + 4 + 4 + 4 + 1 + 8) <= 200 * 1024;
}

struct Smem {
  unsigned long long* keys;  // [np] sort keys, then rank order
  double* exps;              // [n] by rank: exp(logit - max), then that over the sum
  double* ed;                // [n] the kept ids' exp terms in index order, or null (no room)
  float* lg;                 // [n] logits in index order
  float* pf;                 // [n] probabilities in index order (kept ids only)
  int* kept;                 // [n] the kept ids' indices, ascending
  uint8_t* keep;             // [n] kept flags in index order
};

// Compact the kept flags into an ascending index list (block-wide exclusive scan).
__device__ void compact_kept(const Smem& m, int n) {
  __shared__ int s_warp[kThreadsS / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (n + kThreadsS - 1) / kThreadsS, i0 = tid * per, i1 = min(n, i0 + per);
  int c = 0;
  for (int i = i0; i < i1; i++) c += m.keep[i];
  int incl = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kThreadsS / 32 ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += v;
    }
    if (lane < kThreadsS / 32) s_warp[lane] = w;  // inclusive totals per warp
  }
  __syncthreads();
  int pos = incl - c + (warp > 0 ? s_warp[warp - 1] : 0);
  for (int i = i0; i < i1; i++)
    if (m.keep[i]) m.kept[pos++] = i;
  __syncthreads();
}

__device__ __forceinline__ int order_at(const Smem& m, int r) { return (int)(0xFFFFFFFFu - (uint32_t)m.keys[r]); }

// One logits_to_probs + multinomial1 with (temperature, top_p, top_k) on the sorted ids.
// Every thread of the CTA calls it; returns the drawn id (an allowed id, or the reference's
// fall-backs: id 0 when nothing has mass, the array's last id if no prefix sum exceeds u).
__device__ uint32_t draw(const SampleArgs& a, const Smem& m, int n, double sum, float temperature, float top_p,
                         int top_k) {
  __shared__ int s_rend;
  __shared__ float s_red[kThreadsS / 32];
  __shared__ uint32_t s_pick;
  const int tid = threadIdx.x;
  if (tid == 0) {
    // the kept ids are the rank prefix [0, rend); exps[r] already holds exps[r] / sum, so
    // the one sequential chain left here is the reference's f64 additions
    const int k_cap = top_k == 0 ? n : top_k;
    double cum = 0.0;
    int r = 0;
    for (; r < n; r++) {
      if (r > 0 && !(cum <= (double)top_p && r < k_cap)) break;
      cum += m.exps[r];
    }
    s_rend = r;
  }
  for (int i = tid; i < n; i += kThreadsS) m.keep[i] = 0;
  __syncthreads();
  const int rend = s_rend;
  const float t = fmaxf(temperature, 1e-5f);
  float mx = -INFINITY;
  for (int r = tid; r < rend; r += kThreadsS) {
    const int i = order_at(m, r);
    m.keep[i] = 1;
    mx = fmaxf(mx, __fdiv_rn(m.lg[i], t));
  }
  mx = warp_max(mx);
  if ((tid & 31) == 0) s_red[tid >> 5] = mx;
  __syncthreads();
  compact_kept(m, n);  // the index-order loops below visit only the rend kept ids
  // The temperature softmax over the kept ids. The terms (an f64 exp each) are independent:
  // every thread makes some; the sums over them stay one thread's sequential f64 chain in
  // index order, as in the reference.
  __shared__ double s_psum;
  float kept_max = -INFINITY;
  for (int w = 0; w < kThreadsS / 32; w++) kept_max = fmaxf(kept_max, s_red[w]);
  if (m.ed) {
    for (int j = tid; j < rend; j += kThreadsS) {
      const int i = m.kept[j];
      const double e = exp((double)(__fdiv_rn(m.lg[i], t) - kept_max));
      m.pf[i] = (float)e;
      m.ed[j] = e;
    }
    __syncthreads();
    if (tid == 0) {
      double psum = 0.0;
      for (int j = 0; j < rend; j++) psum += m.ed[j];
      s_psum = psum;
    }
  } else if (tid == 0) {
    double psum = 0.0;
    for (int j = 0; j < rend; j++) {
      const int i = m.kept[j];
      const double e = exp((double)(__fdiv_rn(m.lg[i], t) - kept_max));
      m.pf[i] = (float)e;
      psum += e;
    }
    s_psum = psum;
  }
  __syncthreads();
  const double psum = s_psum;
  if (psum > 0.0)
    for (int j = tid; j < rend; j += kThreadsS) m.pf[m.kept[j]] = (float)((double)m.pf[m.kept[j]] / psum);
  __syncthreads();
  if (tid == 0) {
    double total = 0.0;
    for (int j = 0; j < rend; j++) total += (double)m.pf[m.kept[j]];
    uint32_t pick = 0;
    if (total > 0.0) {
      const double u = next_f64(a.st) * total;
      double acc = 0.0;
      pick = a.full_last;
      for (int j = 0; j < rend; j++) {
        const int i = m.kept[j];
        acc += (double)m.pf[i];
        if (u < acc) {
          pick = id_of(a, i);
          break;
        }
      }
    }
    s_pick = pick;
  }
  __syncthreads();
  return s_pick;
}

__global__ void __launch_bounds__(kThreadsS, 1) k_sample(const SampleArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  pdl_launch_dependents();
  pdl_wait();
  const int n = (int)(a.hi[0] - a.lo[0]) + (a.ranges > 1 ? (int)(a.hi[1] - a.lo[1]) : 0);
  int np = 1;
  while (np < n) np <<= 1;
  Smem m;
  m.keys = reinterpret_cast<unsigned long long*>(sm);
  m.exps = reinterpret_cast<double*>(m.keys + np);
  m.ed = sample_smem_par(n) ? m.exps + n : nullptr;
  m.lg = reinterpret_cast<float*>(m.exps + (m.ed ? 2 * n : n));
  m.pf = m.lg + n;
  m.kept = reinterpret_cast<int*>(m.pf + n);
  m.keep = reinterpret_cast<uint8_t*>(m.kept + n);
  const int tid = threadIdx.x;
  for (int i = tid; i < np; i += kThreadsS) {
    unsigned long long key = 0ull;  // padding sorts last
    if (i < n) {
      const float v = ld_cg(a.logits + id_of(a, i)) + 0.0f;  // -0 ranks as +0, as the comparator does
      m.lg[i] = v;
      key = ((unsigned long long)f32_order_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
    }
    m.keys[i] = key;
  }
  __syncthreads();
  // bitonic sort, descending: larger logit first, lower index first among equal logits
  for (int k = 2; k <= np; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < np; i += kThreadsS) {
        const int p = i ^ j;
        if (p > i) {
          const unsigned long long x = m.keys[i], y = m.keys[p];
          if ((i & k) == 0 ? x < y : x > y) {
            m.keys[i] = y;
            m.keys[p] = x;
          }
        }
      }
      __syncthreads();
    }
  const float mx = m.lg[order_at(m, 0)];
  for (int r = tid; r < n; r += kThreadsS) m.exps[r] = exp((double)(m.lg[order_at(m, r)] - mx));
  __syncthreads();
  __shared__ double s_sum;
  {
    // The softmax normaliser of the top-p cut, as a fixed-order tree (strided per-thread
    // sums, then warp and block trees): deterministic, and within an ulp or two of the
    // reference's rank-order sum. It only scales the cumulative sums compared with top_p, so
    // like the last bit of exp it can matter only when such a comparison lands within an ulp.
    __shared__ double s_part[kThreadsS / 32];
    double part = 0.0;
    for (int r = tid; r < n; r += kThreadsS) part += m.exps[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if ((tid & 31) == 0) s_part[tid >> 5] = part;
    __syncthreads();
    if (tid < 32) {
      double v = tid < kThreadsS / 32 ? s_part[tid] : 0.0;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (tid == 0) s_sum = v;
    }
  }
  __syncthreads();
  const double sum = s_sum;
  // the top-p cut's terms exps[r] / sum, made once for both draws (independent divisions)
  for (int r = tid; r < n; r += kThreadsS) m.exps[r] = m.exps[r] / sum;
  __syncthreads();
  const sx_sampling_params p = *a.params;
  uint32_t pick = draw(a, m, n, sum, p.temperature, p.top_p, p.top_k);
  if (a.semantic) {
    const uint32_t high = draw(a, m, n, sum, p.ras_high_temp, p.ras_high_top_p, p.top_k);
    if (tid == 0) {
      SampleState* st = a.st;
      const int win = max(1, min(p.ras_win_size, kMaxRasWin));
      const int cnt = __ldcg(&st->win_count);
      bool in_window = false;
      for (int w = 0; w < min(cnt, win); w++) in_window |= __ldcg(&st->win[w]) == pick;
      if (in_window && pick >= a.sem_lo && pick <= a.sem_hi) pick = high;
      // the window holds the last `win` semantic ids of emitted frames (a stop ends the run)
      if (!(pick >= a.stop_lo && pick < a.stop_hi)) {
        st->win[cnt % win] = pick;
        st->win_count = cnt + 1;
      }
    }
  }
  if (tid == 0) *a.amax = argmax_key(0.0f, pick);
}

}  // namespace

size_t sample_smem_bytes(int n) {
  int np = 1;
  while (np < n) np <<= 1;
  return (size_t)np * 8 + (size_t)n * (8 + 4 + 4 + 4 + 1) + (sample_smem_par(n) ? (size_t)n * 8 : 0);
}

cudaError_t launch_sample(const SampleArgs& a, cudaStream_t st) {
  const int n = (int)(a.hi[0] - a.lo[0]) + (a.ranges > 1 ? (int)(a.hi[1] - a.lo[1]) : 0);
  if (n < 1 || n > kSampleMaxIds || a.ranges < 1 || a.ranges > 2) return cudaErrorInvalidValue;
  const size_t smem = sample_smem_bytes(n);
  // the attribute belongs to the current device: set it on every launch (a host-side call,
  // no device work), so sessions on several devices of one process all get it
  cudaError_t e = cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sample_smem_bytes(kSampleMaxIds));
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = launch_cfg(dim3(1), dim3(kThreadsS), smem, st, attr);
  return cudaLaunchKernelEx(&cfg, k_sample, a);
}

}  // namespace sx
