// codec_tc.cu — the codec's convolution / linear product on the 5th-generation tensor cores
// (tcgen05.mma kind::tf32), at f32 accuracy through a three-term split.
//
// The same product as k_conv_gemm (codec.cu): Y[M][N] = W[M][R] * im2col(X)[R][N] with the
// causal im2col formed while the B operand is staged, and the same epilogue (bias, layer
// scale, residual, tanh / GELU, stride-phase scatter). Every f32 operand a is split into
// hi = a with its 13 low mantissa bits cleared (exact in tf32) and lo = a - hi (exact in f32,
// 13 significant bits, of which tf32 keeps 11), and the tensor core accumulates
// hi*hi + hi*lo + lo*hi in f32: the dropped lo*lo term and lo's last bits are below 2^-21 of
// each product, so the result carries f32-level error, which the f32 reference's own
// summation order already has. The weights are split and laid out once at load (one 16 KB
// image per 128-row tile and 16-wide k block: hi then lo, each in the canonical K-major
// layout with the 64-byte swizzle); activations are split by the staging warps.
//
// The tensor core's f32 accumulation is not the round-to-nearest sequence of the CUDA-core
// product: accumulated over a whole reduction of thousands of terms its error reached
// 1.8e-3 on the s2 waveform (the bound is 1e-3). So a tile's reduction runs in chunks of 4
// k blocks (64 terms x 3 products), each into a fresh TMEM accumulator, and the read-back
// warps add the chunks in registers (round to nearest).
//
// One CTA per SM walks output tiles of 128 rows x 128 columns, m-tile fastest so that
// concurrent CTAs share the activations in L2. Warp roles, joined by mbarriers:
//   - warps 0-7: read-back (warp w reads TMEM lanes 32 (w % 4).., columns 64 (w / 4)..) of
//     every chunk into register sums, then the epilogue;
//   - warp 8, one lane: bulk copies of the weight images into a 6-stage ring; the warp also
//     owns the TMEM allocation (4 accumulators of 128 columns);
//   - warp 9, one lane: issues 6 MMAs per k block (2 k steps x 3 products) and the commits;
//   - warps 10-17: stage the B operands (im2col gather, split, swizzled stores), four
//     groups of two warps taking every fourth k block, so four gathers are in flight.
// Every wait is bounded by %globaltimer and raises the error flag; TMEM is freed on every path.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstring>

#include "codec.hpp"
#include "sx_device.cuh"

namespace sx {
namespace codec {
namespace {

constexpr int kRowsTc = 128;  // output rows per tile (M of the MMA)
constexpr int kKB = 16;       // tf32 per 64-byte operand row: one k block
constexpr int kBN = 128;      // output columns per tile (N of the MMA)
constexpr int kStagesTc = 6;
constexpr int kChunkKB = 4;   // k blocks accumulated in TMEM before the register sum
constexpr int kAccBufs = 4;   // TMEM accumulators of kBN columns
constexpr int kEpiW = 8, kProdW = 8;
constexpr int kGroups = kProdW / 2;  // staging groups of two warps
constexpr int kCopyW = kEpiW, kMmaW = kEpiW + 1;
constexpr int kWarpsTc = kEpiW + 2 + kProdW;
constexpr int kThreadsTc = kWarpsTc * 32;
constexpr uint32_t kAImg = 2u * kRowsTc * 64;  // one weight image: hi | lo, 16 KB
constexpr uint32_t kBImg = 2u * kBN * 64;      // one B operand: hi | lo, 16 KB
constexpr uint64_t kWaitNs = 2000000000ull;

struct TcSm {
  uint8_t A[kStagesTc][kAImg];  // weight images
  uint8_t B[kStagesTc][kBImg];  // B hi at 0, B lo at kBN * 64
  uint64_t full[kStagesTc], empty[kStagesTc], acc_full[kAccBufs], acc_empty[kAccBufs];
  uint32_t tmem_base;
};
constexpr size_t kTcSmemBytes = sizeof(TcSm) + 1024;  // + alignment of the base to 1024

__device__ __forceinline__ void tcw(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = global_ns();
  while (!mbar_wait_sleep(bar, parity)) {
    const uint64_t dt = global_ns() - t0;
    if (dt > 1000000ull && err && __ldcg(err) != 0) return;
    if (dt > kWaitNs) {
      if (err) atomicExch(err, 2);
      return;
    }
  }
}

// The K-major, 64-byte-swizzled operand layout (rows of 64 bytes = 16 tf32, 8-row atoms of
// 512 bytes, 16-byte chunk c of row r at chunk c ^ ((r & 7) >> 1)), and its UMMA descriptor:
// the same canonical form the prefill GEMM uses (gemm_tc.cu) with 4-byte elements.
__device__ __forceinline__ uint64_t desc_sw64(const void* p) {
  const uint32_t a = smem_addr(p);
  uint64_t d = 0;
  d |= (uint64_t)((a >> 4) & 0x3fff);
  d |= (uint64_t)1 << 16;           // leading byte offset field: 1
  d |= (uint64_t)(512 >> 4) << 32;  // stride byte offset: 512 (one 8-row atom)
  d |= (uint64_t)1 << 46;           // descriptor version
  d |= (uint64_t)4 << 61;           // SWIZZLE_64B
  return d;
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void commit_to(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float tf32_hi(float v) { return __uint_as_float(__float_as_uint(v) & 0xffffe000u); }

__device__ __forceinline__ float epi_act(float v, int act) {
  if (act == 1) return tanhf(v);
  if (act == 2) return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
  return v;
}

__global__ void __launch_bounds__(kThreadsTc, 1) k_conv_tc(const __grid_constant__ TcConvArgs p) {
  extern __shared__ uint8_t smem_raw[];
  TcSm& sm = *reinterpret_cast<TcSm*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = p.n_mt * p.n_nt;
  const int n_ch = (p.n_kb + kChunkKB - 1) / kChunkKB;  // chunks per tile

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesTc; s++) {
      mbar_init(&sm.full[s], 1 + 2);  // the weight copy (with its bytes) + one staging group
      mbar_init(&sm.empty[s], 1);          // the k block's MMAs (commit)
    }
    for (int b = 0; b < kAccBufs; b++) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], kEpiW);
    }
    mbar_fence_init();
  }
  if (warp == kCopyW) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_addr(&sm.tmem_base)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == kCopyW) {
    if (lane == 0) {
      int g = 0;
      for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
        const int mt = t % p.n_mt;
        for (int kb = 0; kb < p.n_kb; kb++, g++) {
          const int s = g % kStagesTc;
          if (g >= kStagesTc) tcw(&sm.empty[s], (uint32_t)((g / kStagesTc - 1) & 1), p.err);
          mbar_arrive_expect_tx(&sm.full[s], kAImg);
          bulk_g2s(sm.A[s], p.a_img + ((size_t)mt * p.n_kb + kb) * kAImg, kAImg, &sm.full[s]);
        }
      }
      // the last copies have landed before the CTA can leave (already true unless a wait
      // above gave up)
      for (int q = std::max(0, g - kStagesTc); q < g; q++)
        tcw(&sm.full[q % kStagesTc], (uint32_t)((q / kStagesTc) & 1), p.err);
    }
  } else if (warp == kMmaW) {
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kBN >> 3) << 17) |
                                 ((uint32_t)(kRowsTc >> 4) << 24);
      int g = 0, h = 0;
      for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
        for (int kb = 0; kb < p.n_kb; kb++, g++) {
          const int b = h % kAccBufs;
          const bool first = kb % kChunkKB == 0;
          if (first) {
            if (h >= kAccBufs) tcw(&sm.acc_empty[b], (uint32_t)((h / kAccBufs - 1) & 1), p.err);
            fence_after();
          }
          const int s = g % kStagesTc;
          tcw(&sm.full[s], (uint32_t)((g / kStagesTc) & 1), p.err);
          fence_after();
          const uint32_t d = tmem + (uint32_t)(b * kBN);
          const uint8_t* Ah = sm.A[s];
          const uint8_t* Al = Ah + kRowsTc * 64;
          const uint8_t* Bh = sm.B[s];
          const uint8_t* Bl = Bh + kBN * 64;
#pragma unroll
          for (int ks = 0; ks < 2; ks++) {
            const int o = 32 * ks;  // k step of 8 tf32
            mma_tf32(d, desc_sw64(Ah + o), desc_sw64(Bh + o), idesc, (first && ks == 0) ? 0u : 1u);
            mma_tf32(d, desc_sw64(Ah + o), desc_sw64(Bl + o), idesc, 1u);
            mma_tf32(d, desc_sw64(Al + o), desc_sw64(Bh + o), idesc, 1u);
          }
          commit_to(&sm.empty[s]);
          if (kb % kChunkKB == kChunkKB - 1 || kb == p.n_kb - 1) {
            commit_to(&sm.acc_full[b]);
            h++;
          }
        }
      }
    }
  } else if (warp > kMmaW) {
    // ---- staging: kGroups groups of two warps; group j stages the k blocks g with
    // g % kGroups == j, so that kGroups blocks' gathers are in flight at once. In a block,
    // thread i of a group covers rows n = i and i + 64 of each 4-wide k piece c, and all its
    // 32 loads are issued before the first store and before the wait for the ring stage ----
    const int sw = warp - kMmaW - 1, grp = sw >> 1, gt = (sw & 1) * 32 + lane;
    int g = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
      const int n0 = (t / p.n_mt) * kBN;
      for (int kb = 0; kb < p.n_kb; kb++, g++) {
        if (g % kGroups != grp) continue;
        const int s = g % kStagesTc;
        // the k block's 16 reduction rows: lane j (< 16) resolves row kb*16 + j to its
        // channel and causal shift once, the warp reads them by shuffle
        int base = -1, shift = 0;
        if (lane < kKB) {
          const int r = kb * kKB + lane;
          if (r < p.R) {
            const int ci = r / p.k, tap = r - ci * p.k;
            base = ci;
            shift = (p.k - 1 - tap) * p.dil;
          }
        }
        float v[4][2][4];  // [piece c][row n = gt + 64 hh][k in piece]
#pragma unroll
        for (int c = 0; c < 4; c++) {
          int ci[4], sh[4];
#pragma unroll
          for (int q = 0; q < 4; q++) {
            ci[q] = __shfl_sync(0xffffffffu, base, c * 4 + q);
            sh[q] = __shfl_sync(0xffffffffu, shift, c * 4 + q);
          }
#pragma unroll
          for (int hh = 0; hh < 2; hh++) {
            const int col = n0 + gt + 64 * hh;
#pragma unroll
            for (int q = 0; q < 4; q++) {
              const int src = col - sh[q];
              v[c][hh][q] = (ci[q] >= 0 && col < p.N && src >= 0) ? __ldg(p.x + (size_t)ci[q] * p.N + src) : 0.f;
            }
          }
        }
        if (g >= kStagesTc) tcw(&sm.empty[s], (uint32_t)((g / kStagesTc - 1) & 1), p.err);
        uint8_t* Bh = sm.B[s];
        uint8_t* Bl = Bh + kBN * 64;
#pragma unroll
        for (int c = 0; c < 4; c++)
#pragma unroll
          for (int hh = 0; hh < 2; hh++) {
            const int n = gt + 64 * hh;
            const float* w = v[c][hh];
            float4 hi, lo;
            hi.x = tf32_hi(w[0]), hi.y = tf32_hi(w[1]), hi.z = tf32_hi(w[2]), hi.w = tf32_hi(w[3]);
            lo.x = w[0] - hi.x, lo.y = w[1] - hi.y, lo.z = w[2] - hi.z, lo.w = w[3] - hi.w;
            int o = (n >> 3) * 512 + (n & 7) * 64 + c * 16;
            o ^= ((o >> 7) & 3) << 4;
            *reinterpret_cast<float4*>(Bh + o) = hi;
            *reinterpret_cast<float4*>(Bl + o) = lo;
          }
        fence_async();  // generic-proxy stores become visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.full[s]);
      }
    }
  } else {
    // ---- read-back: warp w sums columns 64 (w / 4).. of TMEM lanes 32 (w % 4).. ----
    const int q4 = warp & 3, half = warp >> 2;
    int h = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
      const int mt = t % p.n_mt, n0 = (t / p.n_mt) * kBN;
      float acc[64];
#pragma unroll
      for (int j = 0; j < 64; j++) acc[j] = 0.f;
      for (int ch = 0; ch < n_ch; ch++, h++) {
        const int b = h % kAccBufs;
        tcw(&sm.acc_full[b], (uint32_t)((h / kAccBufs) & 1), p.err);
        fence_after();
        const uint32_t ta = tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(b * kBN + half * 64);
#pragma unroll
        for (int c = 0; c < 64; c += 16) {
          uint32_t r[16];
          ld16(ta + c, r);
          ld_wait();
#pragma unroll
          for (int j = 0; j < 16; j++) acc[c + j] += __uint_as_float(r[j]);
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.acc_empty[b]);
      }
      const int m = mt * kRowsTc + q4 * 32 + lane;
      if (m >= p.M) continue;
      const int co = p.phase > 1 ? m % p.cout : m;
      const int ph = p.phase > 1 ? m / p.cout : 0;
      const float bias = p.bias ? p.bias[co] : 0.f;
      const float sc = p.scale ? p.scale[co] : 1.f;
      const int col0 = n0 + half * 64;
      if (p.phase > 1) {
        float* yr = p.y + (size_t)co * p.N * p.phase + ph;
#pragma unroll
        for (int j = 0; j < 64; j++) {
          const int col = col0 + j;
          if (col < p.N) {
            float v = acc[j] + bias;
            if (p.scale) v *= sc;
            yr[(size_t)col * p.phase] = epi_act(v, p.act);
          }
        }
      } else {
        float* yr = p.y + (size_t)m * p.N;
        const float* rr = p.resid ? p.resid + (size_t)m * p.N : nullptr;
        if (col0 + 64 <= p.N && (p.N & 3) == 0) {
#pragma unroll
          for (int j = 0; j < 64; j += 4) {
            float4 v;
            v.x = acc[j] + bias, v.y = acc[j + 1] + bias, v.z = acc[j + 2] + bias, v.w = acc[j + 3] + bias;
            if (p.scale) v.x *= sc, v.y *= sc, v.z *= sc, v.w *= sc;
            v.x = epi_act(v.x, p.act), v.y = epi_act(v.y, p.act);
            v.z = epi_act(v.z, p.act), v.w = epi_act(v.w, p.act);
            if (rr) {
              const float4 x = *reinterpret_cast<const float4*>(rr + col0 + j);
              v.x += x.x, v.y += x.y, v.z += x.z, v.w += x.w;
            }
            *reinterpret_cast<float4*>(yr + col0 + j) = v;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 64; j++) {
            const int col = col0 + j;
            if (col < p.N) {
              float v = acc[j] + bias;
              if (p.scale) v *= sc;
              v = epi_act(v, p.act);
              if (rr) v += rr[col];
              yr[col] = v;
            }
          }
        }
      }
    }
  }
  // every role is done: the read-back waited for every chunk's commit
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == kCopyW) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

}  // namespace

size_t tc_image_bytes(int M, int R) {
  return (size_t)((M + kRowsTc - 1) / kRowsTc) * (size_t)((R + kKB - 1) / kKB) * kAImg;
}

void tc_image(const float* A, int M, int R, uint32_t* out) {
  const int n_mt = (M + kRowsTc - 1) / kRowsTc, n_kb = (R + kKB - 1) / kKB;
  for (int mt = 0; mt < n_mt; mt++)
    for (int kb = 0; kb < n_kb; kb++) {
      uint8_t* img = reinterpret_cast<uint8_t*>(out) + ((size_t)mt * n_kb + kb) * kAImg;
      for (int rr = 0; rr < kRowsTc; rr++)
        for (int k = 0; k < kKB; k++) {
          const int m = mt * kRowsTc + rr, r = kb * kKB + k;
          const float a = (m < M && r < R) ? A[(size_t)m * R + r] : 0.f;
          uint32_t bits;
          std::memcpy(&bits, &a, 4);
          const uint32_t hb = bits & 0xffffe000u;
          float hi, lo;
          std::memcpy(&hi, &hb, 4);
          lo = a - hi;
          int o = (rr >> 3) * 512 + (rr & 7) * 64 + k * 4;
          o ^= ((o >> 7) & 3) << 4;
          std::memcpy(img + o, &hi, 4);
          std::memcpy(img + kRowsTc * 64 + o, &lo, 4);
        }
    }
}

cudaError_t launch_conv_tc(const TcConvArgs& a0, int sms, cudaStream_t st) {
  TcConvArgs a = a0;
  a.n_mt = (a.M + kRowsTc - 1) / kRowsTc;
  a.n_kb = (a.R + kKB - 1) / kKB;
  a.bn = kBN;
  a.n_nt = (a.N + kBN - 1) / kBN;
  // the attribute is per device; threads that race here both set it, which is harmless
  static std::atomic<bool> attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(k_conv_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmemBytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev].store(true, std::memory_order_release);
  }
  const int grid = std::max(1, std::min(a.n_mt * a.n_nt, sms));
  k_conv_tc<<<grid, kThreadsTc, kTcSmemBytes, st>>>(a);
  return cudaSuccess;  // launch errors surface at the caller's cudaGetLastError
}

}  // namespace codec
}  // namespace sx
