// gemm_tc.cu — Q8_0 prefill GEMM on the 5th-generation tensor cores (tcgen05, kind::i8).
//
// Replaces the prompt forward's quantized linears (`SlowAr::prefill`,
// crates/syrinx-fish/src/s2/slow_ar.rs:250-255, M = prompt chunk; `prefill_batch`
// s2/slow_ar.rs:404-499; `Qwen2Lm::forward_hidden_cached` over candle QMatMul,
// crates/syrinx-lm/src/cv2/mod.rs:195-211, 261-279) for chunks of 9..64 tokens.
//
// It computes exactly what k_gemv_q8<Mt> (gemv_q8.cu) computes and writes the same partial
// buffer [tile][k chunk][token][16], so the same merge kernels apply the epilogues and a
// prefill gives bit-identical results either way. The difference is where the products
// happen: a CTA takes a 128-row group of the weight (8 tile records per 32-wide k block) and
// all the chunk's tokens, and one tcgen05.mma (M = 128, N = 4 limbs x Mt tokens, K = 32)
// per k block yields the exact int32 block sums of every row against every limb of every
// token into tensor memory. The epilogue warps read them back (tcgen05.ld), fold the limbs
// and scale per block in f32 in the GEMV's order, while the tensor core already runs the next
// block's product into the other half of tensor memory.
//
// Data flow per CTA (one CTA per SM, a contiguous range of (row group, k chunk) items):
//   - one lane bulk-copies the 8 tile records of an item (8 x 4352 contiguous bytes) into a
//     3-stage shared-memory ring (cp.async.bulk, mbarrier completion), an item ahead;
//   - all warps repack a block's records into the canonical no-swizzle K-major layout of the
//     A operand (8-row x 16-byte core matrices) and split x into int8 limbs in the same layout
//     for the B operand (row n = 4 * token + limb), then fence the async proxy;
//   - one thread issues the MMA and commits it to an mbarrier;
//   - all warps read back the previous block's sums and accumulate.
// Every wait is bounded by %globaltimer and raises the session's error flag; tensor memory is
// freed on every path.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>

#include "sx_device.cuh"
#include "sx_internal.hpp"

namespace sx {
namespace {

constexpr int kTW = 8;             // warps
constexpr int kTT = kTW * 32;      // threads
constexpr int kRows = 128;         // weight rows per CTA tile (8 Q8_0 tiles)
constexpr int kTiles = kRows / kQ8Tile;
constexpr int kChunkB = 8;         // blocks per k chunk
constexpr int kStageBytes = kTiles * kChunkB * kQ8Rec;  // 34816
constexpr int kStages = 3;
constexpr uint64_t kTcWaitNs = 2000000000ull;

__device__ __forceinline__ void tc_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    const uint64_t dt = global_ns() - t0;
    if (dt > 1000000ull && err && __ldcg(err) != 0) return;
    if (dt > kTcWaitNs) {
      if (err) atomicExch(err, 2);
      return;
    }
  }
}

// UMMA shared-memory descriptor: canonical K-major layout without swizzle, 8-row x 16-byte
// core matrices, LBO = distance between the two 16-byte K halves, SBO = between 8-row groups.
__device__ __forceinline__ uint64_t umma_desc(const void* p, uint32_t lbo, uint32_t sbo) {
  const uint32_t a = smem_addr(p);
  uint64_t d = 0;
  d |= (uint64_t)((a >> 4) & 0x3fff);
  d |= (uint64_t)((lbo >> 4) & 0x3fff) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3fff) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  return d;                // base offset 0, swizzle none
}
// instruction descriptor of kind::i8: s32 accumulator, signed 8-bit A and B, both K-major
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, 0, 0;\n"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive 32-bit columns of this warp's 32 tensor-memory lanes
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

struct TcGeo {
  int K, nb, nc, n_vt, n_rg;  // columns, blocks, k chunks, tiles, 128-row groups
};

// element (row n, k) of a canonical K-major operand of 32 bytes of K per row
__device__ __forceinline__ int canon_off(int n, int k) { return (n >> 3) * 256 + (k >> 4) * 128 + (n & 7) * 16 + (k & 15); }

template <int MT>
struct TcSmem {
  static constexpr int N = 4 * MT;
  uint8_t stage[kStages][kStageBytes];
  uint8_t A[2][kRows * 32];
  uint8_t B[2][N * 32];
  float sxs[2][MT];
  float den[MT];
  float red[kTW][MT];
  int8_t scr[kTW][4][32];
  uint64_t bar_stage[kStages];
  uint64_t bar_mma[2];
  uint32_t tmem_base;
};

template <int MT>
__global__ void __launch_bounds__(kTT, 1) k_gemm_tc(const GemvArgs a, const TcGeo g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  TcSmem<MT>& sm = *reinterpret_cast<TcSmem<MT>*>(smem_raw);
  constexpr int N = TcSmem<MT>::N;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int I = g.n_rg * g.nc;
  const int c0 = (int)((long long)blockIdx.x * I / gridDim.x), c1 = (int)((long long)(blockIdx.x + 1) * I / gridDim.x);
  const uint8_t* W = static_cast<const uint8_t*>(a.w.q);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; i++) mbar_init(&sm.bar_stage[i], 1);
    for (int i = 0; i < 2; i++) mbar_init(&sm.bar_mma[i], 1);
    mbar_fence_init();
  }
  if (warp == 0) {  // two accumulators of up to 256 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_addr(&sm.tmem_base)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  // the item's 8 tile records (weights do not depend on the previous kernel)
  auto issue_item = [&](int it, int stage) {
    const int rg = (int)(it / g.nc), kc = (int)(it % g.nc);
    const int nrec = min(kChunkB, g.nb - kc * kChunkB);
    int ntiles = 0;
    for (int t = 0; t < kTiles; t++)
      if (rg * kTiles + t < g.n_vt) ntiles++;
    mbar_arrive_expect_tx(&sm.bar_stage[stage], (uint32_t)(ntiles * nrec * kQ8Rec));
    for (int t = 0; t < ntiles; t++)
      bulk_g2s(sm.stage[stage] + t * kChunkB * kQ8Rec,
               W + ((size_t)(rg * kTiles + t) * g.nb + (size_t)kc * kChunkB) * kQ8Rec, (uint32_t)(nrec * kQ8Rec),
               &sm.bar_stage[stage]);
  };
  if (threadIdx.x == 0 && c1 > c0) issue_item(c0, 0);

  pdl_launch_dependents();
  pdl_wait();

  // RMSNorm denominators of the chunk's tokens over the full K, in the GEMV's order
  if (a.norm_w) {
    float ss[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) ss[m] = 0.f;
    for (int k = threadIdx.x; k < g.K; k += kTT)
#pragma unroll
      for (int m = 0; m < MT; m++) {
        const float v = (m < a.M) ? ld_cg(a.x + (size_t)m * g.K + k) : 0.f;
        ss[m] = fmaf(v, v, ss[m]);
      }
#pragma unroll
    for (int m = 0; m < MT; m++) {
      const float t = warp_sum(ss[m]);
      if (lane == 0) sm.red[warp][m] = t;
    }
    __syncthreads();
    if (threadIdx.x < MT) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kTW; w++) t += sm.red[w][threadIdx.x];
      sm.den[threadIdx.x] = sqrtf(__fadd_rn(__fdiv_rn(t, (float)g.K), a.eps));
    }
    __syncthreads();
  }

  // epilogue roles: TMEM lane quarter q (rows 32q..32q+31), token half h
  const int q = warp & 3, h = warp >> 2;
  const int row = q * 32 + lane;
  constexpr int TPT = MT / 2;  // tokens per thread
  float acc01[TPT], acc23[TPT];
#pragma unroll
  for (int i = 0; i < TPT; i++) acc01[i] = acc23[i] = 0.f;

  int blk = 0;  // blocks processed by this CTA (selects the A/B buffer and TMEM half)
  int prev_stage = 0, prev_j = 0, prev_rg = 0, prev_kc = 0, prev_nrec = 0;
  bool have_prev = false;

  // read back block (blk - 1)'s sums and accumulate; at the end of its item, store the partials
  auto epilogue = [&]() {
    const int buf = (int)((blk - 1) & 1);
    tc_wait(&sm.bar_mma[buf], (uint32_t)(((blk - 1) >> 1) & 1), a.err);
    tc_fence_after();
    const uint8_t* rec = sm.stage[prev_stage] + ((row >> 4) * kChunkB + prev_j) * kQ8Rec;
    const float ds = __half2float(*reinterpret_cast<const __half*>(rec + q8_scale_off(row & 15)));
#pragma unroll
    for (int part = 0; part < TPT / 8; part++) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 256 + (h * TPT + part * 8) * 4), r);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int tl = part * 8 + i, t = h * TPT + tl;
        const float sx = sm.sxs[buf][t];
        const float dsx = __fmul_rn(ds, sx);
        const int s01 = (int)r[4 * i] * 128 + (int)r[4 * i + 1];
        const int s23 = (int)r[4 * i + 2] * 128 + (int)r[4 * i + 3];
        acc01[tl] = fmaf(dsx, (float)s01, acc01[tl]);
        acc23[tl] = fmaf(dsx, (float)s23, acc23[tl]);
      }
    }
    if (prev_j == prev_nrec - 1) {
      const int vt = prev_rg * kTiles + (row >> 4);
      if (vt < g.n_vt) {
        float* P = a.part + ((size_t)vt * g.nc + prev_kc) * MT * 16 + (row & 15);
#pragma unroll
        for (int tl = 0; tl < TPT; tl++) {
          const int t = h * TPT + tl;
          if (t < a.M) __stcg(P + t * 16, acc01[tl] * 0x1p-7f + acc23[tl] * 0x1p-21f);
          acc01[tl] = acc23[tl] = 0.f;
        }
      } else {
#pragma unroll
        for (int tl = 0; tl < TPT; tl++) acc01[tl] = acc23[tl] = 0.f;
      }
    }
  };

  int n_items = 0;
  for (int it = c0; it < c1; it++, n_items++) {
    const int stage = (int)(n_items % kStages);
    const int rg = (int)(it / g.nc), kc = (int)(it % g.nc);
    const int nrec = min(kChunkB, g.nb - kc * kChunkB);
    // the next item's records into the stage an item ahead (its last reader finished two
    // items ago)
    if (threadIdx.x == 0 && it + 1 < c1) issue_item(it + 1, (int)((n_items + 1) % kStages));
    tc_wait(&sm.bar_stage[stage], (uint32_t)((n_items / kStages) & 1), a.err);
    for (int j = 0; j < nrec; j++, blk++) {
      const int buf = (int)(blk & 1);
      const int b = kc * kChunkB + j;
      // A: the 8 records' quants into the canonical layout (one 16-byte fragment per thread)
      {
        const int t = warp, L = lane;  // tile t, fragment lane L = 4g + c
        const int gg = L >> 2, cc = L & 3;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (rg * kTiles + t < g.n_vt) v = lds128(sm.stage[stage] + (t * kChunkB + j) * kQ8Rec + L * 16);
        uint8_t* A = sm.A[buf];
        const int m0 = t * 16 + gg, m1 = m0 + 8;
        *reinterpret_cast<uint32_t*>(A + canon_off(m0, 4 * cc)) = v.x;
        *reinterpret_cast<uint32_t*>(A + canon_off(m1, 4 * cc)) = v.y;
        *reinterpret_cast<uint32_t*>(A + canon_off(m0, 16 + 4 * cc)) = v.z;
        *reinterpret_cast<uint32_t*>(A + canon_off(m1, 16 + 4 * cc)) = v.w;
      }
      // B: limbs of x (normed) for block b, one warp per token
      for (int m = warp; m < MT; m += kTW) {
        const int k = b * 32 + lane;
        float v = 0.f;
        if (m < a.M) {
          v = ld_cg(a.x + (size_t)m * g.K + k);
          if (a.norm_w) v = __fmul_rn(__fdiv_rn(v, sm.den[m]), a.norm_w[k]);
        }
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
        {  // lane L writes limb L/8's bytes k = 4(L%8) .. 4(L%8)+3 as one word
          const int limb = lane >> 3, kk = 4 * (lane & 7);
          const uint32_t w = *reinterpret_cast<const uint32_t*>(&sm.scr[warp][limb][kk]);
          *reinterpret_cast<uint32_t*>(sm.B[buf] + canon_off(4 * m + limb, kk)) = w;
        }
        if (lane == 0) sm.sxs[buf][m] = sx;
        __syncwarp();
      }
      fence_async_smem();  // the operands written by threads become visible to the tensor core
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      if (threadIdx.x == 0) {
        tc_mma(tmem + (uint32_t)(buf * 256), umma_desc(sm.A[buf], 128, 256), umma_desc(sm.B[buf], 128, 256),
               idesc_i8(kRows, N));
        tc_commit(&sm.bar_mma[buf]);
      }
      if (have_prev) epilogue();
      // the next MMA into this warp's TMEM half must not start before the read-back is done
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      prev_stage = stage;
      prev_j = j;
      prev_rg = rg;
      prev_kc = kc;
      prev_nrec = nrec;
      have_prev = true;
    }
  }
  if (have_prev) epilogue();  // the last block (blk - 1)
  tc_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

template <int MT>
cudaError_t launch_tc_t(const GemvArgs& a, const TcGeo& g, int sms, cudaStream_t st) {
  auto kern = k_gemm_tc<MT>;
  const size_t smem = sizeof(TcSmem<MT>) + 1024;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long I = (long long)g.n_rg * g.nc;
  const int grid = (int)std::max(1LL, std::min<long long>(I, sms));
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = launch_cfg(dim3(grid), dim3(kTT), smem, st, attr);
  return cudaLaunchKernelEx(&cfg, kern, a, g);
}

}  // namespace

// read per launch, so a process can compare both paths (SYRINX_TC=0: the mma.sync GEMV)
bool tc_enabled() {
  const char* v = getenv("SYRINX_TC");
  return !(v && v[0] == '0');
}

// The partials of a Q8_0 GEMV of 9..64 tokens (Mt = 16, 32 or 64) on the tensor cores.
cudaError_t launch_gemm_tc(const GemvArgs& a, int Mt, int K, int nb, int nc, int t_first, int n_vt, int sms,
                           cudaStream_t st) {
  if (t_first != 0 || a.n_extra != 0 || K % 32) return cudaErrorInvalidValue;
  TcGeo g;
  g.K = K;
  g.nb = nb;
  g.nc = nc;
  g.n_vt = n_vt;
  g.n_rg = (n_vt + kTiles - 1) / kTiles;
  switch (Mt) {
    case 16: return launch_tc_t<16>(a, g, sms, st);
    case 32: return launch_tc_t<32>(a, g, sms, st);
    case 64: return launch_tc_t<64>(a, g, sms, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace sx
