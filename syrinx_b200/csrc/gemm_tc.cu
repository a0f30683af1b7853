// gemm_tc.cu — Q8_0 prefill GEMM on the 5th-generation tensor cores (tcgen05, kind::f16).
//
// Replaces the prompt forward's quantized linears (`SlowAr::prefill`,
// crates/syrinx-fish/src/s2/slow_ar.rs:250-255, M = prompt chunk; `prefill_batch`
// s2/slow_ar.rs:404-499; `Qwen2Lm::forward_hidden_cached` over candle QMatMul,
// crates/syrinx-lm/src/cv2/mod.rs:195-211, 261-279) for chunks of 9..64 tokens.
//
// It computes exactly what k_gemv_q8<Mt> (gemv_q8.cu) computes and writes the same partial
// buffer [tile][k chunk][token][16], so the same merge kernels apply the epilogues and a
// prefill gives bit-identical results either way. A CTA takes a 128-row group of the weight
// (8 tile records per 32-wide k block) and all the chunk's tokens. The operands are small
// integers: the Q8_0 quants (-128..127) and the four limbs of each token's activations
// (|limb| <= 128). Both are exact in f16, every product is exact, and every partial sum of a
// 32-wide block stays below 2^24, so two tcgen05.mma kind::f16 (M = 128, N = 4 limbs x Mt
// tokens, K = 16) give the exact integer block sums of every row against every limb of every
// token in f32 in tensor memory, whatever order the tensor core adds them in. The epilogue
// then needs no integer-to-float conversion (the XU pipe, which bounded the kind::i8 form):
// per (row, token) one packed fma.rn.f32x2 folds the limb pairs (l0 * 128 + l1 and
// l2 * 128 + l3, each rounded once, exactly as the GEMV's (float)(int) does) and a second one
// scales and accumulates them, in the GEMV's order.
//
// Data flow:
//   - k_tc_limbs (one CTA per token) stages the token's row in shared memory (one round trip),
//     computes the RMSNorm denominator as k_gemv_q8 does (256 threads, k strided by 256, warp
//     sums added in warp order) and splits the normed values of each 32-wide block into int8
//     limbs, written once per launch as every block's f16 B operand in the canonical
//     K-major layout with the 64-byte swizzle, rows grouped by token pairs (limb_row);
//   - k_gemm_tc (one CTA per SM, a contiguous range of (k chunk, 128-row group) items, k-chunk
//     major so consecutive items share their B operands) runs four warp roles joined by
//     mbarriers: a copy lane bulk-copies each half item's 8 x 4 tile records (three stages) and
//     each chunk's B operands (cp.async.bulk), after prefetching all the CTA's records into L2;
//     four warps widen every block's quants to f16 in the swizzled layout (byte-permute into
//     0x64xx and one packed f16 subtract: exact); one lane issues the block's two MMAs into
//     one of two TMEM accumulators and commits them; sixteen warps read back each block's sums
//     (tcgen05.ld) and accumulate.
// Every wait is bounded by %globaltimer and raises the session's error flag; tensor memory is
// freed on every path.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>

#include "sx_device.cuh"
#include "sx_internal.hpp"

namespace sx {
namespace {

constexpr int kTW = 8;             // warps of the limb kernel
constexpr int kTT = kTW * 32;      // its threads
constexpr int kRows = 128;         // weight rows per CTA tile (8 Q8_0 tiles)
constexpr int kTiles = kRows / kQ8Tile;
constexpr int kChunkB = 8;         // blocks per k chunk
constexpr uint64_t kTcWaitNs = 2000000000ull;

__device__ __forceinline__ void tc_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = global_ns();
  while (!mbar_wait_sleep(bar, parity)) {
    const uint64_t dt = global_ns() - t0;
    if (dt > 1000000ull && err && __ldcg(err) != 0) return;
    if (dt > kTcWaitNs) {
      if (err) atomicExch(err, 2);
      return;
    }
  }
}

// UMMA shared-memory descriptor of the canonical K-major layout with the 64-byte swizzle (one
// 32-wide block of f16 per row): 8-row atoms of 512 bytes (SBO), the leading offset field 1 as the swizzled K-major
// form requires, layout type 4. The second MMA of a block starts 32 bytes further.
__device__ __forceinline__ uint64_t umma_desc_sw64(const void* p) {
  const uint32_t a = smem_addr(p);
  uint64_t d = 0;
  d |= (uint64_t)((a >> 4) & 0x3fff);
  d |= (uint64_t)1 << 16;           // leading byte offset (16 B units): 1
  d |= (uint64_t)(512 >> 4) << 32;  // stride byte offset: 512
  d |= (uint64_t)1 << 46;           // descriptor version (sm_100)
  d |= (uint64_t)4 << 61;           // SWIZZLE_64B
  return d;
}
// instruction descriptor of kind::f16: f32 accumulator, f16 A and B, both K-major
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 16 consecutive 32-bit columns of this warp's 32 tensor-memory lanes
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Four signed int8 (one word) -> four exact f16 (two words): bias to 128 + b, place each byte
// under the f16 exponent of 1024 (0x64xx = 1024 + byte), subtract 1152 in packed f16.
__device__ __forceinline__ uint2 s8x4_to_f16x4(uint32_t w) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t lo = __byte_perm(u, 0x64646464u, 0x5140);
  const uint32_t hi = __byte_perm(u, 0x64646464u, 0x7362);
  const __half2 off = __half2half2(__ushort_as_half((unsigned short)0x6480));  // 1152
  __half2 a = __hsub2(*reinterpret_cast<const __half2*>(&lo), off);
  __half2 b = __hsub2(*reinterpret_cast<const __half2*>(&hi), off);
  return make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
}

struct TcGeo {
  int K, nb, nc, n_vt, n_rg;  // columns, blocks, k chunks, tiles, 128-row groups
};

// byte offset of element (row n, k < 32) of a K-major f16 operand, 64-byte swizzle: rows of 64
// bytes, 8-row atoms of 512 bytes, 16-byte chunk c of row r stored at chunk c ^ ((r & 7) >> 1)
// (address bits 4-5 ^= bits 7-8). Pieces of 4 elements (k % 4 == 0) stay contiguous.
__host__ __device__ __forceinline__ int canon16_off(int n, int k) {
  const int o = (n >> 3) * 512 + (n & 7) * 64 + k * 2;
  return o ^ (((o >> 7) & 3) << 4);
}
// B row of limb l of token t: tokens in pairs, each limb's two tokens adjacent
// (S_l0[t], S_l0[t+1], S_l1[t], S_l1[t+1], ...), so a pair's sums read back as f32x2 operands
__host__ __device__ __forceinline__ int limb_row(int t, int l) { return 8 * (t >> 1) + 2 * l + (t & 1); }

// ---- the B operand: limbs of x for every k block, f16 in the swizzled layout -----------
// One CTA per token: the row into shared memory (every load in flight at once), the RMSNorm
// denominator exactly as k_gemv_q8 computes it (256 threads, k strided by 256, warp sums added
// in warp order), then per 32-wide block the limb split of the normed values (exact to 2^-27
// of the block max) as rows limb_row(t, 0..3) of that block's f16 operand (exact: |limb| <=
// 128), and the block's power-of-two scale.
template <int MT>
__global__ void __launch_bounds__(kTT) k_tc_limbs(const GemvArgs a, const TcGeo g, uint8_t* Bg, float* sxg) {
  extern __shared__ float xrow[];  // [K]
  __shared__ float red[kTW];
  __shared__ float den_s;
  __shared__ __align__(16) int8_t scr[kTW][4][32];
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int N = 4 * MT;
  pdl_launch_dependents();
  pdl_wait();
  const bool live = t < a.M;
  if (live) {
    const float4* src = reinterpret_cast<const float4*>(a.x + (size_t)t * g.K);
    for (int i = threadIdx.x; i < g.K / 4; i += kTT) reinterpret_cast<float4*>(xrow)[i] = __ldcg(src + i);
  }
  __syncthreads();
  if (a.norm_w && live) {
    float ss = 0.f;
    for (int k = threadIdx.x; k < g.K; k += kTT) ss = fmaf(xrow[k], xrow[k], ss);
    const float w = warp_sum(ss);
    if (lane == 0) red[warp] = w;
    __syncthreads();
    if (threadIdx.x == 0) {
      float tot = 0.f;
      for (int i = 0; i < kTW; i++) tot += red[i];
      den_s = sqrtf(__fadd_rn(__fdiv_rn(tot, (float)g.K), a.eps));
    }
    __syncthreads();
  }
  for (int b = warp; b < g.nb; b += kTW) {
    const int k = b * 32 + lane;
    float v = 0.f;
    if (live) {
      v = xrow[k];
      if (a.norm_w) v = __fmul_rn(__fdiv_rn(v, den_s), a.norm_w[k]);
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
    const float sv = v * sc;
    const float l0 = rintf(sv);
    float r = (sv - l0) * 128.f;
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
    const int limb = lane >> 3, kk = 4 * (lane & 7);
    const uint32_t word = *reinterpret_cast<const uint32_t*>(&scr[warp][limb][kk]);
    *reinterpret_cast<uint2*>(Bg + (size_t)b * N * 64 + canon16_off(limb_row(t, limb), kk)) = s8x4_to_f16x4(word);
    if (lane == 0) sxg[(size_t)b * MT + t] = sx;
    __syncwarp();
  }
}

// Warp roles of k_gemm_tc (22 warps):
//   warp 0        one lane bulk-copies the tile records of each half item (4 blocks, three
//                 stages) and each k chunk's f16 B operands and x scales (one chunk resident);
//   warp 1        one lane issues the two MMAs of every block and commits them;
//   warps 2-5     widen each block's 8 records (two tiles each) to the f16 A operand and copy the
//                 block's row and x scales into a ring of four stages, up to four blocks ahead;
//   warps 6-21    read-back: TMEM lane quarter warp % 4, token quarter (warp - 6) / 4.
// Everything between the roles goes through mbarriers, so copies, widening, MMAs and read-backs
// of different blocks overlap: with the operands ahead, a block costs the larger of its MMAs
// and its read-back, which alternate between two TMEM accumulators. Every wait is bounded.
constexpr int kGW = 22;            // warps of the GEMM
constexpr int kGT = kGW * 32;
constexpr int kWidenW = 4;         // widening warps (two tiles each)
constexpr int kEpiW = 16;          // read-back warps
constexpr int kHalfB = kChunkB / 2;  // blocks per staged half item
constexpr int kAStages = 3;        // staged half items
constexpr int kWStages = 4;        // widened blocks

template <int MT>
struct TcSmem {
  static constexpr int N = 4 * MT;
  uint8_t stA[kAStages][kTiles * kHalfB * kQ8Rec];  // a half item: 8 tiles x 4 records
  alignas(512) uint8_t B16[kChunkB][N * 64];        // the k chunk's B operands, f16 swizzled
  float stS[kChunkB * MT];                          // and its blocks' x scales
  alignas(512) uint8_t A16[kWStages][kRows * 64];   // a block's A operand, f16 swizzled
  float dsb[kWStages][kRows];                       // its row scales
  float sxr[kWStages][MT];                          // its x scales
  uint64_t a_full[kAStages], a_empty[kAStages], b_full, b_empty, w_full[kWStages], w_empty[kWStages], t_full[2],
      t_empty[2];
  uint32_t tmem_base;
};

// the CTA's items and the chunk bookkeeping every role walks identically
struct TcWalk {
  int c0, c1, n_rg;
  __device__ int kc(int it) const { return it / n_rg; }
  __device__ bool chunk_starts(int it) const { return it == c0 || kc(it) != kc(it - 1); }
  __device__ bool chunk_ends(int it) const { return it + 1 == c1 || kc(it + 1) != kc(it); }
};

template <int MT>
__global__ void __launch_bounds__(kGT, 1) k_gemm_tc(const GemvArgs a, const TcGeo g, const uint8_t* Bg,
                                                    const float* sxg) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  TcSmem<MT>& sm = *reinterpret_cast<TcSmem<MT>*>(smem_raw);
  constexpr int N = TcSmem<MT>::N;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // items (k chunk, 128-row group), k-chunk-major: consecutive items share the B operand
  const int I = g.n_rg * g.nc;
  TcWalk wk;
  wk.c0 = (int)((long long)blockIdx.x * I / gridDim.x);
  wk.c1 = (int)((long long)(blockIdx.x + 1) * I / gridDim.x);
  wk.n_rg = g.n_rg;
  const uint8_t* W = static_cast<const uint8_t*>(a.w.q);
  auto nrec_of = [&](int kc) { return min(kChunkB, g.nb - kc * kChunkB); };
  auto half_blocks = [&](int nrec, int hf) { return min(kHalfB, nrec - hf * kHalfB); };

  if (threadIdx.x == 0) {
    for (int i = 0; i < kAStages; i++) {
      mbar_init(&sm.a_full[i], 1);
      mbar_init(&sm.a_empty[i], kWidenW);
    }
    for (int i = 0; i < kWStages; i++) {
      mbar_init(&sm.w_full[i], kWidenW);
      mbar_init(&sm.w_empty[i], 1 + kEpiW);  // the block's MMAs (commit) + the read-back warps
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&sm.t_full[i], 1);
      mbar_init(&sm.t_empty[i], kEpiW);
    }
    mbar_init(&sm.b_full, 1);
    mbar_init(&sm.b_empty, 1 + kWidenW);  // the chunk's last MMAs (commit) + the widening warps
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
  pdl_launch_dependents();

  if (warp == 0) {
    // ---- copy lane ----
    if (lane == 0) {
      int ns = 0, chunk = 0;
      for (int it = wk.c0; it < wk.c1; it++) {
        const int kc = wk.kc(it), rg = it % g.n_rg, nrec = nrec_of(kc);
        const int ntiles = min(kTiles, g.n_vt - rg * kTiles);
        for (int hf = 0; hf < 2; hf++) {
          const int nbh = half_blocks(nrec, hf);
          if (nbh <= 0) break;
          const int st = ns % kAStages;
          if (ns >= kAStages) tc_wait(&sm.a_empty[st], (uint32_t)(((ns - kAStages) / kAStages) & 1), a.err);
          mbar_arrive_expect_tx(&sm.a_full[st], (uint32_t)(ntiles * nbh * kQ8Rec));
          for (int t = 0; t < ntiles; t++)
            bulk_g2s(sm.stA[st] + t * kHalfB * kQ8Rec,
                     W + ((size_t)(rg * kTiles + t) * g.nb + (size_t)kc * kChunkB + hf * kHalfB) * kQ8Rec,
                     (uint32_t)(nbh * kQ8Rec), &sm.a_full[st]);
          ns++;
          if (ns == 1) {  // every later record of this CTA into L2 now: the copies then hit L2
            for (int i2 = it; i2 < wk.c1; i2++) {
              const int kc2 = wk.kc(i2), rg2 = i2 % g.n_rg, nr2 = nrec_of(kc2);
              const int nt2 = min(kTiles, g.n_vt - rg2 * kTiles);
              for (int t = 0; t < nt2; t++)
                bulk_prefetch_l2(W + ((size_t)(rg2 * kTiles + t) * g.nb + (size_t)kc2 * kChunkB) * kQ8Rec,
                                 (uint32_t)(nr2 * kQ8Rec));
            }
          }
          if (hf == 0 && wk.chunk_starts(it)) {
            if (chunk == 0) pdl_wait();  // the B operands come from the limb kernel
            if (chunk > 0) tc_wait(&sm.b_empty, (uint32_t)((chunk - 1) & 1), a.err);
            mbar_arrive_expect_tx(&sm.b_full, (uint32_t)(nrec * N * 64 + nrec * MT * 4));
            for (int j = 0; j < nrec; j++)
              bulk_g2s(sm.B16[j], Bg + ((size_t)kc * kChunkB + j) * N * 64, (uint32_t)(N * 64), &sm.b_full);
            bulk_g2s(sm.stS, sxg + (size_t)kc * kChunkB * MT, (uint32_t)(nrec * MT * 4), &sm.b_full);
            chunk++;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA lane ----
    if (lane == 0) {
      int blk = 0, chunk = 0;
      for (int it = wk.c0; it < wk.c1; it++) {
        const int kc = wk.kc(it), nrec = nrec_of(kc);
        if (wk.chunk_starts(it)) tc_wait(&sm.b_full, (uint32_t)(chunk++ & 1), a.err);
        for (int j = 0; j < nrec; j++, blk++) {
          const int r = blk % kWStages, s = blk & 1;
          tc_wait(&sm.w_full[r], (uint32_t)((blk / kWStages) & 1), a.err);
          if (blk >= 2) tc_wait(&sm.t_empty[s], (uint32_t)(((blk - 2) >> 1) & 1), a.err);
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(s * 256);
          tc_mma(d, umma_desc_sw64(sm.A16[r]), umma_desc_sw64(sm.B16[j]), idesc_f16(kRows, N), 0u);
          tc_mma(d, umma_desc_sw64(sm.A16[r] + 32), umma_desc_sw64(sm.B16[j] + 32), idesc_f16(kRows, N), 1u);
          tc_commit(&sm.t_full[s]);
          tc_commit(&sm.w_empty[r]);
          if (j == nrec - 1 && wk.chunk_ends(it)) tc_commit(&sm.b_empty);
        }
      }
    }
  } else if (warp < 2 + kWidenW) {
    // ---- widening: warp w widens tiles w - 2 and w + 2 of each block ----
    const int ww = warp - 2;
    const int gg = lane >> 2, cc = lane & 3;
    int blk = 0, ns = 0, chunk = 0;
    for (int it = wk.c0; it < wk.c1; it++) {
      const int kc = wk.kc(it), rg = it % g.n_rg, nrec = nrec_of(kc);
      if (wk.chunk_starts(it)) tc_wait(&sm.b_full, (uint32_t)(chunk++ & 1), a.err);  // stS
      for (int hf = 0; hf < 2; hf++) {
        const int nbh = half_blocks(nrec, hf);
        if (nbh <= 0) break;
        const int st = ns % kAStages;
        tc_wait(&sm.a_full[st], (uint32_t)((ns / kAStages) & 1), a.err);
        for (int jj = 0; jj < nbh; jj++, blk++) {
          const int j = hf * kHalfB + jj, r = blk % kWStages;
          // ring stage r was last used by block blk - 4 (its MMAs and its read-back)
          if (blk >= kWStages) tc_wait(&sm.w_empty[r], (uint32_t)(((blk - kWStages) / kWStages) & 1), a.err);
          uint8_t* A = sm.A16[r];
          for (int t = ww; t < kTiles; t += kWidenW) {
            const bool tile_ok = rg * kTiles + t < g.n_vt;
            const uint8_t* rec = sm.stA[st] + (t * kHalfB + jj) * kQ8Rec;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (tile_ok) v = lds128(rec + lane * 16);
            const int m0 = t * 16 + gg, m1 = m0 + 8;
            *reinterpret_cast<uint2*>(A + canon16_off(m0, 4 * cc)) = s8x4_to_f16x4(v.x);
            *reinterpret_cast<uint2*>(A + canon16_off(m1, 4 * cc)) = s8x4_to_f16x4(v.y);
            *reinterpret_cast<uint2*>(A + canon16_off(m0, 16 + 4 * cc)) = s8x4_to_f16x4(v.z);
            *reinterpret_cast<uint2*>(A + canon16_off(m1, 16 + 4 * cc)) = s8x4_to_f16x4(v.w);
            if (lane < 16)
              sm.dsb[r][t * 16 + lane] =
                  tile_ok ? __half2float(*reinterpret_cast<const __half*>(rec + q8_scale_off(lane))) : 0.f;
          }
          for (int i = ww * 32 + lane; i < MT; i += kWidenW * 32) sm.sxr[r][i] = sm.stS[j * MT + i];
          fence_async_smem();  // the A operand written by threads becomes visible to the tensor core
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.w_full[r]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.a_empty[st]);
        ns++;
      }
      if (lane == 0 && wk.chunk_ends(it)) mbar_arrive(&sm.b_empty);  // stS of this chunk is no longer read
    }
  } else {
    // ---- read-back ----
    const int e = warp - 2 - kWidenW, q = warp & 3, h = e >> 2;  // a warp reads TMEM lanes 32 (warp % 4)..
    const int row = q * 32 + lane;
    constexpr int TPT = MT / 4;   // tokens per thread
    constexpr int NPR = TPT / 2;  // token pairs per thread
    unsigned long long acc01[NPR], acc23[NPR];  // per token pair the packed {limbs 0/1} and {limbs 2/3}
#pragma unroll
    for (int i = 0; i < NPR; i++) acc01[i] = acc23[i] = 0ull;
    const unsigned long long k128 = pack2(128.f, 128.f);
    int blk = 0;
    for (int it = wk.c0; it < wk.c1; it++) {
      const int kc = wk.kc(it), rg = it % g.n_rg, nrec = nrec_of(kc);
      for (int j = 0; j < nrec; j++, blk++) {
        const int r = blk % kWStages, s = blk & 1;
        tc_wait(&sm.w_full[r], (uint32_t)((blk / kWStages) & 1), a.err);  // acquires dsb[r], sxr[r]
        tc_wait(&sm.t_full[s], (uint32_t)((blk >> 1) & 1), a.err);
        tc_fence_after();
        const unsigned long long ds2 = pack2(sm.dsb[r][row], sm.dsb[r][row]);
        constexpr int LDP = NPR >= 4 ? 4 : NPR;  // token pairs per batch of loads (two per load)
#pragma unroll
        for (int ld = 0; ld < NPR / LDP; ld++) {  // up to two loads of 16 columns in flight
          uint32_t v[8 * LDP];
          const uint32_t col = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(s * 256 + 4 * h * TPT + 8 * LDP * ld);
#pragma unroll
          for (int k = 0; k < LDP / 2; k++) tmem_ld16(col + 16 * k, *reinterpret_cast<uint32_t(*)[16]>(v + 16 * k));
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < LDP; i++) {
            const int p = LDP * ld + i;
            const float2 sx = *reinterpret_cast<const float2*>(&sm.sxr[r][h * TPT + 2 * p]);
            const unsigned long long dsx = mul2(ds2, pack2(sx.x, sx.y));
            // per token: S_l0 * 128 + S_l1 and S_l2 * 128 + S_l3, each rounded once as
            // (float)(int) rounds the GEMV's integer sums
            const uint32_t* w = v + 8 * i;
            const unsigned long long t01 = fma2(pack2u(w[0], w[1]), k128, pack2u(w[2], w[3]));
            const unsigned long long t23 = fma2(pack2u(w[4], w[5]), k128, pack2u(w[6], w[7]));
            acc01[p] = fma2(dsx, t01, acc01[p]);
            acc23[p] = fma2(dsx, t23, acc23[p]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sm.t_empty[s]);
          mbar_arrive(&sm.w_empty[r]);
        }
        if (j == nrec - 1) {
          const int vt = rg * kTiles + (row >> 4);
          if (vt < g.n_vt) {
            float* P = a.part + ((size_t)vt * g.nc + kc) * MT * 16 + (row & 15);
#pragma unroll
            for (int p = 0; p < NPR; p++) {
              const int t = h * TPT + 2 * p;
              float x0, x1, y0, y1;
              unpack2(acc01[p], x0, x1);
              unpack2(acc23[p], y0, y1);
              if (t < a.M) __stcg(P + t * 16, x0 * 0x1p-7f + y0 * 0x1p-21f);
              if (t + 1 < a.M) __stcg(P + (t + 1) * 16, x1 * 0x1p-7f + y1 * 0x1p-21f);
            }
          }
#pragma unroll
          for (int p = 0; p < NPR; p++) acc01[p] = acc23[p] = 0ull;
        }
      }
    }
  }
  // every role is done: the read-back waited for every MMA and read every accumulator.
  // Every thread also waits for the prerequisite grid, so this grid never completes before it.
  pdl_wait();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

template <int MT>
cudaError_t launch_tc_t(const GemvArgs& a, const TcGeo& g, int sms, uint8_t* scratch, cudaStream_t st) {
  constexpr int N = 4 * MT;
  uint8_t* Bg = scratch;
  float* sxg = reinterpret_cast<float*>(scratch + (size_t)g.nb * N * 64);
  const size_t row_bytes = (size_t)g.K * 4;
  cudaError_t e = cudaSuccess;
  if (row_bytes > 48 * 1024) {
    e = cudaFuncSetAttribute(k_tc_limbs<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)row_bytes);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchAttribute attr0[1];
  cudaLaunchConfig_t cfg0 = launch_cfg(dim3(MT), dim3(kTT), row_bytes, st, attr0);
  e = cudaLaunchKernelEx(&cfg0, k_tc_limbs<MT>, a, g, Bg, sxg);
  if (e != cudaSuccess) return e;
  auto kern = k_gemm_tc<MT>;
  const size_t smem = sizeof(TcSmem<MT>) + 1024;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long I = (long long)g.n_rg * g.nc;
  const int grid = (int)std::max(1LL, std::min<long long>(I, sms));
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = launch_cfg(dim3(grid), dim3(kGT), smem, st, attr);
  return cudaLaunchKernelEx(&cfg, kern, a, g, (const uint8_t*)Bg, (const float*)sxg);
}

}  // namespace

// read per launch, so a process can compare both paths (SYRINX_TC=0: the mma.sync GEMV)
bool tc_enabled() {
  const char* v = getenv("SYRINX_TC");
  return !(v && v[0] == '0');
}

// The partials of a Q8_0 GEMV of 9..64 tokens (Mt = 16, 32 or 64) on the tensor cores.
size_t gemm_tc_scratch_bytes(int K, int Mt) { return (size_t)(K / 32) * (4 * Mt * 64 + Mt * 4); }

cudaError_t launch_gemm_tc(const GemvArgs& a, int Mt, int K, int nb, int nc, int t_first, int n_vt, int sms,
                           cudaStream_t st) {
  if (t_first != 0 || a.n_extra != 0 || K % 32 || !a.tc_scratch || gemm_tc_scratch_bytes(K, Mt) > a.tc_scratch_bytes)
    return cudaErrorInvalidValue;
  TcGeo g;
  g.K = K;
  g.nb = nb;
  g.nc = nc;
  g.n_vt = n_vt;
  g.n_rg = (n_vt + kTiles - 1) / kTiles;
  switch (Mt) {
    case 16: return launch_tc_t<16>(a, g, sms, a.tc_scratch, st);
    case 32: return launch_tc_t<32>(a, g, sms, a.tc_scratch, st);
    case 64: return launch_tc_t<64>(a, g, sms, a.tc_scratch, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace sx
