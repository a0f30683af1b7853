// codec.cu — the s2 causal-DAC codec decode on the device: `[num_codebooks, T]` codes to a
// 44.1 kHz waveform (`EvaGanDac::decode`, crates/syrinx-fish/src/s2/codec.rs:342-379).
//
// Every activation is held channels-first, `[C][L]` row-major, so that one kernel serves
// every matrix product of the path: a linear layer over channels-first data is a k=1
// convolution. `k_conv_gemm` computes Y[M][N] = W[M][R] * im2col(X)[R][N] with the im2col
// formed while the B tile is loaded (column n, tap kk of input channel ci reads
// x[ci][n - (K-1-kk)*dil], zero before the start: the causal left pad). Transposed
// convolutions run as the same product over their stride phases: output sample q*s + p
// is a K/s-tap causal convolution of the input with the kernel taps p, p+s, ..., so the
// weights are repacked once at load into [s*Cout][Cin*K/s] and the epilogue scatters row
// p*Cout + co to y[co][q*s + p]. The transpose's right trim (codec.rs:117-137) is then
// implicit: only q < L is computed.
//
// The arithmetic is f32 throughout (the reference's CPU path is f32); the products run on
// the FP32 pipes, 8x8 register tiles per thread.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "blob.hpp"
#include "codec.hpp"

namespace sx {
namespace codec {

// ---- the convolution / linear product --------------------------------------------------

struct ConvGemm {
  const float* w;      // [M][R] row-major, R = cin * k (tap fastest)
  const float* x;      // [cin][N] input rows
  float* y;            // output
  const float* bias;   // [cout] or null
  const float* scale;  // [cout] or null (layer scale, applied after the bias)
  const float* resid;  // [M][N] added last (plain store only) or null
  int M, R, N;         // rows, reduction, columns (= input length)
  int k, dil;          // taps and dilation
  int phase;           // 1: y[m][n]; s > 1: row m = p*cout + co stores y[co][n*s + p]
  int cout;            // output channels (M / phase)
  int act;             // 0 none, 1 tanh, 2 GELU (erf form)
};

constexpr int kBM = 128, kBN = 128, kBK = 8;

__device__ __forceinline__ float gelu_erf(float v) {
  return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
}

// 256 threads, a 128 x 128 output tile per block, 8 x 8 outputs per thread in two 4-wide
// halves of rows and of columns (so that the shared-memory reads are float4 and the two
// row halves of a warp hit distinct banks). Global loads for k-tile t+1 are issued before
// the products of tile t and land in the other shared-memory buffer afterwards.
__global__ void __launch_bounds__(256, 2) k_conv_gemm(const ConvGemm p) {
  __shared__ __align__(16) float As[2][kBK][kBM];
  __shared__ __align__(16) float Bs[2][kBK][kBN];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
  const int am = tid >> 1, ak = (tid & 1) * 4;  // A loader: one row, four reduction steps
  const int bk = tid >> 5, bn = tid & 31;       // B loader: one reduction row, four columns
  const bool avec = (p.R & 3) == 0;
  const float* wrow = p.w + (size_t)(m0 + am) * p.R;
  const bool arow_ok = m0 + am < p.M;

  float ra[4], rb[4];
  auto load_tiles = [&](int kt) {
    const int r0 = kt * kBK + ak;
    if (arow_ok && avec && r0 + 3 < p.R) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(wrow + r0));
      ra[0] = v.x, ra[1] = v.y, ra[2] = v.z, ra[3] = v.w;
    } else {
#pragma unroll
      for (int i = 0; i < 4; i++) ra[i] = (arow_ok && r0 + i < p.R) ? __ldg(wrow + r0 + i) : 0.f;
    }
    const int r = kt * kBK + bk;
    if (r < p.R) {
      const int ci = r / p.k, tap = r - ci * p.k;
      const int shift = (p.k - 1 - tap) * p.dil;
      const float* xr = p.x + (size_t)ci * p.N;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int n = n0 + bn + 32 * j, src = n - shift;
        rb[j] = (n < p.N && src >= 0) ? __ldg(xr + src) : 0.f;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; j++) rb[j] = 0.f;
    }
  };
  auto store_tiles = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; i++) As[buf][ak + i][am] = ra[i];
#pragma unroll
    for (int j = 0; j < 4; j++) Bs[buf][bk][bn + 32 * j] = rb[j];
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

  const int tx = tid & 15, ty = tid >> 4;
  const int nkt = (p.R + kBK - 1) / kBK;
  load_tiles(0);
  store_tiles(0);
  __syncthreads();
  for (int kt = 0; kt < nkt; kt++) {
    const int cur = kt & 1;
    if (kt + 1 < nkt) load_tiles(kt + 1);
#pragma unroll
    for (int kk = 0; kk < kBK; kk++) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][kk][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (kt + 1 < nkt) {
      store_tiles(cur ^ 1);
      __syncthreads();
    }
  }

#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (m >= p.M) continue;
    const int co = p.phase > 1 ? m % p.cout : m;
    const int ph = p.phase > 1 ? m / p.cout : 0;
    const float b = p.bias ? p.bias[co] : 0.f;
    const float sc = p.scale ? p.scale[co] : 1.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (n >= p.N) continue;
      float v = acc[i][j] + b;
      if (p.scale) v *= sc;
      if (p.act == 1) v = tanhf(v);
      else if (p.act == 2) v = gelu_erf(v);
      if (p.phase > 1) {
        p.y[(size_t)co * p.N * p.phase + (size_t)n * p.phase + ph] = v;
      } else {
        const size_t o = (size_t)m * p.N + n;
        if (p.resid) v += p.resid[o];
        p.y[o] = v;
      }
    }
  }
}

// ---- element-wise and per-column kernels -----------------------------------------------

// RVQ from_codes (codec.rs:259-276, summed at 356-367): per codebook, gather the codebook
// row of the (clamped) code, project it by out_proj (a k=1 conv, cbdim -> latent) plus its
// bias, and add the codebooks' latents in codebook order.
__global__ void k_rvq_embed(const uint32_t* __restrict__ codes, int ncb, int T,
                            const CbTab* __restrict__ tabs, int latent, float* __restrict__ z) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int co = blockIdx.y;
  if (t >= T) return;
  float acc = 0.f;
  for (int i = 0; i < ncb; i++) {
    const CbTab tb = tabs[i];
    uint32_t c = codes[(size_t)i * T + t];
    if (c > (uint32_t)(tb.size - 1)) c = (uint32_t)(tb.size - 1);
    const float* e = tb.cb + (size_t)c * tb.dim;
    const float* wr = tb.w + (size_t)co * tb.dim;
    float v = 0.f;
    for (int j = 0; j < tb.dim; j++) v = fmaf(wr[j], e[j], v);
    v += tb.b[co];
    acc = (i == 0) ? v : acc + v;
  }
  z[(size_t)co * T + t] = acc;
}

// Snake1d (codec.rs:139-149): x + (alpha + 1e-9)^-1 * sin(alpha x)^2, alpha per channel.
__global__ void k_snake(const float* __restrict__ x, const float* __restrict__ alpha,
                        float* __restrict__ y, int C, int L) {
  const int c = blockIdx.y;
  const float a = alpha[c];
  const float inv = 1.0f / (a + 1e-9f);
  const size_t base = (size_t)c * L;
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < L; t += gridDim.x * blockDim.x) {
    const float v = x[base + t];
    const float s = sinf(v * a);
    y[base + t] = v + (s * s) * inv;
  }
}

// Per-column normalisation over the channel axis of a [C][L] tensor: RMSNorm
// (s2/nn.rs:100-106, weight only) when `b` is null, else LayerNorm with bias
// (codec.rs:647-655). 32 columns per block, 8 channel groups reduced through shared memory.
__global__ void __launch_bounds__(256) k_chan_norm(const float* __restrict__ x,
                                                   const float* __restrict__ w,
                                                   const float* __restrict__ b,
                                                   float* __restrict__ y, int C, int L,
                                                   float eps) {
  __shared__ float red[8][33];
  const int lx = threadIdx.x & 31, ly = threadIdx.x >> 5;
  const int t = blockIdx.x * 32 + lx;
  const bool ok = t < L;
  float mean = 0.f;
  if (b) {
    float s = 0.f;
    if (ok)
      for (int c = ly; c < C; c += 8) s += x[(size_t)c * L + t];
    red[ly][lx] = s;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) tot += red[i][lx];
    mean = tot / (float)C;
    __syncthreads();
  }
  float s2 = 0.f;
  if (ok)
    for (int c = ly; c < C; c += 8) {
      const float d = x[(size_t)c * L + t] - mean;
      s2 = fmaf(d, d, s2);
    }
  red[ly][lx] = s2;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; i++) tot += red[i][lx];
  const float den = sqrtf(tot / (float)C + eps);
  if (!ok) return;
  for (int c = ly; c < C; c += 8) {
    const size_t o = (size_t)c * L + t;
    const float v = (x[o] - mean) / den * w[c];
    y[o] = b ? v + b[c] : v;
  }
}

// Interleaved RoPE (s2/nn.rs:154-166) on the q and k rows of a channels-first qkv
// [3*dim][T]: the pair (2i, 2i+1) of each 64-wide head at position t turns by t*inv_freq[i].
__global__ void k_rope_cf(float* __restrict__ qkv, int dim, int T, const float* __restrict__ inv_freq,
                          int half) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int pr = blockIdx.y;  // pair index over q and k: 2 * dim / 2 pairs
  if (t >= T) return;
  const int i = pr % half;
  const int row = 2 * pr;  // q rows [0, dim), k rows [dim, 2 dim) are contiguous
  float sn, cs;
  sincosf((float)t * inv_freq[i], &sn, &cs);
  float* r0 = qkv + (size_t)row * T + t;
  float* r1 = r0 + T;
  const float x0 = *r0, x1 = *r1;
  *r0 = x0 * cs - x1 * sn;
  *r1 = x1 * cs + x0 * sn;
}

// Full-causal attention of the codec transformer (codec.rs:576-604 through
// s2/nn.rs:284-373, scale 1/sqrt(64)) on channels-first qkv; ctx is [dim][T]. One block
// per (head, 32 queries); each warp owns 4 queries, a lane owns one key of the 32-key tile
// for the scores and two of the 64 dims for the output; online softmax over key tiles.
constexpr int kHd = 64, kQt = 32;
__global__ void __launch_bounds__(256) k_attn_causal_cf(const float* __restrict__ qkv,
                                                        float* __restrict__ ctx, int dim, int T) {
  __shared__ float Qs[kHd][kQt + 1];
  __shared__ float Ks[kHd][kQt + 1];
  __shared__ float Vs[kQt][kHd + 1];
  const int h = blockIdx.y, q0 = blockIdx.x * kQt;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* Q = qkv + (size_t)(h * kHd) * T;
  const float* K = qkv + (size_t)(dim + h * kHd) * T;
  const float* V = qkv + (size_t)(2 * dim + h * kHd) * T;
  for (int e = threadIdx.x; e < kHd * kQt; e += 256) {
    const int d = e / kQt, q = e % kQt;
    Qs[d][q] = (q0 + q < T) ? Q[(size_t)d * T + q0 + q] : 0.f;
  }
  float m[4], l[4], o0[4], o1[4];
#pragma unroll
  for (int i = 0; i < 4; i++) m[i] = -INFINITY, l[i] = 0.f, o0[i] = 0.f, o1[i] = 0.f;
  const int kend = min(T, q0 + kQt);
  for (int j0 = 0; j0 < kend; j0 += kQt) {
    __syncthreads();
    for (int e = threadIdx.x; e < kHd * kQt; e += 256) {
      const int d = e / kQt, k = e % kQt;
      const bool ok = j0 + k < T;
      Ks[d][k] = ok ? K[(size_t)d * T + j0 + k] : 0.f;
      Vs[k][d] = ok ? V[(size_t)d * T + j0 + k] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int ql = warp * 4 + i, q = q0 + ql;
      const int key = j0 + lane;
      float s = 0.f;
#pragma unroll 16
      for (int d = 0; d < kHd; d++) s = fmaf(Qs[d][ql], Ks[d][lane], s);
      s *= 0.125f;
      const bool valid = key <= q && key < T;
      if (!valid) s = -INFINITY;
      float mt = s;
#pragma unroll
      for (int off = 16; off; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float mn = fmaxf(m[i], mt);
      if (mn == -INFINITY) continue;  // no visible key yet (only for queries past T)
      const float corr = expf(m[i] - mn);
      const float pk = valid ? expf(s - mn) : 0.f;
      float ps = pk;
#pragma unroll
      for (int off = 16; off; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l[i] = l[i] * corr + ps;
      float a0 = o0[i] * corr, a1 = o1[i] * corr;
#pragma unroll 8
      for (int k = 0; k < kQt; k++) {
        const float pj = __shfl_sync(0xffffffffu, pk, k);
        a0 = fmaf(pj, Vs[k][lane], a0);
        a1 = fmaf(pj, Vs[k][lane + 32], a1);
      }
      o0[i] = a0, o1[i] = a1;
      m[i] = mn;
    }
  }
  __syncthreads();
  // stage the 32 x 64 output through shared memory so the channels-first rows store whole
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int ql = warp * 4 + i;
    const float inv = l[i] > 0.f ? 1.0f / l[i] : 0.f;
    Qs[lane][ql] = o0[i] * inv;
    Qs[lane + 32][ql] = o1[i] * inv;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < kHd * kQt; e += 256) {
    const int d = e / kQt, q = e % kQt;
    if (q0 + q < T) ctx[(size_t)(h * kHd + d) * T + q0 + q] = Qs[d][q];
  }
}

// SwiGLU (s2/nn.rs:452-457): out[f][t] = silu(h[f][t]) * h[F + f][t] for the stacked w1|w3.
__global__ void k_swiglu_cf(const float* __restrict__ h, float* __restrict__ out, int F, int T) {
  const size_t n = (size_t)F * T;
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (size_t)gridDim.x * blockDim.x) {
    const float g = h[e];
    out[e] = (g / (1.0f + expf(-g))) * h[n + e];
  }
}

// Causal depthwise convolution, k=7 (the ConvNeXt dwconv, codec.rs:189-199).
__global__ void k_dwconv_causal(const float* __restrict__ x, const float* __restrict__ w,
                                const float* __restrict__ b, float* __restrict__ y, int L, int K) {
  const int c = blockIdx.y;
  const float* xr = x + (size_t)c * L;
  const float* wr = w + (size_t)c * K;
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < L; t += gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int k = 0; k < K; k++) {
      const int src = t - (K - 1 - k);
      if (src >= 0) v = fmaf(wr[k], xr[src], v);
    }
    y[(size_t)c * L + t] = v + b[c];
  }
}

// ConvNeXt-V2 GRN (codec.rs:237-257), step 1: gx[c] = ||x[c][:]||_2 over the time axis.
__global__ void __launch_bounds__(256) k_grn_norm(const float* __restrict__ x, float* __restrict__ gx,
                                                  int L) {
  __shared__ float red[8];
  const int c = blockIdx.x;
  float s = 0.f;
  for (int t = threadIdx.x; t < L; t += 256) {
    const float v = x[(size_t)c * L + t];
    s = fmaf(v, v, s);
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int i = 0; i < 8; i++) tot += red[i];
    gx[c] = sqrtf(tot);
  }
}

// Step 2: nx[c] = gx[c] / (mean_c gx + 1e-6) (one block).
__global__ void __launch_bounds__(1024) k_grn_scale(float* __restrict__ gx, int C) {
  __shared__ float red[32];
  float s = 0.f;
  for (int c = threadIdx.x; c < C; c += blockDim.x) s += gx[c];
#pragma unroll
  for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float den = red[0] / (float)C + 1e-6f;
  for (int c = threadIdx.x; c < C; c += blockDim.x) gx[c] = gx[c] / den;
}

// Step 3: x += x * nx[c] * gamma[c] + beta[c].
__global__ void k_grn_apply(float* __restrict__ x, const float* __restrict__ nx,
                            const float* __restrict__ gamma, const float* __restrict__ beta, int L) {
  const int c = blockIdx.y;
  const float g = nx[c], ga = gamma[c], be = beta[c];
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < L; t += gridDim.x * blockDim.x) {
    const size_t o = (size_t)c * L + t;
    const float v = x[o];
    x[o] = v + ((v * g) * ga + be);
  }
}

// The final conv to one channel (k=7, causal) and tanh (codec.rs:326-339): a thread makes
// 8 consecutive samples from a 14-sample window of each input channel.
constexpr int kOutV = 8, kOutK = 7;
__global__ void __launch_bounds__(256) k_conv_out1(const float* __restrict__ x, const float* __restrict__ w,
                                                   const float* __restrict__ b, float* __restrict__ y,
                                                   int C, int L) {
  extern __shared__ float ws[];
  for (int e = threadIdx.x; e < C * kOutK; e += blockDim.x) ws[e] = w[e];
  __syncthreads();
  const int t0 = (blockIdx.x * blockDim.x + threadIdx.x) * kOutV;
  if (t0 >= L) return;
  float acc[kOutV];
#pragma unroll
  for (int v = 0; v < kOutV; v++) acc[v] = 0.f;
  for (int c = 0; c < C; c++) {
    const float* xr = x + (size_t)c * L;
    float win[kOutV + kOutK - 1];  // win[j] = x[t0 - (K-1) + j]
#pragma unroll
    for (int j = 0; j < kOutV + kOutK - 1; j++) {
      const int src = t0 - (kOutK - 1) + j;
      win[j] = (src >= 0 && src < L) ? __ldg(xr + src) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < kOutK; k++) {
      const float wk = ws[c * kOutK + k];
#pragma unroll
      for (int v = 0; v < kOutV; v++) acc[v] = fmaf(wk, win[k + v], acc[v]);
    }
  }
#pragma unroll
  for (int v = 0; v < kOutV; v++)
    if (t0 + v < L) y[t0 + v] = tanhf(acc[v] + b[0]);
}

}  // namespace codec
}  // namespace sx

// ---- host side: blob loading, weight repacking, the decode sequence -------------------

namespace sx {
namespace codec {
namespace {

constexpr int kHeadDim = 64;          // codec transformer head width (codec.rs:58-60)
constexpr float kRopeBase = 10000.f;  // codec.rs:61-63
constexpr float kNormEps = 1e-5f;     // codec.rs:64-65
constexpr float kLnEps = 1e-6f;       // ConvNeXt LayerNorm (codec.rs:205-210)

// Gathers the codec tensors into one host staging image (each tensor 64-byte aligned) and
// records where each device pointer will point once the image is uploaded.
struct Loader {
  const BlobIndex& ix;
  std::string* err;
  std::vector<float> image;
  std::vector<std::pair<float**, size_t>> fix;
  bool ok = true;

  Loader(const BlobIndex& i, std::string* e) : ix(i), err(e) {}
  void fail(const std::string& m) {
    if (ok) *err = "codec blob: " + m;
    ok = false;
  }
  const BlobTensor* find(const std::string& n) const {
    auto it = ix.t.find(n);
    return it == ix.t.end() ? nullptr : &it->second;
  }
  bool has(const std::string& n) const { return find(n) != nullptr; }
  // The tensor `n` as f32 with `elems` elements (any rank), or null after fail().
  const BlobTensor* need(const std::string& n, int64_t elems) {
    const BlobTensor* t = find(n);
    if (!t) {
      fail("missing tensor " + n);
      return nullptr;
    }
    if (t->dtype != SX_DTYPE_F32) {
      fail(n + " must be f32");
      return nullptr;
    }
    if (elems >= 0 && t->rows * t->cols != elems) {
      fail(n + " has " + std::to_string(t->rows * t->cols) + " elements, expected " +
           std::to_string(elems));
      return nullptr;
    }
    return t;
  }
  // A rank-3 convolution kernel; returns its shape through d.
  const BlobTensor* need3(const std::string& n, int64_t d[3]) {
    const BlobTensor* t = need(n, -1);
    if (!t) return nullptr;
    if (t->ndim != 3) {
      fail(n + " must be rank 3");
      return nullptr;
    }
    for (int i = 0; i < 3; i++) d[i] = t->shape[i];
    return t;
  }
  size_t reserve_floats(size_t n) {
    const size_t off = image.size();
    image.resize(off + ((n + 15) & ~size_t(15)), 0.f);
    return off;
  }
  size_t copy(float** dst, const BlobTensor* t) {
    if (!t) return 0;
    const size_t n = (size_t)(t->rows * t->cols);
    const size_t off = reserve_floats(n);
    std::memcpy(&image[off], t->data, n * sizeof(float));
    fix.push_back({dst, off});
    return off;
  }
  // The tensor-core weight images of the packed matrix at image offset `off` (codec_tc.cu).
  void tc_pack(Conv* c, size_t off) {
    const int M = c->cout * c->stride, R = c->cin * c->taps;
    std::vector<float> a(image.begin() + off, image.begin() + off + (size_t)M * R);
    const size_t bytes = tc_image_bytes(M, R);
    const size_t o = reserve_floats(bytes / sizeof(float));
    tc_image(a.data(), M, R, reinterpret_cast<uint32_t*>(&image[o]));
    fix.push_back({&c->tc, o});
  }
  void vec(float** dst, const std::string& n, int64_t elems) { copy(dst, need(n, elems)); }
  // Stacks two [rows][cols] matrices into one [2 rows][cols].
  // Two [rows][cols] linear weights stacked into one [2 rows][cols] k=1 product.
  void stack2(Conv* c, const BlobTensor* a, const BlobTensor* b) {
    if (!a || !b) return;
    const size_t n = (size_t)(a->rows * a->cols);
    const size_t off = reserve_floats(2 * n);
    std::memcpy(&image[off], a->data, n * sizeof(float));
    std::memcpy(&image[off + n], b->data, n * sizeof(float));
    fix.push_back({&c->w, off});
    c->cout = (int)(2 * a->rows), c->cin = (int)a->cols, c->taps = 1, c->stride = 1, c->dil = 1;
    tc_pack(c, off);
  }
  // A causal convolution [cout][cin][k] (codec.rs:93-115): used as is.
  void conv(Conv* c, const std::string& w, const std::string& b, int64_t cin, int dil,
            int64_t k_expect = -1) {
    int64_t d[3];
    const BlobTensor* t = need3(w, d);
    if (!t) return;
    if ((cin >= 0 && d[1] != cin) || (k_expect >= 0 && d[2] != k_expect)) {
      fail(w + " has an unexpected shape");
      return;
    }
    c->cout = (int)d[0], c->cin = (int)d[1], c->taps = (int)d[2], c->stride = 1, c->dil = dil;
    tc_pack(c, copy(&c->w, t));
    vec(&c->b, b, d[0]);
  }
  // A linear layer [out][in] as a k=1 convolution; no bias when `b` is empty. `out` >= 0
  // requires that many rows.
  void linear(Conv* c, const std::string& w, const std::string& b, int64_t in, int64_t out = -1) {
    const BlobTensor* t = need(w, -1);
    if (!t) return;
    if (t->cols != in || (out >= 0 && t->rows != out) || (t->ndim == 3 && t->shape[2] != 1)) {
      fail(w + " has an unexpected shape");
      return;
    }
    c->cout = (int)t->rows, c->cin = (int)t->cols, c->taps = 1, c->stride = 1, c->dil = 1;
    tc_pack(c, copy(&c->w, t));
    if (!b.empty()) vec(&c->b, b, t->rows);
  }
  // A transposed convolution [cin][cout][kt] of stride s = kt / per (codec.rs:117-137),
  // repacked into its s stride phases of kt / s taps each.
  void tconv(Conv* c, const std::string& w, const std::string& b, int64_t cin, int per) {
    int64_t d[3];
    const BlobTensor* t = need3(w, d);
    if (!t) return;
    if (d[0] != cin || d[2] % per != 0 || d[2] / per < 1) {
      fail(w + " has an unexpected shape");
      return;
    }
    const int Ci = (int)d[0], Co = (int)d[1], Kt = (int)d[2], s = Kt / per, taps = per;
    c->cout = Co, c->cin = Ci, c->taps = taps, c->stride = s, c->dil = 1;
    std::vector<float> src((size_t)Ci * Co * Kt);
    std::memcpy(src.data(), t->data, src.size() * sizeof(float));
    const size_t off = reserve_floats(src.size());
    for (int p = 0; p < s; p++)
      for (int co = 0; co < Co; co++)
        for (int ci = 0; ci < Ci; ci++)
          for (int j = 0; j < taps; j++) {
            const int kk = p + (taps - 1 - j) * s;
            image[off + ((size_t)(p * Co + co) * Ci + ci) * taps + j] =
                src[((size_t)ci * Co + co) * Kt + kk];
          }
    fix.push_back({&c->w, off});
    tc_pack(c, off);
    vec(&c->b, b, Co);
  }
};

// One product on the tensor cores (weight images present, SYRINX_CODEC_TC not 0) or on
// the FP32 CUDA cores.
cudaError_t conv_launch(const Codec& cd, const Conv& c, const float* x, int L, float* y, const float* scale,
                        const float* resid, int act) {
  if (cd.use_tc && c.tc) {
    TcConvArgs t;
    t.a_img = reinterpret_cast<const uint8_t*>(c.tc);
    t.x = x, t.y = y, t.bias = c.b, t.scale = scale, t.resid = resid;
    t.M = c.cout * c.stride, t.R = c.cin * c.taps, t.N = L;
    t.k = c.taps, t.dil = c.dil, t.phase = c.stride, t.cout = c.cout, t.act = act;
    t.err = cd.err;
    return launch_conv_tc(t, cd.sms, cd.stream);
  }
  ConvGemm p;
  p.w = c.w, p.x = x, p.y = y, p.bias = c.b, p.scale = scale, p.resid = resid;
  p.M = c.cout * c.stride, p.R = c.cin * c.taps, p.N = L;
  p.k = c.taps, p.dil = c.dil, p.phase = c.stride, p.cout = c.cout, p.act = act;
  const dim3 grid((L + kBN - 1) / kBN, (p.M + kBM - 1) / kBM);
  k_conv_gemm<<<grid, 256, 0, cd.stream>>>(p);
  return cudaSuccess;
}

inline unsigned cols_grid(int L, int per_block) {
  return (unsigned)std::max(1, std::min((L + per_block - 1) / per_block, 1024));
}

}  // namespace

Codec::~Codec() {
  if (device >= 0) cudaSetDevice(device);
  cudaFree(weights);
  for (float*& b : buf) cudaFree(b);
  cudaFree(grn);
  cudaFree(codes_dev);
  cudaFree(wav_dev);
  cudaFree(err);
}

int Codec::load(const void* blob, size_t size, int dev, std::string* err) {
  device = dev;
  BlobIndex ix;
  int rc = parse_blob(blob, size, &ix, err);
  if (rc) return rc;
  Loader ld(ix, err);

  // Tensor names: the s2 codec nests the RVQ, its upsample and its post_module under
  // `quantizer.` (s2/codec.rs:348-372); the s1 modded DAC has them at the top level and no
  // post_module transformer (s1/codec.rs:255-290).
  const std::string qp = ld.has("quantizer.semantic_quantizer.quantizers.0.codebook.weight") ? "quantizer." : "";
  // RVQ tables (codec.rs:259-276, 342-367)
  const std::string sem = qp + "semantic_quantizer.quantizers.0";
  const BlobTensor* cb0 = ld.need(sem + ".codebook.weight", -1);
  if (!cb0) return SX_E_BLOB;
  sem_size = (int)cb0->rows, cb_dim = (int)cb0->cols;
  {
    int64_t d[3];
    const BlobTensor* op = ld.need3(sem + ".out_proj.weight", d);
    if (!op) return SX_E_BLOB;
    if (d[1] != cb_dim || d[2] != 1) {
      *err = "codec blob: " + sem + ".out_proj.weight has an unexpected shape";
      return SX_E_BLOB;
    }
    latent = (int)d[0];
  }
  while (ld.has(qp + "quantizer.quantizers." + std::to_string(n_res) + ".codebook.weight")) n_res++;
  std::vector<float*> cb(1 + n_res), pw(1 + n_res), pb(1 + n_res);
  std::vector<int> sizes(1 + n_res);
  for (int i = 0; i <= n_res; i++) {
    const std::string pre = i == 0 ? sem : qp + "quantizer.quantizers." + std::to_string(i - 1);
    const BlobTensor* c = ld.need(pre + ".codebook.weight", -1);
    if (!c) return SX_E_BLOB;
    if (c->cols != cb_dim) {
      *err = "codec blob: " + pre + ".codebook.weight has an unexpected width";
      return SX_E_BLOB;
    }
    sizes[i] = (int)c->rows;
    if (i == 1) res_size = (int)c->rows;
    ld.copy(&cb[i], c);
    ld.vec(&pw[i], pre + ".out_proj.weight", (int64_t)latent * cb_dim);
    ld.vec(&pb[i], pre + ".out_proj.bias", latent);
  }
  if (!ld.ok) return SX_E_BLOB;

  // post_module transformer (codec.rs:559-626); the layer count is read from the blob
  const std::string tp = qp + "post_module";
  while (ld.has(tp + ".layers." + std::to_string(n_layers) + ".attention_norm.weight")) n_layers++;
  if (n_layers) {
    if (latent % kHeadDim) {
      *err = "codec blob: transformer width is not a multiple of 64";
      return SX_E_BLOB;
    }
    n_head = latent / kHeadDim;
    const BlobTensor* w1 = ld.need(tp + ".layers.0.feed_forward.w1.weight", -1);
    if (!w1) return SX_E_BLOB;
    ffn = (int)w1->rows;
    layers.resize(n_layers);
    const int64_t D = latent, F = ffn;
    for (int l = 0; l < n_layers; l++) {
      const std::string p = tp + ".layers." + std::to_string(l);
      Layer& y = layers[l];
      ld.vec(&y.attn_norm, p + ".attention_norm.weight", D);
      ld.linear(&y.wqkv, p + ".attention.wqkv.weight", "", D, 3 * D);
      ld.linear(&y.wo, p + ".attention.wo.weight", "", D, D);
      ld.vec(&y.attn_gamma, p + ".attention_layer_scale.gamma", D);
      ld.vec(&y.ffn_norm, p + ".ffn_norm.weight", D);
      ld.stack2(&y.w13, ld.need(p + ".feed_forward.w1.weight", F * D),
                ld.need(p + ".feed_forward.w3.weight", F * D));
      ld.linear(&y.w2, p + ".feed_forward.w2.weight", "", F, D);
      ld.vec(&y.ffn_gamma, p + ".ffn_layer_scale.gamma", D);
    }
    ld.vec(&post_norm, tp + ".norm.weight", D);
    std::vector<float> inv(kHeadDim / 2);
    for (int i = 0; i < kHeadDim / 2; i++)  // s2/nn.rs:124-126, in f32
      inv[i] = 1.0f / powf(kRopeBase, 2.0f * (float)i / (float)kHeadDim);
    const size_t off = ld.reserve_floats(inv.size());
    std::memcpy(&ld.image[off], inv.data(), inv.size() * sizeof(float));
    ld.fix.push_back({&inv_freq, off});
  }
  if (!ld.ok) return SX_E_BLOB;

  // ConvNeXt upsample (codec.rs:278-300): kernel = stride = factor per stage
  int n_up = 0;
  while (ld.has(qp + "upsample." + std::to_string(n_up) + ".0.conv.weight")) n_up++;
  ups.resize(n_up);
  int64_t C = latent;
  for (int s = 0; s < n_up; s++) {
    const std::string p = qp + "upsample." + std::to_string(s);
    UpStage& u = ups[s];
    ld.tconv(&u.up, p + ".0.conv.weight", p + ".0.conv.bias", C, 1);
    if (!ld.ok) return SX_E_BLOB;
    C = u.up.cout;
    u.c = (int)C;
    const std::string b = p + ".1";
    ld.vec(&u.dw_w, b + ".dwconv.conv.weight", C * 7);
    ld.vec(&u.dw_b, b + ".dwconv.conv.bias", C);
    ld.vec(&u.ln_w, b + ".norm.weight", C);
    ld.vec(&u.ln_b, b + ".norm.bias", C);
    ld.linear(&u.pw1, b + ".pwconv1.weight", b + ".pwconv1.bias", C);
    if (!ld.ok) return SX_E_BLOB;
    if (ld.has(b + ".grn.gamma")) {
      ld.vec(&u.grn_g, b + ".grn.gamma", u.pw1.cout);
      ld.vec(&u.grn_b, b + ".grn.beta", u.pw1.cout);
    }
    ld.linear(&u.pw2, b + ".pwconv2.weight", b + ".pwconv2.bias", u.pw1.cout);
    if (ld.ok && u.pw2.cout != C) ld.fail(b + ".pwconv2.weight has an unexpected shape");
    if (ld.has(b + ".gamma")) ld.vec(&u.gamma, b + ".gamma", C);
    hop *= u.up.stride;
  }
  if (!ld.ok) return SX_E_BLOB;

  // DAC decoder (codec.rs:302-340)
  ld.conv(&conv0, "decoder.model.0.conv.weight", "decoder.model.0.conv.bias", C, 1, 7);
  if (!ld.ok) return SX_E_BLOB;
  C = conv0.cout;
  int n_blk = 0;
  while (ld.has("decoder.model." + std::to_string(n_blk + 1) + ".block.1.conv.weight")) n_blk++;
  blocks.resize(n_blk);
  static const int kDil[3] = {1, 3, 9};
  for (int i = 0; i < n_blk; i++) {
    const std::string p = "decoder.model." + std::to_string(i + 1);
    DecBlock& bk = blocks[i];
    ld.vec(&bk.alpha, p + ".block.0.alpha", C);
    ld.tconv(&bk.up, p + ".block.1.conv.weight", p + ".block.1.conv.bias", C, 2);
    if (!ld.ok) return SX_E_BLOB;
    C = bk.up.cout;
    for (int r = 0; r < 3; r++) {
      const std::string q = p + ".block." + std::to_string(r + 2) + ".block";
      ResUnit& u = bk.ru[r];
      ld.vec(&u.a0, q + ".0.alpha", C);
      ld.conv(&u.c1, q + ".1.conv.weight", q + ".1.conv.bias", C, kDil[r], 7);
      ld.vec(&u.a2, q + ".2.alpha", C);
      ld.conv(&u.c3, q + ".3.conv.weight", q + ".3.conv.bias", C, 1, 1);
      if (ld.ok && (u.c1.cout != C || u.c3.cout != C)) ld.fail(q + " convolutions change the width");
    }
    hop *= bk.up.stride;
  }
  const std::string fa = "decoder.model." + std::to_string(n_blk + 1) + ".alpha";
  const std::string fc = "decoder.model." + std::to_string(n_blk + 2) + ".conv";
  ld.vec(&final_alpha, fa, C);
  ld.vec(&final_w, fc + ".weight", C * 7);
  ld.vec(&final_b, fc + ".bias", 1);
  final_cin = (int)C;
  if (!ld.ok) return SX_E_BLOB;

  // upload the image and the quantizer table array
  if (cudaSetDevice(device) != cudaSuccess) {
    *err = "cudaSetDevice failed";
    return SX_E_CUDA;
  }
  const char* tc_env = getenv("SYRINX_CODEC_TC");
  use_tc = !(tc_env && tc_env[0] == '0');
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (cudaMalloc(&this->err, sizeof(int)) != cudaSuccess || cudaMemset(this->err, 0, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    *err = "device allocation failed";
    return SX_E_OOM;
  }
  weight_bytes = ld.image.size() * sizeof(float);
  const size_t tab_off = (weight_bytes + 255) & ~size_t(255);
  if (cudaMalloc(&weights, tab_off + sizeof(CbTab) * (1 + n_res)) != cudaSuccess) {
    cudaGetLastError();
    weights = nullptr;
    *err = "device allocation of the codec weights failed";
    return SX_E_OOM;
  }
  float* base = static_cast<float*>(weights);
  for (auto& f : ld.fix) *f.first = base + f.second;
  std::vector<CbTab> th(1 + n_res);
  for (int i = 0; i <= n_res; i++) th[i] = CbTab{cb[i], pw[i], pb[i], sizes[i], cb_dim};
  tabs = reinterpret_cast<CbTab*>(static_cast<char*>(weights) + tab_off);
  if (cudaMemcpy(weights, ld.image.data(), weight_bytes, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(tabs, th.data(), sizeof(CbTab) * th.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
    *err = "upload of the codec weights failed";
    return SX_E_CUDA;
  }
  return SX_OK;
}

size_t Codec::elems_for(int T) const {
  size_t L = (size_t)T, m = (size_t)latent * L;
  if (n_layers) m = std::max(m, (size_t)std::max(3 * latent, 2 * ffn) * L);
  for (const UpStage& u : ups) {
    L *= (size_t)u.up.stride;
    m = std::max(m, (size_t)std::max(u.c, u.pw1.cout) * L);
  }
  m = std::max(m, (size_t)conv0.cout * L);
  for (const DecBlock& b : blocks) {
    m = std::max(m, (size_t)b.up.cin * L);
    L *= (size_t)b.up.stride;
    m = std::max(m, (size_t)b.up.cout * L);
  }
  return std::max(m, L);
}

int Codec::reserve(int frames, std::string* err) {
  if (frames <= reserved_frames) return SX_OK;
  const size_t need = elems_for(frames);
  int grn_c = 1;
  for (const UpStage& u : ups) grn_c = std::max(grn_c, u.pw1.cout);
  for (float*& b : buf) {
    cudaFree(b);
    b = nullptr;
  }
  cudaFree(grn);
  grn = nullptr;
  reserved_frames = 0;
  buf_elems = 0;
  for (float*& b : buf)
    if (cudaMalloc(&b, need * sizeof(float)) != cudaSuccess) {
      cudaGetLastError();
      b = nullptr;
      *err = "device allocation of the codec activations failed";
      return SX_E_OOM;
    }
  if (cudaMalloc(&grn, (size_t)grn_c * sizeof(float)) != cudaSuccess) {
    cudaGetLastError();
    grn = nullptr;
    *err = "device allocation of the codec activations failed";
    return SX_E_OOM;
  }
  buf_elems = need;
  reserved_frames = frames;
  return SX_OK;
}

int Codec::decode_device(const uint32_t* codes, int ncb, int T, float* wav, std::string* err) {
  if (T == 0) return SX_OK;
  int rc = reserve(T, err);
  if (rc) return rc;
  cudaStream_t st = stream;
  float *X = buf[0], *S = buf[1], *Z = buf[2], *P = buf[3];

  k_rvq_embed<<<dim3((T + 127) / 128, latent), 128, 0, st>>>(codes, ncb, T, tabs, latent, X);

  if (n_layers) {
    const int D = latent, F = ffn;
    for (const Layer& y : layers) {
      k_chan_norm<<<(T + 31) / 32, 256, 0, st>>>(X, y.attn_norm, nullptr, S, D, T, kNormEps);
      conv_launch(*this, y.wqkv, S, T, Z, nullptr, nullptr, 0);
      k_rope_cf<<<dim3((T + 127) / 128, D), 128, 0, st>>>(Z, D, T, inv_freq, kHeadDim / 2);
      k_attn_causal_cf<<<dim3((T + kQt - 1) / kQt, n_head), 256, 0, st>>>(Z, S, D, T);
      conv_launch(*this, y.wo, S, T, X, y.attn_gamma, X, 0);
      k_chan_norm<<<(T + 31) / 32, 256, 0, st>>>(X, y.ffn_norm, nullptr, S, D, T, kNormEps);
      conv_launch(*this, y.w13, S, T, Z, nullptr, nullptr, 0);
      k_swiglu_cf<<<cols_grid(F * T, 256), 256, 0, st>>>(Z, P, F, T);
      conv_launch(*this, y.w2, P, T, X, y.ffn_gamma, X, 0);
    }
    k_chan_norm<<<(T + 31) / 32, 256, 0, st>>>(X, post_norm, nullptr, S, D, T, kNormEps);
    std::swap(X, S);
  }

  int L = T;
  for (const UpStage& u : ups) {
    conv_launch(*this, u.up, X, L, S, nullptr, nullptr, 0);
    L *= u.up.stride;
    std::swap(X, S);
    const int C = u.c, C4 = u.pw1.cout;
    k_dwconv_causal<<<dim3(cols_grid(L, 256), C), 256, 0, st>>>(X, u.dw_w, u.dw_b, S, L, 7);
    k_chan_norm<<<(L + 31) / 32, 256, 0, st>>>(S, u.ln_w, u.ln_b, Z, C, L, kLnEps);
    conv_launch(*this, u.pw1, Z, L, P, nullptr, nullptr, 2);
    if (u.grn_g) {
      k_grn_norm<<<C4, 256, 0, st>>>(P, grn, L);
      k_grn_scale<<<1, 1024, 0, st>>>(grn, C4);
      k_grn_apply<<<dim3(cols_grid(L, 256), C4), 256, 0, st>>>(P, grn, u.grn_g, u.grn_b, L);
    }
    conv_launch(*this, u.pw2, P, L, X, u.gamma, X, 0);
  }

  conv_launch(*this, conv0, X, L, S, nullptr, nullptr, 0);
  std::swap(X, S);
  for (const DecBlock& b : blocks) {
    k_snake<<<dim3(cols_grid(L, 256), b.up.cin), 256, 0, st>>>(X, b.alpha, S, b.up.cin, L);
    conv_launch(*this, b.up, S, L, X, nullptr, nullptr, 0);
    L *= b.up.stride;
    const int C = b.up.cout;
    for (const ResUnit& u : b.ru) {
      k_snake<<<dim3(cols_grid(L, 256), C), 256, 0, st>>>(X, u.a0, S, C, L);
      conv_launch(*this, u.c1, S, L, Z, nullptr, nullptr, 0);
      k_snake<<<dim3(cols_grid(L, 256), C), 256, 0, st>>>(Z, u.a2, S, C, L);
      conv_launch(*this, u.c3, S, L, X, nullptr, X, 0);
    }
  }
  k_snake<<<dim3(cols_grid(L, 256), final_cin), 256, 0, st>>>(X, final_alpha, S, final_cin, L);
  k_conv_out1<<<(L + 256 * kOutV - 1) / (256 * kOutV), 256, final_cin * kOutK * sizeof(float), st>>>(
      S, final_w, final_b, wav, final_cin, L);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = std::string("codec decode launch: ") + cudaGetErrorString(e);
    return SX_E_CUDA;
  }
  return SX_OK;
}

}  // namespace codec
}  // namespace sx
