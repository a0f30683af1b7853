// codec.hpp — host state of the device codec decode (the s2 causal-DAC `EvaGanDac`,
// crates/syrinx-fish/src/s2/codec.rs:67-379), behind include/syrinx_codec.h.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/syrinx_codec.h"

namespace sx {
namespace codec {

// One quantizer's decode tables: codebook [size][dim] and out_proj [latent][dim] + bias.
struct CbTab {
  const float* cb;
  const float* w;
  const float* b;
  int size;
  int dim;
};

// A convolution packed as the product's A operand: [rows][cin * taps], tap fastest. For a
// transposed convolution of stride s > 1 (or a stride-s kernel of s taps) the rows are the
// stride phases: row p*cout + co holds the kernel taps p + (taps-1-j)*s at column ci*taps + j.
struct Conv {
  float* w = nullptr;
  float* b = nullptr;
  int cout = 0, cin = 0;
  int taps = 0;    // taps of the packed (per-phase) kernel
  int stride = 1;  // > 1: transposed convolution of this stride (phase-packed)
  int dil = 1;
  float* tc = nullptr;  // the same matrix as tensor-core weight images (codec_tc.cu)
};

struct Layer {
  float *attn_norm = nullptr, *attn_gamma = nullptr, *ffn_norm = nullptr, *ffn_gamma = nullptr;
  Conv wqkv, wo, w13, w2;  // linear layers (k = 1, no bias); w13 stacks w1 over w3
};

// The product of codec_tc.cu: Y = W * im2col(X) on tcgen05 (kind::tf32, three-term split).
struct TcConvArgs {
  const uint8_t* a_img = nullptr;  // weight images [n_mt][n_kb] of 16 KB
  const float* x = nullptr;
  float* y = nullptr;
  const float* bias = nullptr;
  const float* scale = nullptr;
  const float* resid = nullptr;
  int M = 0, R = 0, N = 0, k = 1, dil = 1, phase = 1, cout = 0, act = 0;
  int n_mt = 0, n_kb = 0, n_nt = 0, bn = 0;  // set by launch_conv_tc
  int* err = nullptr;
};
size_t tc_image_bytes(int M, int R);
// Weight images of the row-major [M][R] matrix A into out (tc_image_bytes(M, R) bytes).
void tc_image(const float* A, int M, int R, uint32_t* out);
cudaError_t launch_conv_tc(const TcConvArgs& a, int sms, cudaStream_t st);

struct UpStage {
  Conv up;  // transposed conv, kernel = stride = factor
  int c = 0;
  float *dw_w = nullptr, *dw_b = nullptr, *ln_w = nullptr, *ln_b = nullptr;
  Conv pw1, pw2;  // linear layers as k=1 convolutions
  float *grn_g = nullptr, *grn_b = nullptr, *gamma = nullptr;  // optional
};

struct ResUnit {
  float* a0 = nullptr;
  Conv c1;  // k=7, dilated
  float* a2 = nullptr;
  Conv c3;  // k=1
};

struct DecBlock {
  float* alpha = nullptr;
  Conv up;  // transposed conv, kernel 2*stride
  ResUnit ru[3];
};

struct Codec {
  int device = 0;
  cudaStream_t stream = nullptr;
  // geometry discovered from the blob
  int latent = 0, n_layers = 0, n_head = 0, ffn = 0;
  int sem_size = 0, res_size = 0, cb_dim = 0, n_res = 0;
  int hop = 1;
  std::vector<Layer> layers;
  float* post_norm = nullptr;
  float* inv_freq = nullptr;
  std::vector<UpStage> ups;
  Conv conv0;
  std::vector<DecBlock> blocks;
  float* final_alpha = nullptr;
  float* final_w = nullptr;
  float* final_b = nullptr;
  int final_cin = 0;
  CbTab* tabs = nullptr;  // device array [1 + n_res]
  int* err = nullptr;     // device error flag of the tensor-core product's bounded waits
  bool use_tc = true;     // SYRINX_CODEC_TC=0 selects the FP32 CUDA-core product
  int sms = 148;
  void* weights = nullptr;
  size_t weight_bytes = 0;
  // activation buffers, grown by reserve()
  float* buf[4] = {nullptr, nullptr, nullptr, nullptr};
  float* grn = nullptr;
  size_t buf_elems = 0;
  int reserved_frames = 0;
  uint32_t* codes_dev = nullptr;
  float* wav_dev = nullptr;
  size_t io_frames = 0;

  ~Codec();
  int load(const void* blob, size_t size, int dev, std::string* err);
  size_t elems_for(int frames) const;
  int reserve(int frames, std::string* err);
  // Enqueue the decode of codes [ncb][frames] (device) into wav (device, frames*hop) on
  // `stream`; grows the buffers first when needed (a synchronising allocation).
  int decode_device(const uint32_t* codes, int ncb, int frames, float* wav, std::string* err);
};

}  // namespace codec
}  // namespace sx

// The opaque handle of include/syrinx_codec.h.
struct sx_codec : sx::codec::Codec {};
