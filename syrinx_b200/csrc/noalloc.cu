// noalloc.cu — sx_dequantize_noalloc: the dequantize entry point without any device
// allocation. It has no reference counterpart (the reference dequantizes GGUF tensors on
// the CPU while loading weights); it exists for hosts that must not allocate device memory
// per call.
//
// Scratch: two file-scope static device arrays, sized for SX_DEQUANTIZE_NOALLOC_MAX_BLOCKS
// blocks of either type — the raw GGML blocks copied in (144 B per block, 144 KB) and the
// f32 values copied out (256 per block, 1 MB). Their addresses are resolved once per device
// with cudaGetSymbolAddress on the first call for that device (which may load the module:
// make that first call before any stream capture on the device). Nothing in the scratch has
// to start at zero: the host copy overwrites every input byte the kernel reads, and the
// kernel writes every output value that is copied back. The scratch is shared by all calls
// on a device, so calls that overlap on one device (from several host threads) race:
// serialize them. The dequant kernel is the one sx_dequantize runs (dequant_blocks), so the
// two entry points give bit-identical values.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/syrinx_dualar.h"
#include "sx_internal.hpp"

namespace sx {
namespace {

constexpr int64_t kMaxBlocks = SX_DEQUANTIZE_NOALLOC_MAX_BLOCKS;
constexpr int64_t kMaxBlockBytes = 144;  // a Q4_K super-block (a Q8_0 block is 34 B)
constexpr int64_t kMaxValues = 256;      // values per Q4_K super-block (32 per Q8_0 block)
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_blocks[kMaxBlocks * kMaxBlockBytes];
static __device__ __align__(256) float g_noalloc_values[kMaxBlocks * kMaxValues];

struct ScratchAddr {
  bool resolved = false;
  uint8_t* blocks = nullptr;
  float* values = nullptr;
};
ScratchAddr g_addr[kMaxDevices];
std::mutex g_addr_mu;

// Device addresses of the scratch on `device` (the current device), resolved once.
int scratch_for(int device, ScratchAddr* out) {
  std::lock_guard<std::mutex> lock(g_addr_mu);
  ScratchAddr& a = g_addr[device];
  if (!a.resolved) {
    void* b = nullptr;
    void* v = nullptr;
    if (cudaGetSymbolAddress(&b, g_noalloc_blocks) != cudaSuccess ||
        cudaGetSymbolAddress(&v, g_noalloc_values) != cudaSuccess) {
      set_error("sx_dequantize_noalloc: cudaGetSymbolAddress failed");
      return SX_E_CUDA;
    }
    a.blocks = static_cast<uint8_t*>(b);
    a.values = static_cast<float*>(v);
    a.resolved = true;
  }
  *out = a;
  return SX_OK;
}

}  // namespace

int dequantize_noalloc(int32_t dtype, const void* blocks, int64_t n_blocks, float* out, int32_t device) {
  if (!blocks || !out || n_blocks < 0 || (dtype != SX_DTYPE_Q8_0 && dtype != SX_DTYPE_Q4_K)) {
    set_error("sx_dequantize_noalloc: bad arguments");
    return SX_E_INVALID;
  }
  if (n_blocks > kMaxBlocks) {
    set_error("sx_dequantize_noalloc: n_blocks = " + std::to_string(n_blocks) +
              " exceeds the static scratch capacity of " + std::to_string(kMaxBlocks) +
              " blocks (use sx_dequantize, which allocates)");
    return SX_E_RANGE;
  }
  if (device < 0 || device >= kMaxDevices) {
    set_error("sx_dequantize_noalloc: device index out of range");
    return SX_E_INVALID;
  }
  if (n_blocks == 0) return SX_OK;
  if (cudaSetDevice(device) != cudaSuccess) {
    set_error("cudaSetDevice failed");
    return SX_E_CUDA;
  }
  ScratchAddr a;
  const int rc = scratch_for(device, &a);
  if (rc) return rc;
  const size_t bb = dtype == SX_DTYPE_Q8_0 ? 34 : 144, per = dtype == SX_DTYPE_Q8_0 ? 32 : 256;
  if (cudaMemcpy(a.blocks, blocks, (size_t)n_blocks * bb, cudaMemcpyHostToDevice) != cudaSuccess ||
      dequant_blocks(dtype, a.blocks, n_blocks, a.values, 0) != cudaSuccess ||
      cudaMemcpy(out, a.values, (size_t)n_blocks * per * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
    set_error("sx_dequantize_noalloc: CUDA failure");
    return SX_E_CUDA;
  }
  return SX_OK;
}

}  // namespace sx
