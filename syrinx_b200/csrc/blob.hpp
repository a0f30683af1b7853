// blob.hpp — SXW1 weight container (parse + seeded synthetic writer), host only.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/syrinx_dualar.h"

namespace sx {

struct BlobTensor {
  std::string name;
  int dtype = -1;
  int64_t rows = 0, cols = 0;  // a rank-3 tensor [d0, d1, d2] is held as rows d0, cols d1*d2
  int ndim = 0;
  int64_t shape[3] = {1, 1, 1};
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
};

struct BlobIndex {
  std::unordered_map<std::string, BlobTensor> t;
};

struct SynthTensor {
  std::string name;
  int dtype;
  int64_t rows, cols;
  int kind;  // 0 matrix N(0,0.02) in wtype, 1 RMSNorm gain = 1.0 (f32), 2 bias N(0,0.02) f32
  size_t offset = 0, nbytes = 0;
};

size_t row_bytes(int dtype, int64_t cols);
int parse_blob(const void* blob, size_t size, BlobIndex* out, std::string* err);
std::vector<SynthTensor> synth_tensors(const sx_model_desc& d, int wtype);
int synth_layout(const sx_model_desc& d, int wtype, std::vector<SynthTensor>* ts, size_t* header,
                 size_t* total);
int synth_write(const sx_model_desc& d, int wtype, uint64_t seed, void* out, size_t size);

}  // namespace sx
