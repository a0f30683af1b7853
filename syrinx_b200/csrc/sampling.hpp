// sampling.hpp — the driver-owned seeded sampler (host side).
//
// Restates crates/syrinx-fish/src/common/sampling.rs: SplitMix64 (19-41), SamplingParams
// defaults (63-77), the semantic constraint (84-106), Sampler::{sample_codebook,
// sample_semantic} (132-167) with RAS, logits_to_probs (189-245) and multinomial1
// (254-268). One Sampler drives a whole utterance; slow and fast draws share its stream.
#pragma once
#include <stdint.h>

#include <vector>

#include "../../include/syrinx_dualar.h"

namespace sx {

struct SplitMix64 {
  uint64_t state;
  uint64_t next_u64();
  double next_f64();
};

struct SemanticConstraint {
  uint32_t begin, end, stop_lo, stop_hi;  // allowed: [begin, end] U [stop_lo, stop_hi)
  bool is_semantic(uint32_t id) const { return id >= begin && id <= end; }
  bool allowed(uint32_t id) const { return is_semantic(id) || (id >= stop_lo && id < stop_hi); }
};

std::vector<float> logits_to_probs(const float* logits, int n, float temperature, float top_p, int top_k);
int multinomial1(const std::vector<float>& probs, SplitMix64* rng);

struct Sampler {
  SplitMix64 rng;
  sx_sampling_params p;
  uint32_t sample_codebook(const float* logits, int n);
  uint32_t sample_semantic(const float* logits, int n, const std::vector<uint32_t>& window,
                           const SemanticConstraint& c);
};

}  // namespace sx
