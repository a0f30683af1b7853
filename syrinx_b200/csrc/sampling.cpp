// sampling.cpp — host sampler; see sampling.hpp for the reference it restates.
#include "sampling.hpp"

#include <algorithm>
#include <cmath>

namespace sx {

uint64_t SplitMix64::next_u64() {
  state += 0x9E3779B97F4A7C15ull;
  uint64_t z = state;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

double SplitMix64::next_f64() { return (double)(next_u64() >> 11) * (1.0 / (double)(1ull << 53)); }

// Sort descending (ties by ascending index), cumulative softmax for the top-p cut, keep
// the top-1 always, then a temperature softmax over the kept ids in index order.
std::vector<float> logits_to_probs(const float* logits, int n, float temperature, float top_p, int top_k) {
  std::vector<int> order(n);
  for (int i = 0; i < n; i++) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
    if (logits[b] < logits[a]) return true;
    if (logits[a] < logits[b]) return false;
    return a < b;
  });
  const float mx = n ? logits[order[0]] : 0.0f;
  std::vector<double> exps(n);
  double sum = 0.0;
  for (int r = 0; r < n; r++) exps[r] = std::exp((double)(logits[order[r]] - mx));
  for (int r = 0; r < n; r++) sum += exps[r];
  const int k_cap = top_k == 0 ? n : top_k;
  std::vector<char> keep(n, 0);
  double cum = 0.0;
  for (int r = 0; r < n; r++) {
    if (r == 0) {
      keep[order[r]] = 1;
    } else if (cum <= (double)top_p && r < k_cap) {
      keep[order[r]] = 1;
    } else {
      break;
    }
    cum += exps[r] / sum;
  }
  const float t = std::max(temperature, 1e-5f);
  float kept_max = -INFINITY;
  for (int i = 0; i < n; i++)
    if (keep[i]) kept_max = std::max(kept_max, logits[i] / t);
  std::vector<float> probs(n, 0.0f);
  double psum = 0.0;
  for (int i = 0; i < n; i++)
    if (keep[i]) {
      const double e = std::exp((double)(logits[i] / t - kept_max));
      probs[i] = (float)e;
      psum += e;
    }
  if (psum > 0.0)
    for (int i = 0; i < n; i++) probs[i] = (float)((double)probs[i] / psum);
  return probs;
}

int multinomial1(const std::vector<float>& probs, SplitMix64* rng) {
  double total = 0.0;
  for (float p : probs) total += (double)p;
  if (total <= 0.0) return 0;
  const double u = rng->next_f64() * total;
  double acc = 0.0;
  for (size_t i = 0; i < probs.size(); i++) {
    acc += (double)probs[i];
    if (u < acc) return (int)i;
  }
  return probs.empty() ? 0 : (int)probs.size() - 1;
}

uint32_t Sampler::sample_codebook(const float* logits, int n) {
  // the fast AR passes an empty `recent` list, so the repetition penalty is a no-op
  const auto probs = logits_to_probs(logits, n, p.temperature, p.top_p, p.top_k);
  return (uint32_t)multinomial1(probs, &rng);
}

uint32_t Sampler::sample_semantic(const float* logits, int n, const std::vector<uint32_t>& window,
                                  const SemanticConstraint& c) {
  std::vector<float> masked(logits, logits + n);
  for (int i = 0; i < n; i++)
    if (!c.allowed((uint32_t)i)) masked[i] = -INFINITY;
  const auto pn = logits_to_probs(masked.data(), n, p.temperature, p.top_p, p.top_k);
  const uint32_t normal = (uint32_t)multinomial1(pn, &rng);
  const auto ph = logits_to_probs(masked.data(), n, p.ras_high_temp, p.ras_high_top_p, p.top_k);
  const uint32_t high = (uint32_t)multinomial1(ph, &rng);
  const bool in_window = std::find(window.begin(), window.end(), normal) != window.end();
  return (in_window && c.is_semantic(normal)) ? high : normal;
}

}  // namespace sx
