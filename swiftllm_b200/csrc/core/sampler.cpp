#include "sampler.h"

#include <algorithm>
#include <cmath>
#include <numeric>
#include <stdexcept>

namespace swift {

static inline uint32_t mulhilo(uint32_t a, uint32_t b, uint32_t* hi) {
  uint64_t p = static_cast<uint64_t>(a) * b;
  *hi = static_cast<uint32_t>(p >> 32);
  return static_cast<uint32_t>(p);
}

void Philox::block(uint64_t key, uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                   uint32_t out[4]) {
  // Philox4x32 round multipliers and Weyl key increments from the SC'11 paper.
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
  uint32_t k0 = static_cast<uint32_t>(key), k1 = static_cast<uint32_t>(key >> 32);
  uint32_t x0 = c0, x1 = c1, x2 = c2, x3 = c3;
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, hi1;
    uint32_t lo0 = mulhilo(M0, x0, &hi0);
    uint32_t lo1 = mulhilo(M1, x2, &hi1);
    uint32_t y0 = hi1 ^ x1 ^ k0;
    uint32_t y1 = lo1;
    uint32_t y2 = hi0 ^ x3 ^ k1;
    uint32_t y3 = lo0;
    x0 = y0; x1 = y1; x2 = y2; x3 = y3;
    k0 += W0;
    k1 += W1;
  }
  out[0] = x0; out[1] = x1; out[2] = x2; out[3] = x3;
}

float Philox::uniform(uint64_t key, uint32_t c0, uint32_t c1) {
  uint32_t o[4];
  block(key, c0, c1, 0, 0, o);
  return static_cast<float>(o[0] >> 8) * (1.0f / 16777216.0f);
}

void apply_penalties(float* logits, int vocab, const SampleParams& p, const int32_t* prompt,
                     int n_prompt, const int32_t* output, int n_output) {
  if (p.repetition == 1.0f && p.presence == 0.0f && p.frequency == 0.0f) return;
  std::unordered_map<int32_t, int> counts;
  for (int i = 0; i < n_output; ++i) counts[output[i]]++;
  if (p.repetition != 1.0f) {
    std::vector<uint8_t> seen(vocab, 0);
    for (int i = 0; i < n_prompt; ++i)
      if (prompt[i] >= 0 && prompt[i] < vocab) seen[prompt[i]] = 1;
    for (auto& kv : counts)
      if (kv.first >= 0 && kv.first < vocab) seen[kv.first] = 1;
    for (int t = 0; t < vocab; ++t)
      if (seen[t]) logits[t] = logits[t] > 0 ? logits[t] / p.repetition : logits[t] * p.repetition;
  }
  for (auto& kv : counts) {
    if (kv.first < 0 || kv.first >= vocab) continue;
    logits[kv.first] -= p.frequency * static_cast<float>(kv.second) + p.presence;
  }
}

std::pair<int, float> sample_row(const float* logits, int vocab, const SampleParams& p, float u) {
  if (vocab <= 0) throw std::invalid_argument("empty vocabulary");
  const bool greedy = p.temperature <= 0.0f || p.top_k == 1;
  const float inv_t = greedy ? 1.0f : 1.0f / p.temperature;
  float mx = -INFINITY;
  int arg = 0;
  for (int t = 0; t < vocab; ++t)
    if (logits[t] > mx) { mx = logits[t]; arg = t; }
  double sum = 0;
  for (int t = 0; t < vocab; ++t) sum += std::exp((logits[t] - mx) * inv_t);
  const float log_z = static_cast<float>(std::log(sum));
  if (greedy) return {arg, -log_z};
  std::vector<float> prob(vocab);
  for (int t = 0; t < vocab; ++t)
    prob[t] = static_cast<float>(std::exp((logits[t] - mx) * inv_t) / sum);
  // min-p relative to the most likely token (probability of `arg`)
  float thresh = p.min_p > 0.f ? p.min_p * prob[arg] : 0.f;
  if (p.top_k > 0 && p.top_k < vocab) {
    std::vector<float> s(prob);
    std::nth_element(s.begin(), s.begin() + (p.top_k - 1), s.end(), std::greater<float>());
    thresh = std::max(thresh, s[p.top_k - 1]);
  }
  if (p.top_p < 1.0f) {
    std::vector<float> kept;
    double mass = 0;
    for (int t = 0; t < vocab; ++t)
      if (prob[t] >= thresh) { kept.push_back(prob[t]); mass += prob[t]; }
    std::sort(kept.begin(), kept.end(), std::greater<float>());
    double target = p.top_p * mass, c = 0;
    for (float v : kept) {
      c += v;
      if (c >= target) { thresh = std::max(thresh, v); break; }
    }
  }
  double total = 0;
  for (int t = 0; t < vocab; ++t)
    if (prob[t] >= thresh) total += prob[t];
  double target = static_cast<double>(u) * total, c = 0;
  int pick = arg;
  for (int t = 0; t < vocab; ++t) {
    if (prob[t] < thresh) continue;
    c += prob[t];
    pick = t;
    if (c > target) break;
  }
  return {pick, (logits[pick] - mx) * inv_t - log_z};
}

SpecVerifyResult spec_verify(const float* dp, const float* tp, const int32_t* draft, int k,
                             int vocab, const float* u) {
  SpecVerifyResult r;
  for (int i = 0; i < k; ++i) {
    int t = draft[i];
    float pd = dp[static_cast<int64_t>(i) * vocab + t];
    float pt = tp[static_cast<int64_t>(i) * vocab + t];
    float accept = pd > 0 ? std::min(1.0f, pt / pd) : 1.0f;
    if (u[i] < accept) {
      r.tokens.push_back(t);
      ++r.num_accepted;
      continue;
    }
    // rejected: draw from normalised max(0, p_t - p_d)
    std::vector<double> adj(vocab);
    double z = 0;
    for (int v = 0; v < vocab; ++v) {
      double d = tp[static_cast<int64_t>(i) * vocab + v] - dp[static_cast<int64_t>(i) * vocab + v];
      adj[v] = d > 0 ? d : 0;
      z += adj[v];
    }
    int pick = 0;
    if (z <= 0) {
      // identical distributions: fall back to the target distribution
      for (int v = 0; v < vocab; ++v) adj[v] = tp[static_cast<int64_t>(i) * vocab + v];
      z = std::accumulate(adj.begin(), adj.end(), 0.0);
    }
    double target = u[k + 1 + i] * z, c = 0;
    for (int v = 0; v < vocab; ++v) {
      if (adj[v] <= 0) continue;
      c += adj[v];
      pick = v;
      if (c > target) break;
    }
    r.tokens.push_back(pick);
    return r;
  }
  // all accepted: bonus token from target row k
  const float* row = tp + static_cast<int64_t>(k) * vocab;
  double z = 0;
  for (int v = 0; v < vocab; ++v) z += row[v];
  double target = u[k] * z, c = 0;
  int pick = 0;
  for (int v = 0; v < vocab; ++v) {
    if (row[v] <= 0) continue;
    c += row[v];
    pick = v;
    if (c > target) break;
  }
  r.tokens.push_back(pick);
  return r;
}

std::vector<int32_t> NgramSpeculator::propose(const int32_t* ctx, int len, int k) const {
  std::vector<int32_t> out;
  k = std::min(k, max_k_);
  if (k <= 0) return out;
  for (int n = std::min(n_, len - 1); n >= 1; --n) {
    const int32_t* suffix = ctx + len - n;
    // scan backwards for the most recent earlier occurrence
    for (int start = len - n - 1; start >= 0; --start) {
      if (std::equal(suffix, suffix + n, ctx + start)) {
        int from = start + n;
        for (int j = 0; j < k && from + j < len; ++j) out.push_back(ctx[from + j]);
        if (!out.empty()) return out;
      }
    }
  }
  return out;
}

void AdaptiveK::update(int proposed, int accepted) {
  proposed_ += proposed;
  accepted_ += accepted;
  if (proposed_ < 100) return;
  double rate = acceptance_rate();
  if (rate > target_ + 0.1 && k_ < max_k_) ++k_;
  else if (rate < target_ - 0.1 && k_ > min_k_) --k_;
}

}  // namespace swift
