// Host (CPU) token sampler and speculative-decoding helpers.
//
// The CPU sampler is the oracle for the GPU sampling kernel: both use the
// same stage order, the same Philox4x32-10 counter-based generator
// (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3",
// SC'11) and the same index-order inverse-CDF draw, so a seeded request draws
// the same token on either side.
//
// Stage order (the reference's TokenSampler, crates/swiftllm-core/src/
// sampling/mod.rs:155-321, and SamplerChain, sampling/strategies.rs:399-439):
//   repetition / frequency / presence penalties -> temperature ->
//   (greedy if temperature == 0 or top_k == 1) -> softmax -> min-p ->
//   top-k (ties at the threshold kept) -> top-p (keeps the token that
//   crosses p) -> draw.
// The returned logprob is the log-softmax after penalties and temperature and
// before the filters (the reference re-softmaxes the filtered distribution,
// sampling/mod.rs:324-333, which we do not reproduce).
//
// Speculative verification parity: crates/swiftllm-core/src/execution/
// speculative.rs (verify :97-167, adjusted distribution max(0, p_t - p_d)
// :170-190, adaptive k :214-231, NgramSpeculator :294-372).
#pragma once
#include <cstdint>
#include <unordered_map>
#include <utility>
#include <vector>

namespace swift {

struct Philox {
  // One 4x32 block for (key, counter); 10 rounds.
  static void block(uint64_t key, uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                    uint32_t out[4]);
  // Uniform in [0, 1) from the first word, 24 bits of mantissa.
  static float uniform(uint64_t key, uint32_t c0, uint32_t c1);
};

struct SampleParams {
  float temperature = 1.0f, top_p = 1.0f, min_p = 0.0f;
  int top_k = -1;
  float presence = 0.0f, frequency = 0.0f, repetition = 1.0f;
};

// Applies penalties in place. `prompt` tokens feed the repetition penalty
// only; `output` tokens feed all three.
void apply_penalties(float* logits, int vocab, const SampleParams& p,
                     const int32_t* prompt, int n_prompt, const int32_t* output, int n_output);

// Samples one token. `u` is the uniform draw (ignored for greedy).
// Returns (token, logprob).
std::pair<int, float> sample_row(const float* logits, int vocab, const SampleParams& p, float u);

struct SpecVerifyResult {
  int num_accepted = 0;
  std::vector<int32_t> tokens;  // accepted drafts + one bonus / corrected token
};

// Rejection sampling (Leviathan et al. 2023, Chen et al. 2023).
// draft_probs: [k, V], target_probs: [k+1, V], uniforms: [2k+1] in [0,1).
SpecVerifyResult spec_verify(const float* draft_probs, const float* target_probs,
                             const int32_t* draft_tokens, int k, int vocab,
                             const float* uniforms);

class NgramSpeculator {
 public:
  NgramSpeculator(int n, int max_k) : n_(n), max_k_(max_k) {}
  // Longest-suffix match of the last n..1 tokens against earlier context;
  // proposes the tokens that followed the most recent match.
  std::vector<int32_t> propose(const int32_t* ctx, int len, int k) const;

 private:
  int n_, max_k_;
};

class AdaptiveK {
 public:
  AdaptiveK(int k, int min_k, int max_k, double target)
      : k_(k), min_k_(min_k), max_k_(max_k), target_(target) {}
  void update(int proposed, int accepted);
  int k() const { return k_; }
  double acceptance_rate() const { return proposed_ ? double(accepted_) / proposed_ : 0.0; }
  int64_t proposed() const { return proposed_; }
  int64_t accepted() const { return accepted_; }

 private:
  int k_, min_k_, max_k_;
  double target_;
  int64_t proposed_ = 0, accepted_ = 0;
};

}  // namespace swift
