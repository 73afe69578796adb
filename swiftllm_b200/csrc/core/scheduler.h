// Continuous-batching scheduler and per-step batch builder.
//
// Parity:
//   crates/swiftllm-core/src/scheduler/mod.rs (Scheduler: waiting / running /
//     swapped queues :78-102, add_request :178-199, abort_request :202-243,
//     schedule :246-435, finish_request :438-464, RequestMetadata :105-158)
//   crates/swiftllm-core/src/scheduler/continuous_batching.rs (FCFS / SJF /
//     priority policies :20-34, :217-222; chunked prefill :352-358)
//   crates/swiftllm-core/src/execution/mod.rs (BatchBuilder :46-126) and
//   crates/swiftllm-core/src/memory/kv_cache.rs (slot = block*BS + off, :186-216)
//
// Semantics (the reference leaves several undefined or buggy; these are ours):
//   * one token budget per step; running sequences are served first
//     (decode-first), then swapped-in, then new prefills;
//   * with chunked prefill a prompt may be split across steps;
//   * when blocks run out, the lowest-priority running group is preempted by
//     recompute (free + requeue at the head of waiting) or swap (to host);
//   * num_computed advances when a chunk is scheduled; a sequence samples a
//     token only on the chunk that reaches the end of its known tokens;
//   * TTFT is stamped when the first output token arrives (the reference
//     stamps admission, scheduler/mod.rs:418-421).
#pragma once
#include <cstdint>
#include <deque>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "block_manager.h"

namespace swift {

enum class Policy : int { FCFS = 0, SJF = 1, PRIORITY = 2 };
enum class Preempt : int { RECOMPUTE = 0, SWAP = 1 };

enum class SeqStatus : int {
  WAITING = 0,
  RUNNING = 1,
  SWAPPED = 2,
  FINISHED_STOPPED = 3,
  FINISHED_LENGTH = 4,
  FINISHED_ABORTED = 5,
};

struct SchedulerConfig {
  int max_num_seqs = 256;
  int max_num_batched_tokens = 8192;
  int max_model_len = 4096;
  bool enable_chunked_prefill = true;
  Policy policy = Policy::FCFS;
  Preempt preemption = Preempt::RECOMPUTE;
  int num_speculative_tokens = 0;  // extra slots reserved per decode step
};

// Per-request sampling and stopping parameters the core needs on the hot path.
struct GroupParams {
  int n = 1;
  int max_tokens = 256;
  int min_tokens = 0;
  bool ignore_eos = false;
  int eos_token_id = -1;
  std::vector<int32_t> stop_token_ids;
  float temperature = 1.0f;
  float top_p = 1.0f;
  int top_k = -1;
  float min_p = 0.0f;
  float presence_penalty = 0.0f;
  float frequency_penalty = 0.0f;
  float repetition_penalty = 1.0f;
  int64_t seed = -1;
  int priority = 0;
};

struct Sequence {
  int64_t id;
  int64_t group;
  std::vector<int32_t> tokens;  // prompt + generated
  int64_t num_prompt = 0;
  int64_t num_computed = 0;
  SeqStatus status = SeqStatus::WAITING;
  double cum_logprob = 0.0;
  int64_t num_draft = 0;  // trailing speculative tokens awaiting verification
  int64_t num_output() const { return static_cast<int64_t>(tokens.size()) - num_prompt; }
};

struct Group {
  int64_t id;
  std::string request_id;
  std::vector<int64_t> seqs;
  GroupParams params;
  double arrival = 0, first_scheduled = -1, first_token = -1, finished = -1;
  int64_t arrival_order = 0;
  bool forked = false;  // n>1 children created
  int num_preemptions = 0;
};

// Flat per-step batch. Decode rows (query length 1) come first.
struct Batch {
  int num_seqs = 0;
  int num_decode_seqs = 0;
  int64_t num_tokens = 0;
  int max_q_len = 0;
  int max_seq_len = 0;
  int max_blocks = 0;
  std::vector<int32_t> input_ids, positions, slot_mapping;
  std::vector<int32_t> q_start, q_len, seq_len;  // q_start has num_seqs+1 entries
  std::vector<int32_t> block_tables;             // [num_seqs, max_blocks], -1 padded
  std::vector<int64_t> seq_ids;
  // sampling rows: one per generated token this step
  std::vector<int32_t> sample_logit_idx;  // row into the last-token logits
  std::vector<int32_t> sample_seq_row;    // row into the seq arrays above
  std::vector<int64_t> sample_target_seq; // seq that receives the token (-1: new child)
  std::vector<int64_t> sample_group;
  std::vector<float> temperature, top_p, min_p, presence, frequency, repetition;
  std::vector<int32_t> top_k;
  std::vector<int64_t> seed;     // -1: engine RNG
  std::vector<int32_t> step_idx; // number of outputs so far, for per-request RNG offsets
  bool any_penalty = false;
  bool any_random = false;
  std::vector<CopyPair> swap_in, swap_out, copies;
  std::vector<int64_t> preempted_groups;
  int64_t num_prefill_tokens = 0;
};

struct StepResult {
  std::vector<int64_t> group, seq;     // one entry per appended token
  std::vector<int32_t> token;
  std::vector<int32_t> row;            // sample row that produced the token
  std::vector<int64_t> finished_groups;
};

struct SchedulerStats {
  int64_t num_preemptions = 0;
  int64_t num_swapped_out = 0;
  int64_t num_swapped_in = 0;
  int64_t prefill_tokens = 0;
  int64_t decode_tokens = 0;
  int64_t steps = 0;
  int64_t finished = 0;
  int64_t aborted = 0;
  int64_t prefix_cache_hit_tokens = 0;
  int64_t prefix_cache_query_tokens = 0;
};

class Scheduler {
 public:
  Scheduler(const SchedulerConfig& cfg, BlockManager* bm);

  int64_t add_request(const std::string& request_id, const std::vector<int32_t>& prompt,
                      const GroupParams& params, double arrival);
  bool abort_request(const std::string& request_id);
  bool abort_group(int64_t gid);
  // Finish a sequence for a reason found outside the core (stop strings).
  void finish_seq(int64_t seq, SeqStatus reason);

  std::unique_ptr<Batch> schedule(double now);
  // tokens: one per sample row of `batch`; logprobs may be null.
  StepResult update(const Batch& batch, const int32_t* tokens, const float* logprobs,
                    double now);

  // Speculative decoding. append_tokens adds draft tokens to a running
  // sequence, so the next schedule() computes them together with the last
  // real token (query length 1 + k). rollback(seq, n) removes n trailing
  // tokens (the drafts) and marks the last remaining token uncomputed, so a
  // sequence whose drafts were not verified is recomputed from there.
  // update_multi then appends the verified tokens of each sample row
  // (counts[r] tokens starting at offsets[r]) with the stop rules applied per
  // token; every appended token but the last keeps the KV written for it.
  void append_tokens(int64_t seq, const std::vector<int32_t>& toks);
  void rollback(int64_t seq, int64_t num_tokens);
  StepResult update_multi(const Batch& batch, const int32_t* tokens, const int32_t* counts,
                          const float* logprobs, double now);
  // running sequences whose next step is a plain decode (one token to compute)
  std::vector<int64_t> decode_ready_seqs() const;

  // Beam search (SamplingParams.use_beam_search; the reference's
  // BeamSearchSampler, crates/swiftllm-core/src/sampling/strategies.rs:
  // 295-357, only keeps the top candidates of one sequence). The caller has
  // ranked the candidates of group `gid` and passes the next step's live
  // beams and the newly finished hypotheses as (parent sequence, token,
  // token logprob). A parent's first live child continues it in place,
  // further children are forks sharing its KV blocks (copy-on-write on
  // append); live beams no child continues are dropped from the group and
  // their blocks freed; a finished hypothesis becomes a finished sequence of
  // the group that holds no blocks. Beams reaching max_tokens or the model
  // length finish with FINISHED_LENGTH.
  StepResult beam_update(int64_t gid, const std::vector<int64_t>& live_parent,
                         const std::vector<int32_t>& live_token, const std::vector<float>& live_logprob,
                         const std::vector<int64_t>& fin_parent, const std::vector<int32_t>& fin_token,
                         const std::vector<float>& fin_logprob, double now);

  int num_waiting() const { return static_cast<int>(waiting_.size()); }
  int num_running() const { return static_cast<int>(running_.size()); }
  int num_swapped() const { return static_cast<int>(swapped_.size()); }
  int num_unfinished() const { return num_waiting() + num_running() + num_swapped(); }
  bool has_unfinished() const { return num_unfinished() > 0; }

  const Group* group(int64_t gid) const;
  const Group* group_by_request(const std::string& rid) const;
  const Sequence* seq(int64_t sid) const;
  // drop a finished group's state once the caller has read it
  void release_group(int64_t gid);
  const SchedulerStats& stats() const { return stats_; }
  const SchedulerConfig& config() const { return cfg_; }
  BlockManager* block_manager() { return bm_; }

 private:
  bool before(const Group& a, const Group& b) const;  // a has higher priority
  void insert_waiting(int64_t gid, bool front);
  void preempt(int64_t gid, Batch* out);
  void finish_group_if_done(int64_t gid, double now, StepResult* res);
  void free_seq(Sequence& s);
  int64_t group_tokens_needed(const Group& g) const;

  SchedulerConfig cfg_;
  BlockManager* bm_;
  std::unordered_map<int64_t, Group> groups_;
  std::unordered_map<int64_t, Sequence> seqs_;
  std::unordered_map<std::string, int64_t> by_request_;
  std::deque<int64_t> waiting_;
  std::vector<int64_t> running_;
  std::deque<int64_t> swapped_;
  int64_t next_group_ = 1, next_seq_ = 1, arrival_counter_ = 0;
  SchedulerStats stats_;
};

}  // namespace swift
