// Randomised stress of the C++ engine core, built with
// -fsanitize=address,undefined by tests/test_sanitizers_cpu.py: scheduler +
// block manager (prefix caching, chunked prefill, recompute and swap
// preemption, n > 1 forks, speculative appends / rollbacks, aborts), the
// sampling oracle, the n-gram speculator and the request queue. Invariants
// are checked with explicit tests (not assert, which NDEBUG would remove);
// any failure prints a message and exits 1.
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "request_queue.h"
#include "sampler.h"
#include "scheduler.h"

using namespace swift;

#define CHECK(c, msg)                                              \
  do {                                                             \
    if (!(c)) {                                                    \
      std::fprintf(stderr, "CHECK failed: %s (%s:%d)\n", msg, __FILE__, __LINE__); \
      std::exit(1);                                                \
    }                                                              \
  } while (0)

static void fuzz_scheduler(uint32_t seed, bool swap, bool caching, bool chunked) {
  std::mt19937 rng(seed);
  const int bs = 4, gpu_blocks = 48, cpu_blocks = swap ? 64 : 0;
  BlockManager bm(bs, gpu_blocks, cpu_blocks, 0.02, caching);
  SchedulerConfig cfg;
  cfg.max_num_seqs = 8;
  cfg.max_num_batched_tokens = chunked ? 64 : 128;
  cfg.max_model_len = 120;
  cfg.enable_chunked_prefill = chunked;
  cfg.preemption = swap ? Preempt::SWAP : Preempt::RECOMPUTE;
  cfg.num_speculative_tokens = (seed % 2) ? 3 : 0;
  Scheduler s(cfg, &bm);
  int next_req = 0, live = 0;
  std::vector<std::string> ids;
  for (int step = 0; step < 600; ++step) {
    if (rng() % 3 == 0 && live < 12) {
      GroupParams p;
      p.max_tokens = 1 + rng() % 30;
      p.n = (rng() % 5 == 0) ? 2 : 1;
      p.ignore_eos = rng() % 2;
      p.eos_token_id = 7;
      const int len = 1 + rng() % 50;
      std::vector<int32_t> prompt(len);
      // shared prefixes exercise the prefix cache
      for (int i = 0; i < len; ++i) prompt[i] = (i < 12 && rng() % 2) ? i : static_cast<int32_t>(rng() % 50);
      std::string id = "r" + std::to_string(next_req++);
      s.add_request(id, prompt, p, step);
      ids.push_back(id);
      ++live;
    }
    if (rng() % 17 == 0 && !ids.empty()) s.abort_request(ids[rng() % ids.size()]);
    // speculative drafts on some decode-ready sequences
    std::vector<std::pair<int64_t, int>> drafted;
    if (cfg.num_speculative_tokens) {
      for (int64_t sid : s.decode_ready_seqs()) {
        if (rng() % 2) continue;
        const Sequence* q = s.seq(sid);
        const int k = 1 + rng() % 3;
        if (static_cast<int>(q->tokens.size()) + k + 1 >= cfg.max_model_len) continue;
        std::vector<int32_t> d(k);
        for (auto& t : d) t = rng() % 50;
        s.append_tokens(sid, d);
        drafted.push_back({sid, k});
      }
    }
    auto b = s.schedule(step);
    CHECK(b->num_tokens <= cfg.max_num_batched_tokens + 16, "token budget");
    CHECK(b->num_seqs <= cfg.max_num_seqs, "sequence budget");
    CHECK(static_cast<int64_t>(b->input_ids.size()) == b->num_tokens, "flat batch size");
    for (size_t i = 0; i < b->slot_mapping.size(); ++i)
      CHECK(b->slot_mapping[i] >= 0 && b->slot_mapping[i] < gpu_blocks * bs, "slot in pool");
    for (int v : b->block_tables) CHECK(v >= -1 && v < gpu_blocks, "block table entry");
    for (auto& d : drafted) {
      const Sequence* q = s.seq(d.first);
      if (q) s.rollback(d.first, std::min<int64_t>(d.second, q->num_output()));
    }
    const size_t rows = b->sample_logit_idx.size();
    std::vector<int32_t> toks;
    std::vector<int32_t> counts(rows);
    for (size_t r = 0; r < rows; ++r) {
      counts[r] = 1 + (cfg.num_speculative_tokens ? rng() % 2 : 0);
      for (int c = 0; c < counts[r]; ++c) toks.push_back(rng() % 50);
    }
    auto res = s.update_multi(*b, toks.data(), counts.data(), nullptr, step);
    for (int64_t g : res.finished_groups) {
      s.release_group(g);
      --live;
    }
    for (int64_t g : b->preempted_groups)
      if (g < 0) {
        s.release_group(-g);
        --live;
      }
    CHECK(bm.num_free_gpu() >= 0 && bm.num_free_gpu() <= gpu_blocks, "free count");
  }
}

static void fuzz_sampler(uint32_t seed) {
  std::mt19937 rng(seed);
  std::normal_distribution<float> nd(0.f, 3.f);
  for (int it = 0; it < 300; ++it) {
    const int V = 1 + rng() % 300;
    std::vector<float> logits(V);
    for (auto& v : logits) v = nd(rng);
    if (rng() % 7 == 0) logits[rng() % V] = 1e30f;
    SampleParams p;
    p.temperature = (rng() % 4 == 0) ? 0.f : 0.1f + (rng() % 20) * 0.1f;
    p.top_k = (rng() % 3 == 0) ? 1 + static_cast<int>(rng() % V) : -1;
    p.top_p = (rng() % 3 == 0) ? 0.05f + (rng() % 19) * 0.05f : 1.f;
    p.min_p = (rng() % 4 == 0) ? 0.1f : 0.f;
    std::vector<int32_t> hist(rng() % 20);
    for (auto& t : hist) t = rng() % V;
    p.repetition = 1.2f;
    p.presence = 0.5f;
    apply_penalties(logits.data(), V, p, hist.data(), static_cast<int>(hist.size()), hist.data(),
                    static_cast<int>(hist.size()));
    auto r = sample_row(logits.data(), V, p, Philox::uniform(seed, it, 0));
    CHECK(r.first >= 0 && r.first < V, "sampled token in range");
  }
  NgramSpeculator ng(3, 8);
  std::vector<int32_t> ctx(200);
  for (auto& t : ctx) t = rng() % 5;
  for (int len = 0; len <= 200; len += 7) {
    auto d = ng.propose(ctx.data(), len, 5);
    CHECK(d.size() <= 5, "draft length");
  }
}

static void fuzz_queue() {
  RequestQueue q(64, true, 0.0);
  std::atomic<int> got{0};
  std::vector<std::thread> th;
  for (int w = 0; w < 4; ++w)
    th.emplace_back([&] {
      QueueEntry e;
      while (q.dequeue(&e, 0.2)) ++got;
    });
  int ok = 0;
  for (int i = 0; i < 2000; ++i)
    if (q.enqueue("x" + std::to_string(i), i, i % 3) == EnqueueStatus::OK) ++ok;
  while (got.load() < ok) std::this_thread::yield();
  q.close();
  for (auto& t : th) t.join();
  CHECK(got.load() == ok, "every queued entry dequeued once");
}

int main() {
  for (uint32_t seed = 1; seed <= 24; ++seed)
    fuzz_scheduler(seed, seed % 3 == 0, seed % 2 == 0, seed % 4 != 1);
  for (uint32_t seed = 1; seed <= 8; ++seed) fuzz_sampler(seed);
  fuzz_queue();
  std::printf("CORE_FUZZ_OK\n");
  return 0;
}
