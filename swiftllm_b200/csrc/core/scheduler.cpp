#include "scheduler.h"

#include <algorithm>
#include <stdexcept>

namespace swift {

Scheduler::Scheduler(const SchedulerConfig& cfg, BlockManager* bm) : cfg_(cfg), bm_(bm) {
  if (cfg_.max_num_seqs <= 0) throw std::invalid_argument("max_num_seqs must be > 0");
  if (cfg_.max_num_batched_tokens <= 0)
    throw std::invalid_argument("max_num_batched_tokens must be > 0");
  if (!cfg_.enable_chunked_prefill && cfg_.max_num_batched_tokens < cfg_.max_model_len)
    throw std::invalid_argument(
        "max_num_batched_tokens must be >= max_model_len when chunked prefill is off");
}

bool Scheduler::before(const Group& a, const Group& b) const {
  switch (cfg_.policy) {
    case Policy::SJF:
      // shortest expected job first (continuous_batching.rs:217-222 uses
      // -max_tokens as the heap key)
      if (a.params.max_tokens != b.params.max_tokens)
        return a.params.max_tokens < b.params.max_tokens;
      break;
    case Policy::PRIORITY:
      if (a.params.priority != b.params.priority) return a.params.priority > b.params.priority;
      break;
    default:
      break;
  }
  return a.arrival_order < b.arrival_order;
}

void Scheduler::insert_waiting(int64_t gid, bool /*front*/) {
  const Group& g = groups_.at(gid);
  auto it = waiting_.begin();
  while (it != waiting_.end() && !before(g, groups_.at(*it))) ++it;
  waiting_.insert(it, gid);
}

int64_t Scheduler::add_request(const std::string& request_id, const std::vector<int32_t>& prompt,
                               const GroupParams& params, double arrival) {
  if (by_request_.count(request_id))
    throw std::invalid_argument("duplicate request id: " + request_id);
  if (prompt.empty()) throw std::invalid_argument("empty prompt");
  if (static_cast<int64_t>(prompt.size()) >= cfg_.max_model_len)
    throw std::invalid_argument("prompt of " + std::to_string(prompt.size()) +
                                " tokens does not fit max_model_len " +
                                std::to_string(cfg_.max_model_len));
  if (params.n < 1) throw std::invalid_argument("n must be >= 1");
  int64_t gid = next_group_++;
  Group g;
  g.id = gid;
  g.request_id = request_id;
  g.params = params;
  g.arrival = arrival;
  g.arrival_order = arrival_counter_++;
  Sequence s;
  s.id = next_seq_++;
  s.group = gid;
  s.tokens = prompt;
  s.num_prompt = static_cast<int64_t>(prompt.size());
  g.seqs.push_back(s.id);
  seqs_.emplace(s.id, std::move(s));
  groups_.emplace(gid, std::move(g));
  by_request_[request_id] = gid;
  insert_waiting(gid, false);
  return gid;
}

void Scheduler::free_seq(Sequence& s) { bm_->free(s.id); }

bool Scheduler::abort_group(int64_t gid) {
  auto git = groups_.find(gid);
  if (git == groups_.end()) return false;
  Group& g = git->second;
  bool live = false;
  for (int64_t sid : g.seqs) {
    Sequence& s = seqs_.at(sid);
    if (s.status == SeqStatus::WAITING || s.status == SeqStatus::RUNNING ||
        s.status == SeqStatus::SWAPPED) {
      live = true;
      free_seq(s);
      s.status = SeqStatus::FINISHED_ABORTED;
    }
  }
  if (!live) return false;
  waiting_.erase(std::remove(waiting_.begin(), waiting_.end(), gid), waiting_.end());
  running_.erase(std::remove(running_.begin(), running_.end(), gid), running_.end());
  swapped_.erase(std::remove(swapped_.begin(), swapped_.end(), gid), swapped_.end());
  ++stats_.aborted;
  return true;
}

bool Scheduler::abort_request(const std::string& request_id) {
  auto it = by_request_.find(request_id);
  if (it == by_request_.end()) return false;
  return abort_group(it->second);
}

void Scheduler::finish_seq(int64_t sid, SeqStatus reason) {
  auto it = seqs_.find(sid);
  if (it == seqs_.end()) return;
  Sequence& s = it->second;
  if (s.status == SeqStatus::RUNNING || s.status == SeqStatus::WAITING ||
      s.status == SeqStatus::SWAPPED) {
    free_seq(s);
    s.status = reason;
    Group& g = groups_.at(s.group);
    bool all = true;
    for (int64_t q : g.seqs) {
      auto st = seqs_.at(q).status;
      if (st == SeqStatus::RUNNING || st == SeqStatus::WAITING || st == SeqStatus::SWAPPED)
        all = false;
    }
    if (all) {
      running_.erase(std::remove(running_.begin(), running_.end(), g.id), running_.end());
      waiting_.erase(std::remove(waiting_.begin(), waiting_.end(), g.id), waiting_.end());
      swapped_.erase(std::remove(swapped_.begin(), swapped_.end(), g.id), swapped_.end());
      ++stats_.finished;
    }
  }
}

void Scheduler::preempt(int64_t gid, Batch* out) {
  Group& g = groups_.at(gid);
  ++stats_.num_preemptions;
  ++g.num_preemptions;
  out->preempted_groups.push_back(gid);
  bool can_swap = cfg_.preemption == Preempt::SWAP;
  if (can_swap) {
    int need = 0;
    for (int64_t sid : g.seqs)
      if (seqs_.at(sid).status == SeqStatus::RUNNING)
        need += static_cast<int>(bm_->table(sid).size());
    can_swap = need <= bm_->num_free_cpu();
  }
  if (can_swap) {
    for (int64_t sid : g.seqs) {
      Sequence& s = seqs_.at(sid);
      if (s.status != SeqStatus::RUNNING) continue;
      bm_->swap_out(sid, &out->swap_out);
      s.status = SeqStatus::SWAPPED;
    }
    ++stats_.num_swapped_out;
    swapped_.push_back(gid);
  } else {
    for (int64_t sid : g.seqs) {
      Sequence& s = seqs_.at(sid);
      if (s.status != SeqStatus::RUNNING) continue;
      bm_->free(sid);
      s.num_computed = 0;
      s.status = SeqStatus::WAITING;
    }
    insert_waiting(gid, true);
  }
}

std::unique_ptr<Batch> Scheduler::schedule(double now) {
  auto out = std::make_unique<Batch>();
  ++stats_.steps;
  int64_t budget = cfg_.max_num_batched_tokens;
  int seq_budget = cfg_.max_num_seqs;
  struct Item {
    int64_t seq, n, gid;
  };
  std::vector<Item> items;
  bool preempted = false;
  const int extra = cfg_.num_speculative_tokens;

  // Try to give a RUNNING group its next tokens. Returns 1 = scheduled,
  // 0 = did not fit the budget (stop), -1 = the group itself was preempted.
  auto schedule_running = [&](size_t idx) -> int {
    int64_t gid = running_[idx];
    Group& g = groups_.at(gid);
    std::vector<std::pair<int64_t, int64_t>> want;  // seq, n
    int64_t total = 0;
    for (int64_t sid : g.seqs) {
      Sequence& s = seqs_.at(sid);
      if (s.status != SeqStatus::RUNNING) continue;
      int64_t rem = static_cast<int64_t>(s.tokens.size()) - s.num_computed;
      if (rem <= 0) continue;
      want.push_back({sid, rem});
      total += rem;
    }
    if (want.empty()) return 1;
    if (total > budget) {
      if (!cfg_.enable_chunked_prefill || want.size() != 1 || budget <= 0) return 0;
      want[0].second = budget;
      total = budget;
    }
    if (static_cast<int>(want.size()) > seq_budget) return 0;
    for (;;) {
      int need = 0;
      for (auto& w : want) {
        const Sequence& s = seqs_.at(w.first);
        int64_t end = s.num_computed + w.second;
        // reserve speculative slots whenever the step reaches the last token
        if (extra > 0 && end == static_cast<int64_t>(s.tokens.size())) end += extra;
        need += bm_->blocks_to_grow(w.first, s.num_computed, end);
      }
      if (bm_->can_allocate(need, false)) break;
      preempted = true;
      if (running_.size() - 1 > idx) {
        int64_t victim = running_.back();
        running_.pop_back();
        preempt(victim, out.get());
      } else {
        running_.erase(running_.begin() + idx);
        preempt(gid, out.get());
        return -1;
      }
    }
    for (auto& w : want) {
      Sequence& s = seqs_.at(w.first);
      int64_t end = s.num_computed + w.second;
      if (extra > 0 && end == static_cast<int64_t>(s.tokens.size())) end += extra;
      bm_->ensure_slots(w.first, s.num_computed, end, &out->copies);
      items.push_back({w.first, w.second, gid});
    }
    budget -= total;
    seq_budget -= static_cast<int>(want.size());
    if (g.first_scheduled < 0) g.first_scheduled = now;
    return 1;
  };

  // 1. running groups, highest priority first
  for (size_t i = 0; i < running_.size();) {
    int r = schedule_running(i);
    if (r == 0) break;
    if (r == 1) ++i;
  }

  // 2. swapped groups come back before anything new is admitted
  if (!preempted) {
    while (!swapped_.empty() && budget > 0 && seq_budget > 0) {
      int64_t gid = swapped_.front();
      Group& g = groups_.at(gid);
      int need = 0;
      for (int64_t sid : g.seqs) {
        Sequence& s = seqs_.at(sid);
        if (s.status == SeqStatus::SWAPPED)
          need += bm_->blocks_needed(static_cast<int64_t>(s.tokens.size()) + extra);
      }
      if (!bm_->can_allocate(need, true)) {
        if (running_.empty() && items.empty() &&
            need > bm_->num_gpu_blocks() - bm_->watermark_blocks()) {
          // can never come back: end it rather than wait forever
          swapped_.pop_front();
          for (int64_t sid : g.seqs) {
            Sequence& s = seqs_.at(sid);
            if (s.status != SeqStatus::SWAPPED) continue;
            bm_->free(sid);
            s.status = SeqStatus::FINISHED_LENGTH;
          }
          ++stats_.finished;
          out->preempted_groups.push_back(-gid);
          continue;
        }
        break;
      }
      swapped_.pop_front();
      for (int64_t sid : g.seqs) {
        Sequence& s = seqs_.at(sid);
        if (s.status != SeqStatus::SWAPPED) continue;
        bm_->swap_in(sid, &out->swap_in);
        s.status = SeqStatus::RUNNING;
      }
      ++stats_.num_swapped_in;
      // keep running_ ordered by priority
      auto it = running_.begin();
      while (it != running_.end() && !before(g, groups_.at(*it))) ++it;
      size_t pos = static_cast<size_t>(it - running_.begin());
      running_.insert(it, gid);
      int r = schedule_running(pos);
      if (r == 0) break;
    }
  }

  // 3. new (or recompute-preempted) prefills
  if (!preempted && swapped_.empty()) {
    while (!waiting_.empty() && budget > 0 && seq_budget > 0) {
      int64_t gid = waiting_.front();
      Group& g = groups_.at(gid);
      std::vector<std::pair<int64_t, int64_t>> want;
      int64_t total = 0;
      for (int64_t sid : g.seqs) {
        Sequence& s = seqs_.at(sid);
        if (s.status != SeqStatus::WAITING) continue;
        if (!bm_->has(sid)) {
          int64_t len = static_cast<int64_t>(s.tokens.size());
          int maxb = static_cast<int>((len - 1) / bm_->block_size());
          int64_t hit = bm_->allocate_cached_prefix(sid, s.tokens.data(), len, maxb);
          stats_.prefix_cache_query_tokens += len;
          stats_.prefix_cache_hit_tokens += hit;
          s.num_computed = hit;
        }
        int64_t rem = static_cast<int64_t>(s.tokens.size()) - s.num_computed;
        want.push_back({sid, rem});
        total += rem;
      }
      bool fits = true;
      if (total > budget) {
        if (cfg_.enable_chunked_prefill && want.size() == 1) {
          want[0].second = budget;
          total = budget;
        } else {
          fits = false;
        }
      }
      if (static_cast<int>(want.size()) > seq_budget) fits = false;
      int need = 0;
      if (fits) {
        for (auto& w : want) {
          const Sequence& s = seqs_.at(w.first);
          need += bm_->blocks_to_grow(w.first, s.num_computed, s.num_computed + w.second);
        }
        fits = bm_->can_allocate(need, true);
      }
      if (!fits) {
        // give back prefix-cache references taken above; they are retaken next step
        for (auto& w : want) {
          Sequence& s = seqs_.at(w.first);
          bm_->free(w.first);
          s.num_computed = 0;
        }
        // a prompt that can never fit must not block the queue forever
        if (items.empty() && running_.empty() &&
            need > bm_->num_gpu_blocks() - bm_->watermark_blocks()) {
          waiting_.pop_front();
          for (auto& w : want) seqs_.at(w.first).status = SeqStatus::FINISHED_LENGTH;
          ++stats_.finished;
          out->preempted_groups.push_back(-gid);  // negative: rejected
          continue;
        }
        break;
      }
      waiting_.pop_front();
      for (auto& w : want) {
        Sequence& s = seqs_.at(w.first);
        bm_->ensure_slots(w.first, s.num_computed, s.num_computed + w.second, &out->copies);
        s.status = SeqStatus::RUNNING;
        items.push_back({w.first, w.second, gid});
      }
      budget -= total;
      seq_budget -= static_cast<int>(want.size());
      if (g.first_scheduled < 0) g.first_scheduled = now;
      auto it = running_.begin();
      while (it != running_.end() && !before(g, groups_.at(*it))) ++it;
      running_.insert(it, gid);
    }
  }

  // ---- build the flat batch: query length 1 first (decode kernel), then the rest
  std::stable_sort(items.begin(), items.end(),
                   [](const Item& a, const Item& b) { return (a.n == 1) > (b.n == 1); });
  Batch& b = *out;
  b.num_seqs = static_cast<int>(items.size());
  int max_blocks = 0;
  for (auto& it : items) {
    const Sequence& s = seqs_.at(it.seq);
    max_blocks = std::max(max_blocks, bm_->blocks_needed(s.num_computed + it.n));
    b.num_tokens += it.n;
    if (it.n == 1) ++b.num_decode_seqs;
  }
  b.max_blocks = max_blocks;
  b.input_ids.reserve(b.num_tokens);
  b.positions.reserve(b.num_tokens);
  b.slot_mapping.reserve(b.num_tokens);
  b.block_tables.assign(static_cast<size_t>(b.num_seqs) * max_blocks, -1);
  b.q_start.push_back(0);
  const int bs = bm_->block_size();
  int logits_rows = 0;
  for (int r = 0; r < b.num_seqs; ++r) {
    const Item& it = items[r];
    Sequence& s = seqs_.at(it.seq);
    Group& g = groups_.at(it.gid);
    const auto& tab = bm_->table(it.seq);
    for (size_t j = 0; j < tab.size() && static_cast<int>(j) < max_blocks; ++j)
      b.block_tables[static_cast<size_t>(r) * max_blocks + j] = tab[j];
    for (int64_t p = s.num_computed; p < s.num_computed + it.n; ++p) {
      b.input_ids.push_back(s.tokens[p]);
      b.positions.push_back(static_cast<int32_t>(p));
      b.slot_mapping.push_back(tab[p / bs] * bs + static_cast<int32_t>(p % bs));
    }
    int64_t end = s.num_computed + it.n;
    b.q_len.push_back(static_cast<int32_t>(it.n));
    b.seq_len.push_back(static_cast<int32_t>(end));
    b.q_start.push_back(b.q_start.back() + static_cast<int32_t>(it.n));
    b.seq_ids.push_back(it.seq);
    b.max_q_len = std::max<int>(b.max_q_len, static_cast<int>(it.n));
    b.max_seq_len = std::max<int>(b.max_seq_len, static_cast<int>(end));
    if ((it.n > 1 && s.num_draft == 0) || s.num_output() == 0) b.num_prefill_tokens += it.n;
    else stats_.decode_tokens += it.n;
    bool samples = end == static_cast<int64_t>(s.tokens.size());
    s.num_computed = end;
    if (!samples) continue;
    int lrow = logits_rows++;
    int copies = 1;
    if (g.params.n > 1 && !g.forked && s.num_output() == 0 && g.seqs.size() == 1)
      copies = g.params.n;
    for (int c = 0; c < copies; ++c) {
      const GroupParams& p = g.params;
      b.sample_logit_idx.push_back(lrow);
      b.sample_seq_row.push_back(r);
      b.sample_target_seq.push_back(c == 0 ? it.seq : -1);
      b.sample_group.push_back(it.gid);
      b.temperature.push_back(p.temperature);
      b.top_p.push_back(p.top_p);
      b.top_k.push_back(p.top_k);
      b.min_p.push_back(p.min_p);
      b.presence.push_back(p.presence_penalty);
      b.frequency.push_back(p.frequency_penalty);
      b.repetition.push_back(p.repetition_penalty);
      b.seed.push_back(p.seed);
      int child = 0;
      for (size_t q = 0; q < g.seqs.size(); ++q)
        if (g.seqs[q] == it.seq) child = static_cast<int>(q);
      b.step_idx.push_back(static_cast<int32_t>(s.num_output()) + ((child + c) << 20));
      if (p.presence_penalty != 0.f || p.frequency_penalty != 0.f || p.repetition_penalty != 1.f)
        b.any_penalty = true;
      if (p.temperature > 0.f && p.top_k != 1) b.any_random = true;
    }
  }
  stats_.prefill_tokens += b.num_prefill_tokens;
  return out;
}

void Scheduler::finish_group_if_done(int64_t gid, double now, StepResult* res) {
  Group& g = groups_.at(gid);
  for (int64_t sid : g.seqs) {
    auto st = seqs_.at(sid).status;
    if (st == SeqStatus::RUNNING || st == SeqStatus::WAITING || st == SeqStatus::SWAPPED) return;
  }
  if (g.finished >= 0) return;
  g.finished = now;
  running_.erase(std::remove(running_.begin(), running_.end(), gid), running_.end());
  ++stats_.finished;
  res->finished_groups.push_back(gid);
}

StepResult Scheduler::update(const Batch& b, const int32_t* tokens, const float* logprobs,
                             double now) {
  std::vector<int32_t> ones(b.sample_logit_idx.size(), 1);
  return update_multi(b, tokens, ones.data(), logprobs, now);
}

StepResult Scheduler::update_multi(const Batch& b, const int32_t* tokens, const int32_t* counts,
                                   const float* logprobs, double now) {
  StepResult res;
  std::vector<int64_t> touched;
  // register newly full blocks for prefix caching before any sequence of this
  // step finishes and returns its blocks
  if (bm_->prefix_caching()) {
    for (int64_t sid : b.seq_ids) {
      auto it = seqs_.find(sid);
      if (it == seqs_.end()) continue;
      Sequence& s = it->second;
      if (s.status == SeqStatus::RUNNING)
        bm_->register_full_blocks(sid, s.tokens.data(), s.num_computed);
    }
  }
  const size_t rows = b.sample_logit_idx.size();
  std::vector<int64_t> first(rows + 1, 0);
  for (size_t r = 0; r < rows; ++r) first[r + 1] = first[r] + counts[r];
  // children (n > 1) fork from the parent's prompt before the parent appends
  std::vector<size_t> order;
  order.reserve(rows);
  for (size_t r = 0; r < rows; ++r)
    if (b.sample_target_seq[r] < 0) order.push_back(r);
  for (size_t r = 0; r < rows; ++r)
    if (b.sample_target_seq[r] >= 0) order.push_back(r);
  for (size_t r : order) {
    int64_t gid = b.sample_group[r];
    auto git = groups_.find(gid);
    if (git == groups_.end()) continue;
    Group& g = git->second;
    int64_t sid = b.sample_target_seq[r];
    if (sid < 0) {
      // n > 1: fork a child from the parent's prompt (shares its KV blocks)
      int64_t parent = g.seqs[0];
      Sequence& ps = seqs_.at(parent);
      if (ps.status != SeqStatus::RUNNING) continue;
      Sequence c;
      c.id = next_seq_++;
      c.group = gid;
      c.tokens.assign(ps.tokens.begin(), ps.tokens.begin() + ps.num_prompt);
      c.num_prompt = ps.num_prompt;
      c.num_computed = ps.num_prompt;
      c.status = SeqStatus::RUNNING;
      bm_->fork(parent, c.id);
      sid = c.id;
      g.seqs.push_back(c.id);
      seqs_.emplace(c.id, std::move(c));
      g.forked = true;
    }
    auto sit = seqs_.find(sid);
    if (sit == seqs_.end()) continue;
    Sequence& s = sit->second;
    if (s.status != SeqStatus::RUNNING) continue;  // aborted meanwhile
    // a negative token marks a row the caller handles itself (beam search)
    if (first[r + 1] > first[r] && tokens[first[r]] < 0) continue;
    const GroupParams& p = g.params;
    for (int64_t q = first[r]; q < first[r + 1]; ++q) {
      int32_t tok = tokens[q];
      s.tokens.push_back(tok);
      if (logprobs) s.cum_logprob += logprobs[q];
      if (g.first_token < 0) g.first_token = now;
      res.group.push_back(gid);
      res.seq.push_back(sid);
      res.token.push_back(tok);
      res.row.push_back(static_cast<int32_t>(r));
      int64_t nout = s.num_output();
      SeqStatus fin = SeqStatus::RUNNING;
      if (nout >= p.min_tokens) {
        if (!p.ignore_eos && p.eos_token_id >= 0 && tok == p.eos_token_id)
          fin = SeqStatus::FINISHED_STOPPED;
        else if (std::find(p.stop_token_ids.begin(), p.stop_token_ids.end(), tok) !=
                 p.stop_token_ids.end())
          fin = SeqStatus::FINISHED_STOPPED;
      }
      if (fin == SeqStatus::RUNNING &&
          (nout >= p.max_tokens || static_cast<int64_t>(s.tokens.size()) >= cfg_.max_model_len))
        fin = SeqStatus::FINISHED_LENGTH;
      if (fin != SeqStatus::RUNNING) {
        free_seq(s);
        s.status = fin;
        break;
      }
    }
    // tokens verified by this step already have their KV; only the newest
    // one still needs computing
    if (s.status == SeqStatus::RUNNING)
      s.num_computed = std::max<int64_t>(s.num_computed, static_cast<int64_t>(s.tokens.size()) - 1);
    touched.push_back(gid);
  }
  std::sort(touched.begin(), touched.end());
  touched.erase(std::unique(touched.begin(), touched.end()), touched.end());
  for (int64_t gid : touched) finish_group_if_done(gid, now, &res);
  return res;
}

StepResult Scheduler::beam_update(int64_t gid, const std::vector<int64_t>& live_parent,
                                  const std::vector<int32_t>& live_token,
                                  const std::vector<float>& live_logprob,
                                  const std::vector<int64_t>& fin_parent,
                                  const std::vector<int32_t>& fin_token,
                                  const std::vector<float>& fin_logprob, double now) {
  StepResult res;
  if (live_parent.size() != live_token.size() || live_parent.size() != live_logprob.size() ||
      fin_parent.size() != fin_token.size() || fin_parent.size() != fin_logprob.size())
    throw std::invalid_argument("beam_update: mismatched candidate arrays");
  auto git = groups_.find(gid);
  if (git == groups_.end()) return res;
  Group& g = git->second;
  for (int64_t p : live_parent)
    if (std::find(g.seqs.begin(), g.seqs.end(), p) == g.seqs.end() || seqs_.at(p).status != SeqStatus::RUNNING)
      throw std::invalid_argument("beam_update: parent is not a running beam of the group");
  for (int64_t p : fin_parent)
    if (std::find(g.seqs.begin(), g.seqs.end(), p) == g.seqs.end() || seqs_.at(p).status != SeqStatus::RUNNING)
      throw std::invalid_argument("beam_update: parent is not a running beam of the group");
  if (g.first_token < 0) g.first_token = now;
  auto record = [&](int64_t sid, int32_t tok) {
    res.group.push_back(gid);
    res.seq.push_back(sid);
    res.token.push_back(tok);
    res.row.push_back(-1);
  };
  // finished hypotheses: copies of the parent's tokens plus the final token
  for (size_t j = 0; j < fin_parent.size(); ++j) {
    const Sequence& ps = seqs_.at(fin_parent[j]);
    Sequence c;
    c.id = next_seq_++;
    c.group = gid;
    c.tokens = ps.tokens;
    c.tokens.push_back(fin_token[j]);
    c.num_prompt = ps.num_prompt;
    c.num_computed = 0;
    c.cum_logprob = ps.cum_logprob + fin_logprob[j];
    c.status = SeqStatus::FINISHED_STOPPED;
    record(c.id, fin_token[j]);
    g.seqs.push_back(c.id);
    seqs_.emplace(c.id, std::move(c));
  }
  // live beams: forks first (they copy the parent before it appends)
  std::vector<int64_t> target(live_parent.size(), -1);
  std::vector<int64_t> claimed;
  for (size_t j = 0; j < live_parent.size(); ++j) {
    const int64_t p = live_parent[j];
    if (std::find(claimed.begin(), claimed.end(), p) == claimed.end()) {
      claimed.push_back(p);
      target[j] = p;
    }
  }
  for (size_t j = 0; j < live_parent.size(); ++j) {
    if (target[j] >= 0) continue;
    const Sequence& ps = seqs_.at(live_parent[j]);
    Sequence c;
    c.id = next_seq_++;
    c.group = gid;
    c.tokens = ps.tokens;
    c.num_prompt = ps.num_prompt;
    c.num_computed = ps.num_computed;
    c.cum_logprob = ps.cum_logprob;
    c.status = SeqStatus::RUNNING;
    bm_->fork(ps.id, c.id);
    target[j] = c.id;
    g.seqs.push_back(c.id);
    seqs_.emplace(c.id, std::move(c));
  }
  // running beams that no live child continues leave the group
  std::vector<int64_t> keep;
  for (int64_t sid : g.seqs) {
    Sequence& s = seqs_.at(sid);
    const bool old_live = s.status == SeqStatus::RUNNING &&
                          std::find(target.begin(), target.end(), sid) == target.end();
    if (old_live) {
      free_seq(s);
      seqs_.erase(sid);
    } else {
      keep.push_back(sid);
    }
  }
  g.seqs = keep;
  const GroupParams& p = g.params;
  for (size_t j = 0; j < live_parent.size(); ++j) {
    Sequence& s = seqs_.at(target[j]);
    s.tokens.push_back(live_token[j]);
    s.cum_logprob += live_logprob[j];
    record(s.id, live_token[j]);
    if (s.num_output() >= p.max_tokens || static_cast<int64_t>(s.tokens.size()) >= cfg_.max_model_len) {
      free_seq(s);
      s.status = SeqStatus::FINISHED_LENGTH;
    } else {
      s.num_computed = static_cast<int64_t>(s.tokens.size()) - 1;
    }
  }
  finish_group_if_done(gid, now, &res);
  return res;
}

void Scheduler::append_tokens(int64_t sid, const std::vector<int32_t>& toks) {
  Sequence& s = seqs_.at(sid);
  if (s.status != SeqStatus::RUNNING) throw std::invalid_argument("append to a sequence that is not running");
  s.tokens.insert(s.tokens.end(), toks.begin(), toks.end());
  s.num_draft += static_cast<int64_t>(toks.size());
}

void Scheduler::rollback(int64_t sid, int64_t n) {
  Sequence& s = seqs_.at(sid);
  if (n <= 0) return;
  if (n > s.num_output()) throw std::invalid_argument("rollback past the prompt");
  s.tokens.resize(s.tokens.size() - n);
  s.num_draft = std::max<int64_t>(0, s.num_draft - n);
  const int64_t last = static_cast<int64_t>(s.tokens.size()) - 1;
  if (s.num_computed > last) s.num_computed = last;
}

std::vector<int64_t> Scheduler::decode_ready_seqs() const {
  std::vector<int64_t> out;
  for (int64_t gid : running_) {
    const Group& g = groups_.at(gid);
    for (int64_t sid : g.seqs) {
      const Sequence& s = seqs_.at(sid);
      if (s.status == SeqStatus::RUNNING && s.num_output() > 0 &&
          s.num_computed + 1 == static_cast<int64_t>(s.tokens.size()))
        out.push_back(sid);
    }
  }
  return out;
}

const Group* Scheduler::group(int64_t gid) const {
  auto it = groups_.find(gid);
  return it == groups_.end() ? nullptr : &it->second;
}

const Group* Scheduler::group_by_request(const std::string& rid) const {
  auto it = by_request_.find(rid);
  return it == by_request_.end() ? nullptr : group(it->second);
}

const Sequence* Scheduler::seq(int64_t sid) const {
  auto it = seqs_.find(sid);
  return it == seqs_.end() ? nullptr : &it->second;
}

void Scheduler::release_group(int64_t gid) {
  auto it = groups_.find(gid);
  if (it == groups_.end()) return;
  for (int64_t sid : it->second.seqs) {
    auto s = seqs_.find(sid);
    if (s != seqs_.end()) {
      if (s->second.status == SeqStatus::RUNNING || s->second.status == SeqStatus::WAITING ||
          s->second.status == SeqStatus::SWAPPED)
        return;  // still live
      seqs_.erase(s);
    }
  }
  by_request_.erase(it->second.request_id);
  groups_.erase(it);
}

}  // namespace swift
