// pybind11 module `swiftllm_b200._core`: the native engine core.
//
// Implements the surface declared (but never built) by the reference's
// python/swiftllm/_core.pyi:8-136 (RustEngine, RustBlockManager,
// RustScheduler, RustSampler, cuda_* helpers), under B200-build names, plus
// the request queue, speculative helpers and checkpoint parsers.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "block_manager.h"
#include "loaders.h"
#include "request_queue.h"
#include "sampler.h"
#include "scheduler.h"
#include "shm_channel.h"
#include "http_server.h"

namespace py = pybind11;
using namespace swift;

template <typename T>
static py::array_t<T> to_np(const std::vector<T>& v) {
  py::array_t<T> a(v.size());
  if (!v.empty()) std::memcpy(a.mutable_data(), v.data(), v.size() * sizeof(T));
  return a;
}

static py::array_t<int32_t> pairs_np(const std::vector<CopyPair>& v) {
  py::array_t<int32_t> a({static_cast<py::ssize_t>(v.size()), static_cast<py::ssize_t>(2)});
  auto m = a.mutable_unchecked<2>();
  for (size_t i = 0; i < v.size(); ++i) {
    m(i, 0) = v[i].src;
    m(i, 1) = v[i].dst;
  }
  return a;
}

static const char* status_name(SeqStatus s) {
  switch (s) {
    case SeqStatus::WAITING: return "waiting";
    case SeqStatus::RUNNING: return "running";
    case SeqStatus::SWAPPED: return "swapped";
    case SeqStatus::FINISHED_STOPPED: return "stop";
    case SeqStatus::FINISHED_LENGTH: return "length";
    case SeqStatus::FINISHED_ABORTED: return "abort";
  }
  return "?";
}

PYBIND11_MODULE(_core, m) {
  m.doc() = "swiftllm_b200 native engine core (scheduler, block manager, queue, sampler)";

  py::class_<BlockManager>(m, "BlockManager")
      .def(py::init<int, int, int, double, bool>(), py::arg("block_size"),
           py::arg("num_gpu_blocks"), py::arg("num_cpu_blocks"), py::arg("watermark") = 0.01,
           py::arg("enable_prefix_caching") = false)
      .def_property_readonly("block_size", &BlockManager::block_size)
      .def_property_readonly("num_free_gpu_blocks", &BlockManager::num_free_gpu)
      .def_property_readonly("num_free_cpu_blocks", &BlockManager::num_free_cpu)
      .def_property_readonly("num_gpu_blocks", &BlockManager::num_gpu_blocks)
      .def_property_readonly("num_cpu_blocks", &BlockManager::num_cpu_blocks)
      .def_property_readonly("watermark_blocks", &BlockManager::watermark_blocks)
      .def("blocks_needed", &BlockManager::blocks_needed)
      .def("can_allocate", &BlockManager::can_allocate, py::arg("num_blocks"),
           py::arg("keep_watermark") = false)
      .def("ensure_slots",
           [](BlockManager& bm, int64_t seq, int64_t num_computed, int64_t total) {
             std::vector<CopyPair> cow;
             bool ok = bm.ensure_slots(seq, num_computed, total, &cow);
             return py::make_tuple(ok, pairs_np(cow));
           })
      .def("allocate",
           [](BlockManager& bm, int64_t seq, int64_t num_tokens) {
             std::vector<CopyPair> cow;
             if (!bm.ensure_slots(seq, 0, num_tokens, &cow))
               throw std::runtime_error("out of KV blocks");
             return bm.table(seq);
           })
      .def("free", &BlockManager::free)
      .def("fork", &BlockManager::fork)
      .def("has", &BlockManager::has)
      .def("get_block_table", &BlockManager::table)
      .def("swap_out",
           [](BlockManager& bm, int64_t seq) {
             std::vector<CopyPair> m;
             bm.swap_out(seq, &m);
             return pairs_np(m);
           })
      .def("swap_in",
           [](BlockManager& bm, int64_t seq) {
             std::vector<CopyPair> m;
             bm.swap_in(seq, &m);
             return pairs_np(m);
           })
      .def("can_swap_in", &BlockManager::can_swap_in)
      .def("can_swap_out", &BlockManager::can_swap_out)
      .def("is_swapped", &BlockManager::is_swapped)
      .def("count_cached_blocks",
           [](const BlockManager& bm, py::array_t<int32_t, py::array::c_style> toks) {
             return bm.count_cached_blocks(toks.data(), toks.size());
           })
      .def("allocate_cached_prefix",
           [](BlockManager& bm, int64_t seq, py::array_t<int32_t, py::array::c_style> toks,
              int max_blocks) {
             return bm.allocate_cached_prefix(seq, toks.data(), toks.size(), max_blocks);
           })
      .def("register_full_blocks",
           [](BlockManager& bm, int64_t seq, py::array_t<int32_t, py::array::c_style> toks,
              int64_t n) { bm.register_full_blocks(seq, toks.data(), n); })
      .def("refcount", [](BlockManager& bm, int b) { return bm.gpu().refcount(b); })
      .def("num_cached_blocks", [](BlockManager& bm) { return bm.gpu().num_cached(); })
      .def("reset_prefix_cache", &BlockManager::reset_prefix_cache);

  py::enum_<Policy>(m, "Policy")
      .value("FCFS", Policy::FCFS)
      .value("SJF", Policy::SJF)
      .value("PRIORITY", Policy::PRIORITY);
  py::enum_<Preempt>(m, "Preempt").value("RECOMPUTE", Preempt::RECOMPUTE).value("SWAP", Preempt::SWAP);

  py::class_<SchedulerConfig>(m, "SchedulerConfig")
      .def(py::init<>())
      .def_readwrite("max_num_seqs", &SchedulerConfig::max_num_seqs)
      .def_readwrite("max_num_batched_tokens", &SchedulerConfig::max_num_batched_tokens)
      .def_readwrite("max_model_len", &SchedulerConfig::max_model_len)
      .def_readwrite("enable_chunked_prefill", &SchedulerConfig::enable_chunked_prefill)
      .def_readwrite("policy", &SchedulerConfig::policy)
      .def_readwrite("preemption", &SchedulerConfig::preemption)
      .def_readwrite("num_speculative_tokens", &SchedulerConfig::num_speculative_tokens);

  py::class_<GroupParams>(m, "GroupParams")
      .def(py::init<>())
      .def_readwrite("n", &GroupParams::n)
      .def_readwrite("max_tokens", &GroupParams::max_tokens)
      .def_readwrite("min_tokens", &GroupParams::min_tokens)
      .def_readwrite("ignore_eos", &GroupParams::ignore_eos)
      .def_readwrite("eos_token_id", &GroupParams::eos_token_id)
      .def_readwrite("stop_token_ids", &GroupParams::stop_token_ids)
      .def_readwrite("temperature", &GroupParams::temperature)
      .def_readwrite("top_p", &GroupParams::top_p)
      .def_readwrite("top_k", &GroupParams::top_k)
      .def_readwrite("min_p", &GroupParams::min_p)
      .def_readwrite("presence_penalty", &GroupParams::presence_penalty)
      .def_readwrite("frequency_penalty", &GroupParams::frequency_penalty)
      .def_readwrite("repetition_penalty", &GroupParams::repetition_penalty)
      .def_readwrite("seed", &GroupParams::seed)
      .def_readwrite("priority", &GroupParams::priority);

  py::class_<Batch>(m, "Batch")
      .def_readonly("num_seqs", &Batch::num_seqs)
      .def_readonly("num_decode_seqs", &Batch::num_decode_seqs)
      .def_readonly("num_tokens", &Batch::num_tokens)
      .def_readonly("num_prefill_tokens", &Batch::num_prefill_tokens)
      .def_readonly("max_q_len", &Batch::max_q_len)
      .def_readonly("max_seq_len", &Batch::max_seq_len)
      .def_readonly("max_blocks", &Batch::max_blocks)
      .def_readonly("any_penalty", &Batch::any_penalty)
      .def_readonly("any_random", &Batch::any_random)
      .def_property_readonly("input_ids", [](const Batch& b) { return to_np(b.input_ids); })
      .def_property_readonly("positions", [](const Batch& b) { return to_np(b.positions); })
      .def_property_readonly("slot_mapping", [](const Batch& b) { return to_np(b.slot_mapping); })
      .def_property_readonly("q_start", [](const Batch& b) { return to_np(b.q_start); })
      .def_property_readonly("q_len", [](const Batch& b) { return to_np(b.q_len); })
      .def_property_readonly("seq_len", [](const Batch& b) { return to_np(b.seq_len); })
      .def_property_readonly("seq_ids", [](const Batch& b) { return to_np(b.seq_ids); })
      .def_property_readonly("block_tables",
                             [](const Batch& b) {
                               auto a = to_np(b.block_tables);
                               return a.reshape({static_cast<py::ssize_t>(b.num_seqs),
                                                 static_cast<py::ssize_t>(b.max_blocks)});
                             })
      .def_property_readonly("sample_logit_idx", [](const Batch& b) { return to_np(b.sample_logit_idx); })
      .def_property_readonly("sample_seq_row", [](const Batch& b) { return to_np(b.sample_seq_row); })
      .def_property_readonly("sample_target_seq", [](const Batch& b) { return to_np(b.sample_target_seq); })
      .def_property_readonly("sample_group", [](const Batch& b) { return to_np(b.sample_group); })
      .def_property_readonly("temperature", [](const Batch& b) { return to_np(b.temperature); })
      .def_property_readonly("top_p", [](const Batch& b) { return to_np(b.top_p); })
      .def_property_readonly("top_k", [](const Batch& b) { return to_np(b.top_k); })
      .def_property_readonly("min_p", [](const Batch& b) { return to_np(b.min_p); })
      .def_property_readonly("presence_penalty", [](const Batch& b) { return to_np(b.presence); })
      .def_property_readonly("frequency_penalty", [](const Batch& b) { return to_np(b.frequency); })
      .def_property_readonly("repetition_penalty", [](const Batch& b) { return to_np(b.repetition); })
      .def_property_readonly("seed", [](const Batch& b) { return to_np(b.seed); })
      .def_property_readonly("step_idx", [](const Batch& b) { return to_np(b.step_idx); })
      .def_property_readonly("swap_in", [](const Batch& b) { return pairs_np(b.swap_in); })
      .def_property_readonly("swap_out", [](const Batch& b) { return pairs_np(b.swap_out); })
      .def_property_readonly("copies", [](const Batch& b) { return pairs_np(b.copies); })
      .def_readonly("preempted_groups", &Batch::preempted_groups)
      .def_property_readonly("num_sample_rows", [](const Batch& b) { return b.sample_logit_idx.size(); })
      // Pack every per-step int32 array into one buffer (one H2D copy).
      // Layout: [input_ids T | positions T | slot_mapping T | q_start S+1 |
      //          seq_len S | block_tables S*max_blocks]
      .def("pack_int32",
           [](const Batch& b) {
             size_t T = b.num_tokens, S = b.num_seqs;
             size_t n = 3 * T + (S + 1) + S + S * b.max_blocks;
             py::array_t<int32_t> a(n);
             int32_t* p = a.mutable_data();
             auto put = [&](const std::vector<int32_t>& v) {
               if (!v.empty()) std::memcpy(p, v.data(), v.size() * 4);
               p += v.size();
             };
             put(b.input_ids);
             put(b.positions);
             put(b.slot_mapping);
             put(b.q_start);
             put(b.seq_len);
             put(b.block_tables);
             return a;
           });

  py::class_<StepResult>(m, "StepResult")
      .def_property_readonly("group", [](const StepResult& r) { return to_np(r.group); })
      .def_property_readonly("seq", [](const StepResult& r) { return to_np(r.seq); })
      .def_property_readonly("token", [](const StepResult& r) { return to_np(r.token); })
      .def_property_readonly("row", [](const StepResult& r) { return to_np(r.row); })
      .def_readonly("finished_groups", &StepResult::finished_groups);

  py::class_<SchedulerStats>(m, "SchedulerStats")
      .def_readonly("num_preemptions", &SchedulerStats::num_preemptions)
      .def_readonly("num_swapped_out", &SchedulerStats::num_swapped_out)
      .def_readonly("num_swapped_in", &SchedulerStats::num_swapped_in)
      .def_readonly("prefill_tokens", &SchedulerStats::prefill_tokens)
      .def_readonly("decode_tokens", &SchedulerStats::decode_tokens)
      .def_readonly("steps", &SchedulerStats::steps)
      .def_readonly("finished", &SchedulerStats::finished)
      .def_readonly("aborted", &SchedulerStats::aborted)
      .def_readonly("prefix_cache_hit_tokens", &SchedulerStats::prefix_cache_hit_tokens)
      .def_readonly("prefix_cache_query_tokens", &SchedulerStats::prefix_cache_query_tokens);

  py::class_<Scheduler>(m, "Scheduler")
      .def(py::init<const SchedulerConfig&, BlockManager*>(), py::keep_alive<1, 3>())
      .def("add_request",
           [](Scheduler& s, const std::string& rid, py::array_t<int32_t, py::array::c_style | py::array::forcecast> prompt,
              const GroupParams& p, double arrival) {
             std::vector<int32_t> v(prompt.data(), prompt.data() + prompt.size());
             return s.add_request(rid, v, p, arrival);
           })
      .def("abort_request", &Scheduler::abort_request)
      .def("abort_group", &Scheduler::abort_group)
      .def("finish_seq",
           [](Scheduler& s, int64_t seq, const std::string& reason) {
             s.finish_seq(seq, reason == "length" ? SeqStatus::FINISHED_LENGTH
                               : reason == "abort" ? SeqStatus::FINISHED_ABORTED
                                                   : SeqStatus::FINISHED_STOPPED);
           })
      .def("schedule", &Scheduler::schedule, py::arg("now") = 0.0)
      .def("update",
           [](Scheduler& s, const Batch& b, py::array_t<int32_t, py::array::c_style | py::array::forcecast> toks,
              py::object logprobs, double now) {
             if (static_cast<size_t>(toks.size()) != b.sample_logit_idx.size())
               throw std::invalid_argument("one token per sample row expected");
             const float* lp = nullptr;
             py::array_t<float, py::array::c_style | py::array::forcecast> lpa;
             if (!logprobs.is_none()) {
               lpa = logprobs.cast<py::array_t<float, py::array::c_style | py::array::forcecast>>();
               lp = lpa.data();
             }
             return s.update(b, toks.data(), lp, now);
           },
           py::arg("batch"), py::arg("tokens"), py::arg("logprobs") = py::none(), py::arg("now") = 0.0)
      .def("update_multi",
           [](Scheduler& s, const Batch& b, py::array_t<int32_t, py::array::c_style | py::array::forcecast> toks,
              py::array_t<int32_t, py::array::c_style | py::array::forcecast> counts,
              py::object logprobs, double now) {
             if (static_cast<size_t>(counts.size()) != b.sample_logit_idx.size())
               throw std::invalid_argument("one count per sample row expected");
             int64_t total = 0;
             for (ssize_t i = 0; i < counts.size(); ++i) {
               if (counts.data()[i] < 0) throw std::invalid_argument("negative count");
               total += counts.data()[i];
             }
             if (total != toks.size()) throw std::invalid_argument("tokens do not match counts");
             const float* lp = nullptr;
             py::array_t<float, py::array::c_style | py::array::forcecast> lpa;
             if (!logprobs.is_none()) {
               lpa = logprobs.cast<py::array_t<float, py::array::c_style | py::array::forcecast>>();
               if (lpa.size() != total) throw std::invalid_argument("one logprob per token expected");
               lp = lpa.data();
             }
             return s.update_multi(b, toks.data(), counts.data(), lp, now);
           },
           py::arg("batch"), py::arg("tokens"), py::arg("counts"), py::arg("logprobs") = py::none(),
           py::arg("now") = 0.0)
      .def("decode_ready_seqs", [](const Scheduler& s) { return to_np(s.decode_ready_seqs()); })
      .def("beam_update", &Scheduler::beam_update, py::arg("group"), py::arg("live_parent"),
           py::arg("live_token"), py::arg("live_logprob"), py::arg("fin_parent"), py::arg("fin_token"),
           py::arg("fin_logprob"), py::arg("now") = 0.0)
      .def("append_tokens", &Scheduler::append_tokens)
      .def("rollback", &Scheduler::rollback)
      .def_property_readonly("num_waiting", &Scheduler::num_waiting)
      .def_property_readonly("num_running", &Scheduler::num_running)
      .def_property_readonly("num_swapped", &Scheduler::num_swapped)
      .def_property_readonly("num_unfinished", &Scheduler::num_unfinished)
      .def("has_unfinished", &Scheduler::has_unfinished)
      .def("stats", &Scheduler::stats)
      .def("group_id", [](const Scheduler& s, const std::string& rid) -> int64_t {
        const Group* g = s.group_by_request(rid);
        return g ? g->id : -1;
      })
      .def("group_info",
           [](const Scheduler& s, int64_t gid) -> py::object {
             const Group* g = s.group(gid);
             if (!g) return py::none();
             py::dict d;
             d["request_id"] = g->request_id;
             d["arrival"] = g->arrival;
             d["first_scheduled"] = g->first_scheduled;
             d["first_token"] = g->first_token;
             d["finished"] = g->finished;
             d["num_preemptions"] = g->num_preemptions;
             d["seqs"] = g->seqs;
             return d;
           })
      .def("seq_info",
           [](const Scheduler& s, int64_t sid) -> py::object {
             const Sequence* q = s.seq(sid);
             if (!q) return py::none();
             py::dict d;
             d["num_prompt"] = q->num_prompt;
             d["num_computed"] = q->num_computed;
             d["status"] = status_name(q->status);
             d["cum_logprob"] = q->cum_logprob;
             d["num_output"] = q->num_output();
             d["num_draft"] = q->num_draft;
             d["group"] = q->group;
             d["num_tokens"] = static_cast<int64_t>(q->tokens.size());
             return d;
           })
      .def("seq_tokens",
           [](const Scheduler& s, int64_t sid, bool output_only) {
             const Sequence* q = s.seq(sid);
             if (!q) throw std::invalid_argument("unknown sequence");
             std::vector<int32_t> v(q->tokens.begin() + (output_only ? q->num_prompt : 0),
                                    q->tokens.end());
             return to_np(v);
           },
           py::arg("seq"), py::arg("output_only") = true)
      .def("release_group", &Scheduler::release_group);

  py::class_<QueueEntry>(m, "QueueEntry")
      .def_readonly("id", &QueueEntry::id)
      .def_readonly("handle", &QueueEntry::handle)
      .def_readonly("priority", &QueueEntry::priority)
      .def_readonly("enqueue_time", &QueueEntry::enqueue_time);
  py::class_<QueueStats>(m, "QueueStats")
      .def_readonly("enqueued", &QueueStats::enqueued)
      .def_readonly("dequeued", &QueueStats::dequeued)
      .def_readonly("rejected", &QueueStats::rejected)
      .def_readonly("timed_out", &QueueStats::timed_out)
      .def_readonly("removed", &QueueStats::removed)
      .def_readonly("max_wait", &QueueStats::max_wait)
      .def_property_readonly("avg_wait", &QueueStats::avg_wait);
  py::enum_<EnqueueStatus>(m, "EnqueueStatus")
      .value("OK", EnqueueStatus::OK)
      .value("FULL", EnqueueStatus::FULL)
      .value("CLOSED", EnqueueStatus::CLOSED);
  py::class_<RequestQueue>(m, "RequestQueue")
      .def(py::init<size_t, bool, double>(), py::arg("max_size") = 0,
           py::arg("enable_priority") = false, py::arg("max_wait_secs") = 0.0)
      .def("enqueue", &RequestQueue::enqueue, py::arg("id"), py::arg("handle") = 0,
           py::arg("priority") = 0)
      .def("dequeue",
           [](RequestQueue& q, double timeout) -> py::object {
             QueueEntry e;
             bool ok;
             {
               py::gil_scoped_release nogil;
               ok = q.dequeue(&e, timeout);
             }
             if (!ok) return py::none();
             return py::cast(e);
           },
           py::arg("timeout") = 0.0)
      .def("dequeue_batch", &RequestQueue::dequeue_batch)
      .def("remove", &RequestQueue::remove)
      .def("drain_timeouts", &RequestQueue::drain_timeouts)
      .def("stop_accepting", &RequestQueue::stop_accepting)
      .def("start_accepting", &RequestQueue::start_accepting)
      .def_property_readonly("accepting", &RequestQueue::accepting)
      .def("close", &RequestQueue::close)
      .def("__len__", &RequestQueue::size)
      .def("priority_len", &RequestQueue::priority_size)
      .def("stats", &RequestQueue::stats);

  // ---- sampling oracle + speculative helpers
  py::class_<SampleParams>(m, "SampleParams")
      .def(py::init([](float temperature, float top_p, int top_k, float min_p, float presence,
                       float frequency, float repetition) {
             SampleParams p;
             p.temperature = temperature; p.top_p = top_p; p.top_k = top_k; p.min_p = min_p;
             p.presence = presence; p.frequency = frequency; p.repetition = repetition;
             return p;
           }),
           py::arg("temperature") = 1.0f, py::arg("top_p") = 1.0f, py::arg("top_k") = -1,
           py::arg("min_p") = 0.0f, py::arg("presence_penalty") = 0.0f,
           py::arg("frequency_penalty") = 0.0f, py::arg("repetition_penalty") = 1.0f);
  m.def("philox_uniform", &Philox::uniform, py::arg("key"), py::arg("c0"), py::arg("c1") = 0u);
  m.def("philox_block", [](uint64_t key, uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3) {
    uint32_t o[4];
    Philox::block(key, c0, c1, c2, c3, o);
    return py::make_tuple(o[0], o[1], o[2], o[3]);
  });
  m.def("sample_row",
        [](py::array_t<float, py::array::c_style | py::array::forcecast> logits,
           const SampleParams& p, float u,
           py::array_t<int32_t, py::array::c_style | py::array::forcecast> prompt,
           py::array_t<int32_t, py::array::c_style | py::array::forcecast> output) {
          std::vector<float> l(logits.data(), logits.data() + logits.size());
          apply_penalties(l.data(), static_cast<int>(l.size()), p, prompt.data(),
                          static_cast<int>(prompt.size()), output.data(),
                          static_cast<int>(output.size()));
          return sample_row(l.data(), static_cast<int>(l.size()), p, u);
        },
        py::arg("logits"), py::arg("params"), py::arg("u"),
        py::arg("prompt") = py::array_t<int32_t>(0), py::arg("output") = py::array_t<int32_t>(0));
  m.def("spec_verify",
        [](py::array_t<float, py::array::c_style | py::array::forcecast> dp,
           py::array_t<float, py::array::c_style | py::array::forcecast> tp,
           py::array_t<int32_t, py::array::c_style | py::array::forcecast> draft,
           py::array_t<float, py::array::c_style | py::array::forcecast> u) {
          int k = static_cast<int>(draft.size());
          if (tp.ndim() != 2 || tp.shape(0) != k + 1) throw std::invalid_argument("target_probs must be [k+1, V]");
          int V = static_cast<int>(tp.shape(1));
          if (k > 0 && (dp.ndim() != 2 || dp.shape(0) != k || dp.shape(1) != V))
            throw std::invalid_argument("draft_probs must be [k, V]");
          if (u.size() < 2 * k + 1) throw std::invalid_argument("need 2k+1 uniforms");
          auto r = spec_verify(dp.data(), tp.data(), draft.data(), k, V, u.data());
          return py::make_tuple(r.num_accepted, r.tokens);
        });
  py::class_<NgramSpeculator>(m, "NgramSpeculator")
      .def(py::init<int, int>(), py::arg("n") = 3, py::arg("max_k") = 8)
      .def("propose", [](const NgramSpeculator& s,
                         py::array_t<int32_t, py::array::c_style | py::array::forcecast> ctx, int k) {
        return s.propose(ctx.data(), static_cast<int>(ctx.size()), k);
      });
  py::class_<AdaptiveK>(m, "AdaptiveK")
      .def(py::init<int, int, int, double>(), py::arg("k") = 5, py::arg("min_k") = 1,
           py::arg("max_k") = 10, py::arg("target") = 0.7)
      .def("update", &AdaptiveK::update)
      .def_property_readonly("k", &AdaptiveK::k)
      .def_property_readonly("acceptance_rate", &AdaptiveK::acceptance_rate)
      .def_property_readonly("proposed", &AdaptiveK::proposed)
      .def_property_readonly("accepted", &AdaptiveK::accepted);

  bind_loaders(m);
  bind_shm_channel(m);
  bind_http_server(m);
}
