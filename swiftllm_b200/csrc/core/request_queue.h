// Thread-safe admission queue between API threads and the engine thread.
//
// Parity: crates/swiftllm-core/src/scheduler/request_queue.rs
//   (RequestQueueConfig :15-39, enqueue with QueueFull :114-152,
//    dequeue / dequeue_timeout :155-202, dequeue_batch :205-236, remove
//    :239-262, stop_accepting / start_accepting :285-297, drain_timeouts
//    :300-338, QueueStats :349-405).
// The reference's `remove` keeps stale positions after pops; entries here
// are looked up by id, so removal is always exact.
#pragma once
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <mutex>
#include <string>
#include <vector>

namespace swift {

struct QueueEntry {
  std::string id;
  int64_t handle = 0;  // caller-side payload key
  int priority = 0;
  double enqueue_time = 0;  // seconds, steady clock
};

struct QueueStats {
  int64_t enqueued = 0, dequeued = 0, rejected = 0, timed_out = 0, removed = 0;
  double total_wait = 0, max_wait = 0;
  double avg_wait() const { return dequeued ? total_wait / dequeued : 0.0; }
};

enum class EnqueueStatus : int { OK = 0, FULL = 1, CLOSED = 2 };

class RequestQueue {
 public:
  RequestQueue(size_t max_size, bool enable_priority, double max_wait_secs)
      : max_size_(max_size), enable_priority_(enable_priority), max_wait_(max_wait_secs) {}

  static double now() {
    using namespace std::chrono;
    return duration<double>(steady_clock::now().time_since_epoch()).count();
  }

  EnqueueStatus enqueue(const std::string& id, int64_t handle, int priority) {
    std::lock_guard<std::mutex> lk(mu_);
    if (!accepting_) {
      ++stats_.rejected;
      return EnqueueStatus::CLOSED;
    }
    if (max_size_ && size_locked() >= max_size_) {
      ++stats_.rejected;
      return EnqueueStatus::FULL;
    }
    QueueEntry e{id, handle, priority, now()};
    if (enable_priority_ && priority > 0) high_.push_back(e); else normal_.push_back(e);
    ++stats_.enqueued;
    cv_.notify_one();
    return EnqueueStatus::OK;
  }

  // Pops one entry; waits up to `timeout` seconds (<0: forever, 0: no wait).
  bool dequeue(QueueEntry* out, double timeout) {
    std::unique_lock<std::mutex> lk(mu_);
    auto ready = [&] { return size_locked() > 0 || closed_; };
    if (timeout < 0) cv_.wait(lk, ready);
    else if (timeout > 0)
      cv_.wait_for(lk, std::chrono::duration<double>(timeout), ready);
    return pop_locked(out);
  }

  std::vector<QueueEntry> dequeue_batch(size_t max_n) {
    std::lock_guard<std::mutex> lk(mu_);
    std::vector<QueueEntry> v;
    QueueEntry e;
    while (v.size() < max_n && pop_locked(&e)) v.push_back(e);
    return v;
  }

  bool remove(const std::string& id) {
    std::lock_guard<std::mutex> lk(mu_);
    for (auto* q : {&high_, &normal_})
      for (auto it = q->begin(); it != q->end(); ++it)
        if (it->id == id) {
          q->erase(it);
          ++stats_.removed;
          return true;
        }
    return false;
  }

  // Remove and return entries older than max_wait_secs.
  std::vector<QueueEntry> drain_timeouts() {
    std::lock_guard<std::mutex> lk(mu_);
    std::vector<QueueEntry> out;
    if (max_wait_ <= 0) return out;
    double t = now();
    for (auto* q : {&high_, &normal_})
      for (auto it = q->begin(); it != q->end();) {
        if (t - it->enqueue_time > max_wait_) {
          out.push_back(*it);
          it = q->erase(it);
          ++stats_.timed_out;
        } else {
          ++it;
        }
      }
    return out;
  }

  void stop_accepting() {
    std::lock_guard<std::mutex> lk(mu_);
    accepting_ = false;
  }
  void start_accepting() {
    std::lock_guard<std::mutex> lk(mu_);
    accepting_ = true;
  }
  bool accepting() const {
    std::lock_guard<std::mutex> lk(mu_);
    return accepting_;
  }
  // Wake every waiter; dequeue returns false once empty.
  void close() {
    std::lock_guard<std::mutex> lk(mu_);
    closed_ = true;
    accepting_ = false;
    cv_.notify_all();
  }
  size_t size() const {
    std::lock_guard<std::mutex> lk(mu_);
    return size_locked();
  }
  size_t priority_size() const {
    std::lock_guard<std::mutex> lk(mu_);
    return high_.size();
  }
  QueueStats stats() const {
    std::lock_guard<std::mutex> lk(mu_);
    return stats_;
  }

 private:
  size_t size_locked() const { return high_.size() + normal_.size(); }
  bool pop_locked(QueueEntry* out) {
    std::deque<QueueEntry>* q = !high_.empty() ? &high_ : (!normal_.empty() ? &normal_ : nullptr);
    if (!q) return false;
    *out = q->front();
    q->pop_front();
    double w = now() - out->enqueue_time;
    ++stats_.dequeued;
    stats_.total_wait += w;
    if (w > stats_.max_wait) stats_.max_wait = w;
    return true;
  }

  size_t max_size_;
  bool enable_priority_;
  double max_wait_;
  bool accepting_ = true, closed_ = false;
  mutable std::mutex mu_;
  std::condition_variable cv_;
  std::deque<QueueEntry> high_, normal_;
  QueueStats stats_;
};

}  // namespace swift
