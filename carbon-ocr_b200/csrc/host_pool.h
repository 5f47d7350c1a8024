// A fork-join pool for a recognize call's per-line host work (a run's layout: crop regions,
// checks, descriptors, masks, claim keys).  run(parts, f) calls f(part) for every part of
// [0, parts): the caller and the pool's threads take parts from a shared counter until none is
// left, and run returns once every part is done and no thread still holds the job.  Between
// calls the threads sleep on a condition variable.
#pragma once

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace crec {

class HostPool {
 public:
  explicit HostPool(int workers) {
    for (int i = 0; i < workers; ++i) th_.emplace_back([this] { loop(); });
  }

  ~HostPool() {
    {
      std::lock_guard<std::mutex> lk(m_);
      stop_ = true;
    }
    cv_.notify_all();
    for (std::thread& t : th_) t.join();
  }

  HostPool(const HostPool&) = delete;
  HostPool& operator=(const HostPool&) = delete;

  // threads that work on a job, the caller's included
  int threads() const { return static_cast<int>(th_.size()) + 1; }

  void run(int parts, const std::function<void(int)>& f) {
    if (parts <= 0) return;
    if (th_.empty() || parts == 1) {
      for (int i = 0; i < parts; ++i) f(i);
      return;
    }
    {
      std::lock_guard<std::mutex> lk(m_);
      job_ = &f;
      parts_ = parts;
      next_.store(0, std::memory_order_relaxed);
      done_.store(0, std::memory_order_relaxed);
      ++gen_;
    }
    cv_.notify_all();
    claim(f, parts);
    // every part done, then no thread may still hold this job (a thread takes it under the lock,
    // so once the caller clears it there with none active, none can take it later)
    for (;; std::this_thread::yield()) {
      if (done_.load(std::memory_order_acquire) < parts) continue;
      std::lock_guard<std::mutex> lk(m_);
      if (active_ == 0) {
        job_ = nullptr;
        return;
      }
    }
  }

 private:
  void claim(const std::function<void(int)>& f, int parts) {
    for (int i; (i = next_.fetch_add(1, std::memory_order_relaxed)) < parts;) {
      f(i);
      done_.fetch_add(1, std::memory_order_release);
    }
  }

  void loop() {
    unsigned long long seen = 0;
    std::unique_lock<std::mutex> lk(m_);
    for (;;) {
      cv_.wait(lk, [&] { return stop_ || (job_ && gen_ != seen); });
      if (stop_) return;
      seen = gen_;
      const std::function<void(int)>* f = job_;
      const int parts = parts_;
      ++active_;
      lk.unlock();
      claim(*f, parts);
      lk.lock();
      --active_;
    }
  }

  std::vector<std::thread> th_;
  std::mutex m_;
  std::condition_variable cv_;
  bool stop_ = false;
  const std::function<void(int)>* job_ = nullptr;  // under m_
  int parts_ = 0;                                  // under m_
  int active_ = 0;                                 // threads holding the job, under m_
  unsigned long long gen_ = 0;                     // under m_
  std::atomic<int> next_{0}, done_{0};
};

}  // namespace crec
