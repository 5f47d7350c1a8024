// Host -> device upload of page rows from pageable memory, for crec_set_pages and
// crec_prefetch_pages (the reference's CudaModels::upload, carbon/src/cuda/pipeline_cuda.cpp:606-651,
// stages a group's rows through a pinned mirror of the whole group from one thread).
//
// Here: a few worker threads, each with two pinned chunks of its own.  The rows to send are cut
// into pieces of at most a chunk; piece k goes to worker k % workers, which waits until its chunk's
// previous copy has left (an event), copies the piece's rows into it (memcpy), and queues the chunk's
// copy to the device on the copy stream.  Several memcpys run at once, so the host side keeps up
// with the bus; the copy engine sends one chunk while the workers fill the next ones.  Pages in
// pinned (page-locked) memory skip all this: the caller copies them straight from where they are.
//
// A chunk is written once by its worker and then read only by the copy engine, so the workers
// write it with streaming (non-temporal) stores: no read of each destination line into the cache
// before it is overwritten (an ordinary memcpy's read-for-ownership), one pass over host memory
// fewer for every byte sent, and the caches left to the page rows being read.  A store fence
// orders a chunk's stores before its copy is queued.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>
#if defined(__x86_64__) || defined(_M_X64)
#include <emmintrin.h>
#define CREC_STREAM_STORES 1
#endif

namespace crec {

// n bytes from src to dst with streaming stores of 16 bytes where dst is 16-byte aligned (its
// unaligned head and the tail by memcpy); a plain memcpy where the target has no such stores.
inline void copy_streaming(uint8_t* dst, const uint8_t* src, size_t n) {
#ifdef CREC_STREAM_STORES
  const size_t head = std::min(n, static_cast<size_t>((16 - (reinterpret_cast<uintptr_t>(dst) & 15)) & 15));
  std::memcpy(dst, src, head);
  dst += head;
  src += head;
  n -= head;
  size_t i = 0;
  for (; i + 64 <= n; i += 64) {
    const __m128i a = _mm_loadu_si128(reinterpret_cast<const __m128i*>(src + i));
    const __m128i b = _mm_loadu_si128(reinterpret_cast<const __m128i*>(src + i + 16));
    const __m128i c = _mm_loadu_si128(reinterpret_cast<const __m128i*>(src + i + 32));
    const __m128i d = _mm_loadu_si128(reinterpret_cast<const __m128i*>(src + i + 48));
    _mm_stream_si128(reinterpret_cast<__m128i*>(dst + i), a);
    _mm_stream_si128(reinterpret_cast<__m128i*>(dst + i + 16), b);
    _mm_stream_si128(reinterpret_cast<__m128i*>(dst + i + 32), c);
    _mm_stream_si128(reinterpret_cast<__m128i*>(dst + i + 48), d);
  }
  std::memcpy(dst + i, src + i, n - i);
#else
  std::memcpy(dst, src, n);
#endif
}

// the streaming stores made so far visible before a copy engine reads their chunk
inline void stores_visible() {
#ifdef CREC_STREAM_STORES
  _mm_sfence();
#endif
}

// Rows [y0, y0 + rows) of a page (`stride` bytes apart, `width` bytes each) to device memory at
// dst, rows `width` bytes apart there.
struct RowPiece {
  const uint8_t* src;
  long long stride;
  int width, rows;
  uint8_t* dst;
};

class Stager {
 public:
  static constexpr size_t kChunk = size_t{4} << 20;

  Stager(int device, int workers) : device_(device) {
    workers = std::max(1, workers);
    w_.resize(static_cast<size_t>(workers));
    for (int i = 0; i < workers; ++i) w_[i].th = std::thread([this, i] { run(i); });
  }

  ~Stager() {
    {
      std::lock_guard<std::mutex> lk(m_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& w : w_)
      if (w.th.joinable()) w.th.join();
    for (auto& w : w_)
      for (int c = 0; c < 2; ++c) {
        if (w.host[c]) cudaFreeHost(w.host[c]);
        if (w.ev[c]) cudaEventDestroy(w.ev[c]);
      }
  }

  // Queues every piece's copy on `stream` (cut into chunks) and returns once all are queued (the
  // sources may be reused when the copies have completed on the stream, which the caller
  // orders with an event after this returns).  Returns cudaSuccess or the first error.
  cudaError_t send(const std::vector<RowPiece>& pieces, cudaStream_t stream) {
    // cut into chunk-sized pieces
    std::vector<RowPiece> cut;
    for (const RowPiece& p : pieces) {
      const int per = std::max(1, static_cast<int>(kChunk / static_cast<size_t>(std::max(1, p.width))));
      for (int r = 0; r < p.rows; r += per) {
        const int k = std::min(per, p.rows - r);
        cut.push_back({p.src + static_cast<long long>(r) * p.stride, p.stride, p.width, k,
                       p.dst + static_cast<size_t>(r) * p.width});
      }
    }
    std::unique_lock<std::mutex> lk(m_);
    job_ = &cut;
    stream_ = stream;
    err_ = cudaSuccess;
    pending_ = static_cast<int>(w_.size());
    ++gen_;
    cv_.notify_all();
    done_cv_.wait(lk, [&] { return pending_ == 0; });
    job_ = nullptr;
    return err_;
  }

 private:
  struct Worker {
    std::thread th;
    uint8_t* host[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    bool used[2] = {false, false};
  };

  void run(int i) {
    Worker& me = w_[static_cast<size_t>(i)];
    cudaSetDevice(device_);
    uint64_t seen = 0;
    for (;;) {
      const std::vector<RowPiece>* job;
      cudaStream_t stream;
      {
        std::unique_lock<std::mutex> lk(m_);
        cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
        if (stop_) return;
        seen = gen_;
        job = job_;
        stream = stream_;
      }
      cudaError_t e = cudaSuccess;
      int c = 0;
      for (size_t k = static_cast<size_t>(i); k < job->size() && e == cudaSuccess; k += w_.size()) {
        const RowPiece& p = (*job)[k];
        if (!me.host[c]) {
          e = cudaHostAlloc(reinterpret_cast<void**>(&me.host[c]), kChunk, cudaHostAllocDefault);
          if (e == cudaSuccess) e = cudaEventCreateWithFlags(&me.ev[c], cudaEventDisableTiming);
          if (e != cudaSuccess) break;
        }
        if (me.used[c] && (e = cudaEventSynchronize(me.ev[c])) != cudaSuccess) break;  // its last copy has left
        uint8_t* h = me.host[c];
        if (p.stride == p.width) {
          copy_streaming(h, p.src, static_cast<size_t>(p.rows) * p.width);
        } else {
          for (int r = 0; r < p.rows; ++r)
            copy_streaming(h + static_cast<size_t>(r) * p.width, p.src + static_cast<long long>(r) * p.stride, p.width);
        }
        stores_visible();
        e = cudaMemcpyAsync(p.dst, h, static_cast<size_t>(p.rows) * p.width, cudaMemcpyHostToDevice, stream);
        if (e == cudaSuccess) e = cudaEventRecord(me.ev[c], stream);
        me.used[c] = true;
        c ^= 1;
      }
      std::lock_guard<std::mutex> lk(m_);
      if (e != cudaSuccess && err_ == cudaSuccess) err_ = e;
      if (--pending_ == 0) done_cv_.notify_all();
    }
  }

  int device_;
  std::vector<Worker> w_;
  std::mutex m_;
  std::condition_variable cv_, done_cv_;
  bool stop_ = false;
  uint64_t gen_ = 0;
  const std::vector<RowPiece>* job_ = nullptr;
  cudaStream_t stream_ = nullptr;
  cudaError_t err_ = cudaSuccess;
  int pending_ = 0;
};

}  // namespace crec
