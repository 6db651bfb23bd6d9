// fa_host.cu - pinned host buffers and parallel staging copies for the
// host-pointer path (fa_forward_host). See fa_host.h.
//
// Why: the reference's API hands the library pageable NumPy arrays
// (python/bindings.cpp:129-131) and its own host path memcpy's them into
// shared buffers (src/flash_attn_core.cpp:320-326,388). On a discrete GPU a
// copy from pageable memory goes through the driver's bounce buffers at a
// fraction of PCIe speed; copying into pinned staging on several cores,
// piece by piece, and DMA-ing each piece as soon as it is staged keeps the
// link busy.
#include "fa_host.h"

#include <cuda_runtime.h>

#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <thread>

namespace fa {

namespace {

// ------------------------------------------------------------ pinned pool
class PinnedPool {
 public:
  void* get(size_t bytes) {
    size_t r = 4096;
    while (r < bytes) r <<= 1;
    {
      std::lock_guard<std::mutex> g(mu_);
      auto it = free_.find(r);
      if (it != free_.end() && !it->second.empty()) {
        void* p = it->second.back();
        it->second.pop_back();
        cached_ -= r;
        return p;
      }
    }
    void* p = nullptr;
    if (cudaHostAlloc(&p, r, cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      release_cached();
      if (cudaHostAlloc(&p, r, cudaHostAllocPortable) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
      }
    }
    std::lock_guard<std::mutex> g(mu_);
    size_of_[p] = r;
    return p;
  }

  void put(void* p) {
    if (!p) return;
    size_t r = 0;
    {
      std::lock_guard<std::mutex> g(mu_);
      auto it = size_of_.find(p);
      if (it == size_of_.end()) return;  // not from this pool
      r = it->second;
      if (cached_ + r <= kCachedCap) {
        free_[r].push_back(p);
        cached_ += r;
        return;
      }
      size_of_.erase(it);
    }
    cudaFreeHost(p);
    cudaGetLastError();
  }

  void release_cached() {
    std::lock_guard<std::mutex> g(mu_);
    for (auto& kv : free_)
      for (void* p : kv.second) {
        cudaFreeHost(p);
        size_of_.erase(p);
      }
    cudaGetLastError();
    free_.clear();
    cached_ = 0;
  }

 private:
  // Unused pinned memory kept for reuse; beyond it freed buffers go back to the OS.
  static constexpr size_t kCachedCap = size_t(4) << 30;
  std::mutex mu_;
  std::map<size_t, std::vector<void*>> free_;
  std::map<void*, size_t> size_of_;
  size_t cached_ = 0;
};

PinnedPool& pinned_pool() {
  static PinnedPool* p = new PinnedPool();  // never destroyed: buffers may be returned at exit
  return *p;
}

// ------------------------------------------------------------ copy workers
// Regions are cut into pieces of at most kPiece bytes; workers (and the
// waiting caller) take pieces in list order. A worker that finds no job
// spins for kSpin before sleeping, so calls made back to back (a loop of
// forward calls) find it awake instead of paying a wake-up per call.
constexpr size_t kPiece = size_t(256) << 10;
constexpr std::chrono::microseconds kSpin(2000);

inline void cpu_relax() {
#if defined(__x86_64__) || defined(__i386__)
  __builtin_ia32_pause();
#endif
}

struct Piece {
  size_t region, off, bytes;
};

class CopyPool {
 public:
  static CopyPool& get() {
    static CopyPool* p = new CopyPool();  // threads are never joined: they sleep until exit
    return *p;
  }

  std::mutex job_mu;  // held by one Stager from start() to finish()

  void begin(std::vector<CopyRegion> regions) {
    std::unique_lock<std::mutex> lk(mu_);
    if (threads_.empty()) spawn_locked();
    regions_ = std::move(regions);
    pieces_.clear();
    remaining_.reset(new std::atomic<size_t>[regions_.size() ? regions_.size() : 1]);
    for (size_t r = 0; r < regions_.size(); ++r) {
      size_t n = 0;
      for (size_t off = 0; off < regions_[r].bytes; off += kPiece, ++n)
        pieces_.push_back({r, off, std::min(kPiece, regions_[r].bytes - off)});
      remaining_[r].store(n, std::memory_order_relaxed);
    }
    n_pieces_ = pieces_.size();
    next_.store(0, std::memory_order_relaxed);
    done_.store(0, std::memory_order_relaxed);
    open_ = true;
    ++gen_;
    gen_seen_.store(gen_, std::memory_order_release);
    const bool wake = sleeping_ > 0 && n_pieces_ > 1;
    lk.unlock();
    if (wake) cv_.notify_all();
  }

  void wait(size_t i) {
    while (remaining_[i].load(std::memory_order_acquire) != 0)
      if (!run_one()) cpu_relax();
  }

  void end() {
    while (done_.load(std::memory_order_acquire) != n_pieces_)
      if (!run_one()) cpu_relax();
    // Close the job: a worker waking from now on does not join it, and the
    // ones that joined must be out of it before the next begin() rebuilds
    // the piece list.
    {
      std::lock_guard<std::mutex> g(mu_);
      open_ = false;
    }
    while (busy_.load(std::memory_order_acquire) != 0) std::this_thread::yield();
  }

 private:
  CopyPool() = default;

  void spawn_locked() {
    int n = 0;
    if (const char* env = std::getenv("FA_HOST_COPY_THREADS")) n = std::atoi(env);
    if (n <= 0) {
      // Copies saturate host memory bandwidth with a few cores (measured on
      // a B200 host: ~10 GB/s for one, ~30-37 GB/s for 2-16).
      const unsigned hw = std::thread::hardware_concurrency();
      n = (int)std::min(3u, std::max(1u, hw / 4));
    }
    for (int i = 0; i < n; ++i) threads_.emplace_back([this] { loop(); });
    for (auto& t : threads_) t.detach();
  }

  void loop() {
    uint64_t seen = 0;
    for (;;) {
      const auto t0 = std::chrono::steady_clock::now();
      while (gen_seen_.load(std::memory_order_acquire) == seen &&
             std::chrono::steady_clock::now() - t0 < kSpin)
        for (int i = 0; i < 64; ++i) cpu_relax();
      {
        std::unique_lock<std::mutex> lk(mu_);
        if (gen_ == seen) {
          ++sleeping_;
          cv_.wait(lk, [&] { return gen_ != seen; });
          --sleeping_;
        }
        seen = gen_;
        if (!open_) continue;  // woke after the job ended: wait for the next one
        busy_.fetch_add(1, std::memory_order_acq_rel);
      }
      while (run_one()) {
      }
      busy_.fetch_sub(1, std::memory_order_acq_rel);
    }
  }

  bool run_one() {
    const size_t idx = next_.fetch_add(1, std::memory_order_acq_rel);
    if (idx >= n_pieces_) return false;
    const Piece& pc = pieces_[idx];
    const CopyRegion& rg = regions_[pc.region];
    std::memcpy(static_cast<char*>(rg.dst) + pc.off, static_cast<const char*>(rg.src) + pc.off, pc.bytes);
    remaining_[pc.region].fetch_sub(1, std::memory_order_acq_rel);
    done_.fetch_add(1, std::memory_order_acq_rel);
    return true;
  }

  std::mutex mu_;
  std::condition_variable cv_;
  std::vector<std::thread> threads_;
  uint64_t gen_ = 0;
  std::atomic<uint64_t> gen_seen_{0};  // gen_, readable without the lock (spinning workers)
  int sleeping_ = 0;                   // workers waiting on cv_ (guarded by mu_)
  bool open_ = false;                  // a job is running (guarded by mu_)
  std::vector<CopyRegion> regions_;
  std::vector<Piece> pieces_;
  std::unique_ptr<std::atomic<size_t>[]> remaining_;
  size_t n_pieces_ = 0;
  std::atomic<size_t> next_{0};
  std::atomic<size_t> done_{0};
  std::atomic<int> busy_{0};
};

}  // namespace

void* pinned_get(size_t bytes) { return pinned_pool().get(bytes); }
void pinned_put(void* p) { pinned_pool().put(p); }
void pinned_release_cached() { pinned_pool().release_cached(); }

bool host_is_pinned(const void* p) {
  if (!p) return false;
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeHost;
}

Stager::~Stager() { finish(); }

void Stager::start(std::vector<CopyRegion> regions) {
  finish();
  CopyPool::get().job_mu.lock();
  active_ = true;
  CopyPool::get().begin(std::move(regions));
}

void Stager::wait(size_t i) {
  if (active_) CopyPool::get().wait(i);
}

void Stager::finish() {
  if (!active_) return;
  CopyPool::get().end();
  active_ = false;
  CopyPool::get().job_mu.unlock();
}

}  // namespace fa
