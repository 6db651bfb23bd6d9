// fa_host.h - host-memory side of the host-pointer path: a pool of pinned
// (page-locked) host buffers and a stager that copies pageable host memory
// into pinned staging with a few worker threads, so the host<->device
// copies run as DMA at full PCIe speed instead of through the driver's
// slow pageable-copy route.
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <vector>

namespace fa {

// Pinned host memory (cudaHostAlloc, portable across devices) in
// power-of-two buckets; freed buffers are kept for reuse up to a cap.
void* pinned_get(size_t bytes);   // nullptr when the allocation fails
void pinned_put(void* p);         // p from pinned_get (nullptr is ignored)
void pinned_release_cached();     // free every cached (unused) buffer

// True when `p` lies in page-locked host memory CUDA knows about (pinned
// or registered), i.e. a DMA source or destination without staging.
bool host_is_pinned(const void* p);

// One memcpy of the stager: dst <- src, `bytes` bytes.
struct CopyRegion {
  void* dst;
  const void* src;
  size_t bytes;
};

// Copies a list of regions with the worker pool, in list order. start()
// returns at once; wait(i) returns when region i is complete, the calling
// thread copying pieces itself meanwhile; finish() waits for all. One
// Stager runs at a time (start() takes the pool for the stager's life).
class Stager {
 public:
  Stager() = default;
  Stager(const Stager&) = delete;
  Stager& operator=(const Stager&) = delete;
  ~Stager();
  void start(std::vector<CopyRegion> regions);
  void wait(size_t i);
  void finish();
  bool active() const { return active_; }

 private:
  bool active_ = false;
};

}  // namespace fa
