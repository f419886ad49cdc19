// arena.h -- device memory arena of the CUDA backend.
//
// Replaces Backend::allocate/deallocate (lightship-core/src/backend/cpu.rs:215-249) and the
// executor's per-operator host buffers for device tensors: one cudaMalloc per backend,
// carved first-fit with coalescing free lists.  Frees can be deferred until a stream has
// passed a point (free_after), so per-call scratch never forces a host synchronisation.
// Statistics mirror MemoryStats (lightship-core/src/memory/stats.rs:7-110).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <vector>

namespace lsc {

class Arena {
 public:
  Arena() = default;
  ~Arena();
  Arena(const Arena&) = delete;
  Arena& operator=(const Arena&) = delete;

  // Reserves `bytes` on the current device.  Returns the CUDA error of cudaMalloc.
  cudaError_t init(size_t bytes);
  // nullptr when no free range fits (after reaping completed deferred frees).
  void* alloc(size_t size, size_t align);
  // Immediate free; false when `p` is not a live allocation of this arena.
  bool free(void* p);
  // Frees `p` once all work queued on `stream` so far has completed.
  bool free_after(void* p, cudaStream_t stream);
  bool owns(const void* p) const;

  size_t capacity() const { return cap_; }
  size_t current() const;
  size_t peak() const;

 private:
  void reap_locked();
  bool free_locked(size_t off);

  mutable std::mutex mu_;
  char* base_ = nullptr;
  size_t cap_ = 0;
  size_t current_ = 0, peak_ = 0;
  std::map<size_t, size_t> free_;  // offset -> size
  std::map<size_t, size_t> used_;  // offset -> size
  struct Pending {
    size_t off;
    cudaEvent_t ev;
  };
  std::vector<Pending> pending_;
};

}  // namespace lsc
