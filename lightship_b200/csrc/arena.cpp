// arena.cpp -- first-fit device arena with coalescing and stream-deferred frees.
#include "arena.h"

#include <iterator>

namespace lsc {

Arena::~Arena() {
  std::lock_guard<std::mutex> lock(mu_);
  for (auto& p : pending_) {
    cudaEventSynchronize(p.ev);
    cudaEventDestroy(p.ev);
  }
  pending_.clear();
  if (base_) cudaFree(base_);
}

cudaError_t Arena::init(size_t bytes) {
  std::lock_guard<std::mutex> lock(mu_);
  if (base_) return cudaSuccess;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return e;
  base_ = static_cast<char*>(p);
  cap_ = bytes;
  free_[0] = bytes;
  return cudaSuccess;
}

void Arena::reap_locked() {
  size_t keep = 0;
  for (size_t i = 0; i < pending_.size(); ++i) {
    if (cudaEventQuery(pending_[i].ev) == cudaSuccess) {
      cudaEventDestroy(pending_[i].ev);
      free_locked(pending_[i].off);
    } else {
      pending_[keep++] = pending_[i];
    }
  }
  pending_.resize(keep);
  cudaGetLastError();  // cudaEventQuery's "not ready" is not an error
}

void* Arena::alloc(size_t size, size_t align) {
  if (size == 0) size = 1;
  if (align < 256) align = 256;
  if (align & (align - 1)) return nullptr;
  size = (size + 255) & ~static_cast<size_t>(255);
  std::lock_guard<std::mutex> lock(mu_);
  if (!base_) return nullptr;
  if (!pending_.empty()) reap_locked();
  for (;;) {
    for (auto it = free_.begin(); it != free_.end(); ++it) {
      const size_t off = it->first, len = it->second;
      const size_t aligned = (off + align - 1) & ~(align - 1);
      if (aligned + size > off + len) continue;
      free_.erase(it);
      if (aligned > off) free_[off] = aligned - off;
      if (aligned + size < off + len) free_[aligned + size] = off + len - (aligned + size);
      used_[aligned] = size;
      current_ += size;
      if (current_ > peak_) peak_ = current_;
      return base_ + aligned;
    }
    // no room: wait for the oldest stream-deferred free (launches queued ahead of this one
    // still own their scratch) and try again
    if (pending_.empty()) return nullptr;
    cudaEventSynchronize(pending_.front().ev);
    cudaEventDestroy(pending_.front().ev);
    free_locked(pending_.front().off);
    pending_.erase(pending_.begin());
    cudaGetLastError();
  }
}

bool Arena::free_locked(size_t off) {
  auto it = used_.find(off);
  if (it == used_.end()) return false;
  size_t start = off, size = it->second;
  used_.erase(it);
  current_ -= size;
  // merge with the following free range
  auto next = free_.find(off + size);
  if (next != free_.end()) {
    size += next->second;
    free_.erase(next);
  }
  // merge with the preceding free range
  auto after = free_.lower_bound(off);
  if (after != free_.begin()) {
    auto prev = std::prev(after);
    if (prev->first + prev->second == off) {
      start = prev->first;
      size += prev->second;
      free_.erase(prev);
    }
  }
  free_[start] = size;
  return true;
}

bool Arena::free(void* p) {
  if (!p) return true;
  std::lock_guard<std::mutex> lock(mu_);
  if (!base_ || static_cast<char*>(p) < base_ || static_cast<char*>(p) >= base_ + cap_) return false;
  return free_locked(static_cast<size_t>(static_cast<char*>(p) - base_));
}

bool Arena::free_after(void* p, cudaStream_t stream) {
  if (!p) return true;
  std::lock_guard<std::mutex> lock(mu_);
  if (!base_ || static_cast<char*>(p) < base_ || static_cast<char*>(p) >= base_ + cap_) return false;
  const size_t off = static_cast<size_t>(static_cast<char*>(p) - base_);
  if (used_.find(off) == used_.end()) return false;
  cudaEvent_t ev;
  if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventRecord(ev, stream) != cudaSuccess) {
    // Without an event, fall back to waiting for the stream before the range is reused.
    cudaGetLastError();
    cudaStreamSynchronize(stream);
    return free_locked(off);
  }
  pending_.push_back({off, ev});
  return true;
}

bool Arena::owns(const void* p) const {
  std::lock_guard<std::mutex> lock(mu_);
  return base_ && static_cast<const char*>(p) >= base_ && static_cast<const char*>(p) < base_ + cap_;
}

size_t Arena::current() const {
  std::lock_guard<std::mutex> lock(mu_);
  return current_;
}

size_t Arena::peak() const {
  std::lock_guard<std::mutex> lock(mu_);
  return peak_;
}

}  // namespace lsc
