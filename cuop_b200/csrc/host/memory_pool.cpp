// Per-device, stream-ordered caching pool (see include/cuop/base/memory_pool.hpp).
#include "base/memory_pool.hpp"

#include <algorithm>
#include <cstdio>
#include <memory>

namespace cu_op_mem {

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_pools_mu;
CudaMemoryPool* g_pools[kMaxDevices] = {};

// RAII: make `dev` current for the scope (pools allocate on their own device).
struct DeviceScope {
  int prev = -1;
  explicit DeviceScope(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) cudaSetDevice(dev);
    else prev = -1;
  }
  ~DeviceScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};
}  // namespace

CudaMemoryPool& CudaMemoryPool::Instance() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  return ForDevice(dev);
}

CudaMemoryPool& CudaMemoryPool::ForDevice(int device) {
  if (device < 0 || device >= kMaxDevices) device = 0;
  std::lock_guard<std::mutex> lock(g_pools_mu);
  if (!g_pools[device]) g_pools[device] = new CudaMemoryPool(device);  // lives for the process
  return *g_pools[device];
}

CudaMemoryPool::~CudaMemoryPool() = default;

std::size_t CudaMemoryPool::SizeClass(std::size_t bytes) {
  if (bytes == 0) return 0;
  if (bytes <= (std::size_t(1) << 20)) {
    std::size_t c = 256;
    while (c < bytes) c <<= 1;
    return c;
  }
  const std::size_t g = std::size_t(2) << 20;
  return (bytes + g - 1) / g * g;
}

void* CudaMemoryPool::Alloc(std::size_t bytes, cudaStream_t stream) {
  if (bytes == 0) return nullptr;
  const std::size_t cls = SizeClass(bytes);
  std::lock_guard<std::mutex> lock(mu_);
  ++stats_.alloc_calls;
  auto it = free_.find(cls);
  if (it != free_.end()) {
    auto& v = it->second;
    for (std::size_t i = v.size(); i-- > 0;) {
      Cached c = v[i];
      const bool reusable = c.ready == nullptr || c.stream == stream || cudaEventQuery(c.ready) == cudaSuccess;
      if (!reusable) continue;
      if (c.ready) {
        if (c.stream != stream) {
          // Ordered hand-over to another stream: wait for the last use.
          cudaStreamWaitEvent(stream, c.ready, 0);
        }
        spare_events_.push_back(c.ready);
      }
      v.erase(v.begin() + static_cast<std::ptrdiff_t>(i));
      cached_bytes_ -= cls;
      live_[c.ptr] = cls;
      stats_.bytes_in_use += cls;
      stats_.peak_in_use = std::max(stats_.peak_in_use, stats_.bytes_in_use);
      ++stats_.cache_hits;
      return c.ptr;
    }
  }
  if (config_.memory_limit && stats_.bytes_reserved + cls > config_.memory_limit) {
    release_idle_locked(true);
    if (stats_.bytes_reserved + cls > config_.memory_limit) {
      ++stats_.failed_allocs;
      return nullptr;
    }
  }
  DeviceScope scope(device_);
  void* p = nullptr;
  if (cudaMalloc(&p, cls) != cudaSuccess) {
    cudaGetLastError();
    release_idle_locked(false);
    if (cudaMalloc(&p, cls) != cudaSuccess) {
      cudaGetLastError();
      ++stats_.failed_allocs;
      return nullptr;
    }
  }
  ++stats_.cache_misses;
  stats_.bytes_reserved += cls;
  stats_.bytes_in_use += cls;
  stats_.peak_in_use = std::max(stats_.peak_in_use, stats_.bytes_in_use);
  live_[p] = cls;
  return p;
}

void CudaMemoryPool::Free(void* ptr, std::size_t bytes, cudaStream_t stream) {
  (void)bytes;
  if (!ptr) return;
  std::lock_guard<std::mutex> lock(mu_);
  auto it = live_.find(ptr);
  if (it == live_.end()) return;  // not ours (or already freed): ignore
  const std::size_t cls = it->second;
  live_.erase(it);
  ++stats_.free_calls;
  stats_.bytes_in_use -= cls;
  cudaEvent_t ev = nullptr;
  DeviceScope scope(device_);
  if (!spare_events_.empty()) {
    ev = spare_events_.back();
    spare_events_.pop_back();
  } else if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
    ev = nullptr;
  }
  if (ev && cudaEventRecord(ev, stream) != cudaSuccess) {
    cudaGetLastError();
    cudaEventDestroy(ev);
    ev = nullptr;
    cudaStreamSynchronize(stream);  // no event: make the block safe the slow way
  }
  free_[cls].push_back(Cached{ptr, stream, ev});
  cached_bytes_ += cls;
  if (cached_bytes_ > config_.max_cached_bytes) release_idle_locked(true);
}

void CudaMemoryPool::release_idle_locked(bool only_completed) {
  DeviceScope scope(device_);
  for (auto& kv : free_) {
    auto& v = kv.second;
    for (std::size_t i = v.size(); i-- > 0;) {
      Cached c = v[i];
      if (c.ready) {
        if (cudaEventQuery(c.ready) != cudaSuccess) {
          if (only_completed) continue;
          cudaEventSynchronize(c.ready);
        }
        spare_events_.push_back(c.ready);
      }
      cudaFree(c.ptr);
      v.erase(v.begin() + static_cast<std::ptrdiff_t>(i));
      cached_bytes_ -= kv.first;
      stats_.bytes_reserved -= kv.first;
    }
  }
}

void CudaMemoryPool::ReleaseCached() {
  std::lock_guard<std::mutex> lock(mu_);
  release_idle_locked(false);
}

void CudaMemoryPool::ReleaseAll() { ReleaseCached(); }

void CudaMemoryPool::Defragment() { ReleaseCached(); }

void CudaMemoryPool::TrimCache() {
  std::lock_guard<std::mutex> lock(mu_);
  release_idle_locked(true);
}

void CudaMemoryPool::Preallocate(std::size_t block_size, std::size_t count) {
  std::vector<void*> blocks;
  blocks.reserve(count);
  for (std::size_t i = 0; i < count; ++i) {
    void* p = Alloc(block_size);
    if (!p) break;
    blocks.push_back(p);
  }
  for (void* p : blocks) Free(p, block_size);
}

void CudaMemoryPool::PrintStats() const {
  const MemoryStats s = GetStats();
  std::fprintf(stderr,
               "cuop memory pool, device %d: reserved %zu B, in use %zu B, peak %zu B; %zu allocs (%zu cache hits, "
               "%zu from cudaMalloc, %zu failed), %zu frees\n",
               device_, s.bytes_reserved, s.bytes_in_use, s.peak_in_use, s.alloc_calls, s.cache_hits,
               s.cache_misses, s.failed_allocs, s.free_calls);
}

void CudaMemoryPool::SetConfig(const MemoryPoolConfig& c) {
  std::lock_guard<std::mutex> lock(mu_);
  config_ = c;
}

MemoryPoolConfig CudaMemoryPool::GetConfig() const {
  std::lock_guard<std::mutex> lock(mu_);
  return config_;
}

void CudaMemoryPool::SetMemoryLimit(std::size_t bytes) {
  std::lock_guard<std::mutex> lock(mu_);
  config_.memory_limit = bytes;
}

MemoryStats CudaMemoryPool::GetStats() const {
  std::lock_guard<std::mutex> lock(mu_);
  return stats_;
}

void CudaMemoryPool::ResetStats() {
  std::lock_guard<std::mutex> lock(mu_);
  const std::size_t reserved = stats_.bytes_reserved, in_use = stats_.bytes_in_use;
  stats_ = MemoryStats();
  stats_.bytes_reserved = reserved;
  stats_.bytes_in_use = in_use;
  stats_.peak_in_use = in_use;
}

}  // namespace cu_op_mem
