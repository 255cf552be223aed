// Device memory pool feeding Tensor<T> and operator workspaces.
//
// Replaces the reference's CudaMemoryPool (include/base/memory_pool.hpp:86-170,
// src/base/memory_pool.cu) with the same Alloc/Free interface, redesigned for
// multi-GPU processes:
//  * one pool per device: Instance() returns the pool of the device that is
//    current on the calling thread (the reference had one process-wide pool
//    that handed out pointers of whichever device happened to be current);
//  * stream-ordered reuse: Free(ptr, bytes, stream) records an event on
//    `stream`; a cached block is handed out again only to the same stream or
//    once that event has completed, so a block is never reused while a kernel
//    on another stream may still touch it;
//  * size classes: powers of two from 256 B to 1 MiB, then 2 MiB multiples;
//  * on cudaMalloc failure the pool releases its idle cache and retries once;
//  * SetMemoryLimit caps the bytes the pool may hold (tests use it to inject
//    OUT_OF_MEMORY on the host without touching the GPU).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <map>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace cu_op_mem {

struct MemoryStats {
  std::size_t bytes_reserved = 0;   // device bytes currently held (in use + cached)
  std::size_t bytes_in_use = 0;     // handed out and not yet freed
  std::size_t peak_in_use = 0;
  std::size_t alloc_calls = 0;
  std::size_t free_calls = 0;
  std::size_t cache_hits = 0;
  std::size_t cache_misses = 0;     // served by cudaMalloc
  std::size_t failed_allocs = 0;
};

struct MemoryPoolConfig {
  std::size_t alignment = 256;
  std::size_t max_cached_bytes = std::size_t(8) << 30;  // idle cache above this is released
  std::size_t memory_limit = 0;                          // 0 = no limit
};

class CudaMemoryPool {
 public:
  // Pool of the calling thread's current device.
  static CudaMemoryPool& Instance();
  // Pool of a given device.
  static CudaMemoryPool& ForDevice(int device);

  void* Alloc(std::size_t bytes, cudaStream_t stream = nullptr);
  void Free(void* ptr, std::size_t bytes, cudaStream_t stream = nullptr);

  void SetConfig(const MemoryPoolConfig& config);
  MemoryPoolConfig GetConfig() const;
  void SetMemoryLimit(std::size_t bytes);  // 0 removes the limit
  MemoryStats GetStats() const;
  void ResetStats();
  // Frees every idle cached block, first waiting for the last use of any
  // block whose stream work is still pending.  Blocks in use are untouched.
  void ReleaseCached();
  // The reference pool's maintenance calls (include/base/memory_pool.hpp:93-111).
  // Each block here is its own cudaMalloc, so there is nothing to merge or
  // compact inside the pool; these map onto releasing idle blocks:
  void ReleaseAll();   // = ReleaseCached()
  void Defragment();   // = ReleaseCached(): idle blocks go back to the driver
  void TrimCache();    // frees idle blocks whose last use has completed (no waiting)
  // Allocates `count` blocks of `block_size` bytes into the idle cache, so
  // later requests of that size class are cache hits (stops at the first
  // allocation that fails or would pass the memory limit).
  void Preallocate(std::size_t block_size, std::size_t count);
  // One line of statistics on stderr.
  void PrintStats() const;
  int Device() const { return device_; }

  // Size class a request of `bytes` is served from.
  static std::size_t SizeClass(std::size_t bytes);

  CudaMemoryPool(const CudaMemoryPool&) = delete;
  CudaMemoryPool& operator=(const CudaMemoryPool&) = delete;
  ~CudaMemoryPool();

 private:
  explicit CudaMemoryPool(int device) : device_(device) {}

  struct Cached {
    void* ptr;
    cudaStream_t stream;  // stream of the last use
    cudaEvent_t ready;    // completes when that use is done (nullptr: no pending use)
  };

  void release_idle_locked(bool only_completed);

  int device_;
  mutable std::mutex mu_;
  MemoryPoolConfig config_;
  MemoryStats stats_;
  std::map<std::size_t, std::vector<Cached>> free_;      // size class -> idle blocks
  std::unordered_map<void*, std::size_t> live_;          // handed-out block -> size class
  std::size_t cached_bytes_ = 0;
  std::vector<cudaEvent_t> spare_events_;
};

}  // namespace cu_op_mem
