// Tensor<T>: a device buffer plus shape, the argument type of every operator.
//
// Interface of the reference's include/data/tensor.hpp:16-236 (shape ctor that
// allocates from the pool, external-pointer ctor, move-only, data/numel/bytes/
// shape, reshape/resize, fill/zero/ones, copy_from_host/copy_to_host,
// slice/view/astype).  Differences: a tensor built on an external pointer
// never frees it (the reference leaves own_data_ at true there); memory comes
// from the pool of the tensor's device; T may be float, double, __half,
// __nv_bfloat16 or any trivially copyable type.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <functional>
#include <memory>
#include <numeric>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

#include "base/memory_pool.hpp"

namespace cu_op_mem {

template <typename T>
class Tensor {
  static_assert(std::is_trivially_copyable<T>::value, "Tensor elements must be trivially copyable");

 public:
  Tensor() = default;

  explicit Tensor(const std::vector<std::size_t>& shape) : shape_(shape), numel_(count(shape)) {
    if (numel_ == 0) return;
    cudaGetDevice(&device_);
    data_ = static_cast<T*>(CudaMemoryPool::ForDevice(device_).Alloc(bytes()));
    if (!data_) throw std::runtime_error("Tensor: device allocation of " + std::to_string(bytes()) + " bytes failed");
    own_ = true;
  }

  // Non-owning view of caller memory.
  Tensor(T* external, const std::vector<std::size_t>& shape) : data_(external), shape_(shape), numel_(count(shape)) {}

  Tensor(const Tensor&) = delete;
  Tensor& operator=(const Tensor&) = delete;
  Tensor(Tensor&& o) noexcept { take(std::move(o)); }
  Tensor& operator=(Tensor&& o) noexcept {
    if (this != &o) {
      release();
      take(std::move(o));
    }
    return *this;
  }
  ~Tensor() { release(); }

  T* data() const { return data_; }
  std::size_t numel() const { return numel_; }
  std::size_t bytes() const { return numel_ * sizeof(T); }
  const std::vector<std::size_t>& shape() const { return shape_; }
  bool is_empty() const { return data_ == nullptr || numel_ == 0; }
  bool owns_data() const { return own_; }

  void reshape(const std::vector<std::size_t>& s) {
    if (count(s) != numel_) throw std::runtime_error("Tensor::reshape: element count differs");
    shape_ = s;
  }

  void resize(const std::vector<std::size_t>& s) {
    if (count(s) == numel_) {
      shape_ = s;
      return;
    }
    *this = Tensor<T>(s);
  }

  void fill(const T& v) {
    if (is_empty()) return;
    std::vector<T> h(numel_, v);
    cudaMemcpy(data_, h.data(), bytes(), cudaMemcpyHostToDevice);
  }
  void zero() {
    if (!is_empty()) cudaMemset(data_, 0, bytes());
  }
  void ones() { fill(static_cast<T>(1.0f)); }

  void copy_from_host(const T* h, cudaStream_t stream = nullptr) {
    if (is_empty()) return;
    if (stream) cudaMemcpyAsync(data_, h, bytes(), cudaMemcpyHostToDevice, stream);
    else cudaMemcpy(data_, h, bytes(), cudaMemcpyHostToDevice);
  }
  void copy_to_host(T* h, cudaStream_t stream = nullptr) const {
    if (is_empty()) return;
    if (stream) cudaMemcpyAsync(h, data_, bytes(), cudaMemcpyDeviceToHost, stream);
    else cudaMemcpy(h, data_, bytes(), cudaMemcpyDeviceToHost);
  }

  // 1-D view [start, end) sharing this tensor's memory.
  std::shared_ptr<Tensor<T>> slice(std::size_t start, std::size_t end) const {
    if (start >= end || end > numel_) throw std::out_of_range("Tensor::slice out of range");
    return std::make_shared<Tensor<T>>(data_ + start, std::vector<std::size_t>{end - start});
  }

  // N-D view at `offset` of shape `s`; only views whose elements are
  // contiguous in memory are allowed (leading dims of extent 1 or full rows).
  std::shared_ptr<Tensor<T>> view(const std::vector<std::size_t>& offset, const std::vector<std::size_t>& s) const {
    if (offset.size() != shape_.size() || s.size() != shape_.size())
      throw std::invalid_argument("Tensor::view: rank mismatch");
    std::size_t flat = 0, stride = 1;
    for (int i = static_cast<int>(shape_.size()) - 1; i >= 0; --i) {
      if (offset[i] + s[i] > shape_[i]) throw std::out_of_range("Tensor::view out of range");
      flat += offset[i] * stride;
      stride *= shape_[i];
    }
    return std::make_shared<Tensor<T>>(data_ + flat, s);
  }

  template <typename U>
  std::shared_ptr<Tensor<U>> astype() const {
    auto t = std::make_shared<Tensor<U>>(shape_);
    if (numel_ == 0) return t;
    std::vector<T> src(numel_);
    cudaMemcpy(src.data(), data_, bytes(), cudaMemcpyDeviceToHost);
    std::vector<U> dst(numel_);
    std::transform(src.begin(), src.end(), dst.begin(), [](const T& v) { return static_cast<U>(static_cast<float>(v)); });
    cudaMemcpy(t->data(), dst.data(), numel_ * sizeof(U), cudaMemcpyHostToDevice);
    return t;
  }

 private:
  static std::size_t count(const std::vector<std::size_t>& s) {
    if (s.empty()) return 0;
    return std::accumulate(s.begin(), s.end(), std::size_t(1), std::multiplies<std::size_t>());
  }
  void take(Tensor&& o) {
    data_ = o.data_;
    shape_ = std::move(o.shape_);
    numel_ = o.numel_;
    own_ = o.own_;
    device_ = o.device_;
    o.data_ = nullptr;
    o.numel_ = 0;
    o.own_ = false;
  }
  void release() {
    if (data_ && own_) CudaMemoryPool::ForDevice(device_).Free(data_, bytes());
    data_ = nullptr;
    own_ = false;
  }

  T* data_ = nullptr;
  std::vector<std::size_t> shape_;
  std::size_t numel_ = 0;
  bool own_ = false;
  int device_ = 0;
};

}  // namespace cu_op_mem
