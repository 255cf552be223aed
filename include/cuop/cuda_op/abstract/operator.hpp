// Operator<T>: the reference's operator base (include/cuda_op/abstract/operator.hpp:10-15).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "data/tensor.hpp"
#include "util/status_code.hpp"

namespace cu_op_mem {

// Scalar type of alpha/beta: fp32 for 16-bit element types, else T.
template <typename T> struct ScalarOf { using type = T; };
template <> struct ScalarOf<__half> { using type = float; };
template <> struct ScalarOf<__nv_bfloat16> { using type = float; };

template <typename T>
class Operator {
 public:
  virtual ~Operator() = default;
  virtual StatusCode Forward(const Tensor<T>& input, Tensor<T>& output) = 0;
};

}  // namespace cu_op_mem
