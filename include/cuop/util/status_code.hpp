// cuOP status codes for the B200 build of the dense BLAS path.
//
// Same enumerator names and numeric values as the reference's
// include/util/status_code.hpp:28-161 (callers compare these integers and the
// C ABI in cuopx.h returns them), generated here from one table so that the
// enum, the name strings and the categories cannot drift apart.
#pragma once

#include <cuda_runtime.h>

#include <ostream>
#include <string>

namespace cu_op_mem {

enum class ErrorCategory {
  SUCCESS = 0, SYSTEM, CUDA, MEMORY, VALIDATION, COMPILATION, EXECUTION, JIT, CACHE, PLUGIN, TENSOR,
  OPERATOR, UNKNOWN
};

#define CUOP_STATUS_TABLE(X)                                                                                 \
  X(SUCCESS, 0)                                                                                              \
  X(SYSTEM_ERROR, 1000) X(NOT_IMPLEMENTED, 1001) X(UNSUPPORTED_OPERATION, 1002) X(TIMEOUT, 1003)            \
  X(INTERRUPTED, 1004) X(RESOURCE_UNAVAILABLE, 1005) X(FILE_NOT_FOUND, 1006) X(PERMISSION_DENIED, 1007)     \
  X(CUDA_ERROR, 2000) X(CUDA_DRIVER_ERROR, 2001) X(CUDA_RUNTIME_ERROR, 2002) X(CUDA_MEMORY_ERROR, 2003)     \
  X(CUDA_KERNEL_ERROR, 2004) X(CUDA_LAUNCH_ERROR, 2005) X(CUDA_SYNC_ERROR, 2006) X(CUDA_DEVICE_ERROR, 2007) \
  X(CUDA_CONTEXT_ERROR, 2008) X(CUDA_STREAM_ERROR, 2009) X(CUDA_EVENT_ERROR, 2010)                          \
  X(CUDA_INVALID_DEVICE, 2011) X(CUDA_INVALID_VALUE, 2012) X(CUDA_OUT_OF_MEMORY, 2013)                      \
  X(CUDA_LAUNCH_FAILED, 2014)                                                                                \
  X(MEMORY_ERROR, 3000) X(OUT_OF_MEMORY, 3001) X(MEMORY_ALLOCATION_FAILED, 3002)                            \
  X(MEMORY_DEALLOCATION_FAILED, 3003) X(MEMORY_COPY_FAILED, 3004) X(MEMORY_ALIGNMENT_ERROR, 3005)           \
  X(MEMORY_POOL_ERROR, 3006) X(MEMORY_FREE_FAILED, 3007)                                                     \
  X(VALIDATION_ERROR, 4000) X(INVALID_ARGUMENT, 4001) X(INVALID_CONFIGURATION, 4002) X(INVALID_STATE, 4003) \
  X(INVALID_FORMAT, 4004) X(INVALID_DIMENSION, 4005) X(INVALID_TYPE, 4006) X(INVALID_OPERATION, 4007)       \
  X(INVALID_INPUT, 4008) X(INVALID_OUTPUT, 4009) X(INVALID_DIMENSIONS, 4010) X(INVALID_DATA_TYPE, 4011)     \
  X(COMPILATION_ERROR, 5000) X(COMPILATION_FAILED, 5001) X(COMPILATION_TIMEOUT, 5002)                       \
  X(COMPILATION_INVALID_CODE, 5003) X(COMPILATION_INVALID_OPTIONS, 5004) X(COMPILATION_LINKING_ERROR, 5005) \
  X(COMPILATION_OPTIMIZATION_ERROR, 5006) X(JIT_COMPILATION_FAILED, 5007)                                   \
  X(EXECUTION_ERROR, 6000) X(EXECUTION_FAILED, 6001) X(EXECUTION_TIMEOUT, 6002)                             \
  X(EXECUTION_INTERRUPTED, 6003) X(EXECUTION_INVALID_KERNEL, 6004) X(EXECUTION_KERNEL_NOT_FOUND, 6005)      \
  X(KERNEL_LAUNCH_FAILED, 6006)                                                                              \
  X(JIT_ERROR, 7000) X(JIT_NOT_INITIALIZED, 7001) X(JIT_INITIALIZATION_ERROR, 7002) X(JIT_NOT_COMPILED, 7003) \
  X(JIT_COMPILATION_ERROR, 7004) X(JIT_EXECUTION_ERROR, 7005) X(JIT_PLUGIN_ERROR, 7006)                     \
  X(JIT_TEMPLATE_ERROR, 7007) X(JIT_CACHE_ERROR, 7008)                                                      \
  X(CACHE_ERROR, 8000) X(CACHE_NOT_FOUND, 8001) X(CACHE_CORRUPTED, 8002) X(CACHE_FULL, 8003)                \
  X(CACHE_ACCESS_ERROR, 8004) X(CACHE_SERIALIZATION_ERROR, 8005) X(CACHE_DESERIALIZATION_ERROR, 8006)       \
  X(CACHE_VERSION_MISMATCH, 8007) X(CACHE_MISS, 8008)                                                       \
  X(PLUGIN_ERROR, 9000) X(PLUGIN_NOT_FOUND, 9001) X(PLUGIN_LOAD_ERROR, 9002)                                \
  X(PLUGIN_INITIALIZATION_ERROR, 9003) X(PLUGIN_EXECUTION_ERROR, 9004) X(PLUGIN_VERSION_MISMATCH, 9005)     \
  X(PLUGIN_INCOMPATIBLE, 9006)                                                                               \
  X(TENSOR_ERROR, 10000) X(TENSOR_DIMENSION_MISMATCH, 10001) X(TENSOR_SHAPE_MISMATCH, 10002)                \
  X(TENSOR_TYPE_MISMATCH, 10003) X(TENSOR_SIZE_MISMATCH, 10004) X(TENSOR_INDEX_OUT_OF_BOUNDS, 10005)        \
  X(TENSOR_STRIDE_ERROR, 10006) X(TENSOR_LAYOUT_ERROR, 10007)                                               \
  X(OPERATOR_ERROR, 11000) X(OPERATOR_NOT_SUPPORTED, 11001) X(OPERATOR_INVALID_INPUT, 11002)                \
  X(OPERATOR_INVALID_OUTPUT, 11003) X(OPERATOR_COMPUTATION_ERROR, 11004) X(OPERATOR_GRADIENT_ERROR, 11005)  \
  X(OPERATOR_BACKWARD_ERROR, 11006)

enum class StatusCode {
#define CUOP_STATUS_ENUM(name, value) name = value,
  CUOP_STATUS_TABLE(CUOP_STATUS_ENUM)
#undef CUOP_STATUS_ENUM
  // older spellings kept by the reference for compatibility
  SHAPE_MISMATCH = TENSOR_SHAPE_MISMATCH,
  UNSUPPORTED_TYPE = OPERATOR_NOT_SUPPORTED,
  UNKNOWN_ERROR = SYSTEM_ERROR,
  TENSOR_DIMONSION_MISMATCH = TENSOR_DIMENSION_MISMATCH,
  NOT_INITIALIZED = JIT_NOT_INITIALIZED,
  INITIALIZATION_ERROR = JIT_INITIALIZATION_ERROR,
  KERNEL_NOT_FOUND = EXECUTION_KERNEL_NOT_FOUND,
  NOT_COMPILED = JIT_NOT_COMPILED
};

// Category from the thousands digit(s) of the code (0 -> SUCCESS,
// 1xxx SYSTEM ... 11xxx OPERATOR).
inline ErrorCategory GetErrorCategory(StatusCode code) {
  const int v = static_cast<int>(code);
  if (v == 0) return ErrorCategory::SUCCESS;
  const int band = v / 1000;
  if (band >= 1 && band <= 11) return static_cast<ErrorCategory>(band);
  return ErrorCategory::UNKNOWN;
}

const char* StatusCodeToString(StatusCode code);
std::string GetErrorCategoryString(ErrorCategory category);

inline std::ostream& operator<<(std::ostream& os, StatusCode code) { return os << StatusCodeToString(code); }

struct ErrorInfo {
  StatusCode code = StatusCode::SUCCESS;
  ErrorCategory category = ErrorCategory::SUCCESS;
  std::string message, details, function, file;
  int line = 0;
};

class Status {
 public:
  Status() = default;
  Status(StatusCode code) : code_(code) { info_.code = code; info_.category = GetErrorCategory(code); }
  Status(StatusCode code, const std::string& message, const std::string& function = "", const std::string& file = "",
         int line = 0)
      : Status(code) {
    info_.message = message;
    info_.function = function;
    info_.file = file;
    info_.line = line;
  }
  bool IsSuccess() const { return code_ == StatusCode::SUCCESS; }
  bool IsError() const { return !IsSuccess(); }
  StatusCode GetCode() const { return code_; }
  ErrorCategory GetCategory() const { return info_.category; }
  const std::string& GetMessage() const { return info_.message; }
  const std::string& GetDetails() const { return info_.details; }
  const std::string& GetFunction() const { return info_.function; }
  const std::string& GetFile() const { return info_.file; }
  int GetLine() const { return info_.line; }
  void SetDetails(const std::string& d) { info_.details = d; }
  explicit operator bool() const { return IsSuccess(); }
  std::string ToString() const;
  // ToString plus the details, one field per line.
  std::string ToDetailedString() const;

 private:
  StatusCode code_ = StatusCode::SUCCESS;
  ErrorInfo info_;
};

namespace ErrorUtils {
inline Status Success() { return Status(StatusCode::SUCCESS); }
inline Status Error(StatusCode code, const std::string& message, const std::string& function = "",
                    const std::string& file = "", int line = 0) {
  return Status(code, message, function, file, line);
}
Status CudaError(cudaError_t err, const std::string& function = "", const std::string& file = "", int line = 0);
std::string GetStatusCodeString(StatusCode code);
// One-sentence description of a code for messages and logs.
std::string GetErrorDescription(StatusCode code);
// Critical: the device or process state may be damaged (CUDA device,
// context or launch failures, memory corruption); stop using the GPU path.
bool IsCriticalError(StatusCode code);
// Recoverable: the call can be retried or corrected by the caller (bad
// arguments or shapes, memory pressure, time-outs, unsupported requests).
bool IsRecoverableError(StatusCode code);
// Status objects of one category, with a message and the call site.
Status SystemError(const std::string& message, const std::string& function = "", const std::string& file = "",
                   int line = 0);
Status ValidationError(const std::string& message, const std::string& function = "", const std::string& file = "",
                       int line = 0);
Status MemoryError(const std::string& message, const std::string& function = "", const std::string& file = "",
                   int line = 0);
Status CompilationError(const std::string& message, const std::string& function = "", const std::string& file = "",
                        int line = 0);
Status ExecutionError(const std::string& message, const std::string& function = "", const std::string& file = "",
                      int line = 0);
}  // namespace ErrorUtils

}  // namespace cu_op_mem
