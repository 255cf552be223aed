// Status code names and helpers for the C++ facade.
#include "util/status_code.hpp"

namespace cu_op_mem {

const char* StatusCodeToString(StatusCode code) {
  switch (code) {
#define CUOP_STATUS_NAME(name, value) \
  case StatusCode::name:              \
    return #name;
    CUOP_STATUS_TABLE(CUOP_STATUS_NAME)
#undef CUOP_STATUS_NAME
  }
  return "UNKNOWN_STATUS";
}

std::string GetErrorCategoryString(ErrorCategory c) {
  static const char* names[] = {"SUCCESS", "SYSTEM", "CUDA", "MEMORY", "VALIDATION", "COMPILATION", "EXECUTION",
                                "JIT", "CACHE", "PLUGIN", "TENSOR", "OPERATOR", "UNKNOWN"};
  const int i = static_cast<int>(c);
  return (i >= 0 && i <= static_cast<int>(ErrorCategory::UNKNOWN)) ? names[i] : "UNKNOWN";
}

std::string Status::ToString() const {
  std::string s = std::string("[") + GetErrorCategoryString(GetCategory()) + "] " + StatusCodeToString(code_) +
                  " (" + std::to_string(static_cast<int>(code_)) + ")";
  if (!info_.message.empty()) s += ": " + info_.message;
  if (!info_.function.empty()) s += " in " + info_.function;
  if (!info_.file.empty()) s += " at " + info_.file + ":" + std::to_string(info_.line);
  return s;
}

std::string Status::ToDetailedString() const {
  std::string s = "status:   " + std::string(StatusCodeToString(code_)) + " (" +
                  std::to_string(static_cast<int>(code_)) + ")\ncategory: " + GetErrorCategoryString(GetCategory());
  if (!info_.message.empty()) s += "\nmessage:  " + info_.message;
  if (!info_.details.empty()) s += "\ndetails:  " + info_.details;
  if (!info_.function.empty()) s += "\nfunction: " + info_.function;
  if (!info_.file.empty()) s += "\nlocation: " + info_.file + ":" + std::to_string(info_.line);
  return s;
}

namespace ErrorUtils {

std::string GetErrorDescription(StatusCode code) {
  const char* what = "an unclassified failure";
  switch (GetErrorCategory(code)) {
    case ErrorCategory::SUCCESS: what = "the operation completed"; break;
    case ErrorCategory::SYSTEM:
      what = "a system condition: not implemented, unsupported, timed out, interrupted or out of a resource";
      break;
    case ErrorCategory::CUDA: what = "the CUDA runtime or the device reported a failure"; break;
    case ErrorCategory::MEMORY: what = "memory could not be allocated, copied or freed"; break;
    case ErrorCategory::VALIDATION: what = "an argument, configuration or dimension is invalid"; break;
    case ErrorCategory::COMPILATION: what = "kernel compilation failed"; break;
    case ErrorCategory::EXECUTION: what = "a kernel failed to launch or run, timed out, or was not found"; break;
    case ErrorCategory::JIT: what = "the plugin is not initialised or compiled, or its execution failed"; break;
    case ErrorCategory::CACHE: what = "a kernel or tuning cache entry is missing or unusable"; break;
    case ErrorCategory::PLUGIN: what = "a plugin could not be found, loaded or run"; break;
    case ErrorCategory::TENSOR: what = "tensor shapes, sizes, types or layouts do not fit the operation"; break;
    case ErrorCategory::OPERATOR: what = "the operator does not support the request or failed computing it"; break;
    default: break;
  }
  return std::string(StatusCodeToString(code)) + ": " + what;
}

bool IsCriticalError(StatusCode code) {
  switch (code) {
    case StatusCode::CUDA_OUT_OF_MEMORY:   // memory pressure: free and retry
    case StatusCode::CUDA_INVALID_VALUE:   // a bad argument
    case StatusCode::CUDA_INVALID_DEVICE:  // wrong device chosen
      return false;
    case StatusCode::KERNEL_LAUNCH_FAILED:
    case StatusCode::EXECUTION_INVALID_KERNEL:
    case StatusCode::CACHE_CORRUPTED:
      return true;
    default: return GetErrorCategory(code) == ErrorCategory::CUDA;
  }
}

bool IsRecoverableError(StatusCode code) {
  switch (GetErrorCategory(code)) {
    case ErrorCategory::VALIDATION:
    case ErrorCategory::TENSOR:
      return true;
    default: break;
  }
  switch (code) {
    case StatusCode::TIMEOUT:
    case StatusCode::INTERRUPTED:
    case StatusCode::RESOURCE_UNAVAILABLE:
    case StatusCode::UNSUPPORTED_OPERATION:
    case StatusCode::OPERATOR_NOT_SUPPORTED:
    case StatusCode::OPERATOR_INVALID_INPUT:
    case StatusCode::OPERATOR_INVALID_OUTPUT:
    case StatusCode::OUT_OF_MEMORY:
    case StatusCode::MEMORY_ALLOCATION_FAILED:
    case StatusCode::MEMORY_POOL_ERROR:
    case StatusCode::CUDA_OUT_OF_MEMORY:
    case StatusCode::CUDA_INVALID_VALUE:
    case StatusCode::EXECUTION_TIMEOUT:
    case StatusCode::EXECUTION_INTERRUPTED:
    case StatusCode::EXECUTION_KERNEL_NOT_FOUND:
    case StatusCode::JIT_NOT_INITIALIZED:
    case StatusCode::JIT_NOT_COMPILED:
    case StatusCode::CACHE_MISS:
    case StatusCode::CACHE_NOT_FOUND:
    case StatusCode::PLUGIN_NOT_FOUND:
      return true;
    default: return false;
  }
}

Status SystemError(const std::string& m, const std::string& f, const std::string& file, int line) {
  return Status(StatusCode::SYSTEM_ERROR, m, f, file, line);
}
Status ValidationError(const std::string& m, const std::string& f, const std::string& file, int line) {
  return Status(StatusCode::VALIDATION_ERROR, m, f, file, line);
}
Status MemoryError(const std::string& m, const std::string& f, const std::string& file, int line) {
  return Status(StatusCode::MEMORY_ERROR, m, f, file, line);
}
Status CompilationError(const std::string& m, const std::string& f, const std::string& file, int line) {
  return Status(StatusCode::COMPILATION_ERROR, m, f, file, line);
}
Status ExecutionError(const std::string& m, const std::string& f, const std::string& file, int line) {
  return Status(StatusCode::EXECUTION_ERROR, m, f, file, line);
}

Status CudaError(cudaError_t err, const std::string& function, const std::string& file, int line) {
  StatusCode code = StatusCode::CUDA_ERROR;
  switch (err) {
    case cudaSuccess: return Status(StatusCode::SUCCESS);
    case cudaErrorMemoryAllocation: code = StatusCode::CUDA_OUT_OF_MEMORY; break;
    case cudaErrorInvalidDevice: code = StatusCode::CUDA_INVALID_DEVICE; break;
    case cudaErrorInvalidValue: code = StatusCode::CUDA_INVALID_VALUE; break;
    case cudaErrorLaunchFailure: code = StatusCode::CUDA_LAUNCH_FAILED; break;
    default: break;
  }
  return Status(code, cudaGetErrorString(err), function, file, line);
}

std::string GetStatusCodeString(StatusCode code) { return StatusCodeToString(code); }

}  // namespace ErrorUtils
}  // namespace cu_op_mem
