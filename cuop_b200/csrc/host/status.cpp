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

namespace ErrorUtils {

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
