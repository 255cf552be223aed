// GlobalJITManager (reference include/jit/global_jit_manager.hpp): process-wide
// plugin configuration.  Save/LoadCacheFromFile persist the per-operator
// configurations (kernel_type etc.) as plain text; the library compiles no
// code at run time, so there is no compiled-code cache.
#pragma once

#include <mutex>
#include <string>
#include <unordered_map>

#include "jit/ijit_plugin.hpp"
#include "jit/jit_config.hpp"

namespace cu_op_mem {

class GlobalJITManager {
 public:
  static GlobalJITManager& Instance();
  void SetGlobalConfig(const GlobalJITConfig& config);
  GlobalJITConfig GetGlobalConfig() const;
  void SetOperatorConfig(const std::string& op_name, const JITConfig& config);
  JITConfig GetOperatorConfig(const std::string& op_name) const;
  StatusCode Initialize();
  void Cleanup();
  JITStatistics GetStatistics() const;
  void ResetStatistics();
  void RecordExecution(double seconds);
  void ClearAllCaches();
  void SaveCacheToFile(const std::string& file_path);
  void LoadCacheFromFile(const std::string& file_path);
  bool IsInitialized() const { return initialized_; }
  HardwareSpec GetHardwareSpec() const { return hw_; }

 private:
  GlobalJITManager() = default;
  GlobalJITConfig global_config_;
  std::unordered_map<std::string, JITConfig> operator_configs_;
  JITStatistics stats_;
  HardwareSpec hw_;
  bool initialized_ = false;
  mutable std::mutex mutex_;
};

}  // namespace cu_op_mem
