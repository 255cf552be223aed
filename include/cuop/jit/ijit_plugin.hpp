// Plugin interface of the dense BLAS path: IJITPlugin, IPluginFactory,
// PluginRegistrar, PluginManager and the registration macros, with the
// method names and meanings of the reference's include/jit/ijit_plugin.hpp:
// 18-143.  Compile() selects and validates a precompiled sm_100a variant
// (there is no NVRTC step); Execute() runs it through the C ABI and is
// synchronous, as the reference's plugins are.
#pragma once

#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "data/tensor.hpp"
#include "jit/jit_config.hpp"
#include "util/status_code.hpp"

namespace cu_op_mem {

class IJITPlugin {
 public:
  virtual ~IJITPlugin() = default;

  virtual StatusCode Initialize() = 0;
  virtual StatusCode Compile(const JITConfig& config) = 0;
  virtual StatusCode Execute(const std::vector<Tensor<float>>& inputs, std::vector<Tensor<float>>& outputs) = 0;
  virtual void Optimize(const PerformanceProfile& profile) = 0;
  virtual std::string GetPluginName() const = 0;

  virtual void SetConfig(const JITConfig& config) = 0;
  virtual JITConfig GetConfig() const = 0;

  virtual void EnableAutoTuning(bool enable) = 0;
  virtual bool IsAutoTuningEnabled() const = 0;
  virtual PerformanceProfile GetPerformanceProfile() const = 0;

  virtual bool IsInitialized() const = 0;
  virtual bool IsCompiled() const = 0;
  virtual std::string GetLastError() const = 0;

  virtual void Cleanup() = 0;
  virtual size_t GetMemoryUsage() const = 0;
};

class IPluginFactory {
 public:
  virtual ~IPluginFactory() = default;
  virtual std::unique_ptr<IJITPlugin> CreatePlugin() = 0;
  virtual std::string GetPluginType() const = 0;
  virtual bool SupportsOperator(const std::string& op_name) const = 0;
};

class PluginRegistrar {
 public:
  static PluginRegistrar& Instance();
  void RegisterPluginFactory(const std::string& plugin_type, std::unique_ptr<IPluginFactory> factory);
  std::unique_ptr<IJITPlugin> CreatePlugin(const std::string& plugin_type);
  std::vector<std::string> GetSupportedPluginTypes() const;
  bool IsOperatorSupported(const std::string& op_name) const;

 private:
  std::unordered_map<std::string, std::unique_ptr<IPluginFactory>> factories_;
  mutable std::mutex mutex_;
};

class PluginManager {
 public:
  static PluginManager& Instance();
  void RegisterPlugin(const std::string& name, std::unique_ptr<IJITPlugin> plugin);
  IJITPlugin* GetPlugin(const std::string& name);
  void RemovePlugin(const std::string& name);
  void InitializeAllPlugins();
  void CompileAllPlugins(const JITConfig& config);
  void CleanupAllPlugins();
  std::vector<std::string> GetActivePlugins() const;
  size_t GetTotalMemoryUsage() const;
  JITStatistics GetTotalStatistics() const;

 private:
  std::unordered_map<std::string, std::unique_ptr<IJITPlugin>> plugins_;
  mutable std::mutex mutex_;
};

#define REGISTER_JIT_PLUGIN(plugin_type, plugin_class)                                               \
  static int plugin_type##_registrar_ = []() {                                                       \
    ::cu_op_mem::PluginRegistrar::Instance().RegisterPluginFactory(                                  \
        #plugin_type, std::make_unique<plugin_class##Factory>());                                    \
    return 0;                                                                                        \
  }()

#define CREATE_PLUGIN_FACTORY(plugin_class)                                                          \
  class plugin_class##Factory : public ::cu_op_mem::IPluginFactory {                                 \
   public:                                                                                           \
    std::unique_ptr<::cu_op_mem::IJITPlugin> CreatePlugin() override {                               \
      return std::make_unique<plugin_class>();                                                       \
    }                                                                                                \
    std::string GetPluginType() const override { return #plugin_class; }                             \
    bool SupportsOperator(const std::string& op) const override { return plugin_class::SupportsOperator(op); } \
  }

}  // namespace cu_op_mem
