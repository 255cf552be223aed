// JITWrapper<Op>: run an operator through its plugin when JIT is enabled and
// the plugin is compiled, else through the operator itself (reference
// include/jit/jit_wrapper.hpp:18-235).  In the reference the plugin lookup key
// ("gemm_jit") was never registered and ConvertToTensors returned {}, so every
// call ended in the original operator; here the key is registered and the
// operator's tensors are handed to the plugin as non-owning views.  Both
// branches run the same sm_100a kernels.  A failing plugin call falls back to
// the operator, as in the reference.
#pragma once

#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "cuda_op/detail/cuBlas/gemm.hpp"
#include "cuda_op/detail/cuBlas/gemv.hpp"
#include "jit/Blas/blas_jit_plugins.hpp"
#include "jit/global_jit_manager.hpp"

namespace cu_op_mem {

// How an operator maps onto a plugin.  Specialised for the float operators
// the plugin interface (Tensor<float>) can carry.
template <typename Op>
struct JITBinding {
  static std::string PluginType() { return "unknown_jit"; }
  static StatusCode Run(IJITPlugin&, Op&, const Tensor<float>&, Tensor<float>&) {
    return StatusCode::UNSUPPORTED_OPERATION;
  }
};

template <>
struct JITBinding<Gemm<float>> {
  static std::string PluginType() { return "gemm_jit"; }
  static StatusCode Run(IJITPlugin& plugin, Gemm<float>& op, const Tensor<float>& in, Tensor<float>& out) {
    auto* p = dynamic_cast<GemmJITPlugin*>(&plugin);
    if (!p) return StatusCode::PLUGIN_INCOMPATIBLE;
    p->SetGemmParams(op.TransA(), op.TransB(), op.Alpha(), op.Beta());
    p->BindWeight(op.GetWeight());
    std::vector<Tensor<float>> ins, outs;
    ins.emplace_back(in.data(), in.shape());
    outs.emplace_back(out.data(), out.shape());
    return p->Execute(ins, outs);
  }
};

template <>
struct JITBinding<Gemv<float>> {
  static std::string PluginType() { return "gemv_jit"; }
  // Gemv's Forward(A, y) with weight x  ->  plugin weight A, input x, output y.
  static StatusCode Run(IJITPlugin& plugin, Gemv<float>& op, const Tensor<float>& A, Tensor<float>& y) {
    auto* p = dynamic_cast<GemvJITPlugin*>(&plugin);
    if (!p) return StatusCode::PLUGIN_INCOMPATIBLE;
    p->SetGemvParams(op.TransA(), op.Alpha(), op.Beta());
    p->BindWeight(A);
    std::vector<Tensor<float>> ins, outs;
    ins.emplace_back(op.GetWeight().data(), op.GetWeight().shape());
    outs.emplace_back(y.data(), y.shape());
    return p->Execute(ins, outs);
  }
};

template <typename OperatorType>
class JITWrapper {
 public:
  explicit JITWrapper(OperatorType&& op) : op_(std::move(op)) { InitializeJIT(); }
  JITWrapper(const JITWrapper&) = delete;
  JITWrapper& operator=(const JITWrapper&) = delete;
  JITWrapper(JITWrapper&&) noexcept = default;
  JITWrapper& operator=(JITWrapper&&) noexcept = default;

  StatusCode operator()(const Tensor<float>& input, Tensor<float>& output) {
    if (jit_enabled_ && plugin_ && plugin_->IsCompiled()) return ExecuteJIT(input, output);
    return ExecuteOriginal(input, output);
  }

  StatusCode ExecuteJIT(const Tensor<float>& input, Tensor<float>& output) {
    if (!plugin_ || !plugin_->IsCompiled()) return ExecuteOriginal(input, output);
    try {
      const StatusCode s = JITBinding<OperatorType>::Run(*plugin_, op_, input, output);
      if (s != StatusCode::SUCCESS) return ExecuteOriginal(input, output);
      last_profile_ = plugin_->GetPerformanceProfile();
      return s;
    } catch (const std::exception&) {
      return ExecuteOriginal(input, output);
    }
  }

  StatusCode ExecuteOriginal(const Tensor<float>& input, Tensor<float>& output) { return op_(input, output); }

  void SetJITConfig(const JITConfig& c) {
    config_ = c;
    if (plugin_) plugin_->SetConfig(c);
  }
  JITConfig GetJITConfig() const { return config_; }
  void EnableJIT(bool enable) {
    jit_enabled_ = enable;
    if (enable && plugin_ && !plugin_->IsCompiled()) CompileJIT();
  }
  bool IsJITEnabled() const { return jit_enabled_; }
  void EnableAutoTuning(bool enable) {
    auto_tuning_ = enable;
    if (plugin_) plugin_->EnableAutoTuning(enable);
  }
  bool IsAutoTuningEnabled() const { return auto_tuning_; }
  PerformanceProfile GetPerformanceProfile() const { return last_profile_; }
  void UpdatePerformanceProfile(const PerformanceProfile& p) { last_profile_ = p; }
  bool IsJITCompiled() const { return plugin_ && plugin_->IsCompiled(); }
  bool IsJITInitialized() const { return plugin_ && plugin_->IsInitialized(); }
  std::string GetLastError() const { return plugin_ ? plugin_->GetLastError() : ""; }
  void Cleanup() {
    if (plugin_) plugin_->Cleanup();
  }
  size_t GetMemoryUsage() const { return plugin_ ? plugin_->GetMemoryUsage() : 0; }
  OperatorType& GetOriginalOperator() { return op_; }
  const OperatorType& GetOriginalOperator() const { return op_; }
  IJITPlugin* GetPlugin() { return plugin_.get(); }

  StatusCode CompileJIT() {
    if (!plugin_) return StatusCode::NOT_INITIALIZED;
    const StatusCode s = plugin_->Initialize();
    if (s != StatusCode::SUCCESS) return s;
    return plugin_->Compile(config_);
  }
  void OptimizeJIT() {
    if (plugin_ && auto_tuning_) plugin_->Optimize(last_profile_);
  }

 private:
  void InitializeJIT() {
    if (!GlobalJITManager::Instance().GetGlobalConfig().enable_jit) return;
    plugin_ = PluginRegistrar::Instance().CreatePlugin(JITBinding<OperatorType>::PluginType());
    if (plugin_) {
      plugin_->SetConfig(config_);
      plugin_->EnableAutoTuning(auto_tuning_);
    }
  }

  OperatorType op_;
  std::unique_ptr<IJITPlugin> plugin_;
  JITConfig config_;
  bool jit_enabled_ = false;
  bool auto_tuning_ = false;
  PerformanceProfile last_profile_;
};

template <typename OperatorType>
JITWrapper<OperatorType> MakeJITWrapper(OperatorType&& op) {
  return JITWrapper<OperatorType>(std::move(op));
}

template <typename OperatorType>
JITWrapper<OperatorType> MakeJITWrapper(OperatorType&& op, const JITConfig& config) {
  JITWrapper<OperatorType> w(std::move(op));
  w.SetJITConfig(config);
  w.EnableJIT(true);
  return w;
}

}  // namespace cu_op_mem
