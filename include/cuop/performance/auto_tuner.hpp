// AutoTuner: benchmarks parameter sets through a caller-supplied function
// and keeps the best (reference include/performance/auto_tuner.hpp:28-53,
// src/performance/auto_tuner.cu:100-295).  Strategies: "grid" (every
// combination of the tunable parameters' values, in order, up to
// max_iterations) and "random" (seeded draws without repetition).  Early
// stopping ends a run after `patience` evaluations without an improvement
// larger than improvement_threshold (relative).  optimization_target
// "latency" / "memory" minimise the benchmark value, anything else
// ("throughput", "accuracy") maximises it.  History persists as plain text.
//
// For GEMM, the benchmark function typically forces one variant
// (cuopx_set_gemm_variant) and times it; the winning variant becomes a row
// of the selection table (cuopx_tuning_load).  No background thread: the
// reference's StartTuning/StopTuning loop is not part of this library.
#pragma once

#include <atomic>
#include <chrono>
#include <cstddef>
#include <functional>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

namespace cu_op_mem {

enum class ParameterType { INTEGER, FLOAT, STRING, BOOLEAN, ENUM };

struct ParameterDefinition {
  std::string name;
  ParameterType type = ParameterType::ENUM;
  std::string description;
  std::vector<std::string> values;  // candidate values (tunable parameters)
  std::string default_value;        // used when not tunable or no values
  std::string min_value, max_value;
  double weight = 1.0;
  bool is_tunable = true;
};

struct TuningConfig {
  std::string operator_name;
  std::vector<ParameterDefinition> parameters;
  std::string optimization_target = "throughput";
  std::size_t max_iterations = 100;
  double convergence_threshold = 0.01;
  double improvement_threshold = 0.0;
  bool enable_parallel_tuning = false;  // evaluations always run in order here
  std::size_t parallel_workers = 1;
  bool enable_early_stopping = false;
  std::size_t patience = 10;
  std::string tuning_strategy = "grid";
  std::string result_save_path;
};

using ParameterSet = std::unordered_map<std::string, std::string>;

struct TuningResult {
  ParameterSet best_parameters;
  double best_performance = 0.0;
  std::size_t iterations_used = 0;
  std::vector<double> performance_history;
  std::vector<ParameterSet> parameter_history;
  std::string optimization_summary;
  bool converged = false;
  double convergence_rate = 0.0;
  std::chrono::high_resolution_clock::time_point tuning_start_time;
  std::chrono::high_resolution_clock::time_point tuning_end_time;
  std::vector<std::string> recommendations;
};

using BenchmarkFunction = std::function<double(const ParameterSet&)>;

class AutoTuner {
 public:
  static AutoTuner& Instance();
  AutoTuner() = default;

  void SetTuningConfig(const TuningConfig& config);
  TuningConfig GetTuningConfig() const;
  void AddParameter(const ParameterDefinition& param);
  void RemoveParameter(const std::string& param_name);
  std::vector<ParameterDefinition> GetParameters() const;

  void SetTuningStrategy(const std::string& strategy_name);  // "grid" | "random"
  std::vector<std::string> GetAvailableStrategies() const { return {"grid", "random"}; }

  // Evaluates parameter sets with `benchmark_func` and returns the best.
  // The result is appended to the history (and saved to
  // config.result_save_path when set).
  TuningResult Tune(const std::string& operator_name, BenchmarkFunction benchmark_func);
  // Tune on a worker thread (the benchmark callbacks run there, with the
  // caller's current CUDA device made current first).  The reference's
  // signature returns the result, so this call waits for it; StopTuning()
  // from another thread ends it after the evaluation in progress.
  TuningResult TuneAsync(const std::string& operator_name, BenchmarkFunction benchmark_func);

  // StopTuning() makes running Tune calls return after their current
  // evaluation (result marked not converged); StartTuning() re-arms.
  // IsTuning(): a Tune call is in progress.
  void StartTuning() { stop_.store(false); }
  void StopTuning() { stop_.store(true); }
  bool IsTuning() const { return active_.load() > 0; }

  // Human-readable report, and a CSV of every evaluation
  // (iteration, performance, parameters as name=value;...).
  std::string GenerateTuningReport(const TuningResult& result) const;
  void ExportResults(const TuningResult& result, const std::string& filename) const;

  // Callbacks get each finished result; with real-time monitoring on they
  // also get the partial result during Tune, at most once per interval.
  void RegisterCallback(std::function<void(const TuningResult&)> callback);
  void EnableRealTimeMonitoring(bool enable) { monitoring_.store(enable); }
  void SetMonitoringInterval(int interval_ms) { monitor_ms_.store(interval_ms < 0 ? 0 : interval_ms); }

  void SaveTuningHistory(const std::string& filename) const;
  void LoadTuningHistory(const std::string& filename);
  std::vector<TuningResult> GetTuningHistory() const;
  void Reset();

 private:
  bool better(double a, double b) const;  // is a better than b
  std::vector<ParameterSet> candidate_sets(const TuningConfig& cfg) const;

  void notify(const TuningResult& r);

  mutable std::mutex mu_;
  TuningConfig config_;
  std::vector<TuningResult> history_;
  std::vector<std::function<void(const TuningResult&)>> callbacks_;
  std::atomic<bool> stop_{false};
  std::atomic<int> active_{0};
  std::atomic<bool> monitoring_{false};
  std::atomic<int> monitor_ms_{1000};
};

}  // namespace cu_op_mem
