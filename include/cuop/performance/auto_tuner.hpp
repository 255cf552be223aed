// AutoTuner: benchmarks parameter sets through a caller-supplied function
// and keeps the best (reference include/performance/auto_tuner.hpp:28-53,
// 77-200; src/performance/auto_tuner.cu:100-295).
//
// Strategies, selected by name (SetTuningStrategy or TuningConfig::
// tuning_strategy); the reference's names and the short forms its config
// comment lists are both accepted:
//   "GridSearch"           ("grid")     every combination, first parameter
//                                       outermost, in declaration order;
//   "RandomSearch"         ("random")   the same sets in a seeded random order,
//                                       without repetition;
//   "BayesianOptimization" ("bayesian") sequential model-based search: a few
//                                       seeded random sets, then each next set
//                                       maximises an upper confidence bound of
//                                       a kernel-regression surrogate over the
//                                       (Hamming) distance between sets;
//   "GeneticAlgorithm"     ("genetic")  generations of a seeded population:
//                                       elitism, tournament selection, uniform
//                                       crossover and per-gene mutation.
// An unknown name is refused: it is printed to stderr, kept in
// GetLastError(), and the current strategy stays.  A parameter set is
// never evaluated twice in one Tune call.
//
// optimization_target "latency" / "memory" minimise the benchmark value,
// anything else ("throughput", "accuracy") maximises it.  Early stopping
// ends a run after `patience` evaluations without an improvement larger
// than improvement_threshold (relative).  A benchmark call that throws is
// recorded with performance 0.0, never becomes the best, and the run goes
// on (as in the reference, auto_tuner.cu:159-163).
//
// StartTuning() / StopTuning() / IsTuning() follow the reference: IsTuning()
// reports the enabled flag that StartTuning sets and StopTuning clears;
// Tune does not require it.  StopTuning() also ends the Tune calls running
// at that moment after their current evaluation (later calls are not
// affected).  History persists as plain text (the reference's JSON needs
// jsoncpp).
//
// For GEMM, the benchmark function typically forces one variant
// (cuopx_set_gemm_variant) and times it; the winning variant becomes a row
// of the selection table (cuopx_tuning_load).
#pragma once

#include <atomic>
#include <chrono>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <memory>
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
  // Empty: keep the tuner's current strategy (SetTuningConfig then changes
  // only the other fields, as in the reference, whose config string does not
  // select the strategy object).
  std::string tuning_strategy;
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
  std::string strategy_name;  // the strategy that produced the sets (not in the reference)
};

using BenchmarkFunction = std::function<double(const ParameterSet&)>;

// Strategy interface of the reference (include/performance/auto_tuner.hpp:77-86).
// Tune asks GenerateParameterSets for at most `count` next sets, evaluates
// the new ones in order, calling UpdateStrategy after each, and asks again
// until the iteration budget is spent or a request yields no set that was not
// evaluated yet.  A strategy may return fewer sets than `count` (the
// sequential ones return one at a time).
class ITuningStrategy {
 public:
  virtual ~ITuningStrategy() = default;
  virtual std::vector<ParameterSet> GenerateParameterSets(const TuningConfig& config, std::size_t count) = 0;
  virtual void UpdateStrategy(const std::vector<double>& performance_history,
                              const std::vector<ParameterSet>& parameter_history) = 0;
  virtual std::string GetStrategyName() const = 0;
};

class GridSearchStrategy : public ITuningStrategy {
 public:
  std::vector<ParameterSet> GenerateParameterSets(const TuningConfig& config, std::size_t count) override;
  void UpdateStrategy(const std::vector<double>&, const std::vector<ParameterSet>&) override {}
  std::string GetStrategyName() const override { return "GridSearch"; }
};

class RandomSearchStrategy : public ITuningStrategy {
 public:
  explicit RandomSearchStrategy(uint64_t seed = 0x5eedu) : seed_(seed) {}
  std::vector<ParameterSet> GenerateParameterSets(const TuningConfig& config, std::size_t count) override;
  void UpdateStrategy(const std::vector<double>&, const std::vector<ParameterSet>&) override {}
  std::string GetStrategyName() const override { return "RandomSearch"; }

 private:
  uint64_t seed_;
};

class BayesianOptimizationStrategy : public ITuningStrategy {
 public:
  explicit BayesianOptimizationStrategy(uint64_t seed = 0xb0u) : seed_(seed) {}
  std::vector<ParameterSet> GenerateParameterSets(const TuningConfig& config, std::size_t count) override;
  void UpdateStrategy(const std::vector<double>& performance_history,
                      const std::vector<ParameterSet>& parameter_history) override;
  std::string GetStrategyName() const override { return "BayesianOptimization"; }

 private:
  uint64_t seed_;
  uint64_t calls_ = 0;
  std::vector<double> perf_;
  std::vector<ParameterSet> sets_;
};

class GeneticAlgorithmStrategy : public ITuningStrategy {
 public:
  explicit GeneticAlgorithmStrategy(uint64_t seed = 0x6au) : seed_(seed) {}
  std::vector<ParameterSet> GenerateParameterSets(const TuningConfig& config, std::size_t count) override;
  void UpdateStrategy(const std::vector<double>& performance_history,
                      const std::vector<ParameterSet>& parameter_history) override;
  std::string GetStrategyName() const override { return "GeneticAlgorithm"; }
  std::size_t Generation() const { return generation_; }

 private:
  uint64_t seed_;
  std::size_t generation_ = 0;
  std::vector<double> perf_;
  std::vector<ParameterSet> sets_;
};

// A strategy object for a name ("GridSearch" ... or "grid" ...); nullptr for
// an unknown name.
std::unique_ptr<ITuningStrategy> MakeTuningStrategy(const std::string& name);

class AutoTuner {
 public:
  static AutoTuner& Instance();
  AutoTuner() = default;

  void StartTuning() { enabled_.store(true); }
  // Clears the enabled flag and ends the Tune calls running now after their
  // current evaluation (their results are marked not converged).
  void StopTuning();
  bool IsTuning() const { return enabled_.load(); }
  // Clears the parameters, the history and the performance cache.
  void Reset();

  void SetTuningConfig(const TuningConfig& config);
  TuningConfig GetTuningConfig() const;
  // Parameters added here join config.parameters for every Tune call (a
  // parameter of the same name replaces the config's).
  void AddParameter(const ParameterDefinition& param);
  void RemoveParameter(const std::string& param_name);
  std::vector<ParameterDefinition> GetParameters() const;

  TuningResult Tune(const std::string& operator_name, BenchmarkFunction benchmark_func);
  // Tune on a worker thread (the benchmark callbacks run there, with the
  // caller's current CUDA device made current first).  The reference's
  // signature returns the result, so this call waits for it; StopTuning()
  // from another thread ends it after the evaluation in progress.
  TuningResult TuneAsync(const std::string& operator_name, BenchmarkFunction benchmark_func);

  void SetTuningStrategy(const std::string& strategy_name);
  std::vector<std::string> GetAvailableStrategies() const {
    return {"GridSearch", "RandomSearch", "BayesianOptimization", "GeneticAlgorithm"};
  }
  // Canonical name of the strategy the next Tune call uses.
  std::string GetCurrentStrategy() const;
  // Last refusal (unknown strategy name); empty when none.
  std::string GetLastError() const;

  void SaveTuningHistory(const std::string& filename) const;
  void LoadTuningHistory(const std::string& filename);
  std::vector<TuningResult> GetTuningHistory() const;

  // The measured value when this exact set was evaluated before, else a
  // kernel-regression estimate from every evaluated set (0.0 with none).
  double PredictPerformance(const ParameterSet& parameters) const;
  std::vector<std::string> GetPerformanceInsights() const;

  // Human-readable report, and a CSV of every evaluation
  // (iteration, performance, parameters as name=value;...).
  std::string GenerateTuningReport(const TuningResult& result) const;
  void ExportResults(const TuningResult& result, const std::string& filename) const;

  // Callbacks get each finished result; with real-time monitoring on they
  // also get the partial result during Tune, at most once per interval.
  void RegisterCallback(std::function<void(const TuningResult&)> callback);
  void EnableRealTimeMonitoring(bool enable) { monitoring_.store(enable); }
  void SetMonitoringInterval(int interval_ms) { monitor_ms_.store(interval_ms < 0 ? 0 : interval_ms); }

 private:
  bool minimise(const TuningConfig& cfg) const;
  TuningConfig effective_config() const;  // config + added parameters, under mu_
  void notify(const TuningResult& r);

  mutable std::mutex mu_;
  TuningConfig config_;
  std::vector<ParameterDefinition> parameters_;
  std::string strategy_ = "GridSearch";
  std::string last_error_;
  std::vector<TuningResult> history_;
  std::unordered_map<std::string, double> cache_;  // canonical set -> last measured value
  std::vector<std::function<void(const TuningResult&)>> callbacks_;
  std::atomic<bool> enabled_{false};
  std::atomic<uint64_t> stop_generation_{0};
  std::atomic<bool> monitoring_{false};
  std::atomic<int> monitor_ms_{1000};
};

// Convenience macros of the reference (auto_tuner.hpp:205-236).
#define CUOP_AUTO_TUNE(op_name, benchmark_func) ::cu_op_mem::AutoTuner::Instance().Tune(op_name, benchmark_func)
#define CUOP_AUTO_TUNE_ASYNC(op_name, benchmark_func) \
  ::cu_op_mem::AutoTuner::Instance().TuneAsync(op_name, benchmark_func)
#define CUOP_ADD_PARAMETER(param_def) ::cu_op_mem::AutoTuner::Instance().AddParameter(param_def)
#define CUOP_SET_TUNING_STRATEGY(strategy_name) ::cu_op_mem::AutoTuner::Instance().SetTuningStrategy(strategy_name)
#define CUOP_PARAM_OF_TYPE_(ptype, name, values, default_val, weight) \
  ::cu_op_mem::ParameterDefinition { name, ptype, "", values, default_val, "", "", weight, true }
#define CUOP_PARAM_INT(name, values, default_val, weight) \
  CUOP_PARAM_OF_TYPE_(::cu_op_mem::ParameterType::INTEGER, name, values, default_val, weight)
#define CUOP_PARAM_FLOAT(name, values, default_val, weight) \
  CUOP_PARAM_OF_TYPE_(::cu_op_mem::ParameterType::FLOAT, name, values, default_val, weight)
#define CUOP_PARAM_STRING(name, values, default_val, weight) \
  CUOP_PARAM_OF_TYPE_(::cu_op_mem::ParameterType::STRING, name, values, default_val, weight)
#define CUOP_PARAM_BOOL(name, values, default_val, weight) \
  CUOP_PARAM_OF_TYPE_(::cu_op_mem::ParameterType::BOOLEAN, name, values, default_val, weight)
#define CUOP_PARAM_ENUM(name, values, default_val, weight) \
  CUOP_PARAM_OF_TYPE_(::cu_op_mem::ParameterType::ENUM, name, values, default_val, weight)

}  // namespace cu_op_mem
