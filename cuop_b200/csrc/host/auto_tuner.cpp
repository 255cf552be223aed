// AutoTuner of the C++ facade (include/cuop/performance/auto_tuner.hpp).
#include "performance/auto_tuner.hpp"

#include <algorithm>
#include <cmath>
#include <fstream>
#include <random>
#include <sstream>
#include <thread>

#include <cuda_runtime.h>

namespace cu_op_mem {

AutoTuner& AutoTuner::Instance() {
  static AutoTuner t;
  return t;
}

void AutoTuner::SetTuningConfig(const TuningConfig& config) {
  std::lock_guard<std::mutex> lk(mu_);
  config_ = config;
}

TuningConfig AutoTuner::GetTuningConfig() const {
  std::lock_guard<std::mutex> lk(mu_);
  return config_;
}

void AutoTuner::AddParameter(const ParameterDefinition& param) {
  std::lock_guard<std::mutex> lk(mu_);
  for (auto& p : config_.parameters)
    if (p.name == param.name) {
      p = param;
      return;
    }
  config_.parameters.push_back(param);
}

void AutoTuner::RemoveParameter(const std::string& param_name) {
  std::lock_guard<std::mutex> lk(mu_);
  auto& ps = config_.parameters;
  ps.erase(std::remove_if(ps.begin(), ps.end(), [&](const ParameterDefinition& p) { return p.name == param_name; }),
           ps.end());
}

std::vector<ParameterDefinition> AutoTuner::GetParameters() const {
  std::lock_guard<std::mutex> lk(mu_);
  return config_.parameters;
}

void AutoTuner::SetTuningStrategy(const std::string& strategy_name) {
  std::lock_guard<std::mutex> lk(mu_);
  if (strategy_name == "grid" || strategy_name == "random") config_.tuning_strategy = strategy_name;
}

bool AutoTuner::better(double a, double b) const {
  const bool minimise = config_.optimization_target == "latency" || config_.optimization_target == "memory";
  return minimise ? a < b : a > b;
}

// Every combination of the tunable parameters' values (mixed-radix order,
// first parameter fastest); fixed parameters take their default value.
std::vector<ParameterSet> AutoTuner::candidate_sets(const TuningConfig& cfg) const {
  std::vector<const ParameterDefinition*> axes;
  ParameterSet fixed;
  for (const auto& p : cfg.parameters) {
    if (p.is_tunable && !p.values.empty()) axes.push_back(&p);
    else fixed[p.name] = p.default_value;
  }
  std::vector<ParameterSet> out;
  std::vector<std::size_t> idx(axes.size(), 0);
  while (true) {
    ParameterSet s = fixed;
    for (std::size_t a = 0; a < axes.size(); ++a) s[axes[a]->name] = axes[a]->values[idx[a]];
    out.push_back(std::move(s));
    std::size_t a = 0;
    for (; a < axes.size(); ++a) {
      if (++idx[a] < axes[a]->values.size()) break;
      idx[a] = 0;
    }
    if (a == axes.size()) break;
  }
  return out;
}

TuningResult AutoTuner::Tune(const std::string& operator_name, BenchmarkFunction benchmark_func) {
  struct Active {
    std::atomic<int>& n;
    explicit Active(std::atomic<int>& c) : n(c) { ++n; }
    ~Active() { --n; }
  } active(active_);
  TuningConfig cfg = GetTuningConfig();
  TuningResult r;
  auto last_report = std::chrono::steady_clock::now();
  bool stopped = false;
  r.tuning_start_time = std::chrono::high_resolution_clock::now();
  std::vector<ParameterSet> sets = candidate_sets(cfg);
  if (cfg.tuning_strategy == "random") {
    std::mt19937_64 rng(0x5eedu);
    std::shuffle(sets.begin(), sets.end(), rng);
  }
  const std::size_t limit = std::min(sets.size(), std::max<std::size_t>(1, cfg.max_iterations));
  std::size_t since_improvement = 0;
  bool have = false;
  for (std::size_t i = 0; i < limit && benchmark_func; ++i) {
    if (stop_.load()) {
      stopped = true;
      break;
    }
    const double v = benchmark_func(sets[i]);
    r.performance_history.push_back(v);
    r.parameter_history.push_back(sets[i]);
    ++r.iterations_used;
    const double rel = have && r.best_performance != 0.0 ? (v - r.best_performance) / std::abs(r.best_performance) : 1.0;
    const bool improved = !have || (better(v, r.best_performance) && std::abs(rel) > cfg.improvement_threshold);
    if (improved) {
      r.best_performance = v;
      r.best_parameters = sets[i];
      have = true;
      since_improvement = 0;
    } else if (cfg.enable_early_stopping && ++since_improvement >= cfg.patience) {
      r.converged = true;
      break;
    }
    if (monitoring_.load()) {
      const auto now = std::chrono::steady_clock::now();
      if (now - last_report >= std::chrono::milliseconds(monitor_ms_.load())) {
        last_report = now;
        notify(r);
      }
    }
  }
  if (r.iterations_used == limit && !stopped) r.converged = true;
  r.convergence_rate = sets.empty() ? 0.0 : static_cast<double>(r.iterations_used) / static_cast<double>(sets.size());
  r.tuning_end_time = std::chrono::high_resolution_clock::now();
  std::ostringstream sum;
  sum << operator_name << ": " << r.iterations_used << " of " << sets.size() << " parameter sets, best "
      << r.best_performance << " (" << cfg.optimization_target << ")";
  r.optimization_summary = sum.str();
  {
    std::lock_guard<std::mutex> lk(mu_);
    history_.push_back(r);
  }
  if (!cfg.result_save_path.empty()) SaveTuningHistory(cfg.result_save_path);
  notify(r);
  return r;
}

TuningResult AutoTuner::TuneAsync(const std::string& operator_name, BenchmarkFunction benchmark_func) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = -1;
  }
  TuningResult r;
  std::thread worker([&] {
    if (dev >= 0 && cudaSetDevice(dev) != cudaSuccess) cudaGetLastError();
    r = Tune(operator_name, benchmark_func);
  });
  worker.join();
  return r;
}

void AutoTuner::RegisterCallback(std::function<void(const TuningResult&)> callback) {
  if (!callback) return;
  std::lock_guard<std::mutex> lk(mu_);
  callbacks_.push_back(std::move(callback));
}

void AutoTuner::notify(const TuningResult& r) {
  std::vector<std::function<void(const TuningResult&)>> cbs;
  {
    std::lock_guard<std::mutex> lk(mu_);
    cbs = callbacks_;
  }
  for (const auto& cb : cbs) cb(r);
}

namespace {
std::string format_params(const ParameterSet& p, const char* sep) {
  std::vector<std::pair<std::string, std::string>> kv(p.begin(), p.end());
  std::sort(kv.begin(), kv.end());
  std::string out;
  for (const auto& e : kv) {
    if (!out.empty()) out += sep;
    out += e.first + "=" + e.second;
  }
  return out;
}
}  // namespace

std::string AutoTuner::GenerateTuningReport(const TuningResult& r) const {
  std::ostringstream o;
  const double secs = std::chrono::duration<double>(r.tuning_end_time - r.tuning_start_time).count();
  o << "Tuning report\n"
    << "  summary:     " << r.optimization_summary << "\n"
    << "  best:        " << r.best_performance << "  [" << format_params(r.best_parameters, ", ") << "]\n"
    << "  evaluations: " << r.iterations_used << (r.converged ? " (converged)" : " (stopped early)") << "\n"
    << "  wall time:   " << secs << " s\n";
  if (!r.performance_history.empty()) {
    const auto mm = std::minmax_element(r.performance_history.begin(), r.performance_history.end());
    o << "  range:       " << *mm.first << " .. " << *mm.second << "\n";
  }
  for (const auto& rec : r.recommendations) o << "  note:        " << rec << "\n";
  return o.str();
}

void AutoTuner::ExportResults(const TuningResult& r, const std::string& filename) const {
  std::ofstream f(filename);
  f << "iteration,performance,parameters\n";
  for (std::size_t i = 0; i < r.performance_history.size(); ++i) {
    f << i << ',' << r.performance_history[i] << ",\""
      << (i < r.parameter_history.size() ? format_params(r.parameter_history[i], ";") : std::string()) << "\"\n";
  }
}

// History file: one block per result,
//   result <best_performance> <iterations_used> <converged>
//   best <name>=<value> ...
//   summary <text>
void AutoTuner::SaveTuningHistory(const std::string& filename) const {
  std::lock_guard<std::mutex> lk(mu_);
  std::ofstream f(filename);
  for (const auto& r : history_) {
    f << "result " << r.best_performance << ' ' << r.iterations_used << ' ' << (r.converged ? 1 : 0) << '\n';
    f << "best";
    std::vector<std::pair<std::string, std::string>> kv(r.best_parameters.begin(), r.best_parameters.end());
    std::sort(kv.begin(), kv.end());
    for (const auto& p : kv) f << ' ' << p.first << '=' << p.second;
    f << "\nsummary " << r.optimization_summary << '\n';
  }
}

void AutoTuner::LoadTuningHistory(const std::string& filename) {
  std::ifstream f(filename);
  std::vector<TuningResult> loaded;
  std::string line;
  while (std::getline(f, line)) {
    std::istringstream ls(line);
    std::string tag;
    ls >> tag;
    if (tag == "result") {
      TuningResult r;
      int conv = 0;
      ls >> r.best_performance >> r.iterations_used >> conv;
      r.converged = conv != 0;
      loaded.push_back(r);
    } else if (tag == "best" && !loaded.empty()) {
      for (std::string kv; ls >> kv;) {
        const auto eq = kv.find('=');
        if (eq != std::string::npos) loaded.back().best_parameters[kv.substr(0, eq)] = kv.substr(eq + 1);
      }
    } else if (tag == "summary" && !loaded.empty()) {
      std::getline(ls >> std::ws, loaded.back().optimization_summary);
    }
  }
  std::lock_guard<std::mutex> lk(mu_);
  history_.insert(history_.end(), loaded.begin(), loaded.end());
}

std::vector<TuningResult> AutoTuner::GetTuningHistory() const {
  std::lock_guard<std::mutex> lk(mu_);
  return history_;
}

void AutoTuner::Reset() {
  std::lock_guard<std::mutex> lk(mu_);
  config_ = TuningConfig{};
  history_.clear();
  callbacks_.clear();
  stop_.store(false);
}

}  // namespace cu_op_mem
