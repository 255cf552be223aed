// AutoTuner of the C++ facade (include/cuop/performance/auto_tuner.hpp).
#include "performance/auto_tuner.hpp"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <fstream>
#include <limits>
#include <random>
#include <set>
#include <sstream>
#include <thread>

#include <cuda_runtime.h>

namespace cu_op_mem {

namespace {

// The discrete search space of a config: one axis per tunable parameter with
// candidate values (declaration order); every other parameter is fixed at
// its default value.
struct Space {
  std::vector<const ParameterDefinition*> axes;
  ParameterSet fixed;
  explicit Space(const TuningConfig& cfg) {
    for (const auto& p : cfg.parameters) {
      if (p.is_tunable && !p.values.empty()) axes.push_back(&p);
      else fixed[p.name] = p.default_value;
    }
  }
  // Number of distinct sets, saturating at `cap`.
  std::size_t size(std::size_t cap = std::numeric_limits<std::size_t>::max()) const {
    std::size_t n = 1;
    for (const auto* a : axes) {
      if (n > cap / a->values.size()) return cap;
      n *= a->values.size();
    }
    return n;
  }
  ParameterSet at(const std::vector<std::size_t>& idx) const {
    ParameterSet s = fixed;
    for (std::size_t a = 0; a < axes.size(); ++a) s[axes[a]->name] = axes[a]->values[idx[a]];
    return s;
  }
  // Mixed-radix decode of a linear index, first axis outermost.
  std::vector<std::size_t> decode(std::size_t linear) const {
    std::vector<std::size_t> idx(axes.size(), 0);
    for (std::size_t a = axes.size(); a-- > 0;) {
      idx[a] = linear % axes[a]->values.size();
      linear /= axes[a]->values.size();
    }
    return idx;
  }
  // Value indices of a set (a value not among the candidates maps past the end).
  std::vector<std::size_t> encode(const ParameterSet& s) const {
    std::vector<std::size_t> idx(axes.size(), 0);
    for (std::size_t a = 0; a < axes.size(); ++a) {
      const auto& vals = axes[a]->values;
      auto it = s.find(axes[a]->name);
      idx[a] = it == s.end() ? vals.size() : static_cast<std::size_t>(std::find(vals.begin(), vals.end(), it->second) -
                                                                        vals.begin());
    }
    return idx;
  }
};

// Canonical text of a set (sorted name=value pairs): the identity used to
// avoid evaluating a set twice and to key the performance cache.
std::string canonical(const ParameterSet& p) {
  std::vector<std::pair<std::string, std::string>> kv(p.begin(), p.end());
  std::sort(kv.begin(), kv.end());
  std::string out;
  for (const auto& e : kv) out += e.first + "=" + e.second + ";";
  return out;
}

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

bool minimise_target(const std::string& target) { return target == "latency" || target == "memory"; }

// Fraction of axes on which two encoded sets differ.
double hamming(const std::vector<std::size_t>& a, const std::vector<std::size_t>& b) {
  if (a.empty()) return 0.0;
  std::size_t d = 0;
  for (std::size_t i = 0; i < a.size(); ++i) d += a[i] != b[i];
  return static_cast<double>(d) / static_cast<double>(a.size());
}

// Kernel-regression surrogate over evaluated sets: mean of the scores,
// weighted by exp(-(d/0.5)^2) in Hamming distance d, and the distance to the
// nearest evaluated set as the uncertainty.  Scores are larger-is-better.
struct Surrogate {
  std::vector<std::vector<std::size_t>> x;
  std::vector<double> z;  // standardised scores
  void fit(const std::vector<std::vector<std::size_t>>& xs, const std::vector<double>& scores) {
    x = xs;
    double mean = 0, var = 0;
    for (double s : scores) mean += s;
    mean /= scores.empty() ? 1.0 : static_cast<double>(scores.size());
    for (double s : scores) var += (s - mean) * (s - mean);
    const double sd = scores.size() > 1 ? std::sqrt(var / static_cast<double>(scores.size() - 1)) : 0.0;
    z.clear();
    for (double s : scores) z.push_back(sd > 0 ? (s - mean) / sd : 0.0);
  }
  void predict(const std::vector<std::size_t>& c, double& mu, double& sigma) const {
    double wsum = 0, acc = 0, dmin = 1.0;
    for (std::size_t i = 0; i < x.size(); ++i) {
      const double d = hamming(c, x[i]);
      const double w = std::exp(-(d / 0.5) * (d / 0.5));
      wsum += w;
      acc += w * z[i];
      dmin = std::min(dmin, d);
    }
    mu = wsum > 1e-12 ? acc / wsum : 0.0;
    sigma = x.empty() ? 1.0 : dmin;
  }
};

// Candidate sets a sequential strategy may propose next: the whole space when
// it is small, else seeded random draws plus every one-axis neighbour of
// `around` (the best set so far).
std::vector<std::vector<std::size_t>> candidate_pool(const Space& sp, std::mt19937_64& rng,
                                                     const std::vector<std::size_t>* around) {
  std::vector<std::vector<std::size_t>> pool;
  const std::size_t n = sp.size(4097);
  if (n <= 4096) {
    for (std::size_t i = 0; i < n; ++i) pool.push_back(sp.decode(i));
    return pool;
  }
  for (int i = 0; i < 1024; ++i) {
    std::vector<std::size_t> idx(sp.axes.size());
    for (std::size_t a = 0; a < idx.size(); ++a)
      idx[a] = std::uniform_int_distribution<std::size_t>(0, sp.axes[a]->values.size() - 1)(rng);
    pool.push_back(std::move(idx));
  }
  if (around) {
    for (std::size_t a = 0; a < sp.axes.size(); ++a)
      for (std::size_t v = 0; v < sp.axes[a]->values.size(); ++v) {
        auto idx = *around;
        idx[a] = v;
        pool.push_back(std::move(idx));
      }
  }
  return pool;
}

// Larger-is-better scores of a history (failed evaluations are recorded as
// 0.0 by Tune; a strategy cannot tell them apart and treats them as data).
std::vector<double> scores_of(const std::vector<double>& perf, bool minimise) {
  std::vector<double> s;
  for (double v : perf) s.push_back(minimise ? -v : v);
  return s;
}

}  // namespace

// ------------------------------------------------------------------ strategies
std::vector<ParameterSet> GridSearchStrategy::GenerateParameterSets(const TuningConfig& config, std::size_t count) {
  const Space sp(config);
  const std::size_t n = std::min(sp.size(), count);
  std::vector<ParameterSet> out;
  for (std::size_t i = 0; i < n; ++i) out.push_back(sp.at(sp.decode(i)));
  return out;
}

std::vector<ParameterSet> RandomSearchStrategy::GenerateParameterSets(const TuningConfig& config, std::size_t count) {
  const Space sp(config);
  std::mt19937_64 rng(seed_);
  std::vector<ParameterSet> out;
  const std::size_t n = sp.size(1u << 20);
  if (n < (1u << 20)) {  // a seeded permutation of the whole space
    std::vector<std::size_t> order(n);
    for (std::size_t i = 0; i < n; ++i) order[i] = i;
    std::shuffle(order.begin(), order.end(), rng);
    for (std::size_t i = 0; i < std::min(n, count); ++i) out.push_back(sp.at(sp.decode(order[i])));
    return out;
  }
  std::set<std::string> seen;  // very large spaces: independent draws without repetition
  for (std::size_t tries = 0; out.size() < count && tries < 64 * count; ++tries) {
    std::vector<std::size_t> idx(sp.axes.size());
    for (std::size_t a = 0; a < idx.size(); ++a)
      idx[a] = std::uniform_int_distribution<std::size_t>(0, sp.axes[a]->values.size() - 1)(rng);
    ParameterSet s = sp.at(idx);
    if (seen.insert(canonical(s)).second) out.push_back(std::move(s));
  }
  return out;
}

void BayesianOptimizationStrategy::UpdateStrategy(const std::vector<double>& performance_history,
                                                  const std::vector<ParameterSet>& parameter_history) {
  perf_ = performance_history;
  sets_ = parameter_history;
}

// A few seeded random sets first, then one set per call: the unevaluated
// candidate with the largest upper confidence bound mu + 2 sigma.
std::vector<ParameterSet> BayesianOptimizationStrategy::GenerateParameterSets(const TuningConfig& config,
                                                                              std::size_t count) {
  const Space sp(config);
  std::mt19937_64 rng(seed_ + 0x9E3779B97F4A7C15ull * (++calls_));
  std::set<std::string> done;
  for (const auto& s : sets_) done.insert(canonical(s));
  const std::size_t n_init = std::min<std::size_t>(3, sp.size());
  std::vector<ParameterSet> out;
  if (sets_.size() < n_init) {
    RandomSearchStrategy init(seed_);
    for (auto& s : init.GenerateParameterSets(config, n_init)) {
      if (out.size() >= count) break;
      if (!done.count(canonical(s))) out.push_back(std::move(s));
    }
    if (!out.empty()) return out;
  }
  const bool minimise = minimise_target(config.optimization_target);
  std::vector<std::vector<std::size_t>> xs;
  for (const auto& s : sets_) xs.push_back(sp.encode(s));
  Surrogate model;
  model.fit(xs, scores_of(perf_, minimise));
  const std::vector<std::size_t>* best = nullptr;
  if (!perf_.empty()) {
    const auto sc = scores_of(perf_, minimise);
    best = &xs[static_cast<std::size_t>(std::max_element(sc.begin(), sc.end()) - sc.begin())];
  }
  double best_ucb = -std::numeric_limits<double>::infinity();
  ParameterSet pick;
  bool have = false;
  for (const auto& c : candidate_pool(sp, rng, best)) {
    ParameterSet s = sp.at(c);
    if (done.count(canonical(s))) continue;
    double mu, sigma;
    model.predict(c, mu, sigma);
    const double ucb = mu + 2.0 * sigma;
    if (!have || ucb > best_ucb) {
      best_ucb = ucb;
      pick = std::move(s);
      have = true;
    }
  }
  if (have && count > 0) out.push_back(std::move(pick));
  return out;
}

void GeneticAlgorithmStrategy::UpdateStrategy(const std::vector<double>& performance_history,
                                              const std::vector<ParameterSet>& parameter_history) {
  perf_ = performance_history;
  sets_ = parameter_history;
}

// Generation 0: a seeded random population.  Later generations are bred from
// every set evaluated so far: the two best carry over (already evaluated),
// children come from binary-tournament parents among the better half,
// uniform crossover and per-gene mutation (probability 1 / number of
// parameters, at least 0.1); a child equal to an evaluated set is redrawn.
// An empty answer means no new set could be bred.
std::vector<ParameterSet> GeneticAlgorithmStrategy::GenerateParameterSets(const TuningConfig& config,
                                                                          std::size_t count) {
  const Space sp(config);
  const std::size_t space = sp.size(1u << 20);
  const std::size_t pop = std::max<std::size_t>(1, std::min<std::size_t>({8, space, count}));
  std::mt19937_64 rng(seed_ + 0x2545F4914F6CDD1Dull * (generation_ + 1));
  std::set<std::string> done;
  for (const auto& s : sets_) done.insert(canonical(s));
  std::vector<ParameterSet> out;
  if (generation_ == 0 || sets_.empty()) {
    RandomSearchStrategy init(seed_);
    for (auto& s : init.GenerateParameterSets(config, pop))
      if (!done.count(canonical(s))) out.push_back(std::move(s));
    ++generation_;
    return out;
  }
  const bool minimise = minimise_target(config.optimization_target);
  const auto sc = scores_of(perf_, minimise);
  std::vector<std::size_t> rank(sets_.size());
  for (std::size_t i = 0; i < rank.size(); ++i) rank[i] = i;
  std::stable_sort(rank.begin(), rank.end(), [&](std::size_t a, std::size_t b) { return sc[a] > sc[b]; });
  const std::size_t parents = std::max<std::size_t>(2, (rank.size() + 1) / 2);
  auto tournament = [&]() -> const ParameterSet& {
    std::uniform_int_distribution<std::size_t> d(0, std::min(parents, rank.size()) - 1);
    const std::size_t a = rank[d(rng)], b = rank[d(rng)];
    return sc[a] >= sc[b] ? sets_[a] : sets_[b];
  };
  const double pm = sp.axes.empty() ? 0.0 : std::max(0.1, 1.0 / static_cast<double>(sp.axes.size()));
  std::uniform_real_distribution<double> u01(0.0, 1.0);
  std::set<std::string> fresh;
  for (std::size_t tries = 0; out.size() < pop && tries < 64 * pop; ++tries) {
    const ParameterSet& p1 = tournament();
    const ParameterSet& p2 = tournament();
    ParameterSet child = sp.fixed;
    for (const auto* a : sp.axes) {
      auto i1 = p1.find(a->name), i2 = p2.find(a->name);
      std::string v = u01(rng) < 0.5 ? (i1 != p1.end() ? i1->second : a->default_value)
                                     : (i2 != p2.end() ? i2->second : a->default_value);
      if (u01(rng) < pm) v = a->values[std::uniform_int_distribution<std::size_t>(0, a->values.size() - 1)(rng)];
      child[a->name] = v;
    }
    const std::string key = canonical(child);
    if (done.count(key) || !fresh.insert(key).second) continue;
    out.push_back(std::move(child));
  }
  ++generation_;
  return out;
}

std::unique_ptr<ITuningStrategy> MakeTuningStrategy(const std::string& name) {
  if (name == "GridSearch" || name == "grid") return std::make_unique<GridSearchStrategy>();
  if (name == "RandomSearch" || name == "random") return std::make_unique<RandomSearchStrategy>();
  if (name == "BayesianOptimization" || name == "bayesian") return std::make_unique<BayesianOptimizationStrategy>();
  if (name == "GeneticAlgorithm" || name == "genetic") return std::make_unique<GeneticAlgorithmStrategy>();
  return nullptr;
}

// ------------------------------------------------------------------ AutoTuner
AutoTuner& AutoTuner::Instance() {
  static AutoTuner t;
  return t;
}

void AutoTuner::StopTuning() {
  enabled_.store(false);
  stop_generation_.fetch_add(1);
}

void AutoTuner::Reset() {
  std::lock_guard<std::mutex> lk(mu_);
  config_.parameters.clear();
  parameters_.clear();
  history_.clear();
  cache_.clear();
}

void AutoTuner::SetTuningConfig(const TuningConfig& config) {
  std::string refused, keep;
  {
    std::lock_guard<std::mutex> lk(mu_);
    config_ = config;
    if (!config.tuning_strategy.empty()) {
      auto s = MakeTuningStrategy(config.tuning_strategy);
      if (s) strategy_ = s->GetStrategyName();
      else refused = last_error_ = "unknown tuning strategy '" + config.tuning_strategy + "'";
    }
    config_.tuning_strategy = keep = strategy_;
  }
  if (!refused.empty()) std::fprintf(stderr, "cuop AutoTuner: %s; keeping %s\n", refused.c_str(), keep.c_str());
}

TuningConfig AutoTuner::GetTuningConfig() const {
  std::lock_guard<std::mutex> lk(mu_);
  return config_;
}

void AutoTuner::AddParameter(const ParameterDefinition& param) {
  std::lock_guard<std::mutex> lk(mu_);
  for (auto& p : parameters_)
    if (p.name == param.name) {
      p = param;
      return;
    }
  parameters_.push_back(param);
}

void AutoTuner::RemoveParameter(const std::string& param_name) {
  std::lock_guard<std::mutex> lk(mu_);
  auto drop = [&](std::vector<ParameterDefinition>& ps) {
    ps.erase(std::remove_if(ps.begin(), ps.end(), [&](const ParameterDefinition& p) { return p.name == param_name; }),
             ps.end());
  };
  drop(parameters_);
  drop(config_.parameters);
}

std::vector<ParameterDefinition> AutoTuner::GetParameters() const {
  std::lock_guard<std::mutex> lk(mu_);
  return parameters_;
}

void AutoTuner::SetTuningStrategy(const std::string& strategy_name) {
  auto s = MakeTuningStrategy(strategy_name);
  std::string keep;
  {
    std::lock_guard<std::mutex> lk(mu_);
    if (s) {
      strategy_ = config_.tuning_strategy = s->GetStrategyName();
      return;
    }
    last_error_ = "unknown tuning strategy '" + strategy_name + "'";
    keep = strategy_;
  }
  std::fprintf(stderr, "cuop AutoTuner: unknown tuning strategy '%s'; keeping %s\n", strategy_name.c_str(),
               keep.c_str());
}

std::string AutoTuner::GetCurrentStrategy() const {
  std::lock_guard<std::mutex> lk(mu_);
  return strategy_;
}

std::string AutoTuner::GetLastError() const {
  std::lock_guard<std::mutex> lk(mu_);
  return last_error_;
}

bool AutoTuner::minimise(const TuningConfig& cfg) const { return minimise_target(cfg.optimization_target); }

TuningConfig AutoTuner::effective_config() const {
  TuningConfig cfg = config_;
  for (const auto& p : parameters_) {
    auto it = std::find_if(cfg.parameters.begin(), cfg.parameters.end(),
                           [&](const ParameterDefinition& q) { return q.name == p.name; });
    if (it != cfg.parameters.end()) *it = p;
    else cfg.parameters.push_back(p);
  }
  cfg.tuning_strategy = strategy_;
  return cfg;
}

TuningResult AutoTuner::Tune(const std::string& operator_name, BenchmarkFunction benchmark_func) {
  const uint64_t generation = stop_generation_.load();
  TuningConfig cfg;
  {
    std::lock_guard<std::mutex> lk(mu_);
    cfg = effective_config();
  }
  const bool min = minimise(cfg);
  std::unique_ptr<ITuningStrategy> strategy = MakeTuningStrategy(cfg.tuning_strategy);
  const Space sp(cfg);
  TuningResult r;
  r.strategy_name = strategy->GetStrategyName();
  r.tuning_start_time = std::chrono::high_resolution_clock::now();
  auto last_report = std::chrono::steady_clock::now();
  const std::size_t budget = std::max<std::size_t>(1, cfg.max_iterations);
  std::set<std::string> evaluated;
  std::size_t since_improvement = 0, failures = 0;
  bool have = false, stopped = false, exhausted = false, early = false;
  std::vector<std::pair<std::string, double>> measured;
  while (benchmark_func && !stopped && !early && r.iterations_used < budget) {
    std::vector<ParameterSet> batch = strategy->GenerateParameterSets(cfg, budget - r.iterations_used);
    bool any_new = false;
    for (ParameterSet& s : batch) {
      for (const auto& f : sp.fixed) s.emplace(f.first, f.second);  // parameters the strategy left out
      const std::string key = canonical(s);
      if (!evaluated.insert(key).second) continue;
      any_new = true;
      if (stop_generation_.load() != generation) {
        stopped = true;
        break;
      }
      double v = 0.0;
      bool ok = true;
      try {
        v = benchmark_func(s);
      } catch (const std::exception& e) {
        ok = false;
        r.recommendations.push_back("evaluation " + std::to_string(r.iterations_used + 1) + " [" +
                                    format_params(s, ", ") + "] failed: " + e.what());
      } catch (...) {
        ok = false;
        r.recommendations.push_back("evaluation " + std::to_string(r.iterations_used + 1) + " [" +
                                    format_params(s, ", ") + "] failed with a non-standard exception");
      }
      if (!ok) {
        v = 0.0;
        ++failures;
      } else {
        measured.emplace_back(key, v);
      }
      r.performance_history.push_back(v);
      r.parameter_history.push_back(s);
      ++r.iterations_used;
      strategy->UpdateStrategy(r.performance_history, r.parameter_history);
      const bool better = ok && (!have || (min ? v < r.best_performance : v > r.best_performance));
      const double rel = have && r.best_performance != 0.0 ? std::abs(v - r.best_performance) /
                                                                 std::abs(r.best_performance)
                                                           : 1.0;
      if (better && (!have || rel > cfg.improvement_threshold)) {
        r.best_performance = v;
        r.best_parameters = s;
        have = true;
        since_improvement = 0;
      } else if (cfg.enable_early_stopping && ++since_improvement >= cfg.patience) {
        early = true;
        break;
      }
      if (monitoring_.load()) {
        const auto now = std::chrono::steady_clock::now();
        if (now - last_report >= std::chrono::milliseconds(monitor_ms_.load())) {
          last_report = now;
          notify(r);
        }
      }
      if (r.iterations_used >= budget) break;
    }
    if (!any_new) {
      exhausted = true;
      break;
    }
  }
  r.converged = !stopped && (early || exhausted || r.iterations_used >= budget);
  const std::size_t space = sp.size();
  r.convergence_rate = space == 0 ? 0.0 : std::min(1.0, static_cast<double>(r.iterations_used) /
                                                            static_cast<double>(space));
  r.tuning_end_time = std::chrono::high_resolution_clock::now();
  if (failures) r.recommendations.push_back(std::to_string(failures) + " evaluation(s) threw; recorded as 0.0");
  if (!have && r.iterations_used) r.recommendations.push_back("no evaluation succeeded");
  std::ostringstream sum;
  sum << operator_name << ": " << r.strategy_name << ", " << r.iterations_used << " of " << space
      << " parameter sets, best " << r.best_performance << " (" << cfg.optimization_target << ")";
  if (stopped) sum << ", stopped";
  r.optimization_summary = sum.str();
  {
    std::lock_guard<std::mutex> lk(mu_);
    history_.push_back(r);
    for (const auto& m : measured) cache_[m.first] = m.second;
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

double AutoTuner::PredictPerformance(const ParameterSet& parameters) const {
  std::lock_guard<std::mutex> lk(mu_);
  auto it = cache_.find(canonical(parameters));
  if (it != cache_.end()) return it->second;
  if (cache_.empty()) return 0.0;
  // Kernel regression over every cached evaluation, on the same Hamming
  // distance the Bayesian strategy uses (parameters compared by name).
  double wsum = 0, acc = 0;
  for (const auto& e : cache_) {
    std::size_t n = 0, diff = 0;
    for (const auto& kv : parameters) {
      ++n;
      const std::string needle = kv.first + "=" + kv.second + ";";
      if (e.first.find(needle) == std::string::npos) ++diff;
    }
    const double d = n ? static_cast<double>(diff) / static_cast<double>(n) : 1.0;
    const double w = std::exp(-(d / 0.5) * (d / 0.5));
    wsum += w;
    acc += w * e.second;
  }
  return wsum > 0 ? acc / wsum : 0.0;
}

std::vector<std::string> AutoTuner::GetPerformanceInsights() const {
  std::lock_guard<std::mutex> lk(mu_);
  std::vector<std::string> out;
  if (history_.empty()) {
    out.push_back("No tuning history available");
    return out;
  }
  const TuningResult& r = history_.back();
  out.push_back(r.converged ? "Tuning converged" : "Tuning did not converge (stopped before its budget)");
  out.push_back("Strategy " + (r.strategy_name.empty() ? std::string("unknown") : r.strategy_name) + " evaluated " +
                std::to_string(r.iterations_used) + " parameter sets");
  if (!r.performance_history.empty() && r.performance_history.front() != 0.0) {
    const double first = r.performance_history.front();
    const double gain = minimise_target(config_.optimization_target) ? (first - r.best_performance) / first
                                                                     : (r.best_performance - first) / first;
    out.push_back("Best is " + std::to_string(100.0 * gain) + "% better than the first evaluation");
  }
  return out;
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

std::string AutoTuner::GenerateTuningReport(const TuningResult& r) const {
  std::ostringstream o;
  const double secs = std::chrono::duration<double>(r.tuning_end_time - r.tuning_start_time).count();
  o << "Tuning report\n"
    << "  summary:     " << r.optimization_summary << "\n"
    << "  strategy:    " << r.strategy_name << "\n"
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

}  // namespace cu_op_mem
