// C++ tests of the cuOP-compatible facade over libcuopx.so, written the way
// the reference's GTest suites are (test/cuBlas/test_gemm/test_gemm.cpp,
// test/cuBlas/test_gemv/test_gemv.cpp, test/cuDNN/test_matmul/test_matmul.cpp):
// known-answer cases first, then seeded cases checked against the oracle's
// CPU restatement (oracle/cpu_ref.c, linked as liboracle.so).
//
// Usage: test_facade [--host-only] [filter-substring]
//   --host-only runs only the tests that need no GPU.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <memory>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

#include "cuda_op/detail/cuBlas/axpy.hpp"
#include "cuda_op/detail/cuBlas/copy.hpp"
#include "cuda_op/detail/cuBlas/dot.hpp"
#include "cuda_op/detail/cuBlas/gemm.hpp"
#include "cuda_op/detail/cuBlas/gemm_batched.hpp"
#include "cuda_op/detail/cuBlas/gemv.hpp"
#include "cuda_op/detail/cuBlas/scal.hpp"
#include "cuda_op/detail/cuDNN/batchmatmul.hpp"
#include "cuda_op/detail/cuDNN/kernel_fusion.hpp"
#include "cuda_op/detail/cuDNN/matmul.hpp"
#include "cuopx.h"
#include "jit/Blas/blas_jit_plugins.hpp"
#include "jit/global_jit_manager.hpp"
#include "jit/jit_wrapper.hpp"
#include "performance/auto_tuner.hpp"

extern "C" {
void oracle_fill_uniform_f32(float* out, int64_t n, uint64_t seed, float lo, float hi);
void oracle_gemm_f32(int transA, int transB, int64_t M, int64_t N, int64_t K, float alpha, const float* A,
                     int64_t lda, const float* B, int64_t ldb, float beta, float* C, int64_t ldc, int nthreads);
void oracle_gemv_f32(int trans, int64_t M, int64_t N, float alpha, const float* A, int64_t lda, const float* x,
                     float beta, float* y, int nthreads);
void oracle_epilogue_f32(int64_t M, int64_t N, float* C, int64_t ldc, const float* bias, int epi);
}

using namespace cu_op_mem;

// ------------------------------------------------------------------ harness
struct TestCase {
  const char* name;
  bool needs_gpu;
  std::function<void()> fn;
};
static std::vector<TestCase>& registry() {
  static std::vector<TestCase> r;
  return r;
}
static int g_failures = 0;
struct Reg {
  Reg(const char* n, bool gpu, std::function<void()> f) { registry().push_back({n, gpu, f}); }
};
#define TEST_HOST(name) static void name(); static Reg reg_##name(#name, false, name); static void name()
#define TEST_GPU(name) static void name(); static Reg reg_##name(#name, true, name); static void name()
#define EXPECT_TRUE(c)                                                                     \
  do {                                                                                     \
    if (!(c)) {                                                                            \
      std::printf("    FAILED %s:%d: %s\n", __FILE__, __LINE__, #c);                       \
      ++g_failures;                                                                        \
    }                                                                                      \
  } while (0)
#define EXPECT_EQ(a, b) EXPECT_TRUE((a) == (b))
#define EXPECT_NEAR(a, b, tol)                                                                       \
  do {                                                                                               \
    const double va_ = (a), vb_ = (b);                                                               \
    if (!(std::fabs(va_ - vb_) <= (tol))) {                                                          \
      std::printf("    FAILED %s:%d: %s=%g vs %s=%g (tol %g)\n", __FILE__, __LINE__, #a, va_, #b, vb_, \
                  (double)(tol));                                                                    \
      ++g_failures;                                                                                  \
    }                                                                                                \
  } while (0)

template <typename T>
static std::vector<T> to_host(const Tensor<T>& t) {
  std::vector<T> h(t.numel());
  t.copy_to_host(h.data());
  return h;
}

static double rel_frobenius(const std::vector<float>& c, const std::vector<float>& r) {
  double num = 0, den = 0;
  for (size_t i = 0; i < c.size(); ++i) {
    num += (double(c[i]) - r[i]) * (double(c[i]) - r[i]);
    den += double(r[i]) * r[i];
  }
  return std::sqrt(num) / (den > 0 ? std::sqrt(den) : 1.0);
}

// ------------------------------------------------------------------ host-only
TEST_HOST(StatusCodesMatchReferenceValues) {
  EXPECT_EQ(static_cast<int>(StatusCode::SUCCESS), 0);
  EXPECT_EQ(static_cast<int>(StatusCode::CUDA_ERROR), 2000);
  EXPECT_EQ(static_cast<int>(StatusCode::INVALID_ARGUMENT), 4001);
  EXPECT_EQ(static_cast<int>(StatusCode::SHAPE_MISMATCH), 10002);
  EXPECT_EQ(static_cast<int>(StatusCode::UNSUPPORTED_TYPE), 11001);
  EXPECT_EQ(static_cast<int>(StatusCode::NOT_COMPILED), 7003);
  EXPECT_EQ(static_cast<int>(StatusCode::KERNEL_NOT_FOUND), 6005);
  EXPECT_EQ(static_cast<int>(StatusCode::RESOURCE_UNAVAILABLE), CUOPX_RESOURCE_UNAVAILABLE);
  EXPECT_TRUE(GetErrorCategory(StatusCode::OUT_OF_MEMORY) == ErrorCategory::MEMORY);
  EXPECT_TRUE(GetErrorCategory(StatusCode::PLUGIN_NOT_FOUND) == ErrorCategory::PLUGIN);
  EXPECT_TRUE(std::string(StatusCodeToString(StatusCode::TENSOR_SHAPE_MISMATCH)) == "TENSOR_SHAPE_MISMATCH");
  Status s(StatusCode::INVALID_ARGUMENT, "bad lda", "Forward");
  EXPECT_TRUE(s.IsError() && !s);
  EXPECT_TRUE(s.ToString().find("INVALID_ARGUMENT") != std::string::npos);
}

TEST_HOST(ErrorUtilsClassifyAndDescribe) {
  using namespace ErrorUtils;
  EXPECT_TRUE(IsRecoverableError(StatusCode::INVALID_ARGUMENT) && !IsCriticalError(StatusCode::INVALID_ARGUMENT));
  EXPECT_TRUE(IsRecoverableError(StatusCode::SHAPE_MISMATCH));
  EXPECT_TRUE(IsRecoverableError(StatusCode::OUT_OF_MEMORY) && IsRecoverableError(StatusCode::EXECUTION_TIMEOUT));
  EXPECT_TRUE(IsRecoverableError(StatusCode::NOT_COMPILED));
  EXPECT_TRUE(IsCriticalError(StatusCode::CUDA_ERROR) && !IsRecoverableError(StatusCode::CUDA_ERROR));
  EXPECT_TRUE(IsCriticalError(StatusCode::CUDA_LAUNCH_FAILED));
  EXPECT_TRUE(!IsCriticalError(StatusCode::CUDA_OUT_OF_MEMORY) && IsRecoverableError(StatusCode::CUDA_OUT_OF_MEMORY));
  EXPECT_TRUE(!IsCriticalError(StatusCode::SUCCESS) && !IsRecoverableError(StatusCode::SUCCESS));
  // no code is both
  for (int v : {0, 1000, 1003, 2000, 2013, 3001, 4001, 5000, 6002, 7003, 8002, 9001, 10002, 11001})
    EXPECT_TRUE(!(IsCriticalError(static_cast<StatusCode>(v)) && IsRecoverableError(static_cast<StatusCode>(v))));
  EXPECT_TRUE(GetErrorDescription(StatusCode::TENSOR_SHAPE_MISMATCH).rfind("TENSOR_SHAPE_MISMATCH: ", 0) == 0);
  const Status v = ValidationError("K differs", "Gemm::Forward", "gemm.cpp", 42);
  EXPECT_TRUE(v.GetCode() == StatusCode::VALIDATION_ERROR && v.GetCategory() == ErrorCategory::VALIDATION);
  EXPECT_TRUE(MemoryError("x").GetCategory() == ErrorCategory::MEMORY);
  EXPECT_TRUE(ExecutionError("x").GetCategory() == ErrorCategory::EXECUTION);
  EXPECT_TRUE(CompilationError("x").GetCategory() == ErrorCategory::COMPILATION);
  EXPECT_TRUE(SystemError("x").GetCategory() == ErrorCategory::SYSTEM);
  const std::string d = v.ToDetailedString();
  EXPECT_TRUE(d.find("VALIDATION_ERROR (4000)") != std::string::npos && d.find("K differs") != std::string::npos &&
              d.find("gemm.cpp:42") != std::string::npos);
}

TEST_HOST(BlasPluginManagerRegistersEveryOperatorName) {
  RegisterBlasJITPlugins();
  for (const char* n : {"gemm", "Gemm", "gemv", "Gemv", "gemm_batched", "GemmBatched", "batched_gemm",
                        "BatchedGemm", "dot", "Dot", "axpy", "nrm2", "iamax", "Iamin", "rot", "swap", "scal",
                        "copy", "asum"})
    EXPECT_TRUE(IsBlasOperatorSupported(n));
  EXPECT_TRUE(!IsBlasOperatorSupported("trsm_not_here"));
  auto p = CreateBlasJITPlugin("gemm_batched");
  EXPECT_TRUE(p != nullptr);
  if (p) EXPECT_TRUE(p->GetPluginName() == "gemm_batched_jit");
  auto v = CreateBlasJITPlugin("Iamax");
  auto* vp = dynamic_cast<VectorOpsJITPlugin*>(v.get());
  EXPECT_TRUE(vp && vp->GetOperationType() == VectorOpType::IAMAX);
  EXPECT_TRUE(CreateBlasJITPlugin("unknown") == nullptr);
}

TEST_HOST(PluginRegistrarKnowsJitWrapperKeys) {
  auto& r = PluginRegistrar::Instance();
  for (const char* k : {"gemm", "gemm_jit", "gemv", "gemv_jit", "gemm_batched", "gemm_batched_jit", "vector_ops"})
    EXPECT_TRUE(r.CreatePlugin(k) != nullptr);
  EXPECT_TRUE(r.IsOperatorSupported("Gemm") && r.IsOperatorSupported("dot"));
}

TEST_HOST(CompileRequiresInitializeAndKnownKernelType) {
  GemmJITPlugin p;
  EXPECT_TRUE(p.Compile(JITConfig()) == StatusCode::NOT_INITIALIZED);
  std::vector<Tensor<float>> in, out;
  EXPECT_TRUE(p.Execute(in, out) == StatusCode::NOT_COMPILED);
}

TEST_HOST(HardwareSpecTheoreticalPeaks) {  // B200: 148 SMs at 1965 MHz, 8192-bit HBM3e at 3996 MHz
  HardwareSpec hw;
  hw.compute_capability_major = 10;
  hw.num_sms = 148;
  hw.sm_clock_rate = 1965;
  hw.memory_clock_rate = 3996;
  hw.memory_bus_width = 8192;
  EXPECT_NEAR(hw.GetTheoreticalPeakGFLOPS(), 148 * 128 * 2 * 1.965, 1e-6);
  EXPECT_NEAR(hw.GetTheoreticalMemoryBandwidth(), 3996 * 2 * 1024 / 1000.0, 1e-6);
  EXPECT_EQ(HardwareSpec().GetTheoreticalPeakGFLOPS(), 0.0);
}

TEST_HOST(MemoryPoolSizeClasses) {
  EXPECT_EQ(CudaMemoryPool::SizeClass(1), 256u);
  EXPECT_EQ(CudaMemoryPool::SizeClass(257), 512u);
  EXPECT_EQ(CudaMemoryPool::SizeClass(1 << 20), 1u << 20);
  EXPECT_EQ(CudaMemoryPool::SizeClass((1 << 20) + 1), 2u << 20);
  EXPECT_EQ(CudaMemoryPool::SizeClass((5u << 20) + 3), 6u << 20);
}

TEST_HOST(OperatorConfigPersistence) {
  auto& g = GlobalJITManager::Instance();
  JITConfig c;
  c.kernel_type = "tcgen05";
  c.tile_size = 256;
  c.num_stages = 4;
  g.SetOperatorConfig("gemm", c);
  g.SaveCacheToFile("/tmp/cuopx_opcfg.txt");
  g.Cleanup();
  EXPECT_TRUE(g.GetOperatorConfig("gemm").kernel_type == "default");
  g.LoadCacheFromFile("/tmp/cuopx_opcfg.txt");
  EXPECT_TRUE(g.GetOperatorConfig("gemm").kernel_type == "tcgen05");
  EXPECT_EQ(g.GetOperatorConfig("gemm").num_stages, 4);
}

// ------------------------------------------------------------------ GPU: reference known answers
TEST_GPU(GemmForwardFloatNoTranspose) {  // test/cuBlas/test_gemm/test_gemm.cpp:19-43
  float h_input[6] = {1, 2, 3, 4, 5, 6};
  float h_weight[12] = {1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1, 0};
  Tensor<float> input({2, 3}), weight({3, 4}), output({2, 4});
  input.copy_from_host(h_input);
  weight.copy_from_host(h_weight);
  output.zero();
  Gemm<float> gemm(false, false, 1.0f, 0.0f);
  gemm.SetWeight(weight);
  EXPECT_TRUE(gemm.Forward(input, output) == StatusCode::SUCCESS);
  const float expected[8] = {1, 2, 3, 0, 4, 5, 6, 0};
  auto h = to_host(output);
  for (int i = 0; i < 8; ++i) EXPECT_NEAR(h[i], expected[i], 1e-5);
}

TEST_GPU(GemvForwardFloatNoTranspose) {  // test/cuBlas/test_gemv/test_gemv.cpp:19-44
  float h_input[6] = {1, 2, 3, 4, 5, 6}, h_weight[3] = {1, 2, 3};
  Tensor<float> input({2, 3}), weight({3}), output({2});
  input.copy_from_host(h_input);
  weight.copy_from_host(h_weight);
  output.zero();
  Gemv<float> gemv(false, 1.0f, 0.0f);
  gemv.SetWeight(weight);
  EXPECT_TRUE(gemv.Forward(input, output) == StatusCode::SUCCESS);
  auto h = to_host(output);
  EXPECT_NEAR(h[0], 14, 1e-5);
  EXPECT_NEAR(h[1], 32, 1e-5);
}

// The reference's known answers (test_gemm.cpp:19-43, test_gemv.cpp:19-44,
// test_matmul.cpp:45-67) through Gemm<T>, Gemv<T> and BatchMatMul<T> for the
// element types the reference does not instantiate.  Every input, product
// and sum is a small integer, exact in fp16, bf16 and fp64, so the results
// must match exactly.
template <typename T>
static std::vector<T> cast_vec(const float* v, size_t n) {
  std::vector<T> out(n);
  for (size_t i = 0; i < n; ++i) out[i] = T(v[i]);
  return out;
}
template <typename T>
static float as_float(T v) {
  return float(v);
}
template <typename T>
static void known_answers_for_type() {
  const float h_input[6] = {1, 2, 3, 4, 5, 6}, h_weight[12] = {1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1, 0};
  Tensor<T> input({2, 3}), weight({3, 4}), output({2, 4});
  input.copy_from_host(cast_vec<T>(h_input, 6).data());
  weight.copy_from_host(cast_vec<T>(h_weight, 12).data());
  Gemm<T> gemm(false, false);
  gemm.SetWeight(weight);
  EXPECT_TRUE(gemm.Forward(input, output) == StatusCode::SUCCESS);
  auto h = to_host(output);
  const float expected[8] = {1, 2, 3, 0, 4, 5, 6, 0};
  for (int i = 0; i < 8; ++i) EXPECT_EQ(as_float(h[i]), expected[i]);

  const float h_x[3] = {1, 2, 3};
  Tensor<T> x({3}), y({2});
  x.copy_from_host(cast_vec<T>(h_x, 3).data());
  y.zero();
  Gemv<T> gemv(false);
  gemv.SetWeight(x);
  EXPECT_TRUE(gemv.Forward(input, y) == StatusCode::SUCCESS);
  auto hy = to_host(y);
  EXPECT_EQ(as_float(hy[0]), 14.f);
  EXPECT_EQ(as_float(hy[1]), 32.f);

  const float h_a3[12] = {1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12};
  const float h_b3[24] = {1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1, 0, 2, 0, 0, 0, 0, 2, 0, 0, 0, 0, 2, 0};
  Tensor<T> A3({2, 2, 3}), B3({2, 3, 4}), C3({2, 2, 4});
  A3.copy_from_host(cast_vec<T>(h_a3, 12).data());
  B3.copy_from_host(cast_vec<T>(h_b3, 24).data());
  BatchMatMul<T> bmm;
  EXPECT_TRUE(bmm.Forward(A3, B3, C3) == StatusCode::SUCCESS);
  auto hc = to_host(C3);
  const float e3[16] = {1, 2, 3, 0, 4, 5, 6, 0, 14, 16, 18, 0, 20, 22, 24, 0};
  for (int i = 0; i < 16; ++i) EXPECT_EQ(as_float(hc[i]), e3[i]);
}

TEST_GPU(KnownAnswersForDoubleHalfAndBf16) {
  known_answers_for_type<double>();
  known_answers_for_type<__half>();
  known_answers_for_type<__nv_bfloat16>();
}

TEST_GPU(MatMulForward2DAndBatch3D) {  // test/cuDNN/test_matmul/test_matmul.cpp:21-67
  float h_A[6] = {1, 2, 3, 4, 5, 6}, h_B[12] = {1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1, 0};
  Tensor<float> A({2, 3}), B({3, 4}), C({2, 4});
  A.copy_from_host(h_A);
  B.copy_from_host(h_B);
  MatMul<float> mm;
  EXPECT_TRUE(mm.Forward(A, B, C, -1) == StatusCode::SUCCESS);
  const float e2[8] = {1, 2, 3, 0, 4, 5, 6, 0};
  auto h = to_host(C);
  for (int i = 0; i < 8; ++i) EXPECT_NEAR(h[i], e2[i], 1e-5);

  float h_A3[12] = {1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12};
  float h_B3[24] = {1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1, 0, 2, 0, 0, 0, 0, 2, 0, 0, 0, 0, 2, 0};
  Tensor<float> A3({2, 2, 3}), B3({2, 3, 4}), C3;
  A3.copy_from_host(h_A3);
  B3.copy_from_host(h_B3);
  EXPECT_TRUE(mm.Forward(A3, B3, C3, -1) == StatusCode::SUCCESS);
  const float e3[16] = {1, 2, 3, 0, 4, 5, 6, 0, 14, 16, 18, 0, 20, 22, 24, 0};
  auto h3 = to_host(C3);
  EXPECT_EQ(h3.size(), 16u);
  for (int i = 0; i < 16 && i < (int)h3.size(); ++i) EXPECT_NEAR(h3[i], e3[i], 1e-5);

  BatchMatMul<float> bmm;
  Tensor<float> C4;
  EXPECT_TRUE(bmm.Forward(A3, B3, C4, 0) == StatusCode::SUCCESS);
  auto h4 = to_host(C4);
  for (int i = 0; i < 16 && i < (int)h4.size(); ++i) EXPECT_NEAR(h4[i], e3[i], 1e-5);
  Tensor<float> dummy;
  EXPECT_TRUE(bmm.Forward(A3, dummy) == StatusCode::UNSUPPORTED_TYPE);
}

TEST_GPU(ShapeMismatchIsReported) {
  Tensor<float> A({4, 5}), W({6, 7}), C({4, 7});
  Gemm<float> g;
  g.SetWeight(W);
  EXPECT_TRUE(g.Forward(A, C) == StatusCode::SHAPE_MISMATCH);
  Gemv<float> v;
  Tensor<float> x({3}), y({4});
  v.SetWeight(x);
  EXPECT_TRUE(v.Forward(A, y) == StatusCode::SHAPE_MISMATCH);
}

TEST_HOST(AutoTunerAsyncStopCallbacksAndReports) {
  AutoTuner t;
  TuningConfig cfg;
  cfg.optimization_target = "throughput";
  t.SetTuningConfig(cfg);
  t.AddParameter(ParameterDefinition{"a", ParameterType::INTEGER, "", {"1", "2", "3", "4"}, "1"});
  std::vector<size_t> seen;
  t.RegisterCallback([&](const TuningResult& r) { seen.push_back(r.iterations_used); });
  auto score = [](const ParameterSet& p) { return std::stod(p.at("a")); };
  EXPECT_TRUE(!t.IsTuning());
  TuningResult r = t.TuneAsync("toy", score);  // runs on a worker thread, waits for it
  EXPECT_TRUE(r.best_parameters.at("a") == "4" && r.iterations_used == 4 && r.converged);
  EXPECT_TRUE(seen.size() == 1 && seen[0] == 4);
  // monitoring with a zero interval: one partial report per evaluation, then the final one
  t.EnableRealTimeMonitoring(true);
  t.SetMonitoringInterval(0);
  seen.clear();
  t.Tune("toy", score);
  EXPECT_EQ(seen.size(), size_t(5));
  t.EnableRealTimeMonitoring(false);
  // StopTuning from inside the benchmark: the evaluation in progress
  // finishes, no further one starts, and IsTuning() reports the flag.
  t.StartTuning();
  int calls = 0;
  bool tuning_seen = false;
  r = t.Tune("toy", [&](const ParameterSet& p) {
    tuning_seen = t.IsTuning();
    if (++calls == 2) t.StopTuning();
    return score(p);
  });
  EXPECT_TRUE(tuning_seen && calls == 2 && r.iterations_used == 2 && !r.converged);
  EXPECT_TRUE(!t.IsTuning());
  // The stop ended only the call that was running: a later Tune runs in full
  // without StartTuning (as in the reference, Tune ignores the flag).
  EXPECT_EQ(t.Tune("toy", score).iterations_used, size_t(4));
  const std::string rep = t.GenerateTuningReport(r);
  EXPECT_TRUE(rep.find("a=2") != std::string::npos && rep.find("stopped early") != std::string::npos);
  const std::string path = "/tmp/cuop_autotuner_export.csv";
  t.ExportResults(r, path);
  std::ifstream f(path);
  std::string line, all;
  int lines = 0;
  while (std::getline(f, line)) {
    all += line + "\n";
    ++lines;
  }
  EXPECT_EQ(lines, 3);
  EXPECT_TRUE(all.rfind("iteration,performance,parameters\n0,1,\"a=1\"\n1,2,\"a=2\"", 0) == 0);
}

// test/performance/test_performance_monitor.cpp:296-304 (AutoTunerBasic).
TEST_HOST(AutoTunerBasicStartStop) {
  auto& tuner = AutoTuner::Instance();
  EXPECT_TRUE(!tuner.IsTuning());
  tuner.StartTuning();
  EXPECT_TRUE(tuner.IsTuning());
  tuner.StopTuning();
  EXPECT_TRUE(!tuner.IsTuning());
}

// test/performance/test_performance_monitor.cpp:352-388 (SimpleTuning): the
// parameter is added before a config without parameters is set; Tune uses it.
TEST_HOST(AutoTunerSimpleTuningSequence) {
  AutoTuner t;
  ParameterDefinition param;
  param.name = "test_param";
  param.type = ParameterType::INTEGER;
  param.values = {"1", "2", "3"};
  param.default_value = "2";
  param.is_tunable = true;
  t.AddParameter(param);
  TuningConfig config;
  config.operator_name = "test_operator";
  config.max_iterations = 5;
  config.convergence_threshold = 0.1;
  config.improvement_threshold = 0.05;
  t.SetTuningConfig(config);
  auto r = t.Tune("test_operator", [](const ParameterSet& p) {
    auto it = p.find("test_param");
    return it != p.end() ? std::stod(it->second) : 0.0;
  });
  EXPECT_TRUE(r.iterations_used > 0 && r.best_performance > 0 && !r.best_parameters.empty());
  EXPECT_TRUE(r.best_parameters.at("test_param") == "3");
  EXPECT_EQ(t.GetParameters().size(), size_t(1));
  t.RemoveParameter("test_param");
  EXPECT_EQ(t.GetParameters().size(), size_t(0));
}

// Every strategy name of the reference (auto_tuner.cu:195-216) and its short
// form selects that strategy, which then runs: the result names it, no set is
// evaluated twice, the budget holds, and with a budget as large as the space
// every strategy finds the best set.  An unknown name is refused, not ignored.
TEST_HOST(AutoTunerEveryReferenceStrategyRuns) {
  const std::vector<std::string> names = {"GridSearch", "RandomSearch", "BayesianOptimization", "GeneticAlgorithm"};
  const std::vector<std::string> aliases = {"grid", "random", "bayesian", "genetic"};
  AutoTuner t;
  {
    auto avail = t.GetAvailableStrategies();
    EXPECT_TRUE(avail == names);
  }
  t.AddParameter(ParameterDefinition{"tile", ParameterType::INTEGER, "", {"32", "64", "128", "256", "512", "1024"}, "128"});
  t.AddParameter(ParameterDefinition{"stages", ParameterType::ENUM, "", {"2", "3", "4"}, "3"});
  ParameterDefinition fixed{"dtype", ParameterType::STRING, "", {}, "bf16"};
  fixed.is_tunable = false;
  t.AddParameter(fixed);
  // Best at tile=256, stages=3: 30 - |log2(tile) - 8| * 3 - |stages - 3|.
  auto score = [](const ParameterSet& p) {
    EXPECT_TRUE(p.at("dtype") == "bf16");
    const double lt = std::log2(std::stod(p.at("tile")));
    return 30.0 - std::fabs(lt - 8.0) * 3.0 - std::fabs(std::stod(p.at("stages")) - 3.0);
  };
  for (size_t i = 0; i < names.size(); ++i) {
    for (const std::string& nm : {names[i], aliases[i]}) {
      t.SetTuningStrategy(nm);
      EXPECT_TRUE(t.GetCurrentStrategy() == names[i]);
      for (size_t budget : {size_t(7), size_t(100)}) {
        TuningConfig cfg = t.GetTuningConfig();
        cfg.max_iterations = budget;
        cfg.tuning_strategy.clear();  // keep the strategy just selected
        t.SetTuningConfig(cfg);
        TuningResult r = t.Tune("toy", score);
        EXPECT_TRUE(r.strategy_name == names[i]);
        EXPECT_TRUE(r.optimization_summary.find(names[i]) != std::string::npos);
        EXPECT_TRUE(r.iterations_used <= std::min<size_t>(budget, 18) && r.iterations_used >= 1);
        std::set<std::string> distinct;
        for (const auto& ps : r.parameter_history) distinct.insert(ps.at("tile") + "/" + ps.at("stages"));
        EXPECT_EQ(distinct.size(), r.parameter_history.size());
        const double best_seen = *std::max_element(r.performance_history.begin(), r.performance_history.end());
        EXPECT_NEAR(r.best_performance, best_seen, 0.0);
        if (budget == 100) {
          EXPECT_EQ(r.iterations_used, size_t(18));
          EXPECT_TRUE(r.converged);
          EXPECT_TRUE(r.best_parameters.at("tile") == "256" && r.best_parameters.at("stages") == "3");
        }
      }
    }
  }
  t.SetTuningStrategy("Annealing");
  EXPECT_TRUE(t.GetCurrentStrategy() == "GeneticAlgorithm");
  EXPECT_TRUE(t.GetLastError().find("Annealing") != std::string::npos);
  TuningConfig bad = t.GetTuningConfig();
  bad.tuning_strategy = "Tabu";
  t.SetTuningConfig(bad);
  EXPECT_TRUE(t.GetCurrentStrategy() == "GeneticAlgorithm" && t.GetLastError().find("Tabu") != std::string::npos);
  // The strategy classes of the reference header are usable on their own.
  TuningConfig space;
  space.parameters = t.GetParameters();
  GridSearchStrategy grid;
  auto sets = grid.GenerateParameterSets(space, 100);
  EXPECT_EQ(sets.size(), size_t(18));
  EXPECT_TRUE(sets[0].at("tile") == "32" && sets[0].at("stages") == "2" && sets[1].at("stages") == "3");
  std::unique_ptr<ITuningStrategy> s = MakeTuningStrategy("BayesianOptimization");
  EXPECT_TRUE(s && s->GetStrategyName() == "BayesianOptimization");
  EXPECT_TRUE(!MakeTuningStrategy("Annealing"));
  // Predictions: a measured set returns its measurement.
  ParameterSet best{{"tile", "256"}, {"stages", "3"}, {"dtype", "bf16"}};
  EXPECT_NEAR(t.PredictPerformance(best), 30.0, 0.0);
  EXPECT_TRUE(!t.GetPerformanceInsights().empty());
}

// A benchmark call that throws is recorded as 0.0 and the run goes on
// (auto_tuner.cu:159-163); the failure never becomes the best.
TEST_HOST(AutoTunerBenchmarkExceptionIsRecorded) {
  AutoTuner t;
  TuningConfig cfg;
  cfg.optimization_target = "latency";
  t.SetTuningConfig(cfg);
  t.AddParameter(ParameterDefinition{"v", ParameterType::ENUM, "", {"a", "b", "c"}, "a"});
  int calls = 0;
  TuningResult r = t.Tune("toy", [&](const ParameterSet& p) -> double {
    ++calls;
    if (p.at("v") == "b") throw std::runtime_error("kernel refused");
    return p.at("v") == "a" ? 5.0 : 3.0;
  });
  EXPECT_EQ(calls, 3);
  EXPECT_EQ(r.iterations_used, size_t(3));
  EXPECT_TRUE(r.performance_history.size() == 3 && r.performance_history[1] == 0.0);
  EXPECT_TRUE(r.best_parameters.at("v") == "c");  // 0.0 from the failure is not the best latency
  EXPECT_NEAR(r.best_performance, 3.0, 0.0);
  bool noted = false;
  for (const auto& rec : r.recommendations) noted |= rec.find("kernel refused") != std::string::npos;
  EXPECT_TRUE(noted);
}

TEST_HOST(AutoTunerGridRandomEarlyStopAndHistory) {
  AutoTuner t;
  TuningConfig cfg;
  cfg.operator_name = "toy";
  cfg.optimization_target = "throughput";
  t.SetTuningConfig(cfg);
  ParameterDefinition a{"a", ParameterType::INTEGER, "", {"1", "2", "3"}, "1"};
  ParameterDefinition b{"b", ParameterType::ENUM, "", {"x", "y"}, "x"};
  ParameterDefinition fixed{"c", ParameterType::STRING, "", {}, "keep"};
  fixed.is_tunable = false;
  t.AddParameter(a);
  t.AddParameter(b);
  t.AddParameter(fixed);
  int calls = 0;
  auto score = [&](const ParameterSet& p) {
    ++calls;
    EXPECT_TRUE(p.at("c") == "keep");
    return std::stod(p.at("a")) * (p.at("b") == "y" ? 10.0 : 1.0);
  };
  TuningResult r = t.Tune("toy", score);
  EXPECT_EQ(calls, 6);
  EXPECT_TRUE(r.best_parameters.at("a") == "3" && r.best_parameters.at("b") == "y");
  EXPECT_NEAR(r.best_performance, 30.0, 0.0);
  cfg = t.GetTuningConfig();
  cfg.optimization_target = "latency";  // minimise
  cfg.tuning_strategy = "random";
  t.SetTuningConfig(cfg);
  r = t.Tune("toy", score);
  EXPECT_TRUE(r.best_parameters.at("a") == "1" && r.best_parameters.at("b") == "x");
  EXPECT_EQ(r.iterations_used, size_t(6));
  cfg.tuning_strategy = "grid";
  cfg.enable_early_stopping = true;
  cfg.patience = 2;
  t.SetTuningConfig(cfg);
  r = t.Tune("toy", score);  // latency: 1,x is first and best -> stops after 2 more
  EXPECT_EQ(r.iterations_used, size_t(3));
  EXPECT_TRUE(r.converged);
  const std::string path = "/tmp/cuop_autotuner_history.txt";
  t.SaveTuningHistory(path);
  AutoTuner u;
  u.LoadTuningHistory(path);
  auto h = u.GetTuningHistory();
  EXPECT_EQ(h.size(), size_t(3));
  EXPECT_TRUE(h[0].best_parameters.at("a") == "3");
  EXPECT_NEAR(h[0].best_performance, 30.0, 1e-9);
}

// ------------------------------------------------------------------ GPU: seeded parity vs oracle
TEST_GPU(GemmSeededMatchesOracleBitExact) {
  for (int t = 0; t < 4; ++t) {
    const bool tA = t & 1, tB = t & 2;
    const int M = 257, N = 129, K = 300;
    std::vector<float> a(size_t(M) * K), w(size_t(K) * N), c0(size_t(M) * N), ref;
    oracle_fill_uniform_f32(a.data(), a.size(), 11, -1.f, 1.f);
    oracle_fill_uniform_f32(w.data(), w.size(), 12, -1.f, 1.f);
    oracle_fill_uniform_f32(c0.data(), c0.size(), 13, -1.f, 1.f);
    ref = c0;
    oracle_gemm_f32(tA, tB, M, N, K, 0.5f, a.data(), tA ? M : K, w.data(), tB ? K : N, 1.5f, ref.data(), N, 4);
    Tensor<float> A(tA ? std::vector<size_t>{size_t(K), size_t(M)} : std::vector<size_t>{size_t(M), size_t(K)});
    Tensor<float> W(tB ? std::vector<size_t>{size_t(N), size_t(K)} : std::vector<size_t>{size_t(K), size_t(N)});
    Tensor<float> C({size_t(M), size_t(N)});
    A.copy_from_host(a.data());
    W.copy_from_host(w.data());
    C.copy_from_host(c0.data());
    Gemm<float> g(tA, tB, 0.5f, 1.5f);
    g.SetWeight(W);
    EXPECT_TRUE(g.Forward(A, C) == StatusCode::SUCCESS);
    auto h = to_host(C);
    EXPECT_TRUE(std::memcmp(h.data(), ref.data(), h.size() * sizeof(float)) == 0);
  }
}

// MatMulReluFused (kernel_fusion.cu:330-370): relu(A*W + bias); below 256^3
// the fp32 path is the FFMA chain, so the result is the oracle's bit for bit.
TEST_GPU(MatMulReluFusedMatchesOracleBitExact) {
  const int M = 257, N = 129, K = 300;
  std::vector<float> a(size_t(M) * K), w(size_t(K) * N), b(N);
  oracle_fill_uniform_f32(a.data(), a.size(), 31, -1.f, 1.f);
  oracle_fill_uniform_f32(w.data(), w.size(), 32, -1.f, 1.f);
  oracle_fill_uniform_f32(b.data(), b.size(), 33, -1.f, 1.f);
  Tensor<float> A({size_t(M), size_t(K)}), W({size_t(K), size_t(N)}), B({size_t(N)}), Bbad({size_t(N + 1)});
  A.copy_from_host(a.data());
  W.copy_from_host(w.data());
  B.copy_from_host(b.data());
  for (int with_bias = 0; with_bias < 2; ++with_bias) {
    std::vector<float> ref(size_t(M) * N, 0.f);
    oracle_gemm_f32(0, 0, M, N, K, 1.f, a.data(), K, w.data(), N, 0.f, ref.data(), N, 4);
    oracle_epilogue_f32(M, N, ref.data(), N, b.data(), with_bias ? 3 : 2);
    MatMulReluFused<float> op;
    op.SetWeight(W);
    op.SetBias(with_bias ? B : Bbad);  // a bias of the wrong length is ignored, as in the reference
    Tensor<float> C;
    std::vector<Tensor<float>*> ins{&A}, outs{&C};
    EXPECT_TRUE(op.Forward(ins, outs) == StatusCode::SUCCESS);
    EXPECT_TRUE(C.shape() == (std::vector<size_t>{size_t(M), size_t(N)}));
    auto h = to_host(C);
    EXPECT_TRUE(std::memcmp(h.data(), ref.data(), h.size() * sizeof(float)) == 0);
    EXPECT_TRUE(op.Backward(ins, outs, outs) == StatusCode::UNSUPPORTED_OPERATION);
  }
}

TEST_GPU(VectorOperatorClasses) {
  const int n = 100003;
  std::vector<float> x(n), y(n);
  oracle_fill_uniform_f32(x.data(), n, 41, -1.f, 1.f);
  oracle_fill_uniform_f32(y.data(), n, 42, -1.f, 1.f);
  Tensor<float> X({size_t(n)}), Y({size_t(n)}), Z({size_t(n)});
  X.copy_from_host(x.data());
  Y.copy_from_host(y.data());
  double dot = 0;
  for (int i = 0; i < n; ++i) dot += double(x[i]) * y[i];
  float r = 0.f;
  Dot<float> d;
  EXPECT_TRUE(d.Forward(X, Y, r) == StatusCode::SUCCESS);
  EXPECT_NEAR(r, dot, 1e-3);
  Axpy<float> ax(2.f);
  EXPECT_TRUE(ax.Forward(X, Y) == StatusCode::SUCCESS);  // y = 2x + y
  Scal<float> sc(0.5f);
  EXPECT_TRUE(sc.Forward(Y) == StatusCode::SUCCESS);  // y = x + y/2
  Copy<float> cp;
  EXPECT_TRUE(cp.Forward(Y, Z) == StatusCode::SUCCESS);
  cudaDeviceSynchronize();
  auto z = to_host(Z);
  bool ok = true;
  for (int i = 0; i < n; ++i) ok &= z[i] == 0.5f * (2.f * x[i] + y[i]);
  EXPECT_TRUE(ok);
  Tensor<double> Xd({8}), Yd({8});
  double rd = 0;
  Dot<double> dd;
  EXPECT_TRUE(dd.Forward(Xd, Yd, rd) == StatusCode::UNSUPPORTED_TYPE);
  Tensor<float> short_y({size_t(n - 1)});
  EXPECT_TRUE(ax.Forward(X, short_y) == StatusCode::SHAPE_MISMATCH);
}

// The AutoTuner drives the GEMM variant override with a timing callback;
// the winner becomes a selection-table row that Gemm<bf16> then follows.
TEST_GPU(AutoTunerSelectsGemmVariantIntoTable) {
  const int M = 1024, N = 1024, K = 1024;
  Tensor<__nv_bfloat16> A({size_t(M), size_t(K)}), W({size_t(K), size_t(N)}), C({size_t(M), size_t(N)});
  A.zero();
  W.zero();
  AutoTuner t;
  TuningConfig cfg;
  cfg.operator_name = "gemm_bf16_1024";
  cfg.optimization_target = "latency";
  t.SetTuningConfig(cfg);
  t.AddParameter({"variant", ParameterType::ENUM, "", {"tc2", "tc_128x256", "tc_128x128"}, "tc2"});
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  TuningResult r = t.Tune("gemm", [&](const ParameterSet& p) {
    cuopx_set_gemm_variant(p.at("variant").c_str());
    float ms = 0.f;
    for (int rep = 0; rep < 2; ++rep) {  // first pass warms up
      cudaEventRecord(e0);
      for (int i = 0; i < 5; ++i)
        cuopx_gemm(CUOPX_BF16, 0, 0, M, N, K, 1.0, A.data(), K, W.data(), N, 0.0, C.data(), N, nullptr);
      cudaEventRecord(e1);
      cudaEventSynchronize(e1);
      cudaEventElapsedTime(&ms, e0, e1);
    }
    cuopx_set_gemm_variant(nullptr);
    return static_cast<double>(ms);
  });
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  EXPECT_EQ(r.iterations_used, size_t(3));
  const std::string best = r.best_parameters.at("variant");
  const std::string row = "bf16 0 0 1024:1024 1024:1024 1024:1024 1:1 " + best + "\n";
  EXPECT_EQ(cuopx_tuning_load(row.c_str()), CUOPX_SUCCESS);
  Gemm<__nv_bfloat16> g;
  g.SetWeight(W);
  EXPECT_TRUE(g.Forward(A, C) == StatusCode::SUCCESS);
  const std::string k = cuopx_last_kernel();
  EXPECT_TRUE(best == "tc2" ? k == "gemm_tc2_256x256" : k == "gemm_" + best);
  cuopx_tuning_clear();
}

TEST_GPU(GemvSeededMatchesOracle) {
  for (int trans = 0; trans < 2; ++trans) {
    const int m = 4096, n = 3072;
    std::vector<float> a(size_t(m) * n), x(n), y(m, 0.f);
    oracle_fill_uniform_f32(a.data(), a.size(), 21, -1.f, 1.f);
    oracle_fill_uniform_f32(x.data(), n, 22, -1.f, 1.f);
    // Tensor shape [m, n]; transposed reads A[col*m + row] (n rows of m)
    oracle_gemv_f32(trans, m, n, 1.f, a.data(), trans ? m : n, x.data(), 0.f, y.data(), 4);
    Tensor<float> A({size_t(m), size_t(n)}), X({size_t(n)}), Y({size_t(m)});
    A.copy_from_host(a.data());
    X.copy_from_host(x.data());
    Gemv<float> g(trans != 0, 1.f, 0.f);
    g.SetWeight(X);
    EXPECT_TRUE(g.Forward(A, Y) == StatusCode::SUCCESS);
    EXPECT_TRUE(rel_frobenius(to_host(Y), y) <= 1e-5 * std::sqrt(double(n)));
  }
}

TEST_GPU(Bf16GemmAndBatchedRunOnTensorCores) {
  const int M = 256, N = 384, K = 192, batch = 3;
  std::vector<float> a(size_t(batch) * M * K), b(size_t(batch) * K * N);
  oracle_fill_uniform_f32(a.data(), a.size(), 31, -1.f, 1.f);
  oracle_fill_uniform_f32(b.data(), b.size(), 32, -1.f, 1.f);
  std::vector<__nv_bfloat16> ah(a.size()), bh(b.size());
  for (size_t i = 0; i < a.size(); ++i) ah[i] = __float2bfloat16(a[i]);
  for (size_t i = 0; i < b.size(); ++i) bh[i] = __float2bfloat16(b[i]);
  Tensor<__nv_bfloat16> A({size_t(batch), size_t(M), size_t(K)}), B({size_t(batch), size_t(K), size_t(N)});
  Tensor<__nv_bfloat16> C({size_t(batch), size_t(M), size_t(N)});
  A.copy_from_host(ah.data());
  B.copy_from_host(bh.data());
  GemmBatched<__nv_bfloat16> gb;
  EXPECT_TRUE(gb.Forward(A, B, C) == StatusCode::SUCCESS);
  EXPECT_TRUE(std::string(cuopx_last_kernel()).rfind("gemm_tc_", 0) == 0);
  auto h = to_host(C);
  // fp32 reference of the widened inputs, batch 1
  double maxref = 0, maxerr = 0;
  for (int i = 0; i < M; ++i)
    for (int j = 0; j < N; ++j) {
      double s = 0;
      for (int k = 0; k < K; ++k)
        s += double(__bfloat162float(ah[size_t(M) * K + size_t(i) * K + k])) *
             double(__bfloat162float(bh[size_t(K) * N + size_t(k) * N + j]));
      maxref = std::max(maxref, std::fabs(s));
      maxerr = std::max(maxerr, std::fabs(s - double(__bfloat162float(h[size_t(M) * N + size_t(i) * N + j]))));
    }
  EXPECT_TRUE(maxerr / maxref <= 1e-2);
}

// ------------------------------------------------------------------ GPU: plugins and wrapper
TEST_GPU(GemmPluginExecute) {
  auto plugin = CreateBlasJITPlugin("gemm");
  auto* g = dynamic_cast<GemmJITPlugin*>(plugin.get());
  EXPECT_TRUE(g != nullptr);
  if (!g) return;
  EXPECT_TRUE(g->Initialize() == StatusCode::SUCCESS);
  JITConfig cfg;
  cfg.kernel_type = "tensor_core";
  EXPECT_TRUE(g->Compile(cfg) == StatusCode::SUCCESS);
  float h_input[6] = {1, 2, 3, 4, 5, 6}, h_weight[12] = {1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1, 0};
  Tensor<float> W({3, 4});
  W.copy_from_host(h_weight);
  g->SetGemmParams(false, false, 2.0f, 0.0f);
  g->SetWeight(W);
  std::vector<Tensor<float>> in, out;
  in.emplace_back(std::vector<size_t>{2, 3});
  in[0].copy_from_host(h_input);
  out.emplace_back();  // empty: the plugin allocates [2, 4]
  EXPECT_TRUE(g->Execute(in, out) == StatusCode::SUCCESS);
  const float expected[8] = {2, 4, 6, 0, 8, 10, 12, 0};
  auto h = to_host(out[0]);
  for (int i = 0; i < 8; ++i) EXPECT_NEAR(h[i], expected[i], 1e-5);
  EXPECT_TRUE(!g->GetPerformanceProfile().kernel_name.empty());
}

// JITConfig.kernel_type is a hint into variant selection: the reference's
// SIMT kernel families run the FFMA kernels (bit-identical to the oracle),
// "tensor_core" keeps the tensor-core choice.
TEST_GPU(GemmPluginKernelTypeSelectsVariant) {
  const int M = 384, N = 320, K = 512;  // 3xTF32 by default at this size
  std::vector<float> a(size_t(M) * K), w(size_t(K) * N), ref(size_t(M) * N, 0.f);
  oracle_fill_uniform_f32(a.data(), a.size(), 51, -1.f, 1.f);
  oracle_fill_uniform_f32(w.data(), w.size(), 52, -1.f, 1.f);
  oracle_gemm_f32(0, 0, M, N, K, 1.f, a.data(), K, w.data(), N, 0.f, ref.data(), N, 4);
  Tensor<float> W({size_t(K), size_t(N)});
  W.copy_from_host(w.data());
  const char* types[] = {"tensor_core", "tiled", "basic"};
  const char* kernels[] = {"gemm_tf32x3_", "gemm_f32_", "gemm_simt_generic"};
  for (int i = 0; i < 3; ++i) {
    auto plugin = CreateBlasJITPlugin("gemm");
    auto* g = dynamic_cast<GemmJITPlugin*>(plugin.get());
    EXPECT_TRUE(g && g->Initialize() == StatusCode::SUCCESS);
    if (!g) return;
    JITConfig cfg;
    cfg.kernel_type = types[i];
    EXPECT_TRUE(g->Compile(cfg) == StatusCode::SUCCESS);
    g->SetGemmParams(false, false, 1.0f, 0.0f);
    g->SetWeight(W);
    std::vector<Tensor<float>> in, out;
    in.emplace_back(std::vector<size_t>{size_t(M), size_t(K)});
    in[0].copy_from_host(a.data());
    out.emplace_back();
    EXPECT_TRUE(g->Execute(in, out) == StatusCode::SUCCESS);
    const std::string k = g->GetPerformanceProfile().kernel_name;
    EXPECT_TRUE(k.rfind(kernels[i], 0) == 0);
    EXPECT_EQ(g->GetPerformanceProfile().used_tensor_core, i == 0);
    auto h = to_host(out[0]);
    if (i > 0) EXPECT_TRUE(std::memcmp(h.data(), ref.data(), h.size() * sizeof(float)) == 0);
    else EXPECT_TRUE(rel_frobenius(h, ref) <= 1e-5 * std::sqrt(double(K)));
  }
  // The hint covered only the plugin's own launches: a direct call is back on 3xTF32.
  Tensor<float> A({size_t(M), size_t(K)}), C({size_t(M), size_t(N)});
  A.copy_from_host(a.data());
  EXPECT_EQ(cuopx_gemm(CUOPX_F32, 0, 0, M, N, K, 1.0, A.data(), K, W.data(), N, 0.0, C.data(), N, nullptr),
            CUOPX_SUCCESS);
  EXPECT_TRUE(std::string(cuopx_last_kernel()).rfind("gemm_tf32x3_", 0) == 0);
}

// A bounded device-side wait that runs out (a cross-GPU barrier whose peer
// never arrives, ~5 s) is reported by the next plugin call as
// EXECUTION_TIMEOUT; the context stays usable and clearing the word recovers.
TEST_GPU(DeviceTimeoutReportedAsExecutionTimeout) {
  Tensor<unsigned int> s0({size_t(CUOPX_PEER_SIGNAL_BYTES / 4)}), s1({size_t(CUOPX_PEER_SIGNAL_BYTES / 4)});
  s0.zero();
  s1.zero();
  void* sig[2] = {s0.data(), s1.data()};
  cuopx_clear_device_error();
  EXPECT_EQ(cuopx_peer_barrier(sig, 2, 0, nullptr), CUOPX_SUCCESS);
  auto plugin = CreateBlasJITPlugin("gemm");
  auto* g = dynamic_cast<GemmJITPlugin*>(plugin.get());
  EXPECT_TRUE(g && g->Initialize() == StatusCode::SUCCESS && g->Compile(JITConfig{}) == StatusCode::SUCCESS);
  if (!g) return;
  Tensor<float> W({4, 4});
  W.zero();
  g->SetWeight(W);
  std::vector<Tensor<float>> in, out;
  in.emplace_back(std::vector<size_t>{4, 4});
  in[0].zero();
  out.emplace_back();
  EXPECT_TRUE(g->Execute(in, out) == StatusCode::EXECUTION_TIMEOUT);
  EXPECT_TRUE(g->GetLastError().find("timed out") != std::string::npos);
  EXPECT_EQ(cuopx_clear_device_error(), CUOPX_SUCCESS);
  EXPECT_TRUE(g->Execute(in, out) == StatusCode::SUCCESS);
}

TEST_GPU(BatchedAndGemvAndVectorPlugins) {
  // batched: 2 x (2x3 * 3x4) with the known-answer data, registered under "gemm_batched"
  auto pb = CreateBlasJITPlugin("gemm_batched");
  auto* b = dynamic_cast<GemmBatchedJITPlugin*>(pb.get());
  EXPECT_TRUE(b && b->Initialize() == StatusCode::SUCCESS && b->Compile(JITConfig()) == StatusCode::SUCCESS);
  float h_A[12] = {1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12};
  float h_B[24] = {1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1, 0, 2, 0, 0, 0, 0, 2, 0, 0, 0, 0, 2, 0};
  std::vector<Tensor<float>> in, out;
  in.emplace_back(std::vector<size_t>{2, 2, 3});
  in.emplace_back(std::vector<size_t>{2, 3, 4});
  in[0].copy_from_host(h_A);
  in[1].copy_from_host(h_B);
  out.emplace_back(std::vector<size_t>{2, 2, 4});
  b->SetBatchSize(2);
  b->SetMatrixDimensions(2, 4, 3);
  EXPECT_TRUE(b->Execute(in, out) == StatusCode::SUCCESS);
  const float e3[16] = {1, 2, 3, 0, 4, 5, 6, 0, 14, 16, 18, 0, 20, 22, 24, 0};
  auto h = to_host(out[0]);
  for (int i = 0; i < 16; ++i) EXPECT_NEAR(h[i], e3[i], 1e-5);

  // gemv plugin: weight = A [2,3], input x, output y
  auto pv = CreateBlasJITPlugin("Gemv");
  auto* v = dynamic_cast<GemvJITPlugin*>(pv.get());
  EXPECT_TRUE(v && v->Initialize() == StatusCode::SUCCESS && v->Compile(JITConfig()) == StatusCode::SUCCESS);
  Tensor<float> A({2, 3});
  A.copy_from_host(h_A);
  v->SetWeight(A);
  std::vector<Tensor<float>> vin, vout;
  vin.emplace_back(std::vector<size_t>{3});
  float x[3] = {1, 2, 3};
  vin[0].copy_from_host(x);
  vout.emplace_back(std::vector<size_t>{2});
  EXPECT_TRUE(v->Execute(vin, vout) == StatusCode::SUCCESS);
  auto hy = to_host(vout[0]);
  EXPECT_NEAR(hy[0], 14, 1e-5);
  EXPECT_NEAR(hy[1], 32, 1e-5);

  // vector ops: dot, nrm2, iamax (1-based), axpy
  auto pd = CreateBlasJITPlugin("dot");
  auto* d = dynamic_cast<VectorOpsJITPlugin*>(pd.get());
  EXPECT_TRUE(d && d->Initialize() == StatusCode::SUCCESS && d->Compile(JITConfig()) == StatusCode::SUCCESS);
  float hx[4] = {1, -7, 3, 2}, hy2[4] = {2, 1, 0, 1};
  std::vector<Tensor<float>> din, dout;
  din.emplace_back(std::vector<size_t>{4});
  din.emplace_back(std::vector<size_t>{4});
  din[0].copy_from_host(hx);
  din[1].copy_from_host(hy2);
  dout.emplace_back();
  EXPECT_TRUE(d->Execute(din, dout) == StatusCode::SUCCESS);
  EXPECT_NEAR(to_host(dout[0])[0], 2 - 7 + 0 + 2, 1e-6);
  d->SetOperationType(VectorOpType::NRM2);
  EXPECT_TRUE(d->Execute(din, dout) == StatusCode::SUCCESS);
  EXPECT_NEAR(to_host(dout[0])[0], std::sqrt(1 + 49 + 9 + 4.0), 1e-5);
  d->SetOperationType(VectorOpType::IAMAX);
  EXPECT_TRUE(d->Execute(din, dout) == StatusCode::SUCCESS);
  EXPECT_NEAR(to_host(dout[0])[0], 2, 0);
  d->SetOperationType(VectorOpType::AXPY);
  d->SetAlpha(2.f);
  std::vector<Tensor<float>> ain, aout;
  ain.emplace_back(din[0].data(), din[0].shape());
  aout.emplace_back(din[1].data(), din[1].shape());
  EXPECT_TRUE(d->Execute(ain, aout) == StatusCode::SUCCESS);
  auto ha = to_host(din[1]);
  for (int i = 0; i < 4; ++i) EXPECT_NEAR(ha[i], 2 * hx[i] + hy2[i], 1e-6);
}

TEST_HOST(TypedPluginExecuteRequiresCompile) {
  int dummy = 0;
  GemmJITPlugin g;
  EXPECT_TRUE(g.ExecuteTyped(DataType::FLOAT16, 4, 4, 4, &dummy, &dummy, &dummy) == StatusCode::NOT_COMPILED);
  GemmBatchedJITPlugin b;
  EXPECT_TRUE(b.ExecuteTyped(DataType::FLOAT16, &dummy, &dummy, &dummy) == StatusCode::NOT_COMPILED);
  GemvJITPlugin v;
  EXPECT_TRUE(v.ExecuteTyped(DataType::BFLOAT16, 4, 4, &dummy, &dummy, &dummy) == StatusCode::NOT_COMPILED);
}

// Argument checks of ExecuteTyped, all rejected before any launch.
TEST_GPU(TypedPluginExecuteValidatesArguments) {
  RegisterBlasJITPlugins();  // self-contained when run alone (filter argument)
  int dummy = 0;
  auto pg = CreateBlasJITPlugin("gemm");
  auto* g = dynamic_cast<GemmJITPlugin*>(pg.get());
  EXPECT_TRUE(g && g->Initialize() == StatusCode::SUCCESS && g->Compile(JITConfig()) == StatusCode::SUCCESS);
  if (!g) return;
  EXPECT_TRUE(g->ExecuteTyped(static_cast<DataType>(9), 4, 4, 4, &dummy, &dummy, &dummy) ==
              StatusCode::UNSUPPORTED_TYPE);
  EXPECT_TRUE(g->ExecuteTyped(DataType::BFLOAT16, -1, 4, 4, &dummy, &dummy, &dummy) == StatusCode::INVALID_ARGUMENT);
  EXPECT_TRUE(g->ExecuteTyped(DataType::BFLOAT16, 4, 4, 4, nullptr, &dummy, &dummy) == StatusCode::INVALID_ARGUMENT);
  EXPECT_TRUE(!g->GetLastError().empty());
  auto pb = CreateBlasJITPlugin("gemm_batched");
  auto* b = dynamic_cast<GemmBatchedJITPlugin*>(pb.get());
  EXPECT_TRUE(b && b->Initialize() == StatusCode::SUCCESS && b->Compile(JITConfig()) == StatusCode::SUCCESS);
  if (b) EXPECT_TRUE(b->ExecuteTyped(DataType::FLOAT16, &dummy, &dummy, &dummy) == StatusCode::INVALID_ARGUMENT);
  auto pv = CreateBlasJITPlugin("gemv");
  auto* v = dynamic_cast<GemvJITPlugin*>(pv.get());
  EXPECT_TRUE(v && v->Initialize() == StatusCode::SUCCESS && v->Compile(JITConfig()) == StatusCode::SUCCESS);
  if (v) EXPECT_TRUE(v->ExecuteTyped(DataType::BFLOAT16, 4, 4, &dummy, nullptr, &dummy) == StatusCode::INVALID_ARGUMENT);
}

// ExecuteTyped runs the kernels the C ABI runs: results bit-identical to
// direct cuopx calls on the same fp16/bf16 buffers, and within the 16-bit
// tolerance (max|C-R| / max|R| <= 1e-2) of an fp64 product of the widened inputs.
TEST_GPU(TypedPluginExecuteMatchesCAbi) {
  RegisterBlasJITPlugins();  // self-contained when run alone (filter argument)
  const int M = 256, N = 320, K = 192, batch = 3;
  std::vector<float> a(size_t(batch) * M * K), b(size_t(batch) * K * N);
  oracle_fill_uniform_f32(a.data(), a.size(), 41, -1.f, 1.f);
  oracle_fill_uniform_f32(b.data(), b.size(), 42, -1.f, 1.f);
  std::vector<__half> ah(a.size()), bh(b.size());
  for (size_t i = 0; i < a.size(); ++i) ah[i] = __float2half(a[i]);
  for (size_t i = 0; i < b.size(); ++i) bh[i] = __float2half(b[i]);
  Tensor<__half> A({size_t(batch), size_t(M), size_t(K)}), B({size_t(batch), size_t(K), size_t(N)});
  Tensor<__half> C1({size_t(batch), size_t(M), size_t(N)}), C2({size_t(batch), size_t(M), size_t(N)});
  A.copy_from_host(ah.data());
  B.copy_from_host(bh.data());

  // GEMM plugin on batch 0
  auto pg = CreateBlasJITPlugin("gemm");
  auto* g = dynamic_cast<GemmJITPlugin*>(pg.get());
  EXPECT_TRUE(g && g->Initialize() == StatusCode::SUCCESS && g->Compile(JITConfig()) == StatusCode::SUCCESS);
  if (!g) return;
  g->SetGemmParams(false, false, 1.0f, 0.0f);
  EXPECT_TRUE(g->ExecuteTyped(DataType::FLOAT16, M, N, K, A.data(), B.data(), C1.data()) == StatusCode::SUCCESS);
  EXPECT_TRUE(std::string(cuopx_last_kernel()).rfind("gemm_tc", 0) == 0);
  EXPECT_EQ(cuopx_gemm(CUOPX_F16, 0, 0, M, N, K, 1.0, A.data(), K, B.data(), N, 0.0, C2.data(), N, nullptr),
            CUOPX_SUCCESS);
  EXPECT_TRUE(cudaDeviceSynchronize() == cudaSuccess);
  auto h1 = to_host(C1), h2 = to_host(C2);
  EXPECT_TRUE(std::memcmp(h1.data(), h2.data(), size_t(M) * N * sizeof(__half)) == 0);
  double maxref = 0, maxerr = 0;
  for (int i = 0; i < M; ++i)
    for (int j = 0; j < N; ++j) {
      double s = 0;
      for (int k = 0; k < K; ++k) s += double(__half2float(ah[size_t(i) * K + k])) * __half2float(bh[size_t(k) * N + j]);
      maxref = std::max(maxref, std::fabs(s));
      maxerr = std::max(maxerr, std::fabs(s - double(__half2float(h1[size_t(i) * N + j]))));
    }
  EXPECT_TRUE(maxref > 0 && maxerr / maxref <= 1e-2);

  // batched plugin, all batches, alpha/beta
  auto pb = CreateBlasJITPlugin("batched_gemm");
  auto* bp = dynamic_cast<GemmBatchedJITPlugin*>(pb.get());
  EXPECT_TRUE(bp && bp->Initialize() == StatusCode::SUCCESS && bp->Compile(JITConfig()) == StatusCode::SUCCESS);
  if (!bp) return;
  bp->SetBatchSize(batch);
  bp->SetMatrixDimensions(M, N, K);
  bp->SetAlphaBeta(0.5f, 0.25f);
  const std::vector<__half> ones(C1.numel(), __float2half(1.f));
  C1.copy_from_host(ones.data());
  C2.copy_from_host(ones.data());
  EXPECT_TRUE(bp->ExecuteTyped(DataType::FLOAT16, A.data(), B.data(), C1.data()) == StatusCode::SUCCESS);
  EXPECT_EQ(cuopx_gemm_strided_batched(CUOPX_F16, 0, 0, M, N, K, 0.5, A.data(), K, int64_t(M) * K, B.data(), N,
                                       int64_t(K) * N, 0.25, C2.data(), N, int64_t(M) * N, batch, nullptr),
            CUOPX_SUCCESS);
  EXPECT_TRUE(cudaDeviceSynchronize() == cudaSuccess);
  h1 = to_host(C1);
  h2 = to_host(C2);
  EXPECT_TRUE(std::memcmp(h1.data(), h2.data(), h1.size() * sizeof(__half)) == 0);

  // GEMV plugin, bf16, plain and transposed
  const int gm = 768, gn = 1024;
  std::vector<float> ga(size_t(gm) * gn), gx(gm > gn ? gm : gn);
  oracle_fill_uniform_f32(ga.data(), ga.size(), 43, -1.f, 1.f);
  oracle_fill_uniform_f32(gx.data(), gx.size(), 44, -1.f, 1.f);
  std::vector<__nv_bfloat16> gah(ga.size()), gxh(gx.size());
  for (size_t i = 0; i < ga.size(); ++i) gah[i] = __float2bfloat16(ga[i]);
  for (size_t i = 0; i < gx.size(); ++i) gxh[i] = __float2bfloat16(gx[i]);
  Tensor<__nv_bfloat16> GA({size_t(gm) * gn}), GX({gx.size()}), Y1({size_t(gm)}), Y2({size_t(gm)});
  GA.copy_from_host(gah.data());
  GX.copy_from_host(gxh.data());
  auto pv = CreateBlasJITPlugin("gemv");
  auto* v = dynamic_cast<GemvJITPlugin*>(pv.get());
  EXPECT_TRUE(v && v->Initialize() == StatusCode::SUCCESS && v->Compile(JITConfig()) == StatusCode::SUCCESS);
  if (!v) return;
  for (int trans = 0; trans < 2; ++trans) {
    v->SetGemvParams(trans != 0, 1.0f, 0.0f);
    EXPECT_TRUE(v->ExecuteTyped(DataType::BFLOAT16, gm, gn, GA.data(), GX.data(), Y1.data()) == StatusCode::SUCCESS);
    const size_t ws = cuopx_gemv_workspace_size(CUOPX_BF16, trans, gm, gn);
    Tensor<unsigned char> W({ws > 0 ? ws : 1});
    W.zero();
    EXPECT_EQ(cuopx_gemv(CUOPX_BF16, trans, gm, gn, 1.0, GA.data(), trans ? gm : gn, GX.data(), 0.0, Y2.data(),
                         W.data(), ws, nullptr),
              CUOPX_SUCCESS);
    EXPECT_TRUE(cudaDeviceSynchronize() == cudaSuccess);
    auto y1 = to_host(Y1), y2 = to_host(Y2);
    EXPECT_TRUE(std::memcmp(y1.data(), y2.data(), y1.size() * sizeof(__nv_bfloat16)) == 0);
    double mr = 0, me = 0;
    for (int i = 0; i < gm; ++i) {
      double s = 0;
      for (int j = 0; j < gn; ++j) {
        const size_t idx = trans ? size_t(j) * gm + i : size_t(i) * gn + j;
        s += double(__bfloat162float(gah[idx])) * __bfloat162float(gxh[j]);
      }
      mr = std::max(mr, std::fabs(s));
      me = std::max(me, std::fabs(s - double(__bfloat162float(y1[i]))));
    }
    EXPECT_TRUE(mr > 0 && me / mr <= 1e-2);
  }
}

TEST_GPU(JitWrapperRoutesGemmThroughPlugin) {
  // test/JIT_test/test_jit_system.cpp:99-141 style: original vs wrapper on the same inputs
  const int n = 512;
  std::vector<float> a(size_t(n) * n), w(size_t(n) * n);
  oracle_fill_uniform_f32(a.data(), a.size(), 41, -1.f, 1.f);
  oracle_fill_uniform_f32(w.data(), w.size(), 42, -1.f, 1.f);
  Tensor<float> A({size_t(n), size_t(n)}), W({size_t(n), size_t(n)}), C1({size_t(n), size_t(n)}),
      C2({size_t(n), size_t(n)});
  A.copy_from_host(a.data());
  W.copy_from_host(w.data());
  Gemm<float> g(false, false, 1.f, 0.f);
  g.SetWeight(W);
  EXPECT_TRUE(g.Forward(A, C1) == StatusCode::SUCCESS);
  JITWrapper<Gemm<float>> wrapped(std::move(g));
  wrapped.EnableJIT(true);
  EXPECT_TRUE(wrapped.IsJITCompiled());
  EXPECT_TRUE(wrapped(A, C2) == StatusCode::SUCCESS);
  EXPECT_TRUE(!wrapped.GetPerformanceProfile().kernel_name.empty());  // the plugin ran, not the fallback
  auto h1 = to_host(C1), h2 = to_host(C2);
  EXPECT_TRUE(std::memcmp(h1.data(), h2.data(), h1.size() * sizeof(float)) == 0);
}

// The reference pool's maintenance calls (memory_pool.hpp:93-111):
// Preallocate fills the idle cache, TrimCache / Defragment / ReleaseAll hand
// idle blocks back to the driver, PrintStats reports.
TEST_GPU(HardwareProbeFillsClocks) {
  const HardwareSpec hw = QueryHardwareSpec();
  EXPECT_EQ(hw.compute_capability_major, 10);
  EXPECT_TRUE(hw.num_sms >= 100 && hw.sm_clock_rate > 1000 && hw.memory_clock_rate > 1000);
  const double gbs = hw.GetTheoreticalMemoryBandwidth(), gflops = hw.GetTheoreticalPeakGFLOPS();
  std::printf("    %s: %d SMs, %d MHz SM, %d MHz x %d-bit memory -> %.0f GB/s, %.0f FP32 GFLOP/s\n",
              hw.gpu_name.c_str(), hw.num_sms, hw.sm_clock_rate, hw.memory_clock_rate, hw.memory_bus_width, gbs,
              gflops);
  EXPECT_TRUE(gbs > 4000 && gbs < 12000);  // HBM3e-class
  EXPECT_TRUE(gflops > 40000 && gflops < 120000);
}

TEST_GPU(MemoryPoolMaintenanceCalls) {
  auto& pool = CudaMemoryPool::Instance();
  pool.ReleaseAll();
  pool.ResetStats();
  const auto base = pool.GetStats().bytes_reserved;
  pool.Preallocate(size_t(1) << 20, 3);
  EXPECT_EQ(pool.GetStats().bytes_reserved, base + (size_t(3) << 20));
  void* p = pool.Alloc(size_t(1) << 20);
  EXPECT_TRUE(p != nullptr);
  EXPECT_TRUE(pool.GetStats().cache_hits >= 1 && pool.GetStats().cache_misses == 3);
  pool.Free(p, size_t(1) << 20);
  EXPECT_TRUE(cudaDeviceSynchronize() == cudaSuccess);
  pool.TrimCache();  // every last use has completed: all idle blocks go
  EXPECT_EQ(pool.GetStats().bytes_reserved, base);
  pool.Preallocate(4096, 2);
  EXPECT_EQ(pool.GetStats().bytes_reserved, base + 2 * 4096);
  pool.Defragment();
  EXPECT_EQ(pool.GetStats().bytes_reserved, base);
  pool.Preallocate(4096, 1);
  pool.ReleaseAll();
  EXPECT_EQ(pool.GetStats().bytes_reserved, base);
  pool.PrintStats();
}

TEST_GPU(MemoryPoolReusesAndLimits) {
  auto& pool = CudaMemoryPool::Instance();
  pool.ResetStats();
  void* p = pool.Alloc(3000);
  EXPECT_TRUE(p != nullptr);
  pool.Free(p, 3000);
  void* q = pool.Alloc(4000);  // same 4 KiB class, same stream: cached block comes back
  EXPECT_TRUE(q == p);
  EXPECT_TRUE(pool.GetStats().cache_hits >= 1);
  pool.Free(q, 4000);
  // The limit counts reserved bytes (live + cached); idle cached blocks are
  // released to make room, so start from an empty cache to make 64 MiB
  // certainly exceed it.
  pool.ReleaseCached();
  const auto reserved = pool.GetStats().bytes_reserved;
  pool.SetMemoryLimit(reserved + (1 << 20));
  EXPECT_TRUE(pool.Alloc(size_t(64) << 20) == nullptr);  // over the limit: refused on the host
  EXPECT_TRUE(pool.GetStats().failed_allocs >= 1);
  bool threw = false;
  try {
    Tensor<float> big({size_t(32) << 20});
  } catch (const std::runtime_error&) {
    threw = true;
  }
  EXPECT_TRUE(threw);
  pool.SetMemoryLimit(0);
  Tensor<float> ok({size_t(32) << 20});
  EXPECT_TRUE(ok.data() != nullptr);
}

int main(int argc, char** argv) {
  bool host_only = false;
  std::string filter;
  for (int i = 1; i < argc; ++i) {
    if (std::string(argv[i]) == "--host-only") host_only = true;
    else filter = argv[i];
  }
  int run = 0;
  for (auto& t : registry()) {
    if (host_only && t.needs_gpu) continue;
    if (!filter.empty() && std::string(t.name).find(filter) == std::string::npos) continue;
    const int before = g_failures;
    std::printf("[ RUN  ] %s\n", t.name);
    t.fn();
    std::printf("[ %s ] %s\n", g_failures == before ? " OK " : "FAIL", t.name);
    ++run;
  }
  if (!host_only) {
    int code = 0;
    if (cuopx_get_device_error(&code) != 0 || code != 0) {
      std::printf("device error word: %d\n", code);
      ++g_failures;
    }
  }
  std::printf("%d tests, %d failures\n", run, g_failures);
  return g_failures == 0 && run > 0 ? 0 : 1;
}
