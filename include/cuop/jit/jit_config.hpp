// Configuration and profile structs of the plugin interface, with the field
// names and defaults of the reference's include/jit/jit_config.hpp:11-149 so
// existing configuration code keeps compiling.  The library generates no
// code at run time: JITConfig.kernel_type names a precompiled sm_100a
// variant family ("auto"/"default" = the built-in selection).
#pragma once

#include <string>
#include <vector>

namespace cu_op_mem {

struct GlobalJITConfig {
  bool enable_jit = true;
  bool enable_auto_tuning = true;
  bool enable_caching = true;
  std::string cache_dir = "./jit_cache";
  int max_cache_size = 1024 * 1024 * 1024;
  int compilation_timeout = 30;
  bool enable_tensor_core = true;
  bool enable_tma = true;
  int max_compilation_threads = 4;
  bool enable_debug = false;
};

struct JITConfig {
  bool enable_jit = true;
  std::vector<int> block_sizes = {16, 32, 64, 128};
  std::vector<int> tile_sizes = {16, 32, 64};
  int num_stages = 2;
  bool use_tensor_core = true;
  int block_size = 256;
  int block_size_x = 16;
  int block_size_y = 16;
  std::string kernel_type = "default";
  bool use_tma = true;
  std::string optimization_level = "auto";
  int max_registers = 255;
  bool enable_shared_memory_opt = true;
  bool use_shared_memory = true;
  bool enable_loop_unroll = true;
  bool enable_memory_coalescing = true;
  int tile_size = 16;
  bool enable_tensor_core = true;
  bool enable_tma = true;
  std::string hardware_spec = "";
  std::vector<int> matrix_size = {0, 0, 0};
};

struct JITStatistics {
  int total_compilations = 0;
  int cache_hits = 0;
  int cache_misses = 0;
  double total_compilation_time = 0.0;
  double total_execution_time = 0.0;
  size_t cache_size = 0;
  int active_kernels = 0;
  size_t total_saved_compilation_time = 0;
  double GetCacheHitRate() const {
    const int n = cache_hits + cache_misses;
    return n > 0 ? static_cast<double>(cache_hits) / n : 0.0;
  }
  double GetAverageCompilationTime() const {
    return total_compilations > 0 ? total_compilation_time / total_compilations : 0.0;
  }
  void Reset() { *this = JITStatistics(); }
};

struct PerformanceProfile {
  double gflops = 0.0;
  double bandwidth_gb_s = 0.0;
  double kernel_time_ms = 0.0;     // device time (CUDA events)
  double launch_overhead_ms = 0.0;
  double compilation_time_ms = 0.0;
  int block_size_x = 0;
  int block_size_y = 0;
  int tile_size = 0;
  bool used_tensor_core = false;
  bool used_tma = false;
  std::string kernel_name;         // the sm_100a variant that ran
  std::string optimization_level;
  double execution_time = 0.0;     // seconds
  std::string kernel_type = "";
  double throughput = 0.0;
  std::vector<int> matrix_size = {0, 0, 0};
  size_t memory_usage = 0;
  double GetTotalTime() const { return kernel_time_ms + launch_overhead_ms + compilation_time_ms; }
  double GetEfficiency(double peak_gflops) const { return peak_gflops > 0 ? gflops / peak_gflops : 0.0; }
};

struct HardwareSpec {
  int compute_capability_major = 0;
  int compute_capability_minor = 0;
  int num_sms = 0;
  int max_threads_per_sm = 0;
  int max_shared_memory_per_sm = 0;
  int max_registers_per_sm = 0;
  int max_threads_per_block = 0;
  int max_blocks_per_sm = 0;
  size_t total_global_memory = 0;
  int memory_clock_rate = 0;  // MHz
  int memory_bus_width = 0;   // bits
  int sm_clock_rate = 0;      // MHz (peak)
  bool supports_tensor_core = false;
  bool supports_tma = false;
  std::string gpu_name;
  int multi_processor_count = 0;
  int shared_memory_per_block = 0;
  std::string GetComputeCapabilityString() const {
    return std::to_string(compute_capability_major) + "." + std::to_string(compute_capability_minor);
  }
  // FP32 FFMA peak in GFLOP/s: SMs x FP32 lanes per SM (128 from compute
  // capability 9.0 on, 64 before) x 2 FLOP per FMA x peak SM clock.
  double GetTheoreticalPeakGFLOPS() const {
    const double lanes = compute_capability_major >= 9 ? 128.0 : 64.0;
    return num_sms * lanes * 2.0 * sm_clock_rate / 1000.0;
  }
  // DRAM bandwidth in GB/s: two transfers per memory clock across the bus.
  double GetTheoreticalMemoryBandwidth() const { return memory_clock_rate * 2.0 * memory_bus_width / 8.0 / 1000.0; }
};

// Probe of the current device (empty spec when there is none).
HardwareSpec QueryHardwareSpec();

}  // namespace cu_op_mem
