// Python module `cuop_b200.core`: the Python surface of the reference's
// pybind11 module (python/cuop/core.cpp), bound over the C++ facade, so that
// Python callers of TensorFloat / GemmFloat / GemvFloat / MatMulFloat /
// BatchMatMulFloat / DotFloat / AxpyFloat / ScalFloat / CopyFloat /
// JITGemmFloat / JITGemvFloat (and the Double forms) run the sm_100a
// kernels.  Same class and method names and argument meaning; a failed
// forward raises RuntimeError, as in the reference.  Differences: DotX.forward
// returns the result (a Python float cannot be passed by reference), and
// JITGemmX / JITGemvX copy the operator they wrap instead of binding it.
// Operators outside the BLAS path (Symm, Trsm, Relu, Softmax, norms,
// convolution, pooling) are not part of this library.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <random>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "cuda_op/detail/cuBlas/axpy.hpp"
#include "cuda_op/detail/cuBlas/copy.hpp"
#include "cuda_op/detail/cuBlas/dot.hpp"
#include "cuda_op/detail/cuBlas/gemm.hpp"
#include "cuda_op/detail/cuBlas/gemv.hpp"
#include "cuda_op/detail/cuBlas/scal.hpp"
#include "cuda_op/detail/cuDNN/batchmatmul.hpp"
#include "cuda_op/detail/cuDNN/matmul.hpp"
#include "jit/Blas/blas_jit_plugins.hpp"
#include "jit/jit_wrapper.hpp"

namespace py = pybind11;
using namespace cu_op_mem;

namespace {

void check(StatusCode s, const char* what) {
  if (s != StatusCode::SUCCESS)
    throw std::runtime_error(std::string(what) + " forward failed: status " + std::to_string(static_cast<int>(s)));
}

template <typename T>
void copy_from_numpy(Tensor<T>& t, py::array_t<T, py::array::c_style | py::array::forcecast> arr) {
  std::vector<std::size_t> shape(arr.ndim());
  for (py::ssize_t i = 0; i < arr.ndim(); ++i) shape[i] = static_cast<std::size_t>(arr.shape(i));
  Tensor<T> fresh(shape);
  fresh.copy_from_host(arr.data());
  t = std::move(fresh);
}

template <typename T>
py::array_t<T> to_numpy(const Tensor<T>& t) {
  std::vector<py::ssize_t> shape(t.shape().begin(), t.shape().end());
  py::array_t<T> out(shape);
  if (t.numel()) t.copy_to_host(out.mutable_data());
  return out;
}

template <typename T>
void bind_type(py::module_& m, const std::string& sfx) {
  py::class_<Tensor<T>>(m, ("Tensor" + sfx).c_str())
      .def(py::init<>())
      .def(py::init<const std::vector<std::size_t>&>())
      .def(py::init([](const std::vector<std::size_t>& shape, T value) {
        Tensor<T> t(shape);
        t.fill(value);
        return t;
      }))
      .def("shape", [](const Tensor<T>& t) { return t.shape(); })
      .def("size", &Tensor<T>::numel)
      .def("dtype", [](const Tensor<T>&) { return py::dtype::of<T>(); })
      .def("fill", &Tensor<T>::fill)
      .def("zero", &Tensor<T>::zero)
      .def("copy_from", &copy_from_numpy<T>)
      .def("to_numpy", &to_numpy<T>)
      .def("__repr__", [sfx](const Tensor<T>& t) {
        std::ostringstream ss;
        ss << "Tensor" << sfx << "(";
        for (std::size_t i = 0; i < t.shape().size(); ++i) ss << (i ? ", " : "") << t.shape()[i];
        ss << ")";
        return ss.str();
      });

  py::class_<Scal<T>>(m, ("Scal" + sfx).c_str())
      .def(py::init<T>(), py::arg("alpha") = T(1))
      .def("set_alpha", &Scal<T>::SetAlpha)
      .def("forward", [](Scal<T>& op, Tensor<T>& x) {
        check(op.Forward(x), "SCAL");
        cudaDeviceSynchronize();
      });
  py::class_<Axpy<T>>(m, ("Axpy" + sfx).c_str())
      .def(py::init<T>(), py::arg("alpha") = T(1))
      .def("set_alpha", &Axpy<T>::SetAlpha)
      .def("forward", [](Axpy<T>& op, const Tensor<T>& x, Tensor<T>& y) {
        check(op.Forward(x, y), "AXPY");
        cudaDeviceSynchronize();
      });
  py::class_<Copy<T>>(m, ("Copy" + sfx).c_str())
      .def(py::init<>())
      .def("forward", [](Copy<T>& op, const Tensor<T>& x, Tensor<T>& y) {
        check(op.Forward(x, y), "COPY");
        cudaDeviceSynchronize();
      });
  py::class_<Dot<T>>(m, ("Dot" + sfx).c_str())
      .def(py::init<>())
      .def("forward", [](Dot<T>& op, const Tensor<T>& x, const Tensor<T>& y) {
        T r{};
        check(op.Forward(x, y, r), "DOT");
        return r;
      });

  using S = typename ScalarOf<T>::type;
  py::class_<Gemm<T>>(m, ("Gemm" + sfx).c_str())
      .def(py::init<bool, bool, S, S>(), py::arg("transA") = false, py::arg("transB") = false, py::arg("alpha") = S(1),
           py::arg("beta") = S(0))
      .def("set_weight", &Gemm<T>::SetWeight)
      .def("forward", [](Gemm<T>& op, const Tensor<T>& input, Tensor<T>& output) {
        check(op.Forward(input, output), "GEMM");
        cudaDeviceSynchronize();
      });
  py::class_<Gemv<T>>(m, ("Gemv" + sfx).c_str())
      .def(py::init<bool, S, S>(), py::arg("transA") = false, py::arg("alpha") = S(1), py::arg("beta") = S(0))
      .def("set_weight", &Gemv<T>::SetWeight)
      .def("forward", [](Gemv<T>& op, const Tensor<T>& input, Tensor<T>& output) {
        check(op.Forward(input, output), "GEMV");
        cudaDeviceSynchronize();
      });
  py::class_<MatMul<T>>(m, ("MatMul" + sfx).c_str())
      .def(py::init<bool, bool>(), py::arg("transA") = false, py::arg("transB") = false)
      .def("forward", [](MatMul<T>& op, const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C, int axis) {
        check(op.Forward(A, B, C, axis), "MatMul");
      }, py::arg("A"), py::arg("B"), py::arg("C"), py::arg("axis") = -1);
  py::class_<BatchMatMul<T>>(m, ("BatchMatMul" + sfx).c_str())
      .def(py::init<>())
      .def("forward", [](BatchMatMul<T>& op, const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C) {
        check(op.Forward(A, B, C, 0), "BatchMatMul");
      });
}

template <typename Op>
void bind_jit_common(py::class_<JITWrapper<Op>>& c, const char* what) {
  c.def("enable_jit", &JITWrapper<Op>::EnableJIT)
      .def("enable_persistent_cache", [](JITWrapper<Op>&, bool) {})  // kernels are ahead-of-time: nothing to cache
      .def("set_persistent_cache_directory", [](JITWrapper<Op>&, const std::string&) {})
      .def("set_jit_config", &JITWrapper<Op>::SetJITConfig)
      .def("forward", [what](JITWrapper<Op>& w, const Tensor<float>& in, Tensor<float>& out) {
        check(w(in, out), what);
        cudaDeviceSynchronize();
      })
      .def("get_performance_profile", &JITWrapper<Op>::GetPerformanceProfile)
      .def("is_jit_compiled", &JITWrapper<Op>::IsJITCompiled)
      .def("get_last_error", &JITWrapper<Op>::GetLastError);
}

}  // namespace

PYBIND11_MODULE(core, m) {
  m.doc() = "cuOP operators on the B200 (sm_100a) kernels of libcuopx.so";
  RegisterBlasJITPlugins();
  bind_type<float>(m, "Float");
  bind_type<double>(m, "Double");

  // Tensor construction and device helpers (reference core.cpp's module functions).
  m.def("tensor", [](py::array_t<float, py::array::c_style | py::array::forcecast> arr) {
    Tensor<float> t;
    copy_from_numpy<float>(t, arr);
    return t;
  });
  m.def("zeros", [](const std::vector<std::size_t>& shape) {
    Tensor<float> t(shape);
    t.zero();
    return t;
  });
  m.def("ones", [](const std::vector<std::size_t>& shape) {
    Tensor<float> t(shape);
    t.fill(1.0f);
    return t;
  });
  // Normal(mean, std) samples (the reference's binding fills with `mean`
  // only); `seed` < 0 draws a fresh seed.
  m.def(
      "randn",
      [](const std::vector<std::size_t>& shape, float mean, float stddev, long long seed) {
        Tensor<float> t(shape);
        std::mt19937_64 gen(seed < 0 ? std::random_device{}() : static_cast<std::uint64_t>(seed));
        std::normal_distribution<float> dist(mean, stddev);
        std::vector<float> h(t.numel());
        for (auto& v : h) v = dist(gen);
        if (!h.empty()) t.copy_from_host(h.data());
        return t;
      },
      py::arg("shape"), py::arg("mean") = 0.0f, py::arg("std") = 1.0f, py::arg("seed") = -1);
  m.def("get_device_count", []() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    return n;
  });
  m.def("set_device", [](int d) {
    if (cudaSetDevice(d) != cudaSuccess) throw std::runtime_error("set_device failed");
  });
  m.def("get_device", []() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
  });
  m.def("synchronize", []() {
    if (cudaDeviceSynchronize() != cudaSuccess) throw std::runtime_error("synchronize failed");
  });
  m.def("get_memory_info", []() {
    std::size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);
    return py::make_tuple(free_b, total_b);
  });
  m.def("empty_cache", []() {
    int d = 0;
    cudaGetDevice(&d);
    CudaMemoryPool::ForDevice(d).ReleaseCached();
  });

  py::class_<JITConfig>(m, "JITConfig")
      .def(py::init<>())
      .def_readwrite("enable_jit", &JITConfig::enable_jit)
      .def_readwrite("kernel_type", &JITConfig::kernel_type)
      .def_readwrite("tile_size", &JITConfig::tile_size)
      .def_readwrite("block_size", &JITConfig::block_size)
      .def_readwrite("optimization_level", &JITConfig::optimization_level)
      .def_readwrite("enable_tensor_core", &JITConfig::enable_tensor_core)
      .def_readwrite("enable_tma", &JITConfig::enable_tma)
      .def_readwrite("max_registers", &JITConfig::max_registers)
      .def_readwrite("enable_shared_memory_opt", &JITConfig::enable_shared_memory_opt)
      .def_readwrite("enable_loop_unroll", &JITConfig::enable_loop_unroll)
      .def_readwrite("enable_memory_coalescing", &JITConfig::enable_memory_coalescing)
      .def("__repr__", [](const JITConfig& c) {
        return "JITConfig(enable_jit=" + std::string(c.enable_jit ? "True" : "False") + ", kernel_type='" +
               c.kernel_type + "', tile_size=" + std::to_string(c.tile_size) +
               ", block_size=" + std::to_string(c.block_size) + ", optimization_level='" + c.optimization_level +
               "')";
      });
  py::class_<GlobalJITConfig>(m, "GlobalJITConfig")
      .def(py::init<>())
      .def_readwrite("enable_jit", &GlobalJITConfig::enable_jit)
      .def_readwrite("enable_auto_tuning", &GlobalJITConfig::enable_auto_tuning)
      .def_readwrite("enable_caching", &GlobalJITConfig::enable_caching)
      .def_readwrite("cache_dir", &GlobalJITConfig::cache_dir)
      .def_readwrite("max_cache_size", &GlobalJITConfig::max_cache_size)
      .def_readwrite("compilation_timeout", &GlobalJITConfig::compilation_timeout)
      .def_readwrite("enable_tensor_core", &GlobalJITConfig::enable_tensor_core)
      .def_readwrite("enable_tma", &GlobalJITConfig::enable_tma)
      .def_readwrite("max_compilation_threads", &GlobalJITConfig::max_compilation_threads)
      .def_readwrite("enable_debug", &GlobalJITConfig::enable_debug);
  py::class_<PerformanceProfile>(m, "PerformanceProfile")
      .def_readonly("gflops", &PerformanceProfile::gflops)
      .def_readonly("bandwidth_gb_s", &PerformanceProfile::bandwidth_gb_s)
      .def_readonly("kernel_time_ms", &PerformanceProfile::kernel_time_ms)
      .def_readonly("kernel_name", &PerformanceProfile::kernel_name)
      .def_readonly("execution_time", &PerformanceProfile::execution_time);

  py::class_<JITWrapper<Gemm<float>>> jg(m, "JITGemmFloat");
  jg.def(py::init([](const Gemm<float>& op) {
    Gemm<float> g(op.TransA(), op.TransB(), op.Alpha(), op.Beta());
    g.SetWeight(op.GetWeight());
    return JITWrapper<Gemm<float>>(std::move(g));
  }));
  bind_jit_common(jg, "JIT GEMM");
  py::class_<JITWrapper<Gemv<float>>> jv(m, "JITGemvFloat");
  jv.def(py::init([](const Gemv<float>& op) {
    Gemv<float> g(op.TransA(), op.Alpha(), op.Beta());
    g.SetWeight(op.GetWeight());
    return JITWrapper<Gemv<float>>(std::move(g));
  }));
  bind_jit_common(jv, "JIT GEMV");
}
