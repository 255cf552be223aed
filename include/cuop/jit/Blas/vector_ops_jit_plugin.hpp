// Kept for include compatibility with the reference (include/jit/Blas/vector_ops_jit_plugin.hpp);
// the plugin classes are declared together in blas_jit_plugins.hpp.
#pragma once
#include "jit/Blas/blas_jit_plugins.hpp"
