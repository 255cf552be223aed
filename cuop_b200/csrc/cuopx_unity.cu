// Single translation unit for the device code of libcuopx.so, so that the
// module-wide device error word (cuopx::g_device_error) and every kernel
// live in one CUDA module without relocatable-device-code linking.
#include "capi.cu"
#include "gemv_stream.cu"
#include "gemv.cu"
#include "gemv_noalloc.cu"
#include "gemm_simt.cu"
#include "gemm_tc.cu"
#include "gemm_tc2.cu"
#include "peer.cu"
#include "gemm_tf32x3.cu"
#include "vector_ops.cu"
