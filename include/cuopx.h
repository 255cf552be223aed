/*
 * cuopx.h — C ABI of the B200 (sm_100a) dense BLAS hot path.
 *
 * Plain pointers and sizes only: every matrix/vector argument is a pointer
 * the GPU can dereference — device memory, or pinned (page-locked) host
 * memory, which the kernels reach through unified addressing (a GEMV's y
 * or one side of cuopx_copy, for instance); pageable host memory is not
 * checked for and must not be passed.  Every size is int64_t, every call is
 * asynchronous on the given
 * cudaStream_t (passed as void*, NULL = legacy default stream) and returns
 * a cuOP StatusCode integer (same numeric values as the reference's
 * `enum class StatusCode`, include/util/status_code.hpp:28-161).  No compute
 * call allocates device memory (scratch is passed in by the caller); only
 * the set-up call cuopx_peer_alloc does.
 *
 * Threads: compute calls may come from several host threads at once, on
 * one device or several; the library's per-device caches and its tuning
 * table are synchronised.  The GEMM variant override and the fp32 GEMM mode
 * are process-wide settings; cuopx_set_gemm_variant_thread and
 * cuopx_last_kernel are per host thread.  Work is ordered only by the
 * streams the caller passes, so two calls that share a scratch buffer must
 * share a stream (or be ordered by events).
 *
 * Layout convention: row-major, like the reference operators
 * (src/cuda_op/detail/cuBlas/gemm.cu:14-42, gemv.cu:10-23).
 */
#ifndef CUOPX_H_
#define CUOPX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (numerically identical to cu_op_mem::StatusCode) ---- */
#define CUOPX_SUCCESS 0
#define CUOPX_NOT_IMPLEMENTED 1001
#define CUOPX_TIMEOUT 1003
#define CUOPX_RESOURCE_UNAVAILABLE 1005
#define CUOPX_CUDA_ERROR 2000
#define CUOPX_OUT_OF_MEMORY 3001
#define CUOPX_INVALID_ARGUMENT 4001
#define CUOPX_EXECUTION_TIMEOUT 6002
#define CUOPX_KERNEL_NOT_FOUND 6005
#define CUOPX_NOT_COMPILED 7003
#define CUOPX_SHAPE_MISMATCH 10002
#define CUOPX_UNSUPPORTED_TYPE 11001

/* ---- element types ---- */
#define CUOPX_F32 0
#define CUOPX_F64 1
#define CUOPX_F16 2
#define CUOPX_BF16 3

/* ---- library ---- */
int cuopx_version(void);
/* Name of the kernel variant the last successful call on this host thread
 * launched (e.g. "gemm_tc_128x256", "gemv_t_splitk").  Never NULL. */
const char* cuopx_last_kernel(void);
/* Why the last call on this host thread that returned CUOPX_CUDA_ERROR
 * failed: the CUDA runtime error name (e.g. "cudaErrorLaunchOutOfResources")
 * or a short text for a driver-API failure; "none" before any.  Never NULL. */
const char* cuopx_last_cuda_error(void);
/* Number of cuopx kernels launched by this process so far. */
int64_t cuopx_launch_count(void);
/* First error code recorded by a device-side bounded wait (0 = none).
 * Synchronises the current device. */
int cuopx_get_device_error(int* code_out);
int cuopx_clear_device_error(void);

/*
 * fp32 GEMM arithmetic, process-wide:
 *   CUOPX_FP32_AUTO (default): problems of 256^3 and up with 16-byte-aligned
 *     rows run 3xTF32 on the tensor cores (hi*hi + hi*lo + lo*hi, fp32
 *     accumulate; meets ||C-R||_F/||R||_F <= 1e-5*sqrt(K), not bit-identical
 *     to an FFMA loop); the rest run FFMA.
 *   CUOPX_FP32_FFMA: always FFMA, one fma chain per output in ascending k,
 *     then fma(alpha, sum, beta*C) — the summation order and epilogue of the
 *     reference's kernels (gemm.cu:23-41, 264-291).  fp32 and fp64 GEMV then
 *     also run one ascending fma chain per output (gemv.cu:10-23).  Results
 *     reproduce the reference's own Gemm<float> (every kernel its selector
 *     picks for untransposed operands) and its Gemv<float> for shapes its
 *     gemv_kernel serves, bit for bit; the GPU tests run both side by side.
 *   CUOPX_FP32_TF32X3: 3xTF32 at every size it supports.
 * No reference counterpart (the reference has only FFMA kernels).
 */
#define CUOPX_FP32_AUTO 0
#define CUOPX_FP32_FFMA 1
#define CUOPX_FP32_TF32X3 2
int cuopx_set_fp32_gemm_mode(int mode);
int cuopx_get_fp32_gemm_mode(void);

/*
 * GEMM variant selection.  The built-in choice (size thresholds per dtype,
 * like the reference's selector, src/cuda_op/detail/cuBlas/gemm.cu:305-356)
 * can be refined by a tuning table — text rules
 *   dtype transA transB M N K batch variant
 * (dtype f32|f64|f16|bf16|*, trans 0|1|*, sizes lo:hi inclusive with either
 * side optional, or *) produced by an offline sweep; the first matching row
 * wins, and a variant that cannot run a problem falls back to the built-in
 * choice.  cuopx_set_gemm_variant forces one variant process-wide (NULL or
 * "auto" restores table + built-in choice); used by the sweep.  Variant
 * names: cuopx_gemm_variant_name(0..) until it returns NULL.  Replaces the
 * selection tables and AutoTuner-driven kernel choice of the reference
 * (src/jit/Blas/gemm_jit_plugin.cu:667-738, src/performance/auto_tuner.cu:100-295).
 */
int cuopx_tuning_load(const char* text);
int cuopx_tuning_load_file(const char* path);
int cuopx_tuning_clear(void);
int cuopx_tuning_rows(void);
int cuopx_set_gemm_variant(const char* name);
/* The same override for the calling host thread only (takes precedence over
 * the process-wide one); the BLAS plugins set it from JITConfig.kernel_type
 * around their launches.  NULL or "auto" clears it. */
int cuopx_set_gemm_variant_thread(const char* name);
const char* cuopx_gemm_variant_name(int index);

/*
 * GEMM: C = alpha * op(A) * op(B) + beta * C, all row-major.
 *   op(A) is M x K: A is M x K (lda >= K) or, if transA, K x M (lda >= M).
 *   op(B) is K x N: B is K x N (ldb >= N) or, if transB, N x K (ldb >= K).
 *   C is M x N (ldc >= N).  beta == 0 never reads C.
 * dtype F32/F64: alpha, beta and accumulation in that type.
 * dtype F16/BF16: inputs and C in that type, fp32 accumulate, alpha/beta
 *   applied in fp32, one rounding of the result.
 * Replaces Gemm<T>::Forward (src/cuda_op/detail/cuBlas/gemm.cu:417-511)
 * and GemmJITPlugin::Execute (src/jit/Blas/gemm_jit_plugin.cu:147-265).
 */
int cuopx_gemm(int dtype, int transA, int transB, int64_t M, int64_t N, int64_t K, double alpha, const void* A,
               int64_t lda, const void* B, int64_t ldb, double beta, void* C, int64_t ldc, void* stream);

/*
 * GEMM with a fused epilogue: C = act(alpha * op(A) * op(B) + beta * C + bias)
 *   epilogue = CUOPX_EPI_NONE, CUOPX_EPI_BIAS, CUOPX_EPI_RELU or
 *   CUOPX_EPI_BIAS | CUOPX_EPI_RELU.  bias is a device vector of N elements
 *   of `dtype` (added to every row; may be NULL without CUOPX_EPI_BIAS).
 *   ReLU(x) = x if x > 0 else +0.  The bias add and ReLU happen in the
 *   accumulation type before the one rounding to the output type.
 * Replaces MatMulReluFused<T>::Forward
 * (src/cuda_op/detail/cuDNN/kernel_fusion.cu:330-370: relu(A*W + bias)),
 * and Gemm<T>::Forward when epilogue == CUOPX_EPI_NONE.
 */
#define CUOPX_EPI_NONE 0
#define CUOPX_EPI_BIAS 1
#define CUOPX_EPI_RELU 2
int cuopx_gemm_ex(int dtype, int transA, int transB, int64_t M, int64_t N, int64_t K, double alpha, const void* A,
                  int64_t lda, const void* B, int64_t ldb, double beta, void* C, int64_t ldc, const void* bias,
                  int epilogue, void* stream);

/*
 * Strided batched GEMM: for b in [0, batch):
 *   C_b = alpha * op(A_b) * op(B_b) + beta * C_b,
 *   X_b = X + b * strideX (element strides; strideB may be 0 to share B).
 * Replaces BatchMatMul<T>::Forward (src/cuda_op/detail/cuDNN/batchmatmul.cu:52-94,
 * alpha=1, beta=0) and GemmBatchedJITPlugin::Execute
 * (src/jit/Blas/gemm_batched_jit_plugin.cu:113-188).
 */
int cuopx_gemm_strided_batched(int dtype, int transA, int transB, int64_t M, int64_t N, int64_t K,
                               double alpha, const void* A, int64_t lda, int64_t strideA, const void* B,
                               int64_t ldb, int64_t strideB, double beta, void* C, int64_t ldc, int64_t strideC,
                               int64_t batch, void* stream);

/*
 * GEMV: y[M] = alpha * op(A) * x[N] + beta * y[M].
 *   trans == 0: A is M x N row-major (lda >= N), y_i = sum_j A[i*lda+j] x_j.
 *   trans != 0: A is N x M row-major (lda >= M), y_i = sum_j A[j*lda+i] x_j
 *   (the reference's transA indexing A[col*m+row], gemv.cu:17).
 * `workspace` (device, 256-byte aligned) holds split-K partial sums and
 * arrival counters; size from cuopx_gemv_workspace_size().  With too
 * little workspace a single-pass variant runs instead (same result
 * bits are NOT guaranteed between the two variants; both meet tolerance).
 * Counters are left zeroed on return; a fresh workspace must be zeroed once.
 * Replaces Gemv<T>::Forward (src/cuda_op/detail/cuBlas/gemv.cu:209-256)
 * and GemvJITPlugin::Execute (src/jit/Blas/gemv_jit_plugin.cu:126-200).
 */
size_t cuopx_gemv_workspace_size(int dtype, int trans, int64_t M, int64_t N);
int cuopx_gemv(int dtype, int trans, int64_t M, int64_t N, double alpha, const void* A, int64_t lda,
               const void* x, double beta, void* y, void* workspace, size_t workspace_bytes, void* stream);

/*
 * GEMV that allocates nothing: same arguments and result as cuopx_gemv, but
 * the split-K scratch comes from a fixed 2 MiB array inside the library
 * (per device, held until exit) instead of a caller-provided workspace.
 * For callers that may not allocate device memory while running (plugin
 * hosts that own all device memory, latency-bound serving loops where an
 * allocation can stall or fail).  No counterpart in the reference.
 * Returns CUOPX_RESOURCE_UNAVAILABLE when the kernel chosen for the call
 * needs more than 2 MiB of scratch (rows that are 16-byte aligned and a
 * multiple of 16 bytes long never do, at any size and type; other shapes
 * can, e.g. bf16 transposed 8191 x 8192).  The first call on a device resolves the array's
 * device address; make it before any stream capture.  Calls share the array:
 * calls that overlap on the GPU race, so order them on one stream.  Each call
 * zeroes the array's counter block on `stream` before its kernels run.
 */
int cuopx_gemv_noalloc(int dtype, int trans, int64_t M, int64_t N, double alpha, const void* A, int64_t lda,
                       const void* x, double beta, void* y, void* stream);

/*
 * Column-block gather for N-sharded GEMM: `blocks` is G contiguous
 * [M][Nb] row-major blocks (as an all-gather leaves them); writes the
 * row-major [M][G*Nb] matrix `out` (ldo >= G*Nb).  Element size from dtype.
 * No reference counterpart (the reference has no multi-GPU path); used
 * after ncclAllGather of per-rank GEMM outputs.
 */
int cuopx_gather_column_blocks(int dtype, int64_t G, int64_t M, int64_t Nb, const void* blocks, void* out,
                               int64_t ldo, void* stream);

/*
 * Peer memory for the fused column-sharded GEMM (one process per GPU, GPUs
 * of one NVLink/NVSwitch node).  No reference counterpart: the reference is
 * single-GPU.
 *
 * cuopx_peer_alloc   device allocation on the current GPU, zero-filled, plus
 *                    an opaque CUOPX_PEER_HANDLE_BYTES handle that another
 *                    process passes to cuopx_peer_open to map it.  A set-up
 *                    call: it allocates, the compute entry points never do.
 * cuopx_peer_open    maps a peer's allocation into this process (peer access
 *                    over NVLink); cuopx_peer_close unmaps it.
 * cuopx_peer_free    releases an allocation made by cuopx_peer_alloc (after
 *                    every peer has closed it).
 */
#define CUOPX_PEER_HANDLE_BYTES 64
int cuopx_peer_alloc(size_t bytes, void** ptr, void* handle_out);
int cuopx_peer_open(const void* handle, void** ptr);
int cuopx_peer_close(void* ptr);
int cuopx_peer_free(void* ptr);

/*
 * Cross-GPU barrier on `stream`: signals[r] is rank r's signal block (a
 * cuopx_peer_alloc block of at least CUOPX_PEER_SIGNAL_BYTES, mapped in this
 * process).  Every rank posts an epoch into each rank's block with a
 * system-scope release, then waits (acquire) until all `world` ranks have
 * posted, so that device writes a rank made on its stream before the barrier
 * are visible to every rank's stream after it.  The epoch counter lives in
 * the local block, so the call can be captured in a CUDA graph.  A wait that
 * exceeds 5 s records CUOPX_DEVERR_PEER_TIMEOUT in the device error word and
 * returns.  No reference counterpart.
 */
#define CUOPX_PEER_SIGNAL_BYTES 512
#define CUOPX_DEVERR_PEER_TIMEOUT 8
int cuopx_peer_barrier(void* const* signals, int world, int rank, void* stream);

/*
 * Column-sharded GEMM fused with the all-gather of its output: this rank
 * holds B_local = W[:, rank*N_local : (rank+1)*N_local] and computes
 * C_block = alpha * op(A) * B_local; every output tile is written, from the
 * epilogue, into the column block [rank*N_local, (rank+1)*N_local) of every
 * rank's full output C_ranks[r] (row-major [M][world*N_local], leading
 * dimension ldc, identical layout on every rank; C_ranks[rank] is local, the
 * others peer mappings).  Stores to peers are plain global stores over
 * NVLink, overlapped with the next tile's MMAs; no collective library call.
 * The caller brackets the call with cuopx_peer_barrier (before: peers are
 * done reading their outputs; after: all blocks have landed).
 * fp16/bf16 only, M, N_local, K >= 256, N_local and ldc multiples of 8;
 * other problems return CUOPX_NOT_IMPLEMENTED (the caller then uses
 * cuopx_gemm + an all-gather + cuopx_gather_column_blocks).
 * Replaces, for the multi-GPU case, Gemm<T>::Forward
 * (src/cuda_op/detail/cuBlas/gemm.cu:417-511) followed by an all-gather.
 */
int cuopx_gemm_allgather(int dtype, int transA, int transB, int64_t M, int64_t N_local, int64_t K, double alpha,
                         const void* A, int64_t lda, const void* B, int64_t ldb, void* const* C_ranks, int world,
                         int rank, int64_t ldc, void* stream);

/*
 * Level-1 vector operations (fp32), replacing VectorOpsJITPlugin::Execute
 * (src/jit/Blas/vector_ops_jit_plugin.cu:113-181) with standard BLAS
 * semantics.  Scalar results are written to DEVICE memory (`result`).
 * Reductions use `workspace` (cuopx_vector_workspace_size bytes, zeroed
 * once; counters are left zeroed on return).  Index results are 1-based
 * BLAS indices of the FIRST maximal / minimal |x_i| (0 when n <= 0).
 */
size_t cuopx_vector_workspace_size(int64_t n);
int cuopx_dot(int64_t n, const float* x, int64_t incx, const float* y, int64_t incy, float* result,
              void* workspace, size_t workspace_bytes, void* stream);
int cuopx_axpy(int64_t n, float alpha, const float* x, int64_t incx, float* y, int64_t incy, void* stream);
int cuopx_scal(int64_t n, float alpha, float* x, int64_t incx, void* stream);
int cuopx_copy(int64_t n, const float* x, int64_t incx, float* y, int64_t incy, void* stream);
int cuopx_swap(int64_t n, float* x, int64_t incx, float* y, int64_t incy, void* stream);
int cuopx_rot(int64_t n, float* x, int64_t incx, float* y, int64_t incy, float c, float s, void* stream);
int cuopx_nrm2(int64_t n, const float* x, int64_t incx, float* result, void* workspace, size_t workspace_bytes,
               void* stream);
int cuopx_asum(int64_t n, const float* x, int64_t incx, float* result, void* workspace, size_t workspace_bytes,
               void* stream);
int cuopx_iamax(int64_t n, const float* x, int64_t incx, int64_t* result, void* workspace,
                size_t workspace_bytes, void* stream);
int cuopx_iamin(int64_t n, const float* x, int64_t incx, int64_t* result, void* workspace,
                size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CUOPX_H_ */
