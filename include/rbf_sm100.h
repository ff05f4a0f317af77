/*
 * rbf_sm100.h -- C ABI of the B200 (sm_100a) Gaussian RBF kernel matrix.
 *
 *   forward :  K[i,j] = exp(-gamma * ||x_i - y_j||^2)          X[N,D], Y[M,D] -> K[N,M]
 *   backward:  W = G o K (elementwise), c = -2*gamma
 *              dX[i,:] = c * ( rowsum_j(W)[i] * x_i - (W  Y)[i,:] )
 *              dY[j,:] = c * ( colsum_i(W)[j] * y_j - (W^T X)[j,:] )
 *
 * All matrices are fp32, row-major and contiguous.  Sizes are int64 (N*M reaches 4.3e9 at
 * N=M=65536).  Every entry point below that takes a stream is stream-ordered and non-blocking:
 * it validates its arguments on the host, enqueues its kernels on `stream`, and returns.  No
 * entry point allocates device memory except the legacy host-pointer pair at the end, which
 * mirrors the reference's delivery ABI.  No entry point aborts, traps or prints; each returns
 * an rbf_status code.
 *
 * Error behaviour of the reference: the torch extension raises RuntimeError through
 * TORCH_CHECK (reference cases/rbf/kernels/rbf_forward.cu:95-99, rbf_backward.cu:61-64); the
 * delivery ABI aborts on a CUDA error (reference cases/rbf/delivery/rbf_kernels.cu:26-36).  The
 * Python layer of this library turns a non-zero rbf_status into RuntimeError; the legacy
 * host-pointer pair prints the error and aborts, as the reference's does.
 */
#ifndef RBF_SM100_H_
#define RBF_SM100_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define RBF_API __attribute__((visibility("default")))
#else
#define RBF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st* rbf_stream_t;

typedef enum rbf_status {
  RBF_OK = 0,
  RBF_ERR_INVALID_ARGUMENT = 1, /* negative size, NULL pointer, non-finite gamma        */
  RBF_ERR_MISALIGNED = 2,       /* a pointer is not 16-byte aligned                      */
  RBF_ERR_WORKSPACE = 3,        /* workspace NULL or smaller than the *_workspace_bytes  */
  RBF_ERR_UNSUPPORTED = 4,      /* shape outside what the kernels support (D > 4096)     */
  RBF_ERR_CUDA = 5,             /* a CUDA runtime/driver call failed                     */
  RBF_ERR_NO_DEVICE = 6,        /* no sm_100 device is current                           */
  RBF_ERR_TIMEOUT = 7,          /* a device-side wait exceeded its bound (status word)   */
  RBF_ERR_TOO_LARGE = 8         /* size exceeds a fixed capacity of the entry point      */
} rbf_status;

/* Human-readable message for a status code (static storage; never NULL). */
RBF_API const char* rbf_sm100_strerror(int status);

/* Detail of the last non-OK status returned on the calling thread (names the failing check or
 * the CUDA error).  Thread-local static storage; never NULL. */
RBF_API const char* rbf_sm100_last_error_detail(void);

/* Number of kernels this library has enqueued in this process (all devices, all threads). */
RBF_API uint64_t rbf_sm100_launch_count(void);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
RBF_API int rbf_sm100_version(void);

/* ---------------------------------------------------------------------------------------------
 * Forward.  Replaces the torch-extension call rbf_forward(X, Y, gamma) -> K
 * (reference cases/rbf/kernels/rbf_forward.cu:94-116) and the kernel it launches
 * (rbf_forward.cu:20-92).  Differences from the reference: the caller owns K and the workspace;
 * the call is enqueued on `stream` instead of the legacy default stream.
 *
 * The workspace holds the split (hi/lo TF32) copies of X and Y and their squared norms.  After
 * the call (in stream order) it is a valid "prepared" workspace for rbf_sm100_backward_prepared.
 * ------------------------------------------------------------------------------------------- */
RBF_API size_t rbf_sm100_forward_workspace_bytes(int64_t N, int64_t M, int64_t D);

RBF_API int rbf_sm100_forward(const float* X, const float* Y, float* K,
                      int64_t N, int64_t M, int64_t D, float gamma,
                      void* workspace, size_t workspace_bytes, rbf_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Backward.  Replaces the torch-extension call rbf_backward(X, Y, G, K, gamma) -> [dX, dY]
 * (reference cases/rbf/kernels/rbf_backward.cu:59-84) and its two kernels
 * rbf_backward_dX_kernel / rbf_backward_dY_kernel (rbf_backward.cu:16-57), which read G and K
 * twice.  K is the forward's output (the reference's autograd saves it, cases/rbf/op.py:31-32).
 * dX and dY are fully overwritten.
 * ------------------------------------------------------------------------------------------- */
/* RBF_DETERMINISTIC=1 in the environment (read at every call) makes the backward entries
 * bit-reproducible run to run: each tile's dX / dY contribution goes to its own slot in the
 * workspace and a finalize pass sums the slots in a fixed order, instead of atomic adds.  The
 * workspace then needs about 4 * (ceil(M/128) * N' + ceil(N/128) * M) * (D + 1) more bytes
 * (N' = N rounded up to 128); rbf_sm100_backward_workspace_bytes includes them while the
 * variable is set, so size the workspace after setting it.  A smaller workspace is refused
 * (RBF_ERR_WORKSPACE).  M % 4 != 0 runs CUDA-core kernels that are deterministic already. */
RBF_API size_t rbf_sm100_backward_workspace_bytes(int64_t N, int64_t M, int64_t D);

RBF_API int rbf_sm100_backward(const float* X, const float* Y, const float* G, const float* K,
                       float* dX, float* dY,
                       int64_t N, int64_t M, int64_t D, float gamma,
                       void* workspace, size_t workspace_bytes, rbf_stream_t stream);

/* Same as rbf_sm100_backward, but `workspace` must be the forward workspace of the SAME X, Y
 * (N, M, D) filled by rbf_sm100_forward earlier in stream order, and must be at least
 * rbf_sm100_backward_workspace_bytes(N, M, D) bytes; the X/Y split pass is skipped.  This is
 * the call the autograd op makes (its forward saves the workspace with X, Y and K).  No
 * reference counterpart: the reference backward recomputes nothing it could share. */
RBF_API int rbf_sm100_backward_prepared(const float* X, const float* Y, const float* G, const float* K,
                                float* dX, float* dY,
                                int64_t N, int64_t M, int64_t D, float gamma,
                                void* workspace, size_t workspace_bytes, rbf_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Forward and backward in one call, for callers that hold the upstream gradient G before the
 * forward runs (a fixed loss, a training harness).  Replaces the pair of calls the reference's
 * autograd op makes, RBFFunction.forward then RBFFunction.backward (reference
 * cases/rbf/op.py:27-37): K = exp(-gamma ||x_i - y_j||^2) is written to K and [dX, dY] of
 * sum(G * K) to dX and dY.  The X/Y split is made once and shared by both passes, and the
 * backward kernels follow the forward on `stream` by programmatic dependent launch.  The
 * workspace is the backward's, rbf_sm100_backward_workspace_bytes(N, M, D).  Results are those
 * of rbf_sm100_forward followed by rbf_sm100_backward_prepared.
 * ------------------------------------------------------------------------------------------- */
RBF_API int rbf_sm100_forward_backward(const float* X, const float* Y, const float* G, float* K,
                               float* dX, float* dY,
                               int64_t N, int64_t M, int64_t D, float gamma,
                               void* workspace, size_t workspace_bytes, rbf_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Multi-GPU row sharding helper.  The caller owns rows [row0, row0+N_local) of X, G and K; Y is
 * replicated.  Writes this shard's dX rows (complete) and the shard's PARTIAL dY (sum over the
 * shard's rows only) into dY_partial, which the caller all-reduces (sum) across ranks.  There is
 * no reference counterpart: the reference never runs on more than one GPU.  Same as
 * rbf_sm100_backward on the shard; exposed under its own name so that the partial semantics of
 * dY are explicit at the call site.
 * ------------------------------------------------------------------------------------------- */
RBF_API int rbf_sm100_backward_shard(const float* X_local, const float* Y, const float* G_local,
                             const float* K_local, float* dX_local, float* dY_partial,
                             int64_t N_local, int64_t M, int64_t D, float gamma,
                             void* workspace, size_t workspace_bytes, rbf_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Row-sharded backward with the dY all-reduce done by this library over NVLink peer memory.  No
 * counterpart in the reference (it runs on one GPU); replaces rbf_sm100_backward_shard + an NCCL
 * all-reduce of dY.  `dy_buffers[r]` is rank r's buffer of 2 * M * D floats, mapped in this
 * process (peer memory, e.g. CUDA symmetric memory); every rank passes the same list.  The
 * backward zeroes slot (*step_counter % 2) of dy_buffers[rank] and accumulates this rank's dY
 * partial there; rbf_sm100_dy_exchange then completes dY.  X_local, G_local, K_local, dX_local,
 * workspace: as rbf_sm100_backward_prepared (the forward filled the workspace).  M % 4 == 0.
 * ------------------------------------------------------------------------------------------- */
RBF_API int rbf_sm100_backward_shard_routed(const float* X_local, const float* Y,
                                            const float* G_local, const float* K_local,
                                            float* dX_local, int64_t N_local, int64_t M, int64_t D,
                                            float gamma, void* workspace, size_t workspace_bytes,
                                            float* const* dy_buffers, int world, int rank,
                                            const int* step_counter, rbf_stream_t stream);

/* Completes a routed step on this rank (all ranks call it): barrier; the owner of each 128-row
 * j-block (j-block % world) sums it over every rank's slot; barrier; the full dY [M, D] is
 * gathered from the owners; *step_counter advances (device int, 0 on every rank before the first
 * step).  Both barriers are bounded by RBF_WAIT_TIMEOUT_MS: on expiry the workspace status word
 * reads RBF_ERR_TIMEOUT, dY is not written, the step counter does not advance, and tickets[2]
 * is set: every later exchange on these buffers then skips its work and reports
 * RBF_ERR_TIMEOUT, until the caller sets the buffers up again (flags, counter and tickets
 * zeroed on every rank).  `flag_arrays[r]`: rank r's int[world] signal array (peer memory,
 * zeroed once); `tickets`: three zeroed device unsigned ints of this rank.  D % 4 == 0.  No host
 * synchronisation, so a captured CUDA graph of the step can be replayed. */
RBF_API int rbf_sm100_dy_exchange(float* dY, int64_t M, int64_t D, float* const* dy_buffers,
                                  int* const* flag_arrays, int world, int rank, int* step_counter,
                                  unsigned* tickets, void* workspace, size_t workspace_bytes,
                                  rbf_stream_t stream);

/* Status word written by the device-side bounded waits (RBF_OK or RBF_ERR_TIMEOUT).  Blocking:
 * synchronizes `stream`, then copies the word out of `workspace`.  Resets it to RBF_OK. */
RBF_API int rbf_sm100_read_status(void* workspace, rbf_stream_t stream, int* device_status);

/* ---------------------------------------------------------------------------------------------
 * Allocation-free forward.  No counterpart in the reference.  For callers that cannot allocate
 * device memory (an application whose allocator owns the device heap, a runtime that forbids
 * cudaMalloc on its hot path, a plugin interface with no way to pass a workspace): same result
 * as rbf_sm100_forward, but the workspace is a fixed device array inside this library
 * (rbf_sm100_forward_noalloc_capacity() bytes, 16 MiB, held on every GPU that loads the library
 * until the process exits).  The caller still passes X, Y and K.  Calls whose workspace would
 * exceed the capacity return RBF_ERR_TOO_LARGE (about (N+M)*(2*Dp+1)*4 bytes are needed,
 * Dp = D rounded up to 32; e.g. N = M = 4096 at D = 64 fits).  Allocates nothing: no cudaMalloc,
 * no cudaFree, no allocating library call.  The first call in each CUDA context looks up the
 * array's device address with that context current (cudaGetSymbolAddress) and caches it per
 * context; make that first call before any stream capture.  All calls share the one array, so
 * calls that overlap on the GPU (different streams, or other host threads) race and must be
 * serialised by the caller.  A device-side wait that ran out (RBF_ERR_TIMEOUT: K is then only
 * partly written) is reported by rbf_sm100_forward_noalloc_read_status, which reads the array's
 * status word; the next call resets it.
 * ------------------------------------------------------------------------------------------- */
RBF_API size_t rbf_sm100_forward_noalloc_capacity(void);
RBF_API int rbf_sm100_forward_noalloc(const float* X, const float* Y, float* K,
                                      int64_t N, int64_t M, int64_t D, float gamma,
                                      rbf_stream_t stream);
/* Status word of the allocation-free forward's internal array: RBF_OK, or RBF_ERR_TIMEOUT when a
 * device-side wait of the last call ran out.  Blocking, like rbf_sm100_read_status (synchronizes
 * `stream`, copies the word to the host with a plain cudaMemcpy, resets it); allocates nothing. */
RBF_API int rbf_sm100_forward_noalloc_read_status(rbf_stream_t stream, int* device_status);

/* ---------------------------------------------------------------------------------------------
 * Legacy host-pointer ABI of the reference's standalone delivery
 * (reference cases/rbf/delivery/rbf_kernels.cu:168-220, delivery/README.md:37-41):
 * host pointers, blocking, device memory allocated and freed inside every call.  Like the
 * reference, a CUDA failure prints a message and aborts.  int sizes, as in the reference.
 * ------------------------------------------------------------------------------------------- */
RBF_API void rbf_forward_cuda(const float* X, const float* Y, float* K,
                      int N, int M, int D, float gamma);
RBF_API void rbf_backward_cuda(const float* X, const float* Y, const float* G, const float* K,
                       float* dX, float* dY, int N, int M, int D, float gamma);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* RBF_SM100_H_ */
