/*
 * cos_sm100.h -- C ABI of the B200 (sm_100a) pairwise cosine-similarity matrix, the pairwise
 * case next to the RBF kernel in the same library (librbf_sm100.so) and on the same tcgen05
 * 3xTF32 kernels.
 *
 *   forward :  ah_i = a_i / (|a_i| + eps),  bh_j = b_j / (|b_j| + eps)
 *              S[i,j] = ah_i . bh_j                              A[N,D], B[M,D] -> S[N,M]
 *   backward:  gA = dS Bh,  gB = dS^T Ah
 *              dA_i = gA_i / (|a_i| + eps) - (ah_i . gA_i) ah_i / |a_i|     (dB likewise)
 *
 * This is the gradient torch autograd takes of the reference's broadcast expression
 * (reference cases/cosine_sim/reference.py:14-21); for a zero row the second term is 0.
 * Conventions are those of rbf_sm100.h: fp32, row-major, contiguous; int64 sizes; 16-byte
 * aligned pointers (NULL only for an empty operand); caller-owned outputs and workspace;
 * stream-ordered and non-blocking; an rbf_status code is returned, nothing aborts.
 *
 * The workspace holds the normalised rows of A and B (as TF32 hi/lo pairs) and their norms: the
 * state the reference's extension returns from cos_forward as Ah, Bh, invA, invB and takes back
 * in cos_backward (reference cases/cosine_sim/kernels/cosine_sim.cu:104-125,
 * cases/cosine_sim/op.py:18-32).
 */
#ifndef COS_SM100_H_
#define COS_SM100_H_

#include "rbf_sm100.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Bytes of the forward workspace; the backward needs cos_sm100_backward_workspace_bytes. */
RBF_API size_t cos_sm100_forward_workspace_bytes(int64_t N, int64_t M, int64_t D);
RBF_API size_t cos_sm100_backward_workspace_bytes(int64_t N, int64_t M, int64_t D);

/* Replaces the torch-extension call cos_forward(A, B, eps) -> [S, Ah, Bh, invA, invB]
 * (reference cases/cosine_sim/kernels/cosine_sim.cu:104-115) and its kernels normalize_kernel
 * and cos_fwd_tiled (cosine_sim.cu:25-61).  Writes S; the workspace keeps the normalised rows
 * and norms for cos_sm100_backward_prepared.  eps must be finite. */
RBF_API int cos_sm100_forward(const float* A, const float* B, float* S,
                              int64_t N, int64_t M, int64_t D, float eps,
                              void* workspace, size_t workspace_bytes, rbf_stream_t stream);

/* Replaces cos_backward(Ah, Bh, invA, invB, dS, N, M, D) -> [dA, dB]
 * (reference cosine_sim.cu:117-125, kernels cos_bwd_dA / cos_bwd_dB, cosine_sim.cu:63-102).
 * `workspace` must be the one cos_sm100_forward filled for the same A, B (N, M, D, eps) earlier
 * in stream order, at least cos_sm100_backward_workspace_bytes(N, M, D) bytes.  dA and dB are
 * fully overwritten. */
RBF_API int cos_sm100_backward_prepared(const float* dS, float* dA, float* dB,
                                        int64_t N, int64_t M, int64_t D, float eps,
                                        void* workspace, size_t workspace_bytes,
                                        rbf_stream_t stream);

/* Same, for a caller that did not keep the forward's workspace: normalises A and B again. */
RBF_API int cos_sm100_backward(const float* A, const float* B, const float* dS, float* dA,
                               float* dB, int64_t N, int64_t M, int64_t D, float eps,
                               void* workspace, size_t workspace_bytes, rbf_stream_t stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* COS_SM100_H_ */
