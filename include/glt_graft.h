/*
 * glt_graft.h -- C ABI of the B200-native grafted-MLP training library.
 *
 * Drop-in boundary for the hot path of Hinedes/GLT ("grafting"): a frozen
 * bf16 decoder whose SwiGLU MLPs carry trainable fp32 graft slices (gate/up/
 * down deltas), trained with graft-only AdamW, optionally shadow-baked into
 * the base weights for inference.
 *
 * The reference exposes no FFI; its internal API is free C++ functions
 * taking VramArena& / GraftWeights& plus raw device pointers.  Each entry
 * point below names the reference function(s) it replaces (path:line inside
 * the reference project).  Conventions:
 *   - plain pointers and sizes only; device pointers are marked "dev",
 *     host pointers "host";
 *   - every function returns a GltStatus (0 = ok) and never throws; the
 *     message of the last failure on the calling thread is glt_last_error();
 *     the reference logs file:line and throws std::runtime_error
 *     (src/checks.hpp:10-44) or returns [[nodiscard]] bool for I/O
 *     (src/checkpoint_impl.inc:170, src/data_impl.inc:9);
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default);
 *   - handles are not thread-safe; use one handle per rank thread.
 */
#ifndef GLT_GRAFT_H_
#define GLT_GRAFT_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GLT_API __attribute__((visibility("default")))
#else
#define GLT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Status                                                                   */
/* ------------------------------------------------------------------------ */
typedef enum GltStatus {
  GLT_OK = 0,
  GLT_EINVAL = 1,   /* bad argument / shape / alignment                   */
  GLT_ECUDA = 2,    /* CUDA runtime or driver error                       */
  GLT_ENCCL = 3,    /* NCCL error                                         */
  GLT_EIO = 4,      /* file I/O or format error                           */
  GLT_ETIMEOUT = 5, /* a bounded device wait gave up (see glt_device_error) */
  GLT_ESTATE = 6,   /* call not legal in the current state (e.g. double bake) */
  GLT_ENOMEM = 7    /* allocation failed                                  */
} GltStatus;

/* Message of the last failing call on this thread ("" if none). */
GLT_API const char* glt_last_error(void);
/* Library version string. */
GLT_API const char* glt_version(void);
/* Reads and clears the device error word of the current device
 * (1 = mbarrier wait timed out, 2 = bad shape seen by a kernel). */
GLT_API int glt_device_error(unsigned int* out_code);

/* ------------------------------------------------------------------------ */
/* Generic tensor-core GEMM (bf16 x bf16 -> fp32 accumulate)                */
/* Replaces gemm_core (src/gemm_impl.inc:21-58): one sm_100a tcgen05 kernel */
/* instead of rocblas_gemm_ex.  Row-major view:                            */
/*   C[M,N] = alpha * A[M,K] * B[N,K]^T + beta * C                          */
/* a_mn = 0: A stored [M][lda] (K contiguous); a_mn = 1: A stored [K][lda].   */
/* b_mn = 0: B stored [N][ldb] (K contiguous); b_mn = 1: B stored [K][ldb].   */
/* c_dtype: 0 = fp32, 1 = bf16 (beta must be 0 for bf16).                   */
/* ------------------------------------------------------------------------ */
GLT_API int glt_gemm(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
             void* C, int64_t ldc, int c_dtype, int M, int N, int K, float alpha, float beta,
             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GLT_GRAFT_H_ */
