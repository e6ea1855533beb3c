/*
 * rustane_cuda.h — C ABI of librustane_cuda.so, the B200 (sm_100a) engine for
 * rustane's language-model step: forward pass, backward pass and AdamW.
 *
 * This library is the `cuda-bridge` that replaces the `ane` crate surface the
 * engine crate binds today (crates/ane-bridge/src/lib.rs:1-9; graph build +
 * compile + eval at crates/engine/src/layer.rs:237-275, :600-602), the MIL
 * graph builders (crates/engine/src/kernels/*.rs) and the Accelerate CPU ops
 * (crates/engine/src/cpu/*.rs).  Each entry point below names the reference
 * interface it replaces.
 *
 * Conventions
 *  - Every function returns an int status: RT_OK (0) or a negative RT_ERR_*.
 *    rt_last_error(ctx) returns a human-readable message for the last failure
 *    on that context (the reference panics via .expect(); the Rust binding maps
 *    non-zero status back to that panic).
 *  - Host pointers are borrowed for the duration of the call only.  Device
 *    memory is owned by the context.  Calls on one context are not thread-safe.
 *  - Host tensors use the reference layouts: row-major fp32, wq/wk/wv/wo
 *    [dim, dim], w1/w3/w2 [dim, hidden], embed [vocab, dim], gammas [dim].
 *  - rt_kernel_* entry points take DEVICE pointers and a cudaStream_t (as
 *    void*); they launch one kernel asynchronously and exist for kernel-level
 *    parity checks.
 */
#ifndef RUSTANE_CUDA_H
#define RUSTANE_CUDA_H

#include <stdint.h>

#if defined(__GNUC__)
#define RT_API __attribute__((visibility("default")))
#else
#define RT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes */
#define RT_OK 0
#define RT_ERR_ARG (-1)        /* null pointer / invalid argument            */
#define RT_ERR_SHAPE (-2)      /* shape or alignment the kernels do not take */
#define RT_ERR_CUDA (-3)       /* CUDA runtime error                          */
#define RT_ERR_OOM (-4)        /* device allocation failed                    */
#define RT_ERR_TOKEN (-5)      /* token id >= vocab                           */
#define RT_ERR_DEVICE (-6)     /* a kernel reported an error (device flag)    */
#define RT_ERR_NCCL (-7)       /* NCCL failure / timeout / not initialised    */
#define RT_ERR_STATE (-8)      /* call order (e.g. backward before forward)   */
#define RT_ERR_NONFINITE (-9)  /* loss or gradient norm is NaN / Inf          */

/* GEMM epilogue selector for rt_kernel_gemm (see the kernel sources). */
#define RT_EPI_BF16 0
#define RT_EPI_F32 1
#define RT_EPI_F32_ACC 2
#define RT_EPI_RESIDUAL 3
#define RT_EPI_ROPE 4
#define RT_EPI_SWIGLU 5
#define RT_EPI_SWIGLU_BWD 6

/* -------------------------------------------------- kernel-level entries */

/* tcgen05 GEMM C[M,N] = sum_k A[m,k] B[n,k] (bf16 in, fp32 accumulate) with a
 * fused epilogue.  a_mn/b_mn select MN-major storage ([K][M] / [K][N]).
 * Replaces the DynMatmul / DualDynMatmul ANE graphs
 * (crates/engine/src/kernels/dyn_matmul.rs:15-86), the matmuls inside
 * sdpaFwd/ffnFused (kernels/sdpa_fwd.rs:80-83, kernels/ffn_fused.rs:48-72) and
 * the cblas_sgemm calls (crates/engine/src/cpu/vdsp.rs:128-136, :287-321). */
RT_API int rt_kernel_gemm(const void* a, int64_t lda, int a_mn, const void* b, int64_t ldb, int b_mn, int M, int N,
                          int K, int epi, void* out, int64_t ldo, void* out2, int64_t ldo2, const void* aux,
                          int64_t ld_aux, float alpha, int beta, const float* rope_cos, const float* rope_sin,
                          int seq, int rope_cols, int n_half, int force_bn, int* dev_err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RUSTANE_CUDA_H */
