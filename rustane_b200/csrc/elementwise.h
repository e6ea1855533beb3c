// Launch interface of the memory-bound kernels (internal).  Every reduction
// here is deterministic: fixed partitioning and fixed summation order, so two
// runs on the same inputs produce identical bits.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rt {

// x[m, :] = E[tok[m], :] (fp32 copy); tokens >= V set *err and write zeros.
int embed_gather(const float* E, const uint32_t* tok, float* x, int M, int D, int V, int* err, cudaStream_t s);

// dE[seg_tok[j], :] += sum_{i in [seg_start[j], seg_start[j+1])} dx[perm[i], :], positions in ascending order.
int embed_scatter(const float* dx, const int32_t* perm, const int32_t* seg_start, const uint32_t* seg_tok, int nseg,
                  float* dE, int D, cudaStream_t s);

// out = bf16(x * rms_inv * gamma), rms_inv = 1/sqrt(mean(x^2) + 1e-5), one row per token.
int rmsnorm_fwd(const float* x, const float* gamma, __nv_bfloat16* out, float* rms_inv, int M, int D, cudaStream_t s);

// dx = rms_inv * (dy*gamma - xhat * mean(dy*gamma*xhat)) + resid (resid may be null);
// dx_bf16 (optional) = bf16(bf16_scale * dx); dgamma partials [rmsnorm_bwd_blocks(M)][D]
// (fixed row partition and order) for dgamma_reduce.
int rmsnorm_bwd(const float* dy, const float* x, const float* gamma, const float* rms_inv, const float* resid,
                float* dx, __nv_bfloat16* dx_bf16, float bf16_scale, float* dgamma_part, int M, int D,
                cudaStream_t s);
int rmsnorm_bwd_blocks(int M);
// dgamma[d] = (accumulate ? dgamma[d] : 0) + sum_b part[b][d]   (b ascending)
int dgamma_reduce(const float* part, int nblk, float* dgamma, int D, int accumulate, cudaStream_t s);
// The same for ngamma adjacent gammas in one launch: gamma g's partials at
// part + g * part_stride, its result at dgamma + g * D (identical arithmetic).
int dgamma_reduce_many(const float* part, int64_t part_stride, int nblk, float* dgamma, int D, int ngamma,
                       int accumulate, cudaStream_t s);

// Cross-entropy over rows of fp32 logits (optionally soft-capped):
//   row_loss[m] = lse - z[t], row_lse[m] = lse, z = softcap > 0 ? softcap*tanh(l/softcap) : l.
int ce_forward(const float* logits, const uint32_t* tgt, float* row_loss, float* row_lse, int M, int V,
               float softcap, cudaStream_t s);
// dl[m, v] = bf16(scale * (softmax(z)[v] - [v == t]) * (softcap ? 1 - tanh^2 : 1))
int ce_backward(const float* logits, const float* row_lse, const uint32_t* tgt, __nv_bfloat16* dl, int M, int V,
                float softcap, float scale, cudaStream_t s);
// ce_forward and ce_backward in one read of the logits (the train step, where the
// backward always follows): row_loss, row_lse and dl as the two kernels write them.
int ce_fused(const float* logits, const uint32_t* tgt, float* row_loss, float* row_lse, __nv_bfloat16* dl, int M,
             int V, float softcap, float scale, cudaStream_t s);
// out[0] = sum(row_loss) / M (fixed-order tree, one block)
int mean_reduce(const float* row_loss, int M, float* out, cudaStream_t s);

// Global L2 norm over n fp32 values: partials then a fixed-order final pass.
int sumsq_norm(const float* x, int64_t n, float* partials, float* out_norm, cudaStream_t s);
int sumsq_partials_count();
// Segmented form: sumsq_partials writes sumsq_seg_blocks() partial sums of squares of
// x[0, n) (x 16-byte aligned); sumsq_finish reduces n partials in a fixed order to the
// L2 norm.  The train step reduces each layer's gradients as soon as they are final.
int sumsq_seg_blocks();
int sumsq_partials(const float* x, int64_t n, float* partials, cudaStream_t s);
// out[0] = sum of in[0 .. n) (fixed order), out[1 .. nout) = 0.
int sumsq_fold(const float* in, int n, float* out, int nout, cudaStream_t s);
int sumsq_finish(const float* partials, int n, float* out_norm, cudaStream_t s);
// The same reduction without the square root, in double (for a cross-rank sum),
// and the square root of that sum into a float.
int sumsq_finish_sq(const float* partials, int n, double* out_sq, cudaStream_t s);
int sqrt_to_float(const double* sq, float* out, cudaStream_t s);

// Multi-tensor AdamW over up to 4 contiguous segments of one parameter arena
// (crates/engine/src/cpu/adam.rs:95-132 per element).  The gradient scale is
// either `grad_scale` or, when `norm` is non-null, the train-step clip rule
// (full_model.rs:696-704): raw = *norm; scale = raw*gsc > clip ? clip/raw : gsc.
constexpr int kMaxAdamSegments = 72;  // 3 learning-rate groups, or one chunk per gradient segment (sharded)
struct AdamSegment {
  int64_t begin = 0, end = 0;  // element range in the arena
  float lr = 0.f, wd = 0.f;
  int write_bf16 = 0;  // also write the bf16 compute copy at the same offset
};
struct AdamArgs {
  float* param = nullptr;
  const float* grad = nullptr;
  float* m = nullptr;
  float* v = nullptr;
  __nv_bfloat16* param_bf16 = nullptr;
  AdamSegment seg[kMaxAdamSegments];
  int nseg = 0;
  float beta1 = 0.9f, beta2 = 0.95f, eps = 1e-8f, bc1 = 1.f, bc2 = 1.f;
  float grad_scale = 1.f;
  const float* norm = nullptr;
  float gsc = 1.f, clip = 0.f;
};
int adam_step(const AdamArgs& a, cudaStream_t s);

// Tensor-parallel residual: x_out = x + alpha * p (p = all-reduced bf16 partial
// of a row-parallel GEMM); with gamma, also xn = RMSNorm(x_out) and rms_inv.
int residual_rmsnorm_fwd(const float* x, const __nv_bfloat16* p, float alpha, const float* gamma, float* x_out,
                         __nv_bfloat16* xn, float* rms_inv, int M, int D, cudaStream_t s);
// Fill a [rows, cols] block (row stride dst_ld) with the N(0, std) stream of
// init_normal at global element indices gbase + r * gld + gcol0 + c, so a shard
// gets exactly the values of the same block of the full parameter arena.
int init_normal_block(float* dst, int64_t rows, int64_t cols, int64_t dst_ld, int64_t gbase, int64_t gld,
                      int64_t gcol0, uint64_t seed, float std, cudaStream_t s);

// Elementwise helpers.
int cast_bf16(const float* src, __nv_bfloat16* dst, int64_t n, cudaStream_t s);
// dst = bf16(scale * src)
int cast_bf16_scaled(const float* src, __nv_bfloat16* dst, int64_t n, float scale, cudaStream_t s);
int fill_f32(float* dst, int64_t n, float value, cudaStream_t s);
// Counter-based N(0, std) init: element i of a stream with the given seed.
int init_normal(float* dst, int64_t n, uint64_t seed, float std, cudaStream_t s);
// y = a * x (fp32 -> fp32), used for scaled copies
int scale_f32(const float* x, float* y, int64_t n, float a, cudaStream_t s);
// check all values finite: *flag = 1 if any NaN / Inf
int nonfinite_check(const float* x, int64_t n, int* flag, cudaStream_t s);

}  // namespace rt
