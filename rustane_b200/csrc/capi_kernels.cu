// Kernel-level C entry points: one launch of one kernel on caller-owned device
// buffers.  They exist so that each kernel can be checked on its own against
// the CPU oracle; the model-level API (rustane_cuda.h, rt_ctx_*) is built on
// the same launchers.
#include "kernels.h"
#include "rustane_cuda.h"

extern "C" {

RT_API int rt_kernel_gemm(const void* a, int64_t lda, int a_mn, const void* b, int64_t ldb, int b_mn, int M, int N,
                          int K, int epi, void* out, int64_t ldo, void* out2, int64_t ldo2, const void* aux,
                          int64_t ld_aux, float alpha, int beta, const float* rope_cos, const float* rope_sin,
                          int seq, int rope_cols, int n_half, int force_bn, int* dev_err, void* stream) {
  rt::GemmArgs g;
  g.a = a;
  g.lda = lda;
  g.a_mn = a_mn != 0;
  g.b = b;
  g.ldb = ldb;
  g.b_mn = b_mn != 0;
  g.M = M;
  g.N = N;
  g.K = K;
  g.epi = epi;
  g.out = out;
  g.ldo = ldo;
  g.out2 = out2;
  g.ldo2 = ldo2;
  g.aux = aux;
  g.ld_aux = ld_aux;
  g.alpha = alpha;
  g.beta = beta;
  g.rope_cos = rope_cos;
  g.rope_sin = rope_sin;
  g.seq = seq;
  g.rope_cols = rope_cols;
  g.n_half = n_half;
  g.force_bn = force_bn;
  g.err = dev_err;
  const int rc = rt::gemm_launch(g, static_cast<cudaStream_t>(stream));
  if (rc == 0) return RT_OK;
  if (rc == -1) return RT_ERR_SHAPE;
  return RT_ERR_CUDA;
}

}  // extern "C"

// ------------------------------------------------------------------ others
#include <cmath>

#include "attention.h"
#include "elementwise.h"

namespace {
inline int map_rc(int rc) { return rc == 0 ? RT_OK : (rc == -1 ? RT_ERR_SHAPE : RT_ERR_CUDA); }
inline cudaStream_t st(void* s) { return static_cast<cudaStream_t>(s); }
}  // namespace

extern "C" {

RT_API int rt_kernel_attention_fwd(const void* qkv, void* out, float* lse2, int batch, int seq, int heads,
                                   void* stream) {
  rt::AttnArgs a;
  a.batch = batch;
  a.S = seq;
  a.heads = heads;
  a.hd = 128;
  a.D = heads * 128;
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.ldq = 3 * a.D;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ldo = a.D;
  a.lse2 = lse2;
  return map_rc(rt::attn_forward(a, st(stream)));
}

RT_API int rt_kernel_attention_bwd(const void* qkv, const void* out, const float* lse2, const void* dout,
                                   float* dvec, void* dqkv, const float* rope_cos_b, const float* rope_sin_b,
                                   int batch, int seq, int heads, void* stream) {
  rt::AttnArgs a;
  a.batch = batch;
  a.S = seq;
  a.heads = heads;
  a.hd = 128;
  a.D = heads * 128;
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.ldq = 3 * a.D;
  a.out = const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(out));
  a.ldo = a.D;
  a.lse2 = const_cast<float*>(lse2);
  a.dout = static_cast<const __nv_bfloat16*>(dout);
  a.lddo = a.D;
  a.dvec = dvec;
  a.dqkv = static_cast<__nv_bfloat16*>(dqkv);
  a.lddq = 3 * a.D;
  a.rope_cos_b = rope_cos_b;
  a.rope_sin_b = rope_sin_b;
  return map_rc(rt::attn_backward(a, st(stream)));
}

RT_API int rt_kernel_attention_bwd_tc(const void* qkv, const void* out, const float* lse2, const void* dout,
                                      float* dvec, void* ds_scratch, void* dqkv, const float* rope_cos_b,
                                      const float* rope_sin_b, int batch, int seq, int heads, void* stream) {
  if (!qkv || !out || !lse2 || !dout || !dvec || !ds_scratch || !dqkv || !rope_cos_b || !rope_sin_b)
    return RT_ERR_ARG;
  rt::AttnArgs a;
  a.batch = batch;
  a.S = seq;
  a.heads = heads;
  a.hd = 128;
  a.D = heads * 128;
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.ldq = 3 * a.D;
  a.out = const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(out));
  a.ldo = a.D;
  a.lse2 = const_cast<float*>(lse2);
  a.dout = static_cast<const __nv_bfloat16*>(dout);
  a.lddo = a.D;
  a.dvec = dvec;
  a.ds_scratch = static_cast<__nv_bfloat16*>(ds_scratch);
  a.dqkv = static_cast<__nv_bfloat16*>(dqkv);
  a.lddq = 3 * a.D;
  a.rope_cos_b = rope_cos_b;
  a.rope_sin_b = rope_sin_b;
  return map_rc(rt::attn_backward_tc(a, st(stream)));
}

RT_API int64_t rt_kernel_attention_bwd_scratch_bytes(int batch, int seq, int heads) {
  if (batch <= 0 || seq <= 0 || heads <= 0) return 0;
  return static_cast<int64_t>(rt::attn_bwd_scratch_bytes(batch, seq, heads));
}

RT_API int rt_kernel_rmsnorm_fwd(const float* x, const float* gamma, void* out_bf16, float* rms_inv, int M, int D,
                                 void* stream) {
  return map_rc(rt::rmsnorm_fwd(x, gamma, static_cast<__nv_bfloat16*>(out_bf16), rms_inv, M, D, st(stream)));
}

RT_API int rt_kernel_rmsnorm_bwd_partials(int M) { return rt::rmsnorm_bwd_blocks(M); }

RT_API int rt_kernel_rmsnorm_bwd(const float* dy, const float* x, const float* gamma, const float* rms_inv,
                                 const float* resid, float* dx, void* dx_bf16, float bf16_scale, float* dgamma,
                                 int accumulate, float* partials, int M, int D, void* stream) {
  int rc = rt::rmsnorm_bwd(dy, x, gamma, rms_inv, resid, dx, static_cast<__nv_bfloat16*>(dx_bf16), bf16_scale,
                           partials, M, D, st(stream));
  if (rc) return map_rc(rc);
  return map_rc(rt::dgamma_reduce(partials, rt::rmsnorm_bwd_blocks(M), dgamma, D, accumulate, st(stream)));
}

RT_API int rt_kernel_embed_gather(const float* E, const uint32_t* tok, float* x, int M, int D, int V, int* dev_err,
                                  void* stream) {
  return map_rc(rt::embed_gather(E, tok, x, M, D, V, dev_err, st(stream)));
}

RT_API int rt_kernel_embed_scatter(const float* dx, const int32_t* perm, const int32_t* seg_start,
                                   const uint32_t* seg_tok, int nseg, float* dE, int D, void* stream) {
  return map_rc(rt::embed_scatter(dx, perm, seg_start, seg_tok, nseg, dE, D, st(stream)));
}

RT_API int rt_kernel_ce_fwd(const float* logits, const uint32_t* tgt, float* row_loss, float* row_lse, int M, int V,
                            float softcap, void* stream) {
  return map_rc(rt::ce_forward(logits, tgt, row_loss, row_lse, M, V, softcap, st(stream)));
}

RT_API int rt_kernel_ce_bwd(const float* logits, const float* row_lse, const uint32_t* tgt, void* dl_bf16, int M,
                            int V, float softcap, float scale, void* stream) {
  return map_rc(rt::ce_backward(logits, row_lse, tgt, static_cast<__nv_bfloat16*>(dl_bf16), M, V, softcap, scale,
                                st(stream)));
}

RT_API int rt_kernel_adam(float* param, const float* grad, float* m, float* v, void* param_bf16, int64_t n,
                          uint32_t t, float lr, float beta1, float beta2, float eps, float weight_decay,
                          float grad_scale, void* stream) {
  if (t == 0 || n % 4) return RT_ERR_ARG;
  rt::AdamArgs a;
  a.param = param;
  a.grad = grad;
  a.m = m;
  a.v = v;
  a.param_bf16 = static_cast<__nv_bfloat16*>(param_bf16);
  a.nseg = 1;
  a.seg[0] = {0, n, lr, weight_decay, param_bf16 ? 1 : 0};
  a.beta1 = beta1;
  a.beta2 = beta2;
  a.eps = eps;
  float p1 = 1.f, p2 = 1.f;
  for (uint32_t i = 0; i < t; ++i) {
    p1 *= beta1;
    p2 *= beta2;
  }
  a.bc1 = 1.0f / (1.0f - p1);
  a.bc2 = 1.0f / (1.0f - p2);
  a.grad_scale = grad_scale;
  return map_rc(rt::adam_step(a, st(stream)));
}

RT_API int rt_kernel_l2norm(const float* x, int64_t n, float* partials, float* out_norm, void* stream) {
  return map_rc(rt::sumsq_norm(x, n, partials, out_norm, st(stream)));
}

}  // extern "C"
