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
