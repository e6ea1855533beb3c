// ORACLE — TEST INFRASTRUCTURE ONLY.
//
// CPU fp32 restatement of rustane's language-model step (jackzampolin/rustane,
// crates/engine), used as the correctness checker for librustane_cuda.so and as
// the timed CPU baseline.  It is never linked into, called by, or shipped with
// the product path.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline may load it.
//
// Layouts follow the reference exactly: activations are channel-first [C, S]
// per sequence, weights row-major wq/wk/wv/wo [D, D], w1/w3/w2 [D, H], embed
// [V, D].  The ANE graphs of the reference (fp16 inside the ANE) are restated
// in fp32; the Accelerate sgemm is replaced by the host's cblas_sgemm
// (OpenBLAS, dlopen'ed), or by a plain OpenMP loop nest when none is found.
// Each function cites the reference file:line it follows.
#include <dlfcn.h>
#include <omp.h>
#include <stdint.h>
#include <string.h>

#include <cmath>
#include <string>
#include <vector>

#define OR_API extern "C" __attribute__((visibility("default")))

namespace {

// ------------------------------------------------------------------ BLAS
enum { kRowMajor = 101, kNoTrans = 111, kTrans = 112 };
typedef void (*sgemm32_t)(int, int, int, int, int, int, float, const float*, int, const float*, int, float, float*,
                          int);
typedef void (*sgemm64_t)(int, int, int, int64_t, int64_t, int64_t, float, const float*, int64_t, const float*,
                          int64_t, float, float*, int64_t);
typedef void (*setthreads_t)(int);

sgemm32_t g_sgemm32 = nullptr;
sgemm64_t g_sgemm64 = nullptr;
std::string g_blas_name = "builtin-omp";
int g_threads = 1;

void sgemm_builtin(bool ta, bool tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
                   const float* B, int64_t ldb, float beta, float* C, int64_t ldc) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < M; ++i) {
    std::vector<float> acc(N, 0.f);
    for (int64_t k = 0; k < K; ++k) {
      const float a = ta ? A[k * lda + i] : A[i * lda + k];
      if (a == 0.f) continue;
      if (!tb) {
        const float* brow = B + k * ldb;
        for (int64_t j = 0; j < N; ++j) acc[j] += a * brow[j];
      } else {
        for (int64_t j = 0; j < N; ++j) acc[j] += a * B[j * ldb + k];
      }
    }
    float* crow = C + i * ldc;
    for (int64_t j = 0; j < N; ++j) crow[j] = alpha * acc[j] + (beta == 0.f ? 0.f : beta * crow[j]);
  }
}

// Row-major C = alpha * op(A) op(B) + beta * C (cblas_sgemm semantics,
// crates/engine/src/cpu/vdsp.rs:128-136).
void sgemm(bool ta, bool tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
           const float* B, int64_t ldb, float beta, float* C, int64_t ldc) {
  if (M == 0 || N == 0) return;
  if (g_sgemm64) {
    g_sgemm64(kRowMajor, ta ? kTrans : kNoTrans, tb ? kTrans : kNoTrans, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
  } else if (g_sgemm32) {
    g_sgemm32(kRowMajor, ta ? kTrans : kNoTrans, tb ? kTrans : kNoTrans, int(M), int(N), int(K), alpha, A, int(lda),
              B, int(ldb), beta, C, int(ldc));
  } else {
    sgemm_builtin(ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
  }
}

// sgemm_at: C[m,n] += A[m,k] B[n,k]  (beta = 1; crates/engine/src/cpu/vdsp.rs:287-302)
void sgemm_at(const float* a, int64_t m, int64_t k, const float* b, int64_t n, float* c) {
  sgemm(false, true, m, n, k, 1.f, a, k, b, k, 1.f, c, n);
}

// vDSP_mtrans: c[n_cols x m_rows] = transpose(a[m x n])  (cpu/vdsp.rs:245-251)
void mtrans(const float* a, int64_t m, int64_t n, float* c) {
#pragma omp parallel for schedule(static) if (m * n > 65536)
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) c[j * m + i] = a[i * n + j];
}

constexpr float kRmsEps = 1e-5f;  // crates/engine/src/cpu/rmsnorm.rs:10

}  // namespace

// ------------------------------------------------------------ public types
struct OrConfig {  // crates/engine/src/model.rs:5-17
  int32_t dim, hidden, heads, kv_heads, hd, seq, nlayers, vocab, q_dim, kv_dim, gqa_ratio;
};
struct OrLayer {  // crates/engine/src/layer.rs:16-26 (LayerWeights / LayerGrads / moments)
  float *wq, *wk, *wv, *wo, *w1, *w3, *w2, *gamma1, *gamma2;
};
struct OrModel {  // crates/engine/src/full_model.rs:13-31
  float* embed;
  float* gamma_final;
  OrLayer* layers;
};
struct OrTrainConfig {  // crates/engine/src/full_model.rs:34-70
  float max_lr, min_lr_frac;
  uint32_t warmup_steps, total_steps;
  float beta1, beta2, eps, weight_decay, matrix_lr_scale, embed_lr_scale, loss_scale;
  uint32_t accum_steps;
  float grad_clip, softcap;
};

// Forward cache of one layer for one sequence (crates/engine/src/layer.rs:42-57).
struct OrCache {
  std::vector<float> x, xnorm, rms_inv1, q_rope, k_rope, v, attn_out, o_out, x2, x2norm, rms_inv2, h1, h3, gate;
};
struct OrSeq {  // model-level forward workspace of one sequence (full_model.rs:148-162)
  std::vector<OrCache> caches;
  std::vector<float> x_prenorm, x_final, rms_inv_final, logits, logits_capped, dlogits;
};
struct OrWs {
  OrConfig cfg;
  int batch = 0;
  std::vector<OrSeq> seqs;
  std::vector<float> rope_cos_fwd, rope_sin_fwd;  // [seq][hd] (kernels/sdpa_fwd.rs:18-33)
  std::vector<float> rope_cos_bwd, rope_sin_bwd;  // [pairs][seq] (layer.rs:197-217)
};

// ======================================================= library control
OR_API int or_init(const char* blas_path, int threads) {
  g_threads = threads > 0 ? threads : omp_get_max_threads();
  omp_set_num_threads(g_threads);
  g_sgemm32 = nullptr;
  g_sgemm64 = nullptr;
  g_blas_name = "builtin-omp";
  if (blas_path && *blas_path) {
    void* h = dlopen(blas_path, RTLD_NOW | RTLD_LOCAL);
    if (!h) return -1;
    if (void* f = dlsym(h, "scipy_cblas_sgemm64_")) {
      g_sgemm64 = reinterpret_cast<sgemm64_t>(f);
      if (void* st = dlsym(h, "scipy_openblas_set_num_threads64_")) reinterpret_cast<setthreads_t>(st)(g_threads);
    } else if (void* f2 = dlsym(h, "cblas_sgemm")) {
      g_sgemm32 = reinterpret_cast<sgemm32_t>(f2);
      if (void* st = dlsym(h, "openblas_set_num_threads")) reinterpret_cast<setthreads_t>(st)(g_threads);
    } else {
      return -2;
    }
    g_blas_name = blas_path;
  }
  return 0;
}
OR_API const char* or_blas_name() { return g_blas_name.c_str(); }
OR_API int or_threads() { return g_threads; }

OR_API void or_sgemm(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
                     const float* B, int64_t ldb, float beta, float* C, int64_t ldc) {
  sgemm(ta != 0, tb != 0, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}

// =========================================================== init (LCG)
// random_vec: seed = 42 + n, 64-bit LCG, r = (seed>>32)/u32::MAX * 2 - 1
// (crates/engine/src/layer.rs:404-413, full_model.rs:648-657).
OR_API void or_random_vec(float* out, int64_t n, float scale) {
  uint64_t seed = 42ull + static_cast<uint64_t>(n);
  for (int64_t i = 0; i < n; ++i) {
    seed = seed * 6364136223846793005ull + 1442695040888963407ull;
    const float r = (static_cast<float>(static_cast<uint32_t>(seed >> 32)) / static_cast<float>(UINT32_MAX)) * 2.0f - 1.0f;
    out[i] = r * scale;
  }
}

// =============================================================== cpu ops
// RMSNorm single vector (crates/engine/src/cpu/rmsnorm.rs:15-35); returns rms_inv.
OR_API float or_rmsnorm_forward(const float* x, const float* gamma, float* out, int dim) {
  float ss = 0.f;
  for (int i = 0; i < dim; ++i) ss += x[i] * x[i];
  const float mean_sq = ss / static_cast<float>(dim);
  const float rms_inv = 1.0f / std::sqrt(mean_sq + kRmsEps);
  for (int i = 0; i < dim; ++i) out[i] = x[i] * rms_inv * gamma[i];
  return rms_inv;
}

// Single-vector backward: dx = rms_inv * (dy*g - x_hat * mean(dy*g*x_hat)); dgamma += dy*x_hat
// (crates/engine/src/cpu/rmsnorm.rs header formula and :37-75).
OR_API void or_rmsnorm_backward(const float* dy, const float* x, const float* gamma, float rms_inv, float* dx,
                                float* dgamma, int dim) {
  float dot = 0.f;
  for (int i = 0; i < dim; ++i) {
    const float xh = x[i] * rms_inv;
    dot += dy[i] * gamma[i] * xh;
    dgamma[i] += dy[i] * xh;
  }
  dot /= static_cast<float>(dim);
  for (int i = 0; i < dim; ++i) dx[i] = rms_inv * (dy[i] * gamma[i] - x[i] * rms_inv * dot);
}

// Channel-first forward on [dim, seq] (crates/engine/src/cpu/rmsnorm.rs:149-183).
OR_API void or_rmsnorm_forward_cf(const float* x, const float* gamma, float* out, float* rms_inv, int dim, int seq) {
  for (int s = 0; s < seq; ++s) rms_inv[s] = 0.f;
  for (int d = 0; d < dim; ++d) {
    const float* row = x + static_cast<int64_t>(d) * seq;
    for (int s = 0; s < seq; ++s) rms_inv[s] += row[s] * row[s];
  }
  const float inv_dim = 1.0f / static_cast<float>(dim);
  for (int s = 0; s < seq; ++s) rms_inv[s] = 1.0f / std::sqrt(rms_inv[s] * inv_dim + kRmsEps);
  for (int d = 0; d < dim; ++d) {
    const float* xr = x + static_cast<int64_t>(d) * seq;
    float* orow = out + static_cast<int64_t>(d) * seq;
    const float g = gamma[d];
    for (int s = 0; s < seq; ++s) orow[s] = xr[s] * rms_inv[s] * g;
  }
}

// Channel-first backward (crates/engine/src/cpu/rmsnorm.rs:190-238); dgamma accumulates.
OR_API void or_rmsnorm_backward_cf(const float* dy, const float* x, const float* gamma, const float* rms_inv,
                                   float* dx, float* dgamma, int dim, int seq) {
  std::vector<float> dot(seq, 0.f);
  for (int d = 0; d < dim; ++d) {
    const float* dyr = dy + static_cast<int64_t>(d) * seq;
    const float* xr = x + static_cast<int64_t>(d) * seq;
    float* dxr = dx + static_cast<int64_t>(d) * seq;
    const float g = gamma[d];
    float dg = 0.f;
    for (int s = 0; s < seq; ++s) {
      const float xh = xr[s] * rms_inv[s];
      dxr[s] = xh;
      dg += dyr[s] * xh;
      dot[s] += dyr[s] * g * xh;
    }
    dgamma[d] += dg;
  }
  const float inv_dim = 1.0f / static_cast<float>(dim);
  for (int s = 0; s < seq; ++s) dot[s] *= inv_dim;
  for (int d = 0; d < dim; ++d) {
    const float* dyr = dy + static_cast<int64_t>(d) * seq;
    float* dxr = dx + static_cast<int64_t>(d) * seq;
    const float g = gamma[d];
    for (int s = 0; s < seq; ++s) {
      const float xh = dxr[s];
      dxr[s] = rms_inv[s] * (dyr[s] * g - xh * dot[s]);
    }
  }
}

// Cross-entropy single token (crates/engine/src/cpu/cross_entropy.rs:13-38); writes log-softmax.
OR_API float or_ce_forward(const float* logits, int vocab, int target, float* log_sm) {
  float mx = -INFINITY;
  for (int i = 0; i < vocab; ++i) mx = logits[i] > mx ? logits[i] : mx;
  float sum = 0.f;
  for (int i = 0; i < vocab; ++i) sum += std::exp(logits[i] - mx);
  const float lse = std::log(sum);
  for (int i = 0; i < vocab; ++i) log_sm[i] = (logits[i] - mx) - lse;
  return -log_sm[target];
}
// d_logits = softmax - onehot (cross_entropy.rs:43-53)
OR_API void or_ce_backward(const float* log_sm, int vocab, int target, float* d_logits) {
  for (int i = 0; i < vocab; ++i) d_logits[i] = std::exp(log_sm[i]);
  d_logits[target] -= 1.0f;
}
// Batched forward+backward (cross_entropy.rs:58-96): returns the summed loss,
// dlogits = (softmax - onehot) * inv_seq.
OR_API float or_ce_forward_backward_batch(const float* logits, const uint32_t* targets, int seq, int vocab,
                                          float* dlogits, float inv_seq) {
  std::vector<float> losses(seq);
#pragma omp parallel for schedule(static)
  for (int s = 0; s < seq; ++s) {
    const float* row = logits + static_cast<int64_t>(s) * vocab;
    float* d = dlogits + static_cast<int64_t>(s) * vocab;
    float mx = -INFINITY;
    for (int i = 0; i < vocab; ++i) mx = row[i] > mx ? row[i] : mx;
    float sum = 0.f;
    for (int i = 0; i < vocab; ++i) {
      d[i] = std::exp(row[i] - mx);
      sum += d[i];
    }
    const int t = static_cast<int>(targets[s]);
    losses[s] = -((row[t] - mx) - std::log(sum));
    const float r = 1.0f / sum;
    for (int i = 0; i < vocab; ++i) d[i] = d[i] * r;
    d[t] -= 1.0f;
    for (int i = 0; i < vocab; ++i) d[i] *= inv_seq;
  }
  float total = 0.f;
  for (int s = 0; s < seq; ++s) total += losses[s];
  return total;
}

// AdamW (crates/engine/src/cpu/adam.rs:37-85): unfused vDSP semantics.
OR_API void or_adam_step(float* param, const float* grad, float* m, float* v, int64_t n, uint32_t t, float lr,
                         float beta1, float beta2, float eps, float weight_decay) {
  const float bc1 = 1.0f / (1.0f - std::pow(beta1, static_cast<float>(t)));
  const float bc2 = 1.0f / (1.0f - std::pow(beta2, static_cast<float>(t)));
  for (int64_t i = 0; i < n; ++i) {
    const float tmp = m[i] * beta1;
    m[i] = grad[i] * (1.0f - beta1) + tmp;
    const float g2 = grad[i] * grad[i];
    const float tmp2 = v[i] * beta2;
    v[i] = g2 * (1.0f - beta2) + tmp2;
  }
  for (int64_t i = 0; i < n; ++i) {
    const float mh = m[i] * bc1;
    const float vh = v[i] * bc2;
    const float update = mh / (std::sqrt(vh) + eps);
    param[i] -= lr * (update + weight_decay * param[i]);
  }
}

// Fused AdamW with inline grad scaling (crates/engine/src/cpu/adam.rs:95-132).
OR_API void or_adam_step_fused(float* param, const float* grad, float* m, float* v, int64_t n, uint32_t t, float lr,
                               float beta1, float beta2, float eps, float weight_decay, float grad_scale) {
  float p1 = 1.f, p2 = 1.f;  // powi(t) by repeated multiplication
  for (uint32_t i = 0; i < t; ++i) {
    p1 *= beta1;
    p2 *= beta2;
  }
  const float bc1 = 1.0f / (1.0f - p1);
  const float bc2 = 1.0f / (1.0f - p2);
  const float omb1 = 1.0f - beta1, omb2 = 1.0f - beta2;
#pragma omp parallel for schedule(static) if (n > 65536)
  for (int64_t i = 0; i < n; ++i) {
    const float g = grad[i] * grad_scale;
    const float mi = beta1 * m[i] + omb1 * g;
    const float vi = beta2 * v[i] + omb2 * g * g;
    m[i] = mi;
    v[i] = vi;
    const float mh = mi * bc1;
    const float vh = vi * bc2;
    const float update = mh / (std::sqrt(vh) + eps);
    param[i] -= lr * (update + weight_decay * param[i]);
  }
}

// Embedding (crates/engine/src/cpu/embedding.rs:8-44).
OR_API void or_embedding_forward(const float* table, int dim, const uint32_t* ids, int n, float* out) {
  for (int s = 0; s < n; ++s) memcpy(out + static_cast<int64_t>(s) * dim, table + static_cast<int64_t>(ids[s]) * dim, sizeof(float) * dim);
}
OR_API void or_embedding_backward(const float* d_out, int dim, const uint32_t* ids, int n, float* d_table) {
  for (int s = 0; s < n; ++s) {
    float* row = d_table + static_cast<int64_t>(ids[s]) * dim;
    for (int d = 0; d < dim; ++d) row[d] += d_out[static_cast<int64_t>(s) * dim + d];
  }
}
OR_API void or_embedding_backward_cf(const float* d_out, int dim, const uint32_t* ids, int seq, float* d_table) {
  for (int s = 0; s < seq; ++s) {
    float* row = d_table + static_cast<int64_t>(ids[s]) * dim;
    for (int d = 0; d < dim; ++d) row[d] += d_out[static_cast<int64_t>(d) * seq + s];
  }
}

// SiLU (crates/engine/src/cpu/silu.rs:8-45).
OR_API void or_silu_forward(const float* x, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = x[i] * (1.0f / (1.0f + std::exp(-x[i])));
}
OR_API void or_silu_backward(const float* dy, const float* x, float* dx, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const float sig = 1.0f / (1.0f + std::exp(-x[i]));
    dx[i] = dy[i] * (sig * (1.0f + x[i] * (1.0f - sig)));
  }
}

// ========================================================== model pieces
namespace {

float alpha_of(const OrConfig& c) { return 1.0f / std::sqrt(2.0f * static_cast<float>(c.nlayers)); }

void rope_tables(OrWs& ws) {
  const int S = ws.cfg.seq, hd = ws.cfg.hd, pairs = hd / 2;
  ws.rope_cos_fwd.assign(static_cast<size_t>(S) * hd, 0.f);
  ws.rope_sin_fwd.assign(static_cast<size_t>(S) * hd, 0.f);
  for (int p = 0; p < S; ++p)
    for (int i = 0; i < pairs; ++i) {  // kernels/sdpa_fwd.rs:18-33
      const float theta = static_cast<float>(p) / std::pow(10000.0f, 2.0f * static_cast<float>(i) / static_cast<float>(hd));
      const float c = std::cos(theta), s = std::sin(theta);
      ws.rope_cos_fwd[p * hd + 2 * i] = c;
      ws.rope_cos_fwd[p * hd + 2 * i + 1] = c;
      ws.rope_sin_fwd[p * hd + 2 * i] = s;
      ws.rope_sin_fwd[p * hd + 2 * i + 1] = s;
    }
  ws.rope_cos_bwd.assign(static_cast<size_t>(pairs) * S, 0.f);
  ws.rope_sin_bwd.assign(static_cast<size_t>(pairs) * S, 0.f);
  for (int i = 0; i < pairs; ++i) {  // layer.rs:203-216
    const float freq = 1.0f / std::pow(10000.0f, 2.0f * static_cast<float>(i) / static_cast<float>(hd));
    for (int p = 0; p < S; ++p) {
      const float theta = static_cast<float>(p) * freq;
      ws.rope_cos_bwd[i * S + p] = std::cos(theta);
      ws.rope_sin_bwd[i * S + p] = std::sin(theta);
    }
  }
}

void alloc_cache(const OrConfig& c, OrCache& k) {
  const size_t DS = size_t(c.dim) * c.seq, QS = size_t(c.q_dim) * c.seq, KS = size_t(c.kv_dim) * c.seq,
               HS = size_t(c.hidden) * c.seq;
  k.x.assign(DS, 0.f);
  k.xnorm.assign(DS, 0.f);
  k.rms_inv1.assign(c.seq, 0.f);
  k.q_rope.assign(QS, 0.f);
  k.k_rope.assign(KS, 0.f);
  k.v.assign(KS, 0.f);
  k.attn_out.assign(QS, 0.f);
  k.o_out.assign(DS, 0.f);
  k.x2.assign(DS, 0.f);
  k.x2norm.assign(DS, 0.f);
  k.rms_inv2.assign(c.seq, 0.f);
  k.h1.assign(HS, 0.f);
  k.h3.assign(HS, 0.f);
  k.gate.assign(HS, 0.f);
}

// Attention probabilities P[t][t2] for one head: softmax(q^T k * scale + mask),
// mask = -65504 where t2 > t (kernels/sdpa_fwd.rs:35-46, 130-142).
void attn_probs(const float* qh, const float* kh, int S, int hd, float* P) {
  const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
  sgemm(true, false, S, S, hd, 1.f, qh, S, kh, S, 0.f, P, S);  // scores[t][t2] = sum_e q[e][t] k[e][t2]
  for (int t = 0; t < S; ++t) {
    float* row = P + static_cast<int64_t>(t) * S;
    float mx = -INFINITY;
    for (int t2 = 0; t2 < S; ++t2) {
      row[t2] = row[t2] * scale + (t2 > t ? -65504.0f : 0.0f);
      mx = row[t2] > mx ? row[t2] : mx;
    }
    float sum = 0.f;
    for (int t2 = 0; t2 < S; ++t2) {
      row[t2] = std::exp(row[t2] - mx);
      sum += row[t2];
    }
    const float r = 1.0f / sum;
    for (int t2 = 0; t2 < S; ++t2) row[t2] *= r;
  }
}

// One transformer layer forward, channel-first [D, S]
// (crates/engine/src/layer.rs:443-548 with kernels/sdpa_fwd.rs, dyn_matmul.rs, ffn_fused.rs).
void layer_forward(const OrConfig& c, const OrWs& ws, const OrLayer& w, const float* x, OrCache& k, float* x_next) {
  const int D = c.dim, S = c.seq, Q = c.q_dim, KV = c.kv_dim, H = c.hidden, nh = c.heads, hd = c.hd;
  const float alpha = alpha_of(c);
  memcpy(k.x.data(), x, sizeof(float) * D * S);
  or_rmsnorm_forward_cf(x, w.gamma1, k.xnorm.data(), k.rms_inv1.data(), D, S);
  // QKV projection: Q[q][s] = sum_d Wq[d][q] xnorm[d][s]
  sgemm(true, false, Q, S, D, 1.f, w.wq, Q, k.xnorm.data(), S, 0.f, k.q_rope.data(), S);
  sgemm(true, false, KV, S, D, 1.f, w.wk, KV, k.xnorm.data(), S, 0.f, k.k_rope.data(), S);
  sgemm(true, false, KV, S, D, 1.f, w.wv, KV, k.xnorm.data(), S, 0.f, k.v.data(), S);
  // RoPE: out = x*cos + rotate_half(x)*sin with rotate_half = [-odd, even] (sdpa_fwd.rs:100-128)
  for (float* buf : {k.q_rope.data(), k.k_rope.data()}) {
#pragma omp parallel for schedule(static)
    for (int h = 0; h < nh; ++h)
      for (int i = 0; i < hd / 2; ++i) {
        float* r0 = buf + static_cast<int64_t>(h * hd + 2 * i) * S;
        float* r1 = buf + static_cast<int64_t>(h * hd + 2 * i + 1) * S;
        for (int p = 0; p < S; ++p) {
          const float cs = ws.rope_cos_fwd[p * hd + 2 * i], sn = ws.rope_sin_fwd[p * hd + 2 * i];
          const float a = r0[p], b = r1[p];
          r0[p] = a * cs + (-b) * sn;
          r1[p] = b * cs + a * sn;
        }
      }
  }
  // attention per head
#pragma omp parallel
  {
    std::vector<float> P(static_cast<size_t>(S) * S);
#pragma omp for schedule(static)
    for (int h = 0; h < nh; ++h) {
      const float* qh = k.q_rope.data() + static_cast<int64_t>(h) * hd * S;
      const float* kh = k.k_rope.data() + static_cast<int64_t>(h) * hd * S;
      const float* vh = k.v.data() + static_cast<int64_t>(h) * hd * S;
      float* oh = k.attn_out.data() + static_cast<int64_t>(h) * hd * S;
      attn_probs(qh, kh, S, hd, P.data());
      sgemm(false, true, hd, S, S, 1.f, vh, S, P.data(), S, 0.f, oh, S);  // o[e][t] = sum_t2 v[e][t2] P[t][t2]
    }
  }
  // woFwd: o[d][s] = sum_q Wo[q][d] attn[q][s]   (dyn_matmul.rs:15-46)
  sgemm(true, false, D, S, Q, 1.f, w.wo, D, k.attn_out.data(), S, 0.f, k.o_out.data(), S);
  // x2 = o*alpha + x   (layer.rs:497-498, vsma)
  for (int64_t i = 0; i < int64_t(D) * S; ++i) k.x2[i] = k.o_out[i] * alpha + x[i];
  or_rmsnorm_forward_cf(k.x2.data(), w.gamma2, k.x2norm.data(), k.rms_inv2.data(), D, S);
  // ffnFused (ffn_fused.rs:22-83)
  sgemm(true, false, H, S, D, 1.f, w.w1, H, k.x2norm.data(), S, 0.f, k.h1.data(), S);
  sgemm(true, false, H, S, D, 1.f, w.w3, H, k.x2norm.data(), S, 0.f, k.h3.data(), S);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < int64_t(H) * S; ++i) {
    const float h1 = k.h1[i];
    const float sig = 1.0f / (1.0f + std::exp(-h1));
    k.gate[i] = (h1 * sig) * k.h3[i];
  }
  std::vector<float> ffn(static_cast<size_t>(D) * S);
  sgemm(false, false, D, S, H, 1.f, w.w2, H, k.gate.data(), S, 0.f, ffn.data(), S);  // gate @ W2^T
  for (int64_t i = 0; i < int64_t(D) * S; ++i) x_next[i] = k.x2[i] + ffn[i] * alpha;
}

void rope_backward(const OrWs& ws, float* dx, int heads, int hd, int S) {  // layer.rs:1880-1897
#pragma omp parallel for schedule(static)
  for (int h = 0; h < heads; ++h)
    for (int i = 0; i < hd / 2; ++i) {
      float* r0 = dx + static_cast<int64_t>(h * hd + 2 * i) * S;
      float* r1 = dx + static_cast<int64_t>(h * hd + 2 * i + 1) * S;
      for (int p = 0; p < S; ++p) {
        const float c = ws.rope_cos_bwd[i * S + p], s = ws.rope_sin_bwd[i * S + p];
        const float d0 = r0[p], d1 = r1[p];
        r0[p] = c * d0 + s * d1;
        r1[p] = -s * d0 + c * d1;
      }
    }
}

// Layer backward (crates/engine/src/layer.rs:1606-1858); grads accumulate.
void layer_backward(const OrConfig& c, const OrWs& ws, const OrLayer& w, const OrCache& k, const float* dy,
                    OrLayer& g, float* dx_out) {
  const int D = c.dim, S = c.seq, Q = c.q_dim, KV = c.kv_dim, H = c.hidden, nh = c.heads, hd = c.hd;
  const float alpha = alpha_of(c);
  const int64_t DS = int64_t(D) * S, HS = int64_t(H) * S, QS = int64_t(Q) * S;
  std::vector<float> dffn(DS), dsilu(HS), dh1(HS), dh3(HS), dx_ffn(DS), dx2(DS), dx2s(DS), da(QS);
  // 1. dffn = alpha * dy
  for (int64_t i = 0; i < DS; ++i) dffn[i] = dy[i] * alpha;
  // 2. ffnBwdW2t: dsilu[h][s] = sum_d W2[d][h] dffn[d][s]
  sgemm(true, false, H, S, D, 1.f, w.w2, H, dffn.data(), S, 0.f, dsilu.data(), S);
  // 3. SiLU backward (layer.rs:1643-1667)
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < HS; ++i) {
    const float sig = 1.0f / (1.0f + std::exp(-k.h1[i]));
    const float silu_val = k.h1[i] * sig;
    const float silu_deriv = sig * (1.0f + k.h1[i] * (1.0f - sig));
    dh3[i] = dsilu[i] * silu_val;
    dh1[i] = dsilu[i] * k.h3[i] * silu_deriv;
  }
  // 4-5. ffnBwdW13t: dx_ffn[d][s] = sum_h W1[d][h] dh1[h][s] + W3[d][h] dh3[h][s]; dW3 += x2norm dh3^T
  sgemm(false, false, D, S, H, 1.f, w.w1, H, dh1.data(), S, 0.f, dx_ffn.data(), S);
  sgemm(false, false, D, S, H, 1.f, w.w3, H, dh3.data(), S, 1.f, dx_ffn.data(), S);
  sgemm_at(k.x2norm.data(), D, S, dh3.data(), H, g.w3);
  // 6. RMSNorm2 backward + residual
  or_rmsnorm_backward_cf(dx_ffn.data(), k.x2.data(), w.gamma2, k.rms_inv2.data(), dx2.data(), g.gamma2, D, S);
  for (int64_t i = 0; i < DS; ++i) dx2[i] = dx2[i] + dy[i];
  // 7. wotBwd: da[q][s] = sum_d Wo[q][d] dx2s[d][s]
  for (int64_t i = 0; i < DS; ++i) dx2s[i] = dx2[i] * alpha;
  sgemm(false, false, Q, S, D, 1.f, w.wo, D, dx2s.data(), S, 0.f, da.data(), S);
  // 9. dWo += attn dx2s^T ; dW2 += dffn gate^T
  sgemm_at(k.attn_out.data(), Q, S, dx2s.data(), D, g.wo);
  sgemm_at(dffn.data(), D, S, k.gate.data(), H, g.w2);
  // 8-10. SDPA backward per head (kernels/sdpa_bwd.rs:44-162)
  std::vector<float> dq(QS), dk(int64_t(KV) * S), dv(int64_t(KV) * S);
  const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
#pragma omp parallel
  {
    std::vector<float> P(static_cast<size_t>(S) * S), dP(static_cast<size_t>(S) * S);
#pragma omp for schedule(static)
    for (int h = 0; h < nh; ++h) {
      const int64_t off = static_cast<int64_t>(h) * hd * S;
      const float* qh = k.q_rope.data() + off;
      const float* kh = k.k_rope.data() + off;
      const float* vh = k.v.data() + off;
      const float* dah = da.data() + off;
      attn_probs(qh, kh, S, hd, P.data());
      // dV[e][t2] = sum_t da[e][t] P[t][t2]
      sgemm(false, false, hd, S, S, 1.f, dah, S, P.data(), S, 0.f, dv.data() + off, S);
      // dP[t][t2] = sum_e da[e][t] v[e][t2]
      sgemm(true, false, S, S, hd, 1.f, dah, S, vh, S, 0.f, dP.data(), S);
      // dS = P * (dP - sum_t2 P*dP) * scale
      for (int t = 0; t < S; ++t) {
        float* pr = P.data() + static_cast<int64_t>(t) * S;
        float* dr = dP.data() + static_cast<int64_t>(t) * S;
        float sp = 0.f;
        for (int t2 = 0; t2 < S; ++t2) sp += pr[t2] * dr[t2];
        for (int t2 = 0; t2 < S; ++t2) dr[t2] = pr[t2] * (dr[t2] - sp) * scale;
      }
      // dQ[e][t] = sum_t2 k[e][t2] dS[t][t2] ; dK[e][t2] = sum_t q[e][t] dS[t][t2]
      sgemm(false, true, hd, S, S, 1.f, kh, S, dP.data(), S, 0.f, dq.data() + off, S);
      sgemm(false, false, hd, S, S, 1.f, qh, S, dP.data(), S, 0.f, dk.data() + off, S);
    }
  }
  // dW1 += x2norm dh1^T   (layer.rs:1787)
  sgemm_at(k.x2norm.data(), D, S, dh1.data(), H, g.w1);
  // 11. RoPE backward
  rope_backward(ws, dq.data(), nh, hd, S);
  rope_backward(ws, dk.data(), nh, hd, S);
  // 13. qBwd + kvBwd: dx[d][s] = sum_q Wq[d][q] dq[q][s] + Wk dk + Wv dv ; dWq/dWk/dWv
  std::vector<float> dx_attn(DS), dx_kv(DS), dx_merged(DS), dx_rms1(DS);
  sgemm(false, false, D, S, Q, 1.f, w.wq, Q, dq.data(), S, 0.f, dx_attn.data(), S);
  sgemm(false, false, D, S, KV, 1.f, w.wk, KV, dk.data(), S, 0.f, dx_kv.data(), S);
  sgemm(false, false, D, S, KV, 1.f, w.wv, KV, dv.data(), S, 1.f, dx_kv.data(), S);
  sgemm_at(k.xnorm.data(), D, S, dq.data(), Q, g.wq);
  sgemm_at(k.xnorm.data(), D, S, dk.data(), KV, g.wk);
  sgemm_at(k.xnorm.data(), D, S, dv.data(), KV, g.wv);
  // 15-16. merge + RMSNorm1 backward + residual
  for (int64_t i = 0; i < DS; ++i) dx_merged[i] = dx_attn[i] + dx_kv[i];
  or_rmsnorm_backward_cf(dx_merged.data(), k.x.data(), w.gamma1, k.rms_inv1.data(), dx_rms1.data(), g.gamma1, D, S);
  for (int64_t i = 0; i < DS; ++i) dx_out[i] = dx_rms1[i] + dx2[i];
}

}  // namespace

// ======================================================= model-level API
OR_API OrWs* or_ws_create(const OrConfig* cfg, int batch) {
  OrWs* ws = new OrWs();
  ws->cfg = *cfg;
  ws->batch = batch;
  ws->seqs.resize(batch);
  const size_t DS = size_t(cfg->dim) * cfg->seq, SV = size_t(cfg->seq) * cfg->vocab;
  for (auto& sq : ws->seqs) {
    sq.caches.resize(cfg->nlayers);
    for (auto& k : sq.caches) alloc_cache(*cfg, k);
    sq.x_prenorm.assign(DS, 0.f);
    sq.x_final.assign(DS, 0.f);
    sq.rms_inv_final.assign(cfg->seq, 0.f);
    sq.logits.assign(SV, 0.f);
    sq.dlogits.assign(SV, 0.f);
  }
  rope_tables(*ws);
  return ws;
}
OR_API void or_ws_destroy(OrWs* ws) { delete ws; }

// Rope tables as the reference builds them: forward [seq][hd], backward [hd/2][seq].
OR_API void or_rope_tables(const OrWs* ws, float* cos_fwd, float* sin_fwd, float* cos_bwd, float* sin_bwd) {
  if (cos_fwd) memcpy(cos_fwd, ws->rope_cos_fwd.data(), ws->rope_cos_fwd.size() * sizeof(float));
  if (sin_fwd) memcpy(sin_fwd, ws->rope_sin_fwd.data(), ws->rope_sin_fwd.size() * sizeof(float));
  if (cos_bwd) memcpy(cos_bwd, ws->rope_cos_bwd.data(), ws->rope_cos_bwd.size() * sizeof(float));
  if (sin_bwd) memcpy(sin_bwd, ws->rope_sin_bwd.data(), ws->rope_sin_bwd.size() * sizeof(float));
}

// Forward of `batch` sequences (full_model::forward_ws, full_model.rs:187-247).
// Returns the mean of the per-sequence losses (each = summed CE / seq).
// logits_out [batch*seq*vocab] and per_token_loss [batch*seq] are optional.
OR_API int or_forward(const OrConfig* cfg, const OrModel* w, const uint32_t* tokens, const uint32_t* targets,
                      int batch, float softcap, OrWs* ws, float* loss_out, float* logits_out, float* per_token_loss) {
  if (batch > ws->batch) return -1;
  const int D = cfg->dim, S = cfg->seq, V = cfg->vocab;
  for (int i = 0; i < batch * S; ++i)
    if (tokens[i] >= uint32_t(V) || targets[i] >= uint32_t(V)) return -5;
  float total = 0.f;
  std::vector<float> x_row(size_t(S) * D), x(size_t(D) * S), x_next(size_t(D) * S), xf_row(size_t(S) * D);
  for (int b = 0; b < batch; ++b) {
    OrSeq& sq = ws->seqs[b];
    const uint32_t* tok = tokens + size_t(b) * S;
    const uint32_t* tgt = targets + size_t(b) * S;
    or_embedding_forward(w->embed, D, tok, S, x_row.data());
    mtrans(x_row.data(), S, D, x.data());
    for (int l = 0; l < cfg->nlayers; ++l) {
      layer_forward(*cfg, *ws, w->layers[l], x.data(), sq.caches[l], x_next.data());
      std::swap(x, x_next);
    }
    sq.x_prenorm = x;
    or_rmsnorm_forward_cf(sq.x_prenorm.data(), w->gamma_final, sq.x_final.data(), sq.rms_inv_final.data(), D, S);
    mtrans(sq.x_final.data(), D, S, xf_row.data());
    std::fill(sq.logits.begin(), sq.logits.end(), 0.f);
    sgemm_at(xf_row.data(), S, D, w->embed, V, sq.logits.data());
    if (softcap > 0.f) {  // full_model.rs:232-239
      sq.logits_capped.assign(sq.logits.size(), 0.f);
      for (size_t i = 0; i < sq.logits.size(); ++i) {
        sq.logits[i] *= 1.0f / softcap;
        sq.logits_capped[i] = std::tanh(sq.logits[i]);
        sq.logits[i] = sq.logits_capped[i] * softcap;
      }
    }
    if (logits_out) memcpy(logits_out + size_t(b) * S * V, sq.logits.data(), sizeof(float) * S * V);
    if (per_token_loss) {  // forward_losses (full_model.rs:717-767)
      std::vector<float> lsm(V);
      for (int s = 0; s < S; ++s)
        per_token_loss[size_t(b) * S + s] = or_ce_forward(sq.logits.data() + size_t(s) * V, V, int(tgt[s]), lsm.data());
    }
    const float seq_loss = or_ce_forward_backward_batch(sq.logits.data(), tgt, S, V, sq.dlogits.data(), 1.0f / float(S));
    total += seq_loss / float(S);
  }
  if (loss_out) *loss_out = total / float(batch);
  return 0;
}

// Backward of the sequences of the last or_forward (full_model::backward_ws,
// full_model.rs:250-331); gradients accumulate (beta = 1).
OR_API int or_backward(const OrConfig* cfg, const OrModel* w, OrWs* ws, const uint32_t* tokens, int batch,
                       float softcap, float loss_scale, OrModel* g) {
  const int D = cfg->dim, S = cfg->seq, V = cfg->vocab;
  std::vector<float> dl(size_t(S) * V), dx_final(size_t(D) * S), dy(size_t(D) * S), dy_buf(size_t(D) * S);
  for (int b = 0; b < batch; ++b) {
    OrSeq& sq = ws->seqs[b];
    const uint32_t* tok = tokens + size_t(b) * S;
    if (softcap > 0.f) {
      for (size_t i = 0; i < dl.size(); ++i)
        dl[i] = sq.dlogits[i] * loss_scale * (1.0f - sq.logits_capped[i] * sq.logits_capped[i]);
    } else {
      for (size_t i = 0; i < dl.size(); ++i) dl[i] = sq.dlogits[i] * loss_scale;
    }
    // dx_final[d][s] = sum_v embed[v][d] dl[s][v]
    sgemm(true, true, D, S, V, 1.f, w->embed, D, dl.data(), V, 0.f, dx_final.data(), S);
    // dembed[v][d] += sum_s dl[s][v] x_final[d][s]
    sgemm(true, true, V, D, S, 1.f, dl.data(), V, sq.x_final.data(), S, 1.f, g->embed, D);
    or_rmsnorm_backward_cf(dx_final.data(), sq.x_prenorm.data(), w->gamma_final, sq.rms_inv_final.data(), dy.data(),
                           g->gamma_final, D, S);
    for (int l = cfg->nlayers - 1; l >= 0; --l) {
      layer_backward(*cfg, *ws, w->layers[l], sq.caches[l], dy.data(), g->layers[l], dy_buf.data());
      std::swap(dy, dy_buf);
    }
    or_embedding_backward_cf(dy.data(), D, tok, S, g->embed);
  }
  return 0;
}

namespace {
template <typename F>
void for_each_tensor(const OrConfig& c, OrModel* m, F&& f) {
  const int64_t D = c.dim, Q = c.q_dim, KV = c.kv_dim, H = c.hidden, V = c.vocab;
  f(m->embed, V * D, 0);
  f(m->gamma_final, D, 1);
  for (int l = 0; l < c.nlayers; ++l) {
    OrLayer& L = m->layers[l];
    f(L.wq, D * Q, 2);
    f(L.wk, D * KV, 2);
    f(L.wv, D * KV, 2);
    f(L.wo, Q * D, 2);
    f(L.w1, D * H, 2);
    f(L.w3, D * H, 2);
    f(L.w2, D * H, 2);
    f(L.gamma1, D, 1);
    f(L.gamma2, D, 1);
  }
}
}  // namespace

// Global L2 norm of all gradients (full_model.rs:598-624): sum of per-tensor
// sums of squares, tensors in the reference's order.
OR_API float or_grad_norm(const OrConfig* cfg, const OrModel* g) {
  double total = 0.0;
  for_each_tensor(*cfg, const_cast<OrModel*>(g), [&](float* p, int64_t n, int) {
    double s = 0.0;
#pragma omp parallel for reduction(+ : s) schedule(static) if (n > 65536)
    for (int64_t i = 0; i < n; ++i) s += double(p[i]) * double(p[i]);
    total += s;
  });
  return static_cast<float>(std::sqrt(total));
}

// clip_grads (full_model.rs:627-645)
OR_API void or_clip_grads(const OrConfig* cfg, OrModel* g, float max_norm) {
  const float norm = or_grad_norm(cfg, g);
  if (norm > max_norm) {
    const float scale = max_norm / norm;
    for_each_tensor(*cfg, g, [&](float* p, int64_t n, int) {
      for (int64_t i = 0; i < n; ++i) p[i] *= scale;
    });
  }
}

// learning_rate (full_model.rs:334-342)
OR_API float or_learning_rate(uint32_t step, const OrTrainConfig* tc) {
  if (step < tc->warmup_steps) return tc->max_lr * float(step + 1) / float(tc->warmup_steps);
  const float decay = float(step - tc->warmup_steps) / float(tc->total_steps - tc->warmup_steps);
  const float min_lr = tc->max_lr * tc->min_lr_frac;
  return min_lr + 0.5f * (1.0f + std::cos(3.14159265358979323846f * decay)) * (tc->max_lr - min_lr);
}

// update_weights (full_model.rs:490-593): embed lr*embed_lr_scale wd 0, gamma_final lr wd 0,
// matrices lr*matrix_lr_scale wd, gamma1/2 lr wd 0; all via step_fused.
OR_API void or_update_weights(const OrConfig* cfg, OrModel* w, const OrModel* g, OrModel* m, OrModel* v, uint32_t t,
                              float lr, const OrTrainConfig* tc, float grad_scale) {
  const float matrix_lr = lr * tc->matrix_lr_scale, embed_lr = lr * tc->embed_lr_scale;
  std::vector<float*> ws, gs, ms, vs;
  std::vector<int64_t> ns;
  std::vector<int> kinds;
  for_each_tensor(*cfg, w, [&](float* p, int64_t n, int kind) {
    ws.push_back(p);
    ns.push_back(n);
    kinds.push_back(kind);
  });
  for_each_tensor(*cfg, const_cast<OrModel*>(g), [&](float* p, int64_t, int) { gs.push_back(p); });
  for_each_tensor(*cfg, m, [&](float* p, int64_t, int) { ms.push_back(p); });
  for_each_tensor(*cfg, v, [&](float* p, int64_t, int) { vs.push_back(p); });
  for (size_t i = 0; i < ws.size(); ++i) {
    const float tlr = kinds[i] == 0 ? embed_lr : (kinds[i] == 2 ? matrix_lr : lr);
    const float wd = kinds[i] == 2 ? tc->weight_decay : 0.f;
    or_adam_step_fused(ws[i], gs[i], ms[i], vs[i], ns[i], t, tlr, tc->beta1, tc->beta2, tc->eps, wd, grad_scale);
  }
}

OR_API void or_grads_zero(const OrConfig* cfg, OrModel* g) {
  for_each_tensor(*cfg, g, [&](float* p, int64_t n, int) { memset(p, 0, sizeof(float) * n); });
}

// One optimizer step over `batch` explicit sequences, equivalent to
// ------------------------------------------------------- single layer
// layer::forward / layer::backward of one sequence (layer.rs:443-..., 1355-...):
// x, x_next, dy, dx in the reference's channel-first [D][S] layout.  The forward
// cache lives in the first cache slot of ws and is what the next backward reads.
OR_API void or_layer_forward(const OrConfig* cfg, OrWs* ws, const OrLayer* w, const float* x, float* x_next) {
  layer_forward(*cfg, *ws, *w, x, ws->seqs[0].caches[0], x_next);
}
// Accumulates into g (LayerGrads semantics).
OR_API void or_layer_backward(const OrConfig* cfg, OrWs* ws, const OrLayer* w, const float* dy, OrLayer* g,
                              float* dx) {
  layer_backward(*cfg, *ws, *w, ws->seqs[0].caches[0], dy, *g, dx);
}

namespace {
template <class F>
void for_each_layer_tensor(const OrConfig& c, OrLayer* l, F&& f) {
  const int64_t D = c.dim, Q = c.q_dim, KV = c.kv_dim, H = c.hidden;
  f(l->wq, D * Q);
  f(l->wk, D * KV);
  f(l->wv, D * KV);
  f(l->wo, Q * D);
  f(l->w1, D * H);
  f(l->w3, D * H);
  f(l->w2, D * H);
  f(l->gamma1, D);
  f(l->gamma2, D);
}
}  // namespace

// training::train_step (training.rs:61-97): forward, loss = mean(x_next^2) (an MSE
// against zero, summed in f32 order), dy = 2 x_next / n, grads zeroed, backward,
// then training::update_weights (training.rs:41-59): adam::step on each tensor
// with one AdamConfig (no lr groups, no clipping).  Returns the loss.
OR_API float or_layer_train_step(const OrConfig* cfg, OrWs* ws, OrLayer* w, OrLayer* g, OrLayer* m, OrLayer* v,
                                 const float* x, uint32_t t, float lr, float beta1, float beta2, float eps,
                                 float weight_decay) {
  const int64_t n = int64_t(cfg->dim) * cfg->seq;
  std::vector<float> y(n), dy(n), dx(n);
  or_layer_forward(cfg, ws, w, x, y.data());
  float loss = 0.f;
  for (int64_t i = 0; i < n; ++i) loss += y[i] * y[i];
  loss /= static_cast<float>(n);
  const float scale = 2.0f / static_cast<float>(n);
  for (int64_t i = 0; i < n; ++i) dy[i] = y[i] * scale;
  for_each_layer_tensor(*cfg, g, [](float* p, int64_t k) { std::fill(p, p + k, 0.f); });
  or_layer_backward(cfg, ws, w, dy.data(), g, dx.data());
  float* wp[9];
  float* gp[9];
  float* mp[9];
  float* vp[9];
  int64_t np[9];
  int i = 0;
  for_each_layer_tensor(*cfg, w, [&](float* p, int64_t k) { wp[i] = p; np[i++] = k; });
  i = 0;
  for_each_layer_tensor(*cfg, g, [&](float* p, int64_t) { gp[i++] = p; });
  i = 0;
  for_each_layer_tensor(*cfg, m, [&](float* p, int64_t) { mp[i++] = p; });
  i = 0;
  for_each_layer_tensor(*cfg, v, [&](float* p, int64_t) { vp[i++] = p; });
  for (int k = 0; k < 9; ++k) or_adam_step(wp[k], gp[k], mp[k], vp[k], np[k], t, lr, beta1, beta2, eps, weight_decay);
  return loss;
}

// full_model::train_step (full_model.rs:661-714) with accum_steps = batch:
// zero grads, forward+backward per sequence, clip decision, lr, AdamW(t = step+1).
OR_API float or_train_step_batch(const OrConfig* cfg, OrModel* w, OrModel* g, OrModel* m, OrModel* v,
                                 const uint32_t* tokens, const uint32_t* targets, int batch, uint32_t step,
                                 const OrTrainConfig* tc, OrWs* ws, float* raw_norm_out) {
  or_grads_zero(cfg, g);
  float loss = 0.f;
  if (or_forward(cfg, w, tokens, targets, batch, tc->softcap, ws, &loss, nullptr, nullptr) != 0) return NAN;
  or_backward(cfg, w, ws, tokens, batch, tc->softcap, tc->loss_scale, g);
  const float gsc = 1.0f / (float(batch) * tc->loss_scale);
  const float raw = or_grad_norm(cfg, g);
  const float combined = (raw * gsc > tc->grad_clip) ? tc->grad_clip / raw : gsc;
  const float lr = or_learning_rate(step, tc);
  or_update_weights(cfg, w, g, m, v, step + 1, lr, tc, combined);
  if (raw_norm_out) *raw_norm_out = raw;
  return loss;
}

// The reference's train_step on a u16 token stream: microbatch positions from
// its LCG, pos = (step*7919 + micro*104729) % (len - seq - 1) (full_model.rs:678-694).
OR_API void or_train_positions(uint32_t step, uint32_t accum_steps, int64_t n_data, int seq, int64_t* pos_out) {
  const uint64_t max_pos = uint64_t(n_data - seq - 1);
  for (uint32_t micro = 0; micro < accum_steps; ++micro)
    pos_out[micro] = int64_t((uint64_t(step) * 7919ull + uint64_t(micro) * 104729ull) % max_pos);
}
